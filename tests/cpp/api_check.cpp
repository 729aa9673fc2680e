// Host-side check of include/b4gemv.hpp written the way the reference's
// benchmark driver calls its header (int4_gemv.cu:139-168): srand(0), uniform
// rand() weights, then quantise()/quantise_nf4() with the same arguments.
// Prints the outputs as hex for tests/test_cpp_api.py to compare with the
// reference-generated fixture.
#define B4GEMV_GLOBAL_NAMES
#include "b4gemv.hpp"

#include <cstdio>
#include <cstdlib>
#include <cstring>

int main()
{
    const int out_f = 2, in_f = 256;
    std::vector<float> W((size_t)out_f * in_f), xh(in_f);
    std::srand(0);
    for (auto& w : W) w = ((float)std::rand() / RAND_MAX - 0.5f) * 0.04f;
    for (auto& v : xh) v = ((float)std::rand() / RAND_MAX - 0.5f);

    std::vector<uint32_t> p4; std::vector<half> s4; std::vector<float> d4;
    quantise(W, out_f, in_f, p4, s4, d4);
    std::vector<uint32_t> pn; std::vector<float> an, dn;
    quantise_nf4(W, out_f, in_f, pn, an, dn);

    std::printf("int4_packed");
    for (auto v : p4) std::printf(" %08x", v);
    std::printf("\nint4_scales");
    for (auto h : s4) { uint16_t b; std::memcpy(&b, &h, 2); std::printf(" %04x", b); }
    std::printf("\nnf4_packed");
    for (auto v : pn) std::printf(" %08x", v);
    std::printf("\nnf4_absmax");
    for (auto a : an) { uint32_t b; std::memcpy(&b, &a, 4); std::printf(" %08x", b); }
    std::printf("\n");
    std::vector<float> t = {3.f, 1.f, 2.f, 4.f};
    std::printf("median %g\n", median(t));
    // bad shape: a status, not an exit
    try {
        quantise(W, out_f, 100, p4, s4, d4);
        std::printf("bad_shape no_throw\n");
    } catch (const b4gemv::error& e) {
        std::printf("bad_shape status %d\n", e.status);
    }
    return 0;
}
