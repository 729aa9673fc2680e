// b4_quant_host.cpp -- host quantisers of the C ABI (b4_quantise_int4_g128,
// b4_quantise_nf4_b64): the reference's quantise() and quantise_nf4()
// (kernels.cuh:268-339) with byte-identical output, rows spread over host
// threads.  Compiled with -ffp-contract=off and without fast-math: every
// value is one IEEE operation, as in the reference.
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

#include "../../include/b4gemv.h"

namespace {

const float kNf4[16] = {
    -1.0f,                 -0.6961928009986877f,  -0.5250730514526367f,
    -0.39491748809814453f, -0.28444138169288635f, -0.18477343022823334f,
    -0.09105003625154495f, 0.0f,                  0.07958029955625534f,
    0.16093020141124725f,  0.24611230194568634f,  0.33791524171829224f,
    0.44070982933044434f,  0.5626170039176941f,   0.7229568362236023f,
    1.0f};

// (int)std::lround(q) on glibc x86-64 (kernels.cuh:286): non-finite or
// out-of-range quotients give LONG_MIN, whose low 32 bits are 0.
inline int lround_int(float q)
{
    if (!(std::fabs(q) < 0x1p63f)) return 0;
    const long l = std::lround(q);
    return static_cast<int>(static_cast<uint32_t>(static_cast<unsigned long>(l)));
}

template <typename Fn>
void parallel_rows(int out_f, int nthreads, Fn fn)
{
    if (nthreads <= 0) nthreads = (int)std::max(1u, std::thread::hardware_concurrency());
    nthreads = std::max(1, std::min(nthreads, out_f));
    if (nthreads == 1) { fn(0, out_f); return; }
    std::vector<std::thread> th;
    th.reserve(nthreads - 1);
    for (int t = 1; t < nthreads; ++t) {
        const int r0 = (int)((long long)out_f * t / nthreads);
        const int r1 = (int)((long long)out_f * (t + 1) / nthreads);
        th.emplace_back(fn, r0, r1);
    }
    fn(0, (int)((long long)out_f / nthreads));
    for (auto& t : th) t.join();
}

}  // namespace

extern "C" {

int b4_quantise_int4_g128(const float* W, int out_f, int in_f, uint32_t* packed,
                          uint16_t* scales, float* deq, int nthreads)
{
    if (!W || !packed || !scales || out_f <= 0 || in_f <= 0 || in_f % B4_GROUP) return 1;
    const int groups = in_f / B4_GROUP, words = in_f / 8;
    parallel_rows(out_f, nthreads, [=](int r0, int r1) {
        for (int r = r0; r < r1; ++r) {
            std::memset(packed + (size_t)r * words, 0, sizeof(uint32_t) * words);
            for (int g = 0; g < groups; ++g) {
                const size_t off = (size_t)r * in_f + (size_t)g * B4_GROUP;
                float amax = 0.0f;
                for (int i = 0; i < B4_GROUP; ++i) amax = std::max(amax, std::fabs(W[off + i]));
                const float s = (amax > 0.0f) ? amax / 7.0f : 1.0f;
                const __half sh = __float2half(s);
                uint16_t bits;
                std::memcpy(&bits, &sh, 2);
                scales[(size_t)r * groups + g] = bits;
                const float s_used = __half2float(sh);
                for (int i = 0; i < B4_GROUP; ++i) {
                    int code = lround_int(W[off + i] / s_used) + 8;
                    code = std::min(15, std::max(0, code));
                    const int idx = g * B4_GROUP + i;
                    packed[(size_t)r * words + idx / 8] |= (uint32_t)code << ((idx % 8) * 4);
                    if (deq) deq[off + i] = (float)(code - 8) * s_used;
                }
            }
        }
    });
    return 0;
}

int b4_quantise_nf4_b64(const float* W, int out_f, int in_f, uint32_t* packed,
                        float* absmax, float* deq, int nthreads)
{
    if (!W || !packed || !absmax || out_f <= 0 || in_f <= 0 || in_f % B4_NF4_BLOCK) return 1;
    const int blocks = in_f / B4_NF4_BLOCK, words = in_f / 8;
    parallel_rows(out_f, nthreads, [=](int r0, int r1) {
        for (int r = r0; r < r1; ++r) {
            std::memset(packed + (size_t)r * words, 0, sizeof(uint32_t) * words);
            for (int b = 0; b < blocks; ++b) {
                const size_t off = (size_t)r * in_f + (size_t)b * B4_NF4_BLOCK;
                float amax = 0.0f;
                for (int i = 0; i < B4_NF4_BLOCK; ++i) amax = std::max(amax, std::fabs(W[off + i]));
                if (amax == 0.0f) amax = 1.0f;
                absmax[(size_t)r * blocks + b] = amax;
                for (int i = 0; i < B4_NF4_BLOCK; ++i) {
                    const float norm = W[off + i] / amax;
                    int best = 0;
                    float bd = std::fabs(norm - kNf4[0]);
                    for (int c = 1; c < 16; ++c) {
                        const float d = std::fabs(norm - kNf4[c]);
                        if (d < bd) { bd = d; best = c; }
                    }
                    const int idx = b * B4_NF4_BLOCK + i;
                    packed[(size_t)r * words + idx / 8] |= (uint32_t)best << ((idx % 8) * 4);
                    if (deq) deq[off + i] = kNf4[best] * amax;
                }
            }
        }
    });
    return 0;
}

}  // extern "C"
