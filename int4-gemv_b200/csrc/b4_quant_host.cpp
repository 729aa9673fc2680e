// b4_quant_host.cpp -- host quantisers of the C ABI (b4_quantise_int4_g128,
// b4_quantise_nf4_b64).  Output is byte-identical to the reference's host
// quantisers (kernels.cuh:268-339); the code here is organised differently:
//
//   * a format is a "codec" with three rules -- the scale of a run of weights,
//     the code of one weight under that scale, the dequantised value of a
//     code -- and one driver applies a codec to every run of every row;
//   * codes are packed through a small nibble writer (column k goes to
//     nibble k % 8 of word k / 8, the reference's low-nibble-first layout);
//   * host threads take rows from a shared atomic cursor.
//
// Both formats' numerics are fixed by the format (they define the bytes a
// drop-in must produce): INT4 scale = fp16(amax / 7), code = clamp(round(w /
// scale) + 8, 0, 15) with glibc's lround; NF4 absmax = amax (1 for an all-zero
// block), code = the first index of the smallest |w / absmax - NF4[c]|.
// Compiled with -ffp-contract=off and without fast-math: every value is one
// IEEE operation.
#include <cuda_fp16.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

#include "../../include/b4gemv.h"

namespace {

// The canonical NormalFloat code book (the same 16 literals as kernels.cuh:78-83).
constexpr float kNormalFloat[16] = {
    -1.0f,                 -0.6961928009986877f,  -0.5250730514526367f,
    -0.39491748809814453f, -0.28444138169288635f, -0.18477343022823334f,
    -0.09105003625154495f, 0.0f,                  0.07958029955625534f,
    0.16093020141124725f,  0.24611230194568634f,  0.33791524171829224f,
    0.44070982933044434f,  0.5626170039176941f,   0.7229568362236023f,
    1.0f};

// glibc x86-64's (int)std::lround(q): a quotient that is NaN, infinite or
// beyond the range of long rounds to LONG_MIN, and the int conversion keeps
// its low 32 bits, which are 0.
int glibc_lround_to_int(float q)
{
    if (!(std::fabs(q) < 0x1p63f)) return 0;
    return static_cast<int>(static_cast<uint32_t>(static_cast<unsigned long>(std::lround(q))));
}

float largest_magnitude(const float* w, int n)
{
    float m = 0.0f;
    for (const float* e = w + n; w != e; ++w) m = std::max(m, std::fabs(*w));
    return m;
}

// INT4 with one fp16 scale per 128 columns.
struct Int4Codec {
    static constexpr int kRun = B4_GROUP;
    using Scale = uint16_t;   // fp16 bits
    float step = 1.0f;        // the fp16 scale, widened

    Scale begin_run(const float* w)
    {
        const float m = largest_magnitude(w, kRun);
        const __half h = __float2half(m > 0.0f ? m / 7.0f : 1.0f);
        step = __half2float(h);
        Scale bits;
        std::memcpy(&bits, &h, sizeof(bits));
        return bits;
    }
    int code(float w) const { return std::clamp(glibc_lround_to_int(w / step) + 8, 0, 15); }
    float value(int c) const { return static_cast<float>(c - 8) * step; }
};

// NF4 with one fp32 absmax per 64 columns.
struct Nf4Codec {
    static constexpr int kRun = B4_NF4_BLOCK;
    using Scale = float;
    float amax = 1.0f;

    Scale begin_run(const float* w)
    {
        const float m = largest_magnitude(w, kRun);
        amax = m == 0.0f ? 1.0f : m;
        return amax;
    }
    int code(float w) const
    {
        const float t = w / amax;
        float dist[16];
        for (int c = 0; c < 16; ++c) dist[c] = std::fabs(t - kNormalFloat[c]);
        // the smallest distance, the lowest index among equals (a NaN distance never wins)
        int pick = 0;
        for (int c = 1; c < 16; ++c) pick = dist[c] < dist[pick] ? c : pick;
        return pick;
    }
    float value(int c) const { return kNormalFloat[c] * amax; }
};

// Packs one row's codes, eight per 32-bit word, low nibble first.
class NibbleWriter {
public:
    explicit NibbleWriter(uint32_t* words) : out_(words) {}
    void put(int code)
    {
        acc_ |= static_cast<uint32_t>(code) << (4 * fill_);
        if (++fill_ == 8) {
            *out_++ = acc_;
            acc_ = 0;
            fill_ = 0;
        }
    }

private:
    uint32_t* out_;
    uint32_t acc_ = 0;
    int fill_ = 0;
};

// Quantises rows with `codec` on up to `nthreads` host threads (<= 0: every
// online core); each row's runs write their scale, their codes and, when
// `deq` is given, the dequantised weights.
template <typename Codec>
void quantise_rows(const float* W, int out_f, int in_f, uint32_t* packed, typename Codec::Scale* scales,
                   float* deq, int nthreads)
{
    const int runs = in_f / Codec::kRun;
    std::atomic<int> next_row{0};
    auto worker = [&]() {
        Codec codec;
        for (int r; (r = next_row.fetch_add(1, std::memory_order_relaxed)) < out_f;) {
            const float* w = W + static_cast<size_t>(r) * in_f;
            float* d = deq ? deq + static_cast<size_t>(r) * in_f : nullptr;
            NibbleWriter nibbles(packed + static_cast<size_t>(r) * (in_f / 8));
            for (int run = 0; run < runs; ++run, w += Codec::kRun) {
                scales[static_cast<size_t>(r) * runs + run] = codec.begin_run(w);
                for (int k = 0; k < Codec::kRun; ++k) {
                    const int c = codec.code(w[k]);
                    nibbles.put(c);
                    if (d) *d++ = codec.value(c);
                }
            }
        }
    };
    int n = nthreads > 0 ? nthreads : static_cast<int>(std::max(1u, std::thread::hardware_concurrency()));
    n = std::max(1, std::min(n, out_f));
    std::vector<std::thread> helpers;
    helpers.reserve(n - 1);
    for (int t = 1; t < n; ++t) helpers.emplace_back(worker);
    worker();
    for (auto& h : helpers) h.join();
}

}  // namespace

extern "C" {

int b4_quantise_int4_g128(const float* W, int out_f, int in_f, uint32_t* packed, uint16_t* scales, float* deq,
                          int nthreads)
{
    if (!W || !packed || !scales || out_f <= 0 || in_f <= 0 || in_f % B4_GROUP) return 1;
    quantise_rows<Int4Codec>(W, out_f, in_f, packed, scales, deq, nthreads);
    return 0;
}

int b4_quantise_nf4_b64(const float* W, int out_f, int in_f, uint32_t* packed, float* absmax, float* deq,
                        int nthreads)
{
    if (!W || !packed || !absmax || out_f <= 0 || in_f <= 0 || in_f % B4_NF4_BLOCK) return 1;
    quantise_rows<Nf4Codec>(W, out_f, in_f, packed, absmax, deq, nthreads);
    return 0;
}

}  // extern "C"
