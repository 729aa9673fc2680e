// b4_common.cuh -- formats and device helpers shared by the sm_100a kernels.
//
// Weight formats (byte-identical to QuantumDrizzy/int4-gemv, src/kernels.cuh):
//   packed codes : uint32 [out_f][in_f/8]; column k is nibble k%8 of word k/8,
//                  low nibble first                          (kernels.cuh:289)
//   INT4 g128    : fp16 scale [out_f][in_f/128], w = (code-8) * scale
//                                                     (kernels.cuh:12,50,282)
//   NF4  b64     : fp32 absmax [out_f][in_f/64],  w = NF4[code] * absmax
//                                                  (kernels.cuh:78-85,121,322)
#pragma once

#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace b4 {

constexpr int kGroup = 128;     // INT4 columns per fp16 scale
constexpr int kNf4Block = 64;   // NF4 columns per fp32 absmax

enum Format : int { kInt4 = 0, kNf4 = 1 };

// The canonical 16-entry NormalFloat table (the bitsandbytes NF4 code book),
// the same 16 float literals as kernels.cuh:78-83.
#define B4_NF4_VALUES                                                          \
    -1.0f, -0.6961928009986877f, -0.5250730514526367f, -0.39491748809814453f, \
        -0.28444138169288635f, -0.18477343022823334f, -0.09105003625154495f,  \
        0.0f, 0.07958029955625534f, 0.16093020141124725f,                     \
        0.24611230194568634f, 0.33791524171829224f, 0.44070982933044434f,     \
        0.5626170039176941f, 0.7229568362236023f, 1.0f

// One copy per translation unit (no relocatable device code).
static __constant__ float c_nf4_table[16] = {B4_NF4_VALUES};

// ---- global loads -----------------------------------------------------------
// Packed codes are read exactly once per GEMV: non-coherent path, no L1
// allocation, so they do not evict x, scales or the reduction scratch.
template <int VW>
struct WordVec;
template <>
struct WordVec<1> { uint32_t w[1]; };
template <>
struct WordVec<2> { uint32_t w[2]; };
template <>
struct WordVec<4> { uint32_t w[4]; };

template <int VW>
__device__ __forceinline__ WordVec<VW> ld_stream(const uint32_t* p);

template <>
__device__ __forceinline__ WordVec<1> ld_stream<1>(const uint32_t* p)
{
    WordVec<1> v;
    asm("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v.w[0]) : "l"(p));
    return v;
}
template <>
__device__ __forceinline__ WordVec<2> ld_stream<2>(const uint32_t* p)
{
    WordVec<2> v;
    asm("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];"
        : "=r"(v.w[0]), "=r"(v.w[1]) : "l"(p));
    return v;
}
template <>
__device__ __forceinline__ WordVec<4> ld_stream<4>(const uint32_t* p)
{
    WordVec<4> v;
    asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
        : "=r"(v.w[0]), "=r"(v.w[1]), "=r"(v.w[2]), "=r"(v.w[3]) : "l"(p));
    return v;
}

// ---- INT4 decode ------------------------------------------------------------
// One LOP3 turns two nibbles into two exact fp16 integers: OR-ing a nibble into
// the mantissa of 1024.0 (0x6400) gives 1024+n, into bits 4..7 of the mantissa
// of 64.0 (0x5400) gives 64+n.  One HSUB2 then yields code-8 exactly (all
// values are small integers).  For a word w with nibbles n0..n7 this returns
//   h[0] = (n0-8, n4-8)   h[1] = (n1-8, n5-8)
//   h[2] = (n2-8, n6-8)   h[3] = (n3-8, n7-8)
// as half2 (low half first).  x is staged in the matching pair order.
// The mask-and-OR is one PTX lop3 with the mask as an immediate and the magic
// constant as a register operand (shared by every use with the same magic):
// measured on sm_100a, the equivalent C expression `(a & m) | k` compiles to
// two logic instructions per use, which doubled the integer work of the
// decode.
template <uint32_t MASK, uint32_t MAGIC>
__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a)
{
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, 0xea;" : "=r"(r) : "r"(a), "n"(MASK), "r"(MAGIC));   // (a & b) | c
    return r;
}

__device__ __forceinline__ uint32_t hsub2_bits(uint32_t a, uint16_t k)
{
    __half2_raw kr;
    kr.x = k;
    kr.y = k;
    const __half2 r = __hsub2(*reinterpret_cast<const __half2*>(&a), __half2(kr));
    return *reinterpret_cast<const uint32_t*>(&r);
}

__device__ __forceinline__ void int4_word_to_half2(uint32_t w, uint32_t h[4])
{
    const uint32_t w8 = w >> 8;
    h[0] = hsub2_bits(lop3_and_or<0x000f000fu, 0x64006400u>(w), 0x6408);   // - 1032
    h[1] = hsub2_bits(lop3_and_or<0x00f000f0u, 0x54005400u>(w), 0x5480);   // - 72
    h[2] = hsub2_bits(lop3_and_or<0x000f000fu, 0x64006400u>(w8), 0x6408);
    h[3] = hsub2_bits(lop3_and_or<0x00f000f0u, 0x54005400u>(w8), 0x5480);
}

// INT4 decode to fp32 for the CUDA-core kernel: OR-ing nibble j into the
// mantissa of 2^23 (0x4b000000) gives 2^23 + n_j * 2^p_j exactly, for nibble
// positions p_j <= 19; nibbles 5..7 are taken from w >> 12 so that
// p = {0, 4, 8, 12, 16, 8, 12, 16}.  Subtracting 2^23 + 8 * 2^p_j (exact:
// integers below 2^24) leaves (n_j - 8) * 2^p_j; d[k] holds codes 2k, 2k+1.
__device__ __forceinline__ void int4_word_to_f32x2(uint32_t w, float2 d[4])
{
    const uint32_t hi = w >> 12;
    const float f0 = __uint_as_float(lop3_and_or<0x0000000fu, 0x4b000000u>(w));
    const float f1 = __uint_as_float(lop3_and_or<0x000000f0u, 0x4b000000u>(w));
    const float f2 = __uint_as_float(lop3_and_or<0x00000f00u, 0x4b000000u>(w));
    const float f3 = __uint_as_float(lop3_and_or<0x0000f000u, 0x4b000000u>(w));
    const float f4 = __uint_as_float(lop3_and_or<0x000f0000u, 0x4b000000u>(w));
    const float f5 = __uint_as_float(lop3_and_or<0x00000f00u, 0x4b000000u>(hi));
    const float f6 = __uint_as_float(lop3_and_or<0x0000f000u, 0x4b000000u>(hi));
    const float f7 = __uint_as_float(lop3_and_or<0x000f0000u, 0x4b000000u>(hi));
    d[0] = __fadd2_rn(make_float2(f0, f1), make_float2(-(0x1p23f + 8.0f), -(0x1p23f + 128.0f)));
    d[1] = __fadd2_rn(make_float2(f2, f3), make_float2(-(0x1p23f + 2048.0f), -(0x1p23f + 32768.0f)));
    d[2] = __fadd2_rn(make_float2(f4, f5), make_float2(-(0x1p23f + 524288.0f), -(0x1p23f + 2048.0f)));
    d[3] = __fadd2_rn(make_float2(f6, f7), make_float2(-(0x1p23f + 32768.0f), -(0x1p23f + 524288.0f)));
}

// Two fp32 accumulations from fp16 pairs with one rounding each (sm_100
// mixed-precision FMA): acc_lo += a.lo*b.lo, acc_hi += a.hi*b.hi.
__device__ __forceinline__ void fma2_f32_f16(float& acc_lo, float& acc_hi, uint32_t a, uint32_t b)
{
    asm("{\n\t.reg .b16 al, ah, bl, bh;\n\t"
        "mov.b32 {al, ah}, %2;\n\t"
        "mov.b32 {bl, bh}, %3;\n\t"
        "fma.rn.f32.f16 %0, al, bl, %0;\n\t"
        "fma.rn.f32.f16 %1, ah, bh, %1;\n\t}"
        : "+f"(acc_lo), "+f"(acc_hi)
        : "r"(a), "r"(b));
}

// Reorders the 8 fp16 values of one word's columns, x0..x7 held as four
// half2 (x0,x1)(x2,x3)(x4,x5)(x6,x7), into the decode's pair order
// (x0,x4)(x1,x5)(x2,x6)(x3,x7).
__device__ __forceinline__ uint4 int4_pair_order(uint4 v)
{
    uint4 r;
    r.x = __byte_perm(v.x, v.z, 0x5410);  // x0, x4
    r.y = __byte_perm(v.x, v.z, 0x7632);  // x1, x5
    r.z = __byte_perm(v.y, v.w, 0x5410);  // x2, x6
    r.w = __byte_perm(v.y, v.w, 0x7632);  // x3, x7
    return r;
}

// One 16-byte word of x (8 fp16 values at src): a single 16-byte load when x is
// 16-byte aligned, else eight 2-byte loads.
__device__ __forceinline__ uint4 ld_x_word(const __half* src, bool vec)
{
    if (vec) return __ldg(reinterpret_cast<const uint4*>(src));
    const unsigned short* h = reinterpret_cast<const unsigned short*>(src);
    uint4 raw;
    raw.x = (uint32_t)__ldg(h + 0) | ((uint32_t)__ldg(h + 1) << 16);
    raw.y = (uint32_t)__ldg(h + 2) | ((uint32_t)__ldg(h + 3) << 16);
    raw.z = (uint32_t)__ldg(h + 4) | ((uint32_t)__ldg(h + 5) << 16);
    raw.w = (uint32_t)__ldg(h + 6) | ((uint32_t)__ldg(h + 7) << 16);
    return raw;
}

// Stages n 16-byte words of x (word i at x + 8i) into shared memory through
// store(i, word).  Each thread loads XU of its words (i = tid, tid + blockDim,
// ...) into registers before it stores any, so it waits for one memory round
// trip per XU words instead of one per word: x is read after the
// grid-dependency wait, on the kernel's critical path, and a long row (down_proj:
// 2368 words for 256 threads) would otherwise cost ten round trips.
template <int XU, typename Store>
__device__ __forceinline__ void stage_x_words(const __half* x, int n, bool vec, Store store)
{
    for (int i0 = threadIdx.x; i0 < n; i0 += XU * blockDim.x) {
        uint4 r[XU];
#pragma unroll
        for (int u = 0; u < XU; ++u) {
            const int i = i0 + u * (int)blockDim.x;
            r[u] = i < n ? ld_x_word(x + (long long)i * 8, vec) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int u = 0; u < XU; ++u) {
            const int i = i0 + u * (int)blockDim.x;
            if (i < n) store(i, r[u]);
        }
    }
}

constexpr int kXUnroll = 8;   // x words in flight per thread while staging

// The gated activation of the decode layer's MLP: silu(g) = g / (1 + e^-g),
// with the hardware exponential (__expf) and the approximate divide
// (__fdividef): a few instructions, where expf and an IEEE divide cost tens,
// which matters because every CTA of a GEMV that stages its x from gate/up
// rows computes all in_f of them.  The relative error stays near 2^-20 for
// |g| < 20 (far below the fp16 rounding of x that follows); a g below about
// -87 gives -0 (the true value is below 1e-36).  The SwiGLU glue kernel and the
// GEMVs that compute their x from gate/up rows use this one definition, so
// both round the same way.
__device__ __forceinline__ float swiglu_silu(float g) { return __fdividef(g, 1.0f + __expf(-g)); }

// stage_x_words for an x computed as fp16(silu(gate[k]) * up[k]) from fp32
// gate = gu[0 .. n_words * 8), up = gu[n_words * 8 ..): gu 16-byte aligned.
template <int XU, typename Store>
__device__ __forceinline__ void stage_x_swiglu(const float* gu, int n_words, Store store)
{
    const float4* g4 = reinterpret_cast<const float4*>(gu);
    const float4* u4 = g4 + 2 * (size_t)n_words;
    for (int i0 = threadIdx.x; i0 < n_words; i0 += XU * blockDim.x) {
        float4 g[XU][2], u[XU][2];
#pragma unroll
        for (int k = 0; k < XU; ++k) {
            const int i = i0 + k * (int)blockDim.x;
            if (i < n_words) {
                g[k][0] = g4[2 * i];
                g[k][1] = g4[2 * i + 1];
                u[k][0] = u4[2 * i];
                u[k][1] = u4[2 * i + 1];
            }
        }
#pragma unroll
        for (int k = 0; k < XU; ++k) {
            const int i = i0 + k * (int)blockDim.x;
            if (i < n_words) {
                const float gv[8] = {g[k][0].x, g[k][0].y, g[k][0].z, g[k][0].w, g[k][1].x, g[k][1].y, g[k][1].z, g[k][1].w};
                const float uv[8] = {u[k][0].x, u[k][0].y, u[k][0].z, u[k][0].w, u[k][1].x, u[k][1].y, u[k][1].z, u[k][1].w};
                uint32_t h[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const __half lo = __float2half_rn(swiglu_silu(gv[2 * j]) * uv[2 * j]);
                    const __half hi = __float2half_rn(swiglu_silu(gv[2 * j + 1]) * uv[2 * j + 1]);
                    h[j] = (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
                }
                store(i, make_uint4(h[0], h[1], h[2], h[3]));
            }
        }
    }
}

// x of a small batch in shared memory, for B fragments that lane q reads as
// logical words 4q .. 4q + 3 of a 16-word group (one 16-byte load per word):
// each row's 16-word groups are stored transposed (word s at 4 (s & 3) + (s >> 2))
// so that the four q lanes of a load read four consecutive 16-byte slots, and
// rows are kXmbPad words longer than in_f / 8 (a row stride of 4 slots mod 8),
// so the two rows of a quarter warp take the two halves of the 32 banks.
constexpr int kXmbPad = 4;

__host__ __device__ constexpr int xmb_stride(int words) { return words + kXmbPad; }

__device__ __forceinline__ int xmb_slot(int w) { return (w & ~15) | ((w & 3) << 2) | ((w >> 2) & 3); }

// stage_x_words over [m][words] with store(row, word, value)
template <int XU, typename Store>
__device__ __forceinline__ void stage_x_rows(const __half* x, int m, int words, bool vec, Store store)
{
    const int n = m * words;
    const float inv = 1.0f / (float)words;
    for (int i0 = threadIdx.x; i0 < n; i0 += XU * blockDim.x) {
        uint4 r[XU];
#pragma unroll
        for (int u = 0; u < XU; ++u) {
            const int i = i0 + u * (int)blockDim.x;
            r[u] = i < n ? ld_x_word(x + (long long)i * 8, vec) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int u = 0; u < XU; ++u) {
            const int i = i0 + u * (int)blockDim.x;
            if (i < n) {
                int row = __float2int_rz(__int2float_rn(i) * inv);   // i / words, corrected below
                if (row * words > i) --row;
                else if ((row + 1) * words <= i) ++row;
                store(row, i - row * words, r[u]);
            }
        }
    }
}

// the same with source rows src_ld words (of 8 halves) apart
template <int XU, typename Store>
__device__ __forceinline__ void stage_x_rows(const __half* x, int m, int words, int src_ld, bool vec, Store store)
{
    const int n = m * words;
    const float inv = 1.0f / (float)words;
    for (int i0 = threadIdx.x; i0 < n; i0 += XU * blockDim.x) {
        uint4 r[XU];
        int row[XU];
#pragma unroll
        for (int u = 0; u < XU; ++u) {
            const int i = i0 + u * (int)blockDim.x;
            int rr = __float2int_rz(__int2float_rn(i) * inv);   // i / words, corrected below
            if (rr * words > i) --rr;
            else if ((rr + 1) * words <= i) ++rr;
            row[u] = rr;
            r[u] = i < n ? ld_x_word(x + ((long long)rr * src_ld + (i - rr * words)) * 8, vec) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int u = 0; u < XU; ++u) {
            const int i = i0 + u * (int)blockDim.x;
            if (i < n) store(row[u], i - row[u] * words, r[u]);
        }
    }
}

// ---- NF4 decode ---------------------------------------------------------------
// Warp-register code book: lane L holds NF4[L & 15]; a shuffle with the packed
// word shifted right by 4k as the source lane reads NF4[nibble k], since the
// shuffle uses only the low 5 bits of the lane index and lanes 16..31 mirror
// lanes 0..15.
__device__ __forceinline__ float nf4_lane_value(int lane) { return c_nf4_table[lane & 15]; }

__device__ __forceinline__ float nf4_lookup_shfl(float lut, uint32_t idx)
{
    return __shfl_sync(0xffffffffu, lut, (int)idx);
}

}  // namespace b4
