// b4_gemv_kernel.cuh -- the sm_100a fused 4-bit dequantisation GEMV kernel.
//
// Replaces the reference's int4_gemv_warp_per_row (kernels.cuh:26-62),
// nf4_gemv_warp_per_row (kernels.cuh:87-132) and nf4_gemv_block_per_row
// (kernels.cuh:211-266) with one templated kernel:
//
//  * A warp owns RW rows (a "row group") and a slice of in_f; warps_k warps of
//    one CTA share a row group and split in_f between them, then reduce
//    through shared memory in a fixed order (deterministic, no atomics).
//    warps_k = 1 is warp-per-row(s); rows_per_warp = 1 with warps_k = w is the
//    reference's block-per-row with w warps.
//  * Lanes read VW consecutive packed words (VW*8 columns, "a chunk") per row
//    per step with 4/8/16-byte non-allocating loads; consecutive lanes read
//    consecutive chunks, so a warp load is one contiguous 32*VW*4-byte run.
//    The next step's loads for all RW rows are in flight while the current
//    step is decoded (register double buffering), and the first step's loads
//    are issued before the kernel waits on the producer of x (PDL).
//  * x is staged once per CTA in shared memory (INT4: fp16 in decode pair
//    order; NF4: fp32), swizzled so that the 16-byte reads of 8 consecutive
//    lanes hit 8 distinct bank groups.  One staged chunk of x serves all RW
//    rows and all decode work of the chunk is shared by MB batch rows.
//  * Decode.  INT4: one LOP3 per code ORs the nibble into the mantissa of
//    2^23 and one packed FADD2 per two codes subtracts 2^23 + 8*2^p, leaving
//    (code-8)*2^p exactly in fp32; x was staged pre-scaled by 2^-p, so the
//    packed FFMA2 accumulates (code-8)*x with one rounding per product.  The
//    group scale is applied once per chunk (a chunk never crosses a group).
//    NF4: the 16-entry code book sits in the warp's registers (lane L holds
//    NF4[L&15]) and a shuffle does each lookup, as in the reference
//    (kernels.cuh:64-76); optionally a shared-memory copy does it instead.
//    Packed FFMA2 with fp32 x; absmax applied once per chunk.
//  (The INT4 default is the tensor-pipe kernel of b4_gemv_mma.cuh; this one
//   serves INT4 codes that are not 16-byte aligned.)
#pragma once

#include "b4_common.cuh"

namespace b4 {

struct KParams {
    const uint32_t* qw;
    const void* scale;
    const __half* x;
    float* y;
    int in_f, out_f, m;
    long long x_ld, y_ld;
    int kw;           // warps along in_f per row group
    int rg;           // row groups per CTA
    int tile_chunks;  // chunks of x staged per pass
    int x_vec;        // x rows may be read with 16-byte (INT4) / 8-byte (NF4) loads
};

// 16-byte shared-memory slots of staged x per chunk: 8 fp32 values per word.
// The host launcher sizes shared memory with the same function.
__host__ __device__ constexpr int x_slots_per_chunk(int vw) { return 2 * vw; }

template <int F, int VW>
struct XSlots {
    static constexpr int S = x_slots_per_chunk(VW);
};

// Physical slot of logical slot s of tile-relative chunk c: XOR-swizzled so
// that 8 lanes reading slot s of 8 consecutive chunks use 8 distinct 16-byte
// bank groups.
template <int S>
__device__ __forceinline__ int swz(int c, int s)
{
    if constexpr (S >= 8)
        return c * S + (s ^ (c & 7));
    else
        return c * S + (s ^ ((c / (8 / S)) & (S - 1)));
}

// x staged as fp32, 8 values (two 16-byte slots) per packed word.  NF4: the
// values in column order.  INT4: column j of the word pre-multiplied by
// 2^-p_j, p = {0, 4, 8, 12, 16, 8, 12, 16}, the bit position at which the
// magic-number decode leaves nibble j (int4_word_to_f32x2); the scaling is a
// power of two, so every product stays exact.
template <int F, int VW, int MB>
__device__ __forceinline__ void stage_x(const KParams& p, uint4* xs, int mb0, int t0, int tn)
{
    constexpr int S = XSlots<F, VW>::S;
    const int per_b = tn * S;
    const int total = MB * per_b;
    for (int i = threadIdx.x; i < total; i += blockDim.x) {
        const int b = i / per_b;
        const int rem = i - b * per_b;
        const int c = rem / S;
        const int s = rem - c * S;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (mb0 + b < p.m) {
            const __half* xrow = p.x + (long long)(mb0 + b) * p.x_ld;
            const long long col = ((long long)(t0 + c) * VW + (s >> 1)) * 8 + (s & 1) * 4;
            __half2 lo, hi;
            if (p.x_vec) {
                const uint2 raw = __ldg(reinterpret_cast<const uint2*>(xrow + col));
                lo = *reinterpret_cast<const __half2*>(&raw.x);
                hi = *reinterpret_cast<const __half2*>(&raw.y);
            } else {
                lo = __halves2half2(xrow[col + 0], xrow[col + 1]);
                hi = __halves2half2(xrow[col + 2], xrow[col + 3]);
            }
            float2 a = __half22float2(lo), d = __half22float2(hi);
            if constexpr (F == kInt4) {
                if ((s & 1) == 0) {          // columns 0..3: 2^0, 2^-4, 2^-8, 2^-12
                    a.y *= 0x1p-4f;
                    d.x *= 0x1p-8f;
                    d.y *= 0x1p-12f;
                } else {                     // columns 4..7: 2^-16, 2^-8, 2^-12, 2^-16
                    a.x *= 0x1p-16f;
                    a.y *= 0x1p-8f;
                    d.x *= 0x1p-12f;
                    d.y *= 0x1p-16f;
                }
            }
            v = make_uint4(__float_as_uint(a.x), __float_as_uint(a.y), __float_as_uint(d.x), __float_as_uint(d.y));
        }
        xs[b * per_b + swz<S>(c, s)] = v;
    }
}

// One step's worth of packed words and per-chunk scales for RW rows.
template <int VW, int RW>
struct Frag {
    WordVec<VW> w[RW];
    float s[RW];
};

template <int F, int VW, int RW>
__device__ __forceinline__ void load_frag(Frag<VW, RW>& f, const KParams& p, const uint32_t* const* wrow,
                                          const bool* rok, int row0, bool active, int cg)
{
#pragma unroll
    for (int i = 0; i < RW; ++i) {
        const bool ok = active && rok[i];
        if (ok) {
            f.w[i] = ld_stream<VW>(wrow[i] + (long long)cg * VW);
            if constexpr (F == kInt4) {
                const __half* sr = static_cast<const __half*>(p.scale) +
                                   (long long)(row0 + i) * (p.in_f / kGroup);
                f.s[i] = __half2float(__ldg(sr + (cg * VW) / 16));
            } else {
                const float* ar = static_cast<const float*>(p.scale) +
                                  (long long)(row0 + i) * (p.in_f / kNf4Block);
                f.s[i] = __ldg(ar + (cg * VW) / 8);
            }
        } else {
#pragma unroll
            for (int v = 0; v < VW; ++v) f.w[i].w[v] = 0u;
            f.s[i] = 0.0f;
        }
    }
}

template <int F, int VW, int RW, int MB, int LUT>
__device__ __forceinline__ void gemv_step(const Frag<VW, RW>& cur, const uint4 (&xv)[MB][XSlots<F, VW>::S],
                                          float lut, const float* lut_s, float (&acc)[MB][RW])
{
#pragma unroll
    for (int i = 0; i < RW; ++i) {
        float2 pa[MB];
#pragma unroll
        for (int b = 0; b < MB; ++b) pa[b] = make_float2(0.0f, 0.0f);
#pragma unroll
        for (int v = 0; v < VW; ++v) {
            const uint32_t w = cur.w[i].w[v];
            if constexpr (F == kInt4) {
                // decoded pairs come out of FADD2 as register pairs: FFMA2
                float2 d[4];
                int4_word_to_f32x2(w, d);
#pragma unroll
                for (int b = 0; b < MB; ++b) {
                    const uint4 q0 = xv[b][2 * v], q1 = xv[b][2 * v + 1];
                    pa[b] = __ffma2_rn(d[0], make_float2(__uint_as_float(q0.x), __uint_as_float(q0.y)), pa[b]);
                    pa[b] = __ffma2_rn(d[1], make_float2(__uint_as_float(q0.z), __uint_as_float(q0.w)), pa[b]);
                    pa[b] = __ffma2_rn(d[2], make_float2(__uint_as_float(q1.x), __uint_as_float(q1.y)), pa[b]);
                    pa[b] = __ffma2_rn(d[3], make_float2(__uint_as_float(q1.z), __uint_as_float(q1.w)), pa[b]);
                }
            } else {
                // looked-up values land in arbitrary registers: scalar FMA, two chains
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    float t;
                    if constexpr (LUT == 0)
                        t = nf4_lookup_shfl(lut, w >> (4 * k));
                    else
                        t = lut_s[(w >> (4 * k)) & 15u];
#pragma unroll
                    for (int b = 0; b < MB; ++b) {
                        const uint4 q = xv[b][2 * v + (k >> 2)];
                        const uint32_t xb = (k & 3) == 0 ? q.x : (k & 3) == 1 ? q.y : (k & 3) == 2 ? q.z : q.w;
                        if (k & 1)
                            pa[b].y = fmaf(t, __uint_as_float(xb), pa[b].y);
                        else
                            pa[b].x = fmaf(t, __uint_as_float(xb), pa[b].x);
                    }
                }
            }
        }
#pragma unroll
        for (int b = 0; b < MB; ++b) acc[b][i] = fmaf(pa[b].x + pa[b].y, cur.s[i], acc[b][i]);
    }
}

// Threads per CTA the kernel is compiled for: 16 warps only for the
// single-row, single-batch variants (the reference's block-per-row shapes);
// 8 warps otherwise, which leaves up to 255 registers per thread.
template <int RW, int MB>
struct MaxThreads {
    static constexpr int value = (RW == 1 && MB == 1) ? 512 : 256;
};

template <int F, int VW, int RW, int MB, int LUT>
__global__ void __launch_bounds__(MaxThreads<RW, MB>::value) b4_gemv_kernel(const KParams p)
{
    constexpr int S = XSlots<F, VW>::S;
    extern __shared__ uint4 smem_u4[];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int ks = warp % p.kw;
    const int grp = warp / p.kw;
    const int words = p.in_f >> 3;
    const int chunks = words / VW;
    const int rows_per_tile = p.rg * RW;
    const int n_row_tiles = (p.out_f + rows_per_tile - 1) / rows_per_tile;
    const bool one_xtile = chunks <= p.tile_chunks;

    uint4* xs = smem_u4;
    float* red = reinterpret_cast<float*>(xs + MB * p.tile_chunks * S);
    float* lut_s = red + p.rg * p.kw * MB * RW;

    float lut = 0.0f;
    if constexpr (F == kNf4) {
        lut = nf4_lane_value(lane);
        if constexpr (LUT == 1) {
            if (threadIdx.x < 16) lut_s[threadIdx.x] = c_nf4_table[threadIdx.x];
        }
    }

    // Dependents may start their own weight streams now; they wait for this
    // grid's completion before they read its y.
    asm volatile("griddepcontrol.launch_dependents;");

    const int cw = ks * 32;            // first tile-relative chunk of this warp
    const int stride = 32 * p.kw;      // chunks between this warp's steps
    bool waited = false;

    for (int mb0 = 0; mb0 < p.m; mb0 += MB) {
        bool staged = false;
        for (int rt = blockIdx.x; rt < n_row_tiles; rt += gridDim.x) {
            const int row0 = (rt * p.rg + grp) * RW;
            const uint32_t* wrow[RW];
            bool rok[RW];
#pragma unroll
            for (int i = 0; i < RW; ++i) {
                rok[i] = (row0 + i) < p.out_f;
                wrow[i] = p.qw + (long long)(rok[i] ? row0 + i : 0) * words;
            }
            float acc[MB][RW];
#pragma unroll
            for (int b = 0; b < MB; ++b)
#pragma unroll
                for (int i = 0; i < RW; ++i) acc[b][i] = 0.0f;

            for (int t0 = 0; t0 < chunks; t0 += p.tile_chunks) {
                const int tn = min(p.tile_chunks, chunks - t0);
                const int n_it = tn > cw ? (tn - cw + stride - 1) / stride : 0;

                Frag<VW, RW> cur;
                load_frag<F, VW, RW>(cur, p, wrow, rok, row0, n_it > 0 && cw + lane < tn, t0 + cw + lane);
                if (!waited) {
                    // x may be written by the previous kernel in the stream.
                    asm volatile("griddepcontrol.wait;" ::: "memory");
                    waited = true;
                }
                if (!(one_xtile && staged)) {
                    __syncthreads();  // the previous pass is done reading xs
                    stage_x<F, VW, MB>(p, xs, mb0, t0, tn);
                    __syncthreads();
                    staged = true;
                }

                for (int it = 0; it < n_it; ++it) {
                    const int c = cw + it * stride + lane;
                    const bool active = c < tn;
                    Frag<VW, RW> nxt;
                    if (it + 1 < n_it) {
                        const int cn = c + stride;
                        load_frag<F, VW, RW>(nxt, p, wrow, rok, row0, cn < tn, t0 + cn);
                    }
                    uint4 xv[MB][S];
#pragma unroll
                    for (int b = 0; b < MB; ++b)
#pragma unroll
                        for (int s = 0; s < S; ++s)
                            xv[b][s] = active ? xs[b * tn * S + swz<S>(c, s)] : make_uint4(0u, 0u, 0u, 0u);
                    gemv_step<F, VW, RW, MB, LUT>(cur, xv, lut, lut_s, acc);
                    if (it + 1 < n_it) cur = nxt;
                }
            }

            // Close the rows: butterfly within the warp, then the warps_k
            // partials in warp order through shared memory.
#pragma unroll
            for (int b = 0; b < MB; ++b)
#pragma unroll
                for (int i = 0; i < RW; ++i) {
                    float v = acc[b][i];
#pragma unroll
                    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
                    acc[b][i] = v;
                }
            if (p.kw == 1) {
                if (lane == 0) {
#pragma unroll
                    for (int b = 0; b < MB; ++b)
#pragma unroll
                        for (int i = 0; i < RW; ++i)
                            if (rok[i] && mb0 + b < p.m)
                                p.y[(long long)(mb0 + b) * p.y_ld + row0 + i] = acc[b][i];
                }
            } else {
                if (lane == 0) {
#pragma unroll
                    for (int b = 0; b < MB; ++b)
#pragma unroll
                        for (int i = 0; i < RW; ++i) red[((grp * p.kw + ks) * MB + b) * RW + i] = acc[b][i];
                }
                __syncthreads();
                if (ks == 0 && lane < MB * RW) {
                    const int b = lane / RW, i = lane - (lane / RW) * RW;
                    float t = 0.0f;
                    for (int q = 0; q < p.kw; ++q) t += red[((grp * p.kw + q) * MB + b) * RW + i];
                    if (row0 + i < p.out_f && mb0 + b < p.m) p.y[(long long)(mb0 + b) * p.y_ld + row0 + i] = t;
                }
                __syncthreads();
            }
        }
    }
    if (!waited) asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Kernel lookup for one (format, VW) translation unit; nullptr if that
// (RW, MB, LUT) combination is not instantiated.
void* gemv_kernel_int4_v1(int rw, int mb, int lut);
void* gemv_kernel_int4_v2(int rw, int mb, int lut);
void* gemv_kernel_int4_v4(int rw, int mb, int lut);
void* gemv_kernel_nf4_v1(int rw, int mb, int lut);
void* gemv_kernel_nf4_v2(int rw, int mb, int lut);
void* gemv_kernel_nf4_v4(int rw, int mb, int lut);

}  // namespace b4

// Instantiation helper for the per-(format, VW) translation units.
#define B4_GEMV_PICK(F, VW, RW, MB, LUT) \
    if (rw == RW && mb == MB && lut == LUT) return (void*)&b4::b4_gemv_kernel<F, VW, RW, MB, LUT>;
