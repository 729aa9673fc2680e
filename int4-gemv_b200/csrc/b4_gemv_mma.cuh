// b4_gemv_mma.cuh -- INT4 g128 GEMV with the multiply-accumulates on the
// tensor pipe (register-operand mma.sync.m16n8k16, fp16 x fp16 -> fp32).
//
// Why the tensor pipe at batch 1: the GEMV is memory-bound only if the SMs
// can decode 4-bit codes as fast as HBM delivers them (about 46 codes per
// clock per SM on B200).  On CUDA cores every code costs a conversion and an
// FMA; here one LOP3 + one HSUB2 turn two codes into exact fp16 (code-8)
// values and a single MMA consumes 8 codes per lane, so the instruction count
// per code roughly halves.  The tensor pipe itself is nearly idle (1/8 of its
// N dimension is used at m = 1; up to 8 batch rows ride along for free).
//
// Exactness: (code-8) in [-8, 7] and fp16 x are exact fp16 operands, their
// products are exact in the fp32 accumulator; a 128-column group (one scale)
// is summed by 8 chained MMAs from zero and then scaled once in fp32, which is
// dequant(W) . x with fp32 accumulation (different order than the reference).
//
// Fragment mapping (m16n8k16, A row-major, B col-major; lane = 4g + q):
//   A: a0a1 = (row g,   k 2q..2q+1)   a2a3 = (row g+8, k 2q..2q+1)
//      a4a5 = (row g,   k 2q+8..+9)   a6a7 = (row g+8, k 2q+8..+9)
//   B: b0b1 = (k 2q..2q+1, n g)       b2b3 = (k 2q+8..+9, n g)
//   D: d0d1 = (row g, n 2q..2q+1)     d2d3 = (row g+8, n 2q..2q+1)
// The k order inside an MMA is free as long as A and B agree.  Lane q loads
// words 4q..4q+3 of a 128-column group (one 16-byte load per row), decodes
// word v into the pairs (n0,n4)(n1,n5)(n2,n6)(n3,n7) and feeds MMA (v, p) with
// pairs 2p and 2p+1; x is staged in shared memory in exactly that pair order.
#pragma once

#include "b4_gemv_kernel.cuh"

namespace b4 {

__device__ __forceinline__ uint32_t smem_addr_u32(const void* p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Per-thread asynchronous global -> shared copies (completion tracked per
// thread with commit/wait groups).
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr_u32(smem_dst)), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1,
                                          const float (&c)[4])
{
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%12,%13};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]), "f"(c[2]),
          "f"(c[3]));
}

// Shared-memory slot (16 bytes = one word's 8 pair-ordered x values) of word
// w of batch row b: lanes q = 0..3 of two adjacent batch rows read 8 distinct
// 16-byte bank groups.
__device__ __forceinline__ int mma_xslot(int b, int w, int tile_words)
{
    return b * tile_words + (w ^ (((w >> 3) & 1) << 1) ^ (b & 1));
}

// Stages x[mb0 .. mb0+nb) columns [8*w0, 8*(w0+tw)) in pair order.
__device__ __forceinline__ void mma_stage_x(const KParams& p, uint4* xs, int mb0, int nb, int w0, int tw)
{
    const int total = nb * tw;
    for (int i = threadIdx.x; i < total; i += blockDim.x) {
        const int b = i / tw;
        const int w = i - b * tw;
        const __half* xrow = p.x + (long long)(mb0 + b) * p.x_ld + (long long)(w0 + w) * 8;
        uint4 raw;
        if (p.x_vec) {
            raw = __ldg(reinterpret_cast<const uint4*>(xrow));
        } else {
            const unsigned short* h = reinterpret_cast<const unsigned short*>(xrow);
            raw.x = (uint32_t)__ldg(h + 0) | ((uint32_t)__ldg(h + 1) << 16);
            raw.y = (uint32_t)__ldg(h + 2) | ((uint32_t)__ldg(h + 3) << 16);
            raw.z = (uint32_t)__ldg(h + 4) | ((uint32_t)__ldg(h + 5) << 16);
            raw.w = (uint32_t)__ldg(h + 6) | ((uint32_t)__ldg(h + 7) << 16);
        }
        xs[mma_xslot(b, w, tw)] = int4_pair_order(raw);
    }
}

template <int RT>
struct MmaFrag {
    uint4 wa[RT], wb[RT];  // words 4q..4q+3 of rows g and g+8 of each 16-row tile
    float sa[RT], sb[RT];  // their group scales
};

// Grid: any number of CTAs; CTA j handles row tiles j, j + gridDim.x, ...
// A row tile is rg row groups of 16*RT rows; warps_k warps share a row group
// and take 128-column groups ks, ks + warps_k, ...  Batch rows are processed
// 8*NT at a time (the MMA's N); x_tile columns of x are staged per pass.
template <int RT, int NT>
__global__ void __launch_bounds__(256) b4_gemv_mma_kernel(const KParams p)
{
    constexpr int NB = 8 * NT;              // batch rows per pass
    extern __shared__ uint4 smem_u4[];
    const int lane = threadIdx.x & 31;
    const int g = lane >> 2, q = lane & 3;
    const int warp = threadIdx.x >> 5;
    const int ks = warp % p.kw;
    const int grp = warp / p.kw;
    const int words = p.in_f >> 3;
    const int groups = p.in_f / kGroup;
    const int rows_per_tile = p.rg * 16 * RT;
    const int n_row_tiles = (p.out_f + rows_per_tile - 1) / rows_per_tile;
    const int tile_groups = p.tile_chunks;   // 128-column groups of x staged per pass
    const bool one_xtile = groups <= tile_groups;
    const int nb_max = min(p.m, NB);

    uint4* xs = smem_u4;
    float* red = reinterpret_cast<float*>(xs + nb_max * tile_groups * 16);

    asm volatile("griddepcontrol.launch_dependents;");
    bool waited = false;

    for (int mb0 = 0; mb0 < p.m; mb0 += NB) {
        const int nb = min(NB, p.m - mb0);
        bool staged = false;
        for (int rt_i = blockIdx.x; rt_i < n_row_tiles; rt_i += gridDim.x) {
            const int row0 = rt_i * rows_per_tile + grp * 16 * RT;
            const uint4* wra[RT];
            const uint4* wrb[RT];
            const __half* sra[RT];
            const __half* srb[RT];
            bool oka[RT], okb[RT];
#pragma unroll
            for (int t = 0; t < RT; ++t) {
                const int ra = row0 + 16 * t + g, rb = ra + 8;
                oka[t] = ra < p.out_f;
                okb[t] = rb < p.out_f;
                wra[t] = reinterpret_cast<const uint4*>(p.qw + (long long)(oka[t] ? ra : 0) * words) + q;
                wrb[t] = reinterpret_cast<const uint4*>(p.qw + (long long)(okb[t] ? rb : 0) * words) + q;
                sra[t] = static_cast<const __half*>(p.scale) + (long long)(oka[t] ? ra : 0) * groups;
                srb[t] = static_cast<const __half*>(p.scale) + (long long)(okb[t] ? rb : 0) * groups;
            }
            float acc[RT][NT][4];
#pragma unroll
            for (int t = 0; t < RT; ++t)
#pragma unroll
                for (int n = 0; n < NT; ++n)
#pragma unroll
                    for (int j = 0; j < 4; ++j) acc[t][n][j] = 0.0f;

            for (int G0 = 0; G0 < groups; G0 += tile_groups) {
                const int tg = min(tile_groups, groups - G0);
                const int n_it = tg > ks ? (tg - ks + p.kw - 1) / p.kw : 0;

                auto load = [&](MmaFrag<RT>& f, int G) {
#pragma unroll
                    for (int t = 0; t < RT; ++t) {
                        if (oka[t]) {
                            const WordVec<4> v = ld_stream<4>(reinterpret_cast<const uint32_t*>(wra[t] + G * 4));
                            f.wa[t] = make_uint4(v.w[0], v.w[1], v.w[2], v.w[3]);
                            f.sa[t] = __half2float(__ldg(sra[t] + G));
                        } else {
                            f.wa[t] = make_uint4(0u, 0u, 0u, 0u);
                            f.sa[t] = 0.0f;
                        }
                        if (okb[t]) {
                            const WordVec<4> v = ld_stream<4>(reinterpret_cast<const uint32_t*>(wrb[t] + G * 4));
                            f.wb[t] = make_uint4(v.w[0], v.w[1], v.w[2], v.w[3]);
                            f.sb[t] = __half2float(__ldg(srb[t] + G));
                        } else {
                            f.wb[t] = make_uint4(0u, 0u, 0u, 0u);
                            f.sb[t] = 0.0f;
                        }
                    }
                };

                MmaFrag<RT> cur;
                if (n_it > 0) load(cur, G0 + ks);
                if (!waited) {
                    asm volatile("griddepcontrol.wait;" ::: "memory");
                    waited = true;
                }
                if (!(one_xtile && staged)) {
                    __syncthreads();
                    mma_stage_x(p, xs, mb0, nb, G0 * 16, tg * 16);
                    __syncthreads();
                    staged = true;
                }

                for (int it = 0; it < n_it; ++it) {
                    const int G = G0 + ks + it * p.kw;   // absolute group
                    const int gl = G - G0;               // group within the staged tile
                    MmaFrag<RT> nxt;
                    if (it + 1 < n_it) load(nxt, G + p.kw);

                    // B fragments: batch row n = 8*nt + g, words 4q..4q+3 of group gl
                    uint4 xb[NT][4];
#pragma unroll
                    for (int n = 0; n < NT; ++n) {
                        const int b = 8 * n + g;
#pragma unroll
                        for (int v = 0; v < 4; ++v)
                            xb[n][v] = b < nb ? xs[mma_xslot(b, gl * 16 + 4 * q + v, tg * 16)]
                                              : make_uint4(0u, 0u, 0u, 0u);
                    }
#pragma unroll
                    for (int t = 0; t < RT; ++t) {
                        float d[NT][4];
                        const uint32_t wa[4] = {cur.wa[t].x, cur.wa[t].y, cur.wa[t].z, cur.wa[t].w};
                        const uint32_t wb[4] = {cur.wb[t].x, cur.wb[t].y, cur.wb[t].z, cur.wb[t].w};
#pragma unroll
                        for (int v = 0; v < 4; ++v) {
                            uint32_t ha[4], hb[4];
                            int4_word_to_half2(wa[v], ha);
                            int4_word_to_half2(wb[v], hb);
#pragma unroll
                            for (int pp = 0; pp < 2; ++pp) {
                                const uint32_t a[4] = {ha[2 * pp], hb[2 * pp], ha[2 * pp + 1], hb[2 * pp + 1]};
#pragma unroll
                                for (int n = 0; n < NT; ++n) {
                                    const uint32_t b0 = pp ? xb[n][v].z : xb[n][v].x;
                                    const uint32_t b1 = pp ? xb[n][v].w : xb[n][v].y;
                                    if (v == 0 && pp == 0) {
                                        const float z[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                                        mma_16816(d[n], a, b0, b1, z);
                                    } else {
                                        mma_16816(d[n], a, b0, b1, d[n]);
                                    }
                                }
                            }
                        }
#pragma unroll
                        for (int n = 0; n < NT; ++n) {
                            acc[t][n][0] = fmaf(d[n][0], cur.sa[t], acc[t][n][0]);
                            acc[t][n][1] = fmaf(d[n][1], cur.sa[t], acc[t][n][1]);
                            acc[t][n][2] = fmaf(d[n][2], cur.sb[t], acc[t][n][2]);
                            acc[t][n][3] = fmaf(d[n][3], cur.sb[t], acc[t][n][3]);
                        }
                    }
                    if (it + 1 < n_it) cur = nxt;
                }
            }

            // y: lane (g, q) holds rows g, g+8 of each tile for batch rows 2q, 2q+1
            // (+8 per n tile).  warps_k partials are summed in warp order.
            auto store = [&](int t, int n, int j, float v) {
                const int row = row0 + 16 * t + g + ((j & 2) ? 8 : 0);
                const int b = mb0 + 8 * n + 2 * q + (j & 1);
                if (row < p.out_f && b < p.m) p.y[(long long)b * p.y_ld + row] = v;
            };
            if (p.kw == 1) {
#pragma unroll
                for (int t = 0; t < RT; ++t)
#pragma unroll
                    for (int n = 0; n < NT; ++n)
#pragma unroll
                        for (int j = 0; j < 4; ++j) store(t, n, j, acc[t][n][j]);
            } else {
                constexpr int PER = RT * NT * 4;
                float* mine = red + ((grp * p.kw + ks) * PER) * 32;
#pragma unroll
                for (int t = 0; t < RT; ++t)
#pragma unroll
                    for (int n = 0; n < NT; ++n)
#pragma unroll
                        for (int j = 0; j < 4; ++j) mine[((t * NT + n) * 4 + j) * 32 + lane] = acc[t][n][j];
                __syncthreads();
                if (ks == 0) {
#pragma unroll
                    for (int t = 0; t < RT; ++t)
#pragma unroll
                        for (int n = 0; n < NT; ++n)
#pragma unroll
                            for (int j = 0; j < 4; ++j) {
                                float s = 0.0f;
                                for (int k2 = 0; k2 < p.kw; ++k2)
                                    s += red[((grp * p.kw + k2) * PER + (t * NT + n) * 4 + j) * 32 + lane];
                                store(t, n, j, s);
                            }
                }
                __syncthreads();
            }
        }
    }
    if (!waited) asm volatile("griddepcontrol.wait;" ::: "memory");
}

void* gemv_kernel_int4_mma(int rt, int nt);

}  // namespace b4
