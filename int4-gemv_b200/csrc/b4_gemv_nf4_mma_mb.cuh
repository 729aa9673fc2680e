// b4_gemv_nf4_mma_mb.cuh -- the NF4 b64 tensor-pipe GEMV for small batches
// (m = 2..16).
//
// The batch-1 kernel (b4_gemv_nf4_mma.cuh) uses two of the MMA's eight N
// columns: column 0 carries x at the positions of the step's first NF4 block,
// column 1 at the second's.  Here each 8-column MMA block carries four batch
// rows for both NF4 blocks: column c is NF4 block c >> 2 of batch row
// 4*nb + (c & 3), and NB = ceil(m / 4) blocks cover the batch.  The code-book
// lookups (PRMT + one 8-byte shared load per byte) are done once per lane and
// shared by every batch row; only the MMAs and the x fragments grow with m.
// From 5 batch rows (NB >= 2) one MMA covers an 8-row set as in the batch-1
// kernel: A rows 0-7 hold the rows' high parts and rows 8-15 their low parts,
// the two added after the MMA; at NB = 1 the high and low parts of all 16 rows
// take an MMA each (measured faster there).
//
// B fragments: lane (g, q) supplies column g at the k-slots of lanes q, whose
// codes lie in NF4 block q >> 1, so it carries x of batch row 4*nb + (g & 3)
// when (g >> 2) == (q >> 1) and zero otherwise (16 of 32 lanes load x).
// D: lane (g, q) holds columns 2q, 2q+1 = NF4 block q >> 1 of batch rows
// 4*nb + 2(q & 1) and +1, for weight rows g and g+8; it scales them by that
// block's absmax, and lanes q and q ^ 2 (the two blocks) are added with one
// shuffle at the end.  x is staged per CTA for all m rows in natural order
// within the bank-spread layout of xmb_slot.
#pragma once

#include "b4_gemv_nf4_mma.cuh"

namespace b4 {

struct Nf4MmaMbParams {
    LeanNf4Params base;   // seg[].y is [m][out_f_s]
    int m;                // batch rows, 2..4*NB
    // Row strides and k slices as in LeanMbParams (ld_scales: absmax per row).
    int ld_words, ld_scales, x_ld;
    int xoff[kLeanMaxSeg];
};

template <int D, int NB, int SL = 0>
__global__ void __launch_bounds__(256, 1) b4_gemv_nf4_mma_mb_kernel(const Nf4MmaMbParams pm)
{
    const LeanNf4Params& p = pm.base;
    const int m = pm.m;
    extern __shared__ __align__(16) uint4 lsm[];
    unsigned char* base = reinterpret_cast<unsigned char*>(lsm);
    uint4* xs = reinterpret_cast<uint4*>(base + kNf4PairTableBytes);        // [m][xmb_stride] slots
    const int lane = threadIdx.x & 31;
    const int g = lane >> 2, q = lane & 3;
    const int warp = threadIdx.x >> 5;
    const int ks = warp % p.kw;
    const int grp = warp / p.kw;
    const int words = p.in_f >> 3;
    const int nblk = p.in_f >> 6;
    const int nst = p.in_f >> 7;
    constexpr int NR = 4 * NB;                                             // batch rows per pass
    const int xst = xmb_stride(words);
    float* red = reinterpret_cast<float*>(xs + (size_t)m * xst);          // rg*kw*16*NR
    const int rows_per_tile = p.rg * p.tr;
    const int n_tiles = p.n_tiles;
    const int n_it = nst > ks ? (nst - ks + p.kw - 1) / p.kw : 0;
    const uint32_t lane8 = (uint32_t)lane * 8;

    const uint4 *pa = nullptr, *pb = nullptr;
    const float2 *sa_p = nullptr, *sb_p = nullptr;
    uint4 bufa[D] = {}, bufb[D] = {};
    float2 ama[D] = {}, amb[D] = {};
    int r0 = 0, out_f = 0;
    bool va = false, vb = false;
    float* y = nullptr;
    const int wstep = 4 * p.kw;
    auto setup = [&](int tile) {
        const uint32_t* qw = p.seg[0].qw;
        const float* am = p.seg[0].absmax;
        y = p.seg[0].y;
        out_f = p.seg[0].out_f;
        int t0 = 0;
#pragma unroll
        for (int s = 1; s < kLeanMaxSeg; ++s) {
            if (s < p.nseg && tile >= p.seg[s - 1].tile_end) {
                qw = p.seg[s].qw;
                am = p.seg[s].absmax;
                y = p.seg[s].y;
                out_f = p.seg[s].out_f;
                t0 = p.seg[s - 1].tile_end;
            }
        }
        r0 = (tile - t0) * rows_per_tile + grp * p.tr;
        va = g < p.tr && r0 + g < out_f;
        vb = g + 8 < p.tr && r0 + g + 8 < out_f;
        const int ra = min(r0 + g, out_f - 1);
        const int rb = min(r0 + g + 8, out_f - 1);
        const int lw = SL ? pm.ld_words : words, ls = SL ? pm.ld_scales : nblk;   // row strides
        pa = reinterpret_cast<const uint4*>(qw + (long long)ra * lw) + ks * 4 + q;
        pb = reinterpret_cast<const uint4*>(qw + (long long)rb * lw) + ks * 4 + q;
        sa_p = reinterpret_cast<const float2*>(am + (long long)ra * ls) + ks;
        sb_p = reinterpret_cast<const float2*>(am + (long long)rb * ls) + ks;
    };
    auto fetch = [&](int slot) {
        if (va) {
            const WordVec<4> v = ld_stream<4>(reinterpret_cast<const uint32_t*>(pa));
            bufa[slot] = make_uint4(v.w[0], v.w[1], v.w[2], v.w[3]);
            ama[slot] = __ldg(sa_p);
        }
        if (vb) {
            const WordVec<4> v = ld_stream<4>(reinterpret_cast<const uint32_t*>(pb));
            bufb[slot] = make_uint4(v.w[0], v.w[1], v.w[2], v.w[3]);
            amb[slot] = __ldg(sb_p);
        }
        pa += wstep;
        pb += wstep;
        sa_p += p.kw;
        sb_p += p.kw;
    };
    auto prologue = [&]() {
#pragma unroll
        for (int d = 0; d < D - 1; ++d)
            if (d < n_it) fetch(d);
    };

    // tiles of this CTA: every gridDim.x-th, or (k-sliced) a contiguous run;
    // computed where used, so that they hold no registers in the tile loop
    auto first_tile = [&]() {
        return SL ? (int)((long long)blockIdx.x * n_tiles / gridDim.x) : (int)blockIdx.x;
    };
    auto end_tile = [&]() {
        return SL ? (int)((long long)(blockIdx.x + 1) * n_tiles / gridDim.x) : n_tiles;
    };
    // the segment of a tile (its x columns start at pm.xoff[segment])
    auto seg_of = [&](int t) {
        int sg = 0;
#pragma unroll
        for (int s = 1; s < kLeanMaxSeg; ++s)
            if (s < p.nseg && t >= p.seg[s - 1].tile_end) sg = s;
        return sg;
    };
    int tile = first_tile();
    if (tile < end_tile()) {
        setup(tile);
        prologue();
    }
    nf4_pair_table_fill(base);
    asm volatile("griddepcontrol.launch_dependents;");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // x rows are x_ld halves apart; a segment's columns start at pm.xoff[segment]
    auto stage_x = [&](int sg) {
        if constexpr (SL) {
            int xo = pm.xoff[0];   // pm.xoff[sg], by constant indices
#pragma unroll
            for (int s = 1; s < kLeanMaxSeg; ++s)
                if (sg == s) xo = pm.xoff[s];
            stage_x_rows<kXUnroll>(p.x + xo, m, words, pm.x_ld >> 3, p.x_vec,
                                   [&](int r, int w, uint4 v) { xs[r * xst + xmb_slot(w)] = v; });
        } else {   // x is [m][in_f], contiguous
            stage_x_rows<kXUnroll>(p.x, m, words, p.x_vec, [&](int r, int w, uint4 v) { xs[r * xst + xmb_slot(w)] = v; });
        }
    };
    stage_x(seg_of(tile));
    __syncthreads();

    // B: this lane carries batch row 4*nb + (g & 3) when (g >> 2) == (q >> 1)
    const bool x_lane = (g >> 2) == (q >> 1);
    const uint4* xrow[NB];
    bool x_on[NB];
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) {
        const int b = 4 * nb + (g & 3);
        x_on[nb] = x_lane && b < m;
        xrow[nb] = xs + (size_t)min(b, m - 1) * xst + ks * 16 + q;
    }
    const unsigned char* tb = base;
    const bool hi_blk = q >= 2;   // the NF4 block of this lane's D columns

    for (; tile < end_tile(); tile += SL ? 1 : (int)gridDim.x) {
        if (tile != first_tile()) {
            setup(tile);
            prologue();
            if constexpr (SL) {
                const int sg = seg_of(tile);
                if (sg != seg_of(tile - 1)) {   // the next column slice (uniform per CTA)
                    __syncthreads();
                    stage_x(sg);
                    __syncthreads();
                }
            }
        }
        float acc[NB][4];
#pragma unroll
        for (int nb = 0; nb < NB; ++nb) acc[nb][0] = acc[nb][1] = acc[nb][2] = acc[nb][3] = 0.0f;
        int xoff = 0;

        for (int it0 = 0; it0 < n_it; it0 += D) {
#pragma unroll
            for (int d = 0; d < D; ++d) {
                const int it = it0 + d;
                if (it < n_it) {
                    const int nxt = (d + D - 1) % D;
                    if (it + D - 1 < n_it) fetch(nxt);
                    const uint32_t wa[4] = {bufa[d].x, bufa[d].y, bufa[d].z, bufa[d].w};
                    const uint32_t wb[4] = {bufb[d].x, bufb[d].y, bufb[d].z, bufb[d].w};
                    // the A operands of the step's 8 MMA pairs.  NB >= 2: one MMA
                    // per 8-row set, A rows 0-7 = the rows' high parts, rows 8-15
                    // = their low parts (a lookup's two words are A registers as
                    // loaded; m = 8: 23.2 -> 22.5 us, m = 16: 34.9 -> 32.5 us on
                    // gate_proj).  NB = 1: one MMA for the 16 rows' high parts and
                    // one for their low parts (m = 2: 15.9 us, 23.8 the other way)
                    uint32_t a0[8][4], a1[8][4];
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const uint32_t ua = wa[j >> 1], ub = wb[j >> 1];
                        uint32_t oa0, oa1, ob0, ob1;
                        if (j & 1) {
                            oa0 = nf4_pair_offset<2>(ua, lane8);
                            oa1 = nf4_pair_offset<3>(ua, lane8);
                            ob0 = nf4_pair_offset<2>(ub, lane8);
                            ob1 = nf4_pair_offset<3>(ub, lane8);
                        } else {
                            oa0 = nf4_pair_offset<0>(ua, lane8);
                            oa1 = nf4_pair_offset<1>(ua, lane8);
                            ob0 = nf4_pair_offset<0>(ub, lane8);
                            ob1 = nf4_pair_offset<1>(ub, lane8);
                        }
                        const uint2 ea0 = nf4_pair_lookup(tb, oa0), eb0 = nf4_pair_lookup(tb, ob0);
                        const uint2 ea1 = nf4_pair_lookup(tb, oa1), eb1 = nf4_pair_lookup(tb, ob1);
                        if constexpr (NB >= 2) {
                            a0[j][0] = ea0.x;
                            a0[j][1] = ea0.y;
                            a0[j][2] = ea1.x;
                            a0[j][3] = ea1.y;
                            a1[j][0] = eb0.x;
                            a1[j][1] = eb0.y;
                            a1[j][2] = eb1.x;
                            a1[j][3] = eb1.y;
                        } else {
                            a0[j][0] = ea0.x;
                            a0[j][1] = eb0.x;
                            a0[j][2] = ea1.x;
                            a0[j][3] = eb1.x;
                            a1[j][0] = ea0.y;
                            a1[j][1] = eb0.y;
                            a1[j][2] = ea1.y;
                            a1[j][3] = eb1.y;
                        }
                    }
                    const float am_a = hi_blk ? ama[d].y : ama[d].x;
                    const float am_b = hi_blk ? amb[d].y : amb[d].x;
#pragma unroll
                    for (int nb = 0; nb < NB; ++nb) {
                        uint4 xv[4] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0),
                                       make_uint4(0, 0, 0, 0)};
                        if (x_on[nb]) {
                            const uint4* xp = xrow[nb] + xoff;
#pragma unroll
                            for (int i = 0; i < 4; ++i) xv[i] = xp[4 * i];   // logical words 4q + i
                        }
                        float c[4][4];
#pragma unroll
                        for (int h2 = 0; h2 < 4; ++h2) c[h2][0] = c[h2][1] = c[h2][2] = c[h2][3] = 0.0f;
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            const uint4 xq = xv[j >> 1];
                            const uint32_t b0 = (j & 1) ? xq.z : xq.x, b1 = (j & 1) ? xq.w : xq.y;
                            const int ch = (j & 1) * 2;
                            mma_16816_pure(c[ch], a0[j], b0, b1, c[ch]);
                            mma_16816_pure(c[ch + 1], a1[j], b0, b1, c[ch + 1]);
                        }
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            float s;
                            if constexpr (NB >= 2) {
                                // a set's D: [0], [1] high parts of batch columns 2q,
                                // 2q+1, [2], [3] their low parts; e < 2: row g
                                // (chains 0, 2), else row g+8 (chains 1, 3)
                                const int r = e >> 1, col = e & 1;
                                s = (c[r][col] + c[r][col + 2]) + (c[r + 2][col] + c[r + 2][col + 2]);
                            } else {
                                s = (c[0][e] + c[1][e]) + (c[2][e] + c[3][e]);
                            }
                            acc[nb][e] = fmaf(s, e < 2 ? am_a : am_b, acc[nb][e]);
                        }
                    }
                    xoff += 16 * p.kw;
                }
            }
        }

        // add the two NF4 blocks' sums (lanes q and q ^ 2); lanes q < 2 then hold
        // rows g, g+8 of batch rows 4*nb + 2q, +1
#pragma unroll
        for (int nb = 0; nb < NB; ++nb)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[nb][e] += __shfl_xor_sync(0xffffffffu, acc[nb][e], 2);
        if (p.kw == 1) {
            if (q < 2) {
#pragma unroll
                for (int nb = 0; nb < NB; ++nb) {
                    const int b = 4 * nb + 2 * q;
                    if (va && b < m) y[(long long)b * out_f + r0 + g] = acc[nb][0];
                    if (va && b + 1 < m) y[(long long)(b + 1) * out_f + r0 + g] = acc[nb][1];
                    if (vb && b < m) y[(long long)b * out_f + r0 + g + 8] = acc[nb][2];
                    if (vb && b + 1 < m) y[(long long)(b + 1) * out_f + r0 + g + 8] = acc[nb][3];
                }
            }
        } else {
            float* mine = red + (size_t)(grp * p.kw + ks) * 16 * NR;   // [16 rows][NR batch rows]
            if (q < 2) {
#pragma unroll
                for (int nb = 0; nb < NB; ++nb) {
                    const int b = 4 * nb + 2 * q;
                    mine[g * NR + b] = acc[nb][0];
                    mine[g * NR + b + 1] = acc[nb][1];
                    mine[(g + 8) * NR + b] = acc[nb][2];
                    mine[(g + 8) * NR + b + 1] = acc[nb][3];
                }
            }
            __syncthreads();
            if (ks == 0) {
                for (int e = lane; e < 16 * NR; e += 32) {
                    const int row = e / NR, b = e - row * NR;
                    if (row < p.tr && b < m && r0 + row < out_f) {
                        float t = 0.0f;
                        for (int k2 = 0; k2 < p.kw; ++k2) t += red[(size_t)(grp * p.kw + k2) * 16 * NR + e];
                        y[(long long)b * out_f + r0 + row] = t;
                    }
                }
            }
            __syncthreads();
        }
    }
}

void* gemv_kernel_nf4_mma_mb(int depth, int nb, int sliced = 0);

}  // namespace b4
