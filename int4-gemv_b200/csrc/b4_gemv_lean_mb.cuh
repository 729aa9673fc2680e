// b4_gemv_lean_mb.cuh -- the lean INT4 g128 GEMV for small batches (m = 2..16).
//
// The batch-1 kernel (b4_gemv_lean.cuh) fills every column of the MMA's B
// operand with the same x and keeps column 0 of D.  Here the N = 8 columns of
// an m16n8k16 MMA carry up to 8 different batch rows of x (NB = 2 blocks of 8
// columns for up to 16 rows), so one pass over the weights serves the whole
// batch: the weights are decoded once per lane and multiplied by every batch
// row on the tensor pipe, and the time stays close to the batch-1 time while
// the weights dominate the bytes.
//
// Everything else follows the batch-1 kernel: 16-row MMA blocks with tr rows
// that carry weights, warps_k warps splitting in_f by stages of G groups, a
// per-lane cp.async ring of D stages, weights requested before
// griddepcontrol.wait, up to four matrices sharing x in one launch.  x is
// staged per CTA for all m rows in pair order ([row][word] 16-byte slots, the
// bank-spread layout of xmb_slot);
// lane (g, q) reads the B fragments of batch row nb*8 + g (clamped to m - 1:
// columns past m are computed and dropped).  D's columns 2q, 2q+1 of rows
// g, g+8 are batch rows 2q, 2q+1 of those weight rows, so each lane keeps four
// sums per column block.
#pragma once

#include "b4_gemv_lean.cuh"

namespace b4 {

struct LeanMbParams {
    LeanParams base;   // seg[].y is [m][out_f_s] (leading dimension out_f_s)
    int m;             // batch rows, 2..8*NB
    // Rows of the weights hold ld_words code words and ld_scales scales, rows
    // of x hold x_ld halves; segment s reads x from column xoff[s] (base.in_f
    // columns).  In a k-sliced launch (the kernel's SL = 1) the segments are
    // column slices of one matrix; each CTA then takes a contiguous run of
    // tiles and restages x when the segment changes.
    int ld_words, ld_scales, x_ld;
    int xoff[kLeanMaxSeg];
};

// MAXT = 512: CTAs of 16 warps, one per SM, for batches of 9..16 rows, whose x
// fills most of the shared memory: the 16 warps share one copy of x where two
// CTAs of 8 warps would not fit.  An explicit config only: on B200 it ran
// gate_proj at m = 16 in 23.5 us against 22.2 us for one 8-warp CTA per SM
// with 3 stages of 2 groups, which the dispatch rule keeps.
template <int D, int G, int NB, int MAXT = 256, int SL = 0>
__global__ void __launch_bounds__(MAXT, MAXT == 512 ? 1 : 3 - NB) b4_gemv_lean_mb_kernel(const LeanMbParams pm)
{
    using ST = typename LeanScale<G>::T;
    const LeanParams& p = pm.base;
    const int m = pm.m;
    extern __shared__ __align__(16) uint4 lsm[];
    const int lane = threadIdx.x & 31;
    const int g = lane >> 2, q = lane & 3;
    const int warp = threadIdx.x >> 5;
    const int ks = warp % p.kw;
    const int grp = warp / p.kw;
    const int words = p.in_f >> 3;
    const int ng = p.in_f >> 7;
    const int nst = ng / G;
    const int rows_per_tile = p.rg * p.tr;
    const int n_tiles = p.n_tiles;
    constexpr int NC = 8 * NB;                               // batch columns of D
    const int xst = xmb_stride(words);
    uint4* xs = lsm;                                         // [m][xst] slots, groups transposed
    float* red = reinterpret_cast<float*>(xs + (size_t)m * xst);   // rg*kw*16*NC
    uint4* ring = reinterpret_cast<uint4*>(red + p.rg * p.kw * 16 * NC) + warp * (D * G * 64);

    const int n_it = nst > ks ? (nst - ks + p.kw - 1) / p.kw : 0;
    const int wstep = 4 * G * p.kw;

    const uint4 *pa = nullptr, *pb = nullptr;
    const ST *sa_p = nullptr, *sb_p = nullptr;
    ST bsa[D] = {}, bsb[D] = {};
    int r0 = 0, out_f = 0;
    bool va = false, vb = false;
    float* y = nullptr;
    auto setup = [&](int tile) {
        const uint32_t* qw = p.seg[0].qw;
        const __half* sc = p.seg[0].scale;
        y = p.seg[0].y;
        out_f = p.seg[0].out_f;
        int t0 = 0;
#pragma unroll
        for (int s = 1; s < kLeanMaxSeg; ++s) {
            if (s < p.nseg && tile >= p.seg[s - 1].tile_end) {
                qw = p.seg[s].qw;
                sc = p.seg[s].scale;
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
        const int lw = SL ? pm.ld_words : words, ls = SL ? pm.ld_scales : ng;   // row strides
        pa = reinterpret_cast<const uint4*>(qw + (long long)ra * lw) + ks * 4 * G + q;
        pb = reinterpret_cast<const uint4*>(qw + (long long)rb * lw) + ks * 4 * G + q;
        sa_p = reinterpret_cast<const ST*>(sc + (long long)ra * ls) + ks;
        sb_p = reinterpret_cast<const ST*>(sc + (long long)rb * ls) + ks;
    };
    auto fetch = [&](int slot) {
#pragma unroll
        for (int h = 0; h < G; ++h) {
            if (va) cp_async16(ring + ((slot * G + h) * 2) * 32 + lane, pa + 4 * h);
            if (vb) cp_async16(ring + ((slot * G + h) * 2 + 1) * 32 + lane, pb + 4 * h);
        }
        if (va) bsa[slot] = __ldg(sa_p);
        if (vb) bsb[slot] = __ldg(sb_p);
        pa += wstep;
        pb += wstep;
        sa_p += p.kw;
        sb_p += p.kw;
    };
    auto prologue = [&]() {
#pragma unroll
        for (int d = 0; d < D - 1; ++d) {
            if (d < n_it) fetch(d);
            cp_async_commit();
        }
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
                                   [&](int r, int w, uint4 v) { xs[r * xst + xmb_slot(w)] = int4_pair_order(v); });
        } else {   // x is [m][in_f], contiguous
            stage_x_rows<kXUnroll>(p.x, m, words, p.x_vec, [&](int r, int w, uint4 v) { xs[r * xst + xmb_slot(w)] = int4_pair_order(v); });
        }
    };
    stage_x(seg_of(tile));
    __syncthreads();

    // the batch rows this lane feeds into B (columns g of each block)
    const uint4* xrow[NB];
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) xrow[nb] = xs + (size_t)min(nb * 8 + g, m - 1) * xst + ks * 16 * G + q;

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
        int xoff = 0;                                        // + 16*G*kw slots per stage step

        for (int it0 = 0; it0 < n_it; it0 += D) {
#pragma unroll
            for (int d = 0; d < D; ++d) {
                const int it = it0 + d;
                if (it < n_it) {
                    const int nxt = (d + D - 1) % D;
                    if (it + D - 1 < n_it) fetch(nxt);
                    cp_async_commit();
                    cp_async_wait<D - 1>();
                    float sa[G], sb[G];
                    lean_scales_to_f32<G>(bsa[d], sa);
                    lean_scales_to_f32<G>(bsb[d], sb);
#pragma unroll
                    for (int h = 0; h < G; ++h) {
                        const uint4 wav = ring[((d * G + h) * 2) * 32 + lane];
                        const uint4 wbv = ring[((d * G + h) * 2 + 1) * 32 + lane];
                        const uint32_t wa[4] = {wav.x, wav.y, wav.z, wav.w};
                        const uint32_t wb[4] = {wbv.x, wbv.y, wbv.z, wbv.w};
                        uint32_t ha[4][4], hb[4][4];
#pragma unroll
                        for (int v = 0; v < 4; ++v) {
                            int4_word_to_half2(wa[v], ha[v]);
                            int4_word_to_half2(wb[v], hb[v]);
                        }
#pragma unroll
                        for (int nb = 0; nb < NB; ++nb) {
                            const uint4* xp = xrow[nb] + xoff + 16 * h;
                            const uint4 xv[4] = {xp[0], xp[4], xp[8], xp[12]};   // logical words 4q .. 4q + 3
                            float c0[4] = {0.f, 0.f, 0.f, 0.f}, c1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                            for (int j = 0; j < 4; ++j) {
                                const int v0 = j >> 1, hf = j & 1, v1 = v0 + 2;
                                const uint32_t a0[4] = {ha[v0][2 * hf], hb[v0][2 * hf], ha[v0][2 * hf + 1],
                                                        hb[v0][2 * hf + 1]};
                                mma_16816_pure(c0, a0, hf ? xv[v0].z : xv[v0].x, hf ? xv[v0].w : xv[v0].y, c0);
                                const uint32_t a1[4] = {ha[v1][2 * hf], hb[v1][2 * hf], ha[v1][2 * hf + 1],
                                                        hb[v1][2 * hf + 1]};
                                mma_16816_pure(c1, a1, hf ? xv[v1].z : xv[v1].x, hf ? xv[v1].w : xv[v1].y, c1);
                            }
                            acc[nb][0] = fmaf(c0[0] + c1[0], sa[h], acc[nb][0]);   // row g,   col 2q
                            acc[nb][1] = fmaf(c0[1] + c1[1], sa[h], acc[nb][1]);   // row g,   col 2q+1
                            acc[nb][2] = fmaf(c0[2] + c1[2], sb[h], acc[nb][2]);   // row g+8, col 2q
                            acc[nb][3] = fmaf(c0[3] + c1[3], sb[h], acc[nb][3]);   // row g+8, col 2q+1
                        }
                    }
                    xoff += 16 * G * p.kw;
                }
            }
        }
        cp_async_wait<0>();

        // lane (g, q): rows r0+g, r0+g+8 of batch rows nb*8 + 2q, nb*8 + 2q + 1
        const int out_ld = out_f;
        if (p.kw == 1) {
#pragma unroll
            for (int nb = 0; nb < NB; ++nb) {
                const int c = nb * 8 + 2 * q;
                if (va && c < m) y[(long long)c * out_ld + r0 + g] = acc[nb][0];
                if (va && c + 1 < m) y[(long long)(c + 1) * out_ld + r0 + g] = acc[nb][1];
                if (vb && c < m) y[(long long)c * out_ld + r0 + g + 8] = acc[nb][2];
                if (vb && c + 1 < m) y[(long long)(c + 1) * out_ld + r0 + g + 8] = acc[nb][3];
            }
        } else {
            float* mine = red + (size_t)(grp * p.kw + ks) * 16 * NC;   // [16 rows][NC columns]
#pragma unroll
            for (int nb = 0; nb < NB; ++nb) {
                const int c = nb * 8 + 2 * q;
                mine[g * NC + c] = acc[nb][0];
                mine[g * NC + c + 1] = acc[nb][1];
                mine[(g + 8) * NC + c] = acc[nb][2];
                mine[(g + 8) * NC + c + 1] = acc[nb][3];
            }
            __syncthreads();
            if (ks == 0) {
                for (int e = lane; e < 16 * NC; e += 32) {
                    const int row = e / NC, c = e - row * NC;
                    if (row < p.tr && c < m && r0 + row < out_f) {
                        float t = 0.0f;
                        for (int k2 = 0; k2 < p.kw; ++k2) t += red[(size_t)(grp * p.kw + k2) * 16 * NC + e];
                        y[(long long)c * out_ld + r0 + row] = t;
                    }
                }
            }
            __syncthreads();
        }
    }
}

void* gemv_kernel_int4_lean_mb(int depth, int groups, int nb, int wide = 0, int sliced = 0);

}  // namespace b4
