// b4_gemv_nf4_mma.cuh -- the batch-1 NF4 b64 GEMV on the tensor pipe.
//
// Every NF4 code must be looked up in the 16-entry code book, and the lookups
// are what bound the CUDA-core kernel (b4_gemv_lean_nf4.cuh): one shared load
// or shuffle per code or code pair, plus shared-memory traffic for x and the
// code ring, plus an FFMA per code.  Here a lookup is one PRMT and one 8-byte
// shared load per byte (two codes), and it yields tensor-core operands:
//
//   * the table has a 256-byte row per byte value b (codes b & 15 and b >> 4
//     of two adjacent columns): 32 copies of the 8-byte entry (the pair's
//     high parts, then its low parts), so lane l reads its own copy at
//     b*256 + 8l with one 8-byte load (each half-warp covers the 32 banks
//     once: the two shared-memory wavefronts an 8-byte load takes anyway, no
//     conflicts).  PRMT builds that offset from a packed word in one
//     instruction (byte b of the word into bits 8..15, 8l in bits 0..7); the
//     load's two words are MMA operands as they are.
//   * the code-book values T are split exactly enough for fp32 work:
//     high part h = fp16(T) and low part fp16(T - h), stored as half2 pairs.
//     h + l represents each of the 16 fp32 code-book values (kernels.cuh:78-83)
//     to within 2^-22 relative; the MMA multiplies both by fp16 x exactly and
//     accumulates in fp32, so y carries fp32-level rounding, like an FMA
//     chain over the fp32 dequantised weights.
//   * MMA m16n8k16, one per weight row set: lane (g, q) streams rows r0+g and
//     r0+g+8; a 128-column step of a row is 64 bytes, lane q taking bytes
//     16q .. 16q+15 (columns 32q .. 32q+31, NF4 block q >> 1).  MMA j of row
//     r0+g uses bytes 2j and 2j+1: A row g holds their high parts and A row
//     g+8 their low parts, so the two words of one lookup are A registers
//     (a0, a1) or (a2, a3) as loaded, and D row g + D row g+8 is the sum.
//     Rows r0+8 .. r0+15 take a second MMA with the same B.  The two NF4 blocks of the step are kept apart by B's columns:
//     column 0 of B holds x at block 0's positions (zero elsewhere), column 1
//     x at block 1's, the rest zero, so D[row][0] and D[row][1] are the two
//     blocks' partial sums and the absmax of each block scales its own sum
//     (deq = T[c] * absmax as in kernels.cuh:331, one block at a time).  Only
//     lanes 0, 1 (block 0) and 6, 7 (block 1) load x; the others hold zeros.
//   * codes and absmax come straight from global memory into registers, a
//     D-deep software pipeline, no shared-memory ring.
//
// Work split as in the other lean kernels: warps_k warps share a 16-row MMA
// block and take steps ks, ks + warps_k, ...; CTAs loop over tiles of rg
// blocks of up to four matrices that share x (LeanNf4Params); only the first
// tr rows of a block carry weights (see b4_gemv_lean.cuh).  The table and the first
// stages' loads come before griddepcontrol.wait; x after it.
#pragma once

#include "b4_gemv_lean_nf4.cuh"

namespace b4 {

constexpr int kNf4PairTableBytes = 256 * 256;   // 256 byte values x 32 copies x (4 + 4) bytes

// offset of (byte m of word w) in the table, for the copy at lane*8
template <int M>
__device__ __forceinline__ uint32_t nf4_pair_offset(uint32_t w, uint32_t lane8)
{
    return __byte_perm(w, lane8, 0x5504u | (M << 4));
}

// The table entry at `off`: .x = the high-part pair, .y = the low-part pair.
__device__ __forceinline__ uint2 nf4_pair_lookup(const unsigned char* tb, uint32_t off)
{
    return *reinterpret_cast<const uint2*>(tb + off);
}

// The code book: row b = 32 copies of (high-part pair, low-part pair) of
// (T[b & 15], T[b >> 4]); one thread per byte value computes its pairs and
// writes its row.  Called by all threads of a CTA; the caller synchronises
// before reading.
__device__ __forceinline__ void nf4_pair_table_fill(unsigned char* base)
{
    for (int b = threadIdx.x; b < 256; b += blockDim.x) {
        const float t0 = c_nf4_table[b & 15], t1 = c_nf4_table[b >> 4];
        const __half h0 = __float2half_rn(t0), h1 = __float2half_rn(t1);
        const __half l0 = __float2half_rn(t0 - __half2float(h0)), l1 = __float2half_rn(t1 - __half2float(h1));
        const __half2 hp = __halves2half2(h0, h1), lp = __halves2half2(l0, l1);
        const uint32_t hw = *reinterpret_cast<const uint32_t*>(&hp), lw = *reinterpret_cast<const uint32_t*>(&lp);
        uint4* row = reinterpret_cast<uint4*>(base + b * 256);
        // the 16-byte chunk order rotates with b: the 8 threads of a store
        // phase write 8 different chunks, hence 8 different bank quads
#pragma unroll 4
        for (int c2 = 0; c2 < 16; ++c2) row[(c2 + b) & 15] = make_uint4(hw, lw, hw, lw);
    }
}

// P2P = 1: a row-parallel shard of a tensor-parallel GEMV, y all-reduced over
// the ranks through peer memory as in the INT4 lean kernel (b4_p2p.cuh): each
// 16-row block's partial rows are pushed to every rank as soon as they are
// done, and summed in rank order after the CTA's last block.  One segment.
template <int D, int P2P = 0>   // D >= 2
__global__ void __launch_bounds__(256, 2) b4_gemv_nf4_mma_kernel(const LeanNf4Params p)
{
    extern __shared__ __align__(16) uint4 lsm[];
    unsigned char* base = reinterpret_cast<unsigned char*>(lsm);
    uint4* xs = reinterpret_cast<uint4*>(base + kNf4PairTableBytes);        // in_f / 8 slots of 8 halves
    const int lane = threadIdx.x & 31;
    const int g = lane >> 2, q = lane & 3;
    const int warp = threadIdx.x >> 5;
    const int ks = warp % p.kw;
    const int grp = warp / p.kw;
    const int words = p.in_f >> 3;
    const int nblk = p.in_f >> 6;
    const int nst = p.in_f >> 7;                                           // 128-column steps per row
    float* red = reinterpret_cast<float*>(xs + words);                    // rg*kw*16
    const int rows_per_tile = p.rg * p.tr;
    const int n_tiles = p.n_tiles;
    const int n_it = nst > ks ? (nst - ks + p.kw - 1) / p.kw : 0;
    const uint32_t lane8 = (uint32_t)lane * 8;

    const uint4 *pa = nullptr, *pb = nullptr;
    const float2 *sa_p = nullptr, *sb_p = nullptr;
    uint4 bufa[D] = {}, bufb[D] = {};
    float2 ama[D] = {}, amb[D] = {};
    int r0 = 0, out_f = 0;
    bool va = false, vb = false;   // this lane's rows r0+g, r0+g+8 carry weights
    float* y = nullptr;
    const int wstep = 4 * p.kw;                                            // uint4 per step step (64 B per row)
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
        pa = reinterpret_cast<const uint4*>(qw + (long long)ra * words) + ks * 4 + q;
        pb = reinterpret_cast<const uint4*>(qw + (long long)rb * words) + ks * 4 + q;
        sa_p = reinterpret_cast<const float2*>(am + (long long)ra * nblk) + ks;
        sb_p = reinterpret_cast<const float2*>(am + (long long)rb * nblk) + ks;
    };
    auto fetch = [&](int slot) {
        // rows that carry no weights load nothing (their MMA rows are never stored)
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

    int tile = blockIdx.x;
    if (tile < n_tiles) {   // weights first: they do not depend on the preceding grid
        setup(tile);
        prologue();
    }
    nf4_pair_table_fill(base);
    asm volatile("griddepcontrol.launch_dependents;");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // x slot w is stored at w ^ 2 when bit 3 of w is set: the four x lanes read
    // slots 4q + i (+ 16 per step), and without the swap lanes q and q + 2 hit
    // the same banks (two wavefronts per load instead of one)
    if (P2P && p.p2p.xgu)   // x = the SwiGLU of this rank's gate/up rows
        stage_x_swiglu<(D >= 4 ? 2 : 4)>(p.p2p.xgu, words, [&](int w, uint4 v) { xs[w ^ ((w >> 2) & 2)] = v; });
    else
        stage_x_words<kXUnroll>(p.x, words, p.x_vec, [&](int w, uint4 v) { xs[w ^ ((w >> 2) & 2)] = v; });
    __syncthreads();
    const uint32_t epoch = P2P ? p2p_epoch(p.p2p) : 0u;

    // B carries x only on lanes (g, q) with g == q >> 1 (columns 0/1 = blocks 0/1)
    const bool x_lane = g == (q >> 1);
    const int xsw = (q >> 1) << 1;   // the slot swap of this lane's x slots
    const unsigned char* tb = base;

    for (; tile < n_tiles; tile += gridDim.x) {
        if (tile != (int)blockIdx.x) {
            setup(tile);
            prologue();
        }
        float acc_a = 0.0f, acc_b = 0.0f;
        const uint4* xp = xs + ks * 16 + q * 4;                            // + 16*kw per step
        uint4 xv[4] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0),
                       make_uint4(0, 0, 0, 0)};

        for (int it0 = 0; it0 < n_it; it0 += D) {
#pragma unroll
            for (int d = 0; d < D; ++d) {
                const int it = it0 + d;
                if (it < n_it) {
                    const int nxt = (d + D - 1) % D;
                    if (it + D - 1 < n_it) fetch(nxt);
                    if (x_lane) {
#pragma unroll
                        for (int i = 0; i < 4; ++i) xv[i] = xp[i ^ xsw];
                    }
                    xp += 16 * p.kw;
                    const uint32_t wa[4] = {bufa[d].x, bufa[d].y, bufa[d].z, bufa[d].w};
                    const uint32_t wb[4] = {bufb[d].x, bufb[d].y, bufb[d].z, bufb[d].w};
                    // four chains: (j odd?, row g + 8?)
                    float c[4][4];
#pragma unroll
                    for (int h = 0; h < 4; ++h) c[h][0] = c[h][1] = c[h][2] = c[h][3] = 0.0f;
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        // bytes 2j, 2j+1 of this lane's 16 bytes: word j >> 1, bytes (2j) & 3 and +1
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
                        // one MMA per 8-row set: A rows 0-7 = the rows' high parts,
                        // rows 8-15 = their low parts, so each lookup's two words
                        // are A registers (a0, a1) or (a2, a3) as they come
                        const uint32_t a_ra[4] = {ea0.x, ea0.y, ea1.x, ea1.y};
                        const uint32_t a_rb[4] = {eb0.x, eb0.y, eb1.x, eb1.y};
                        // x[32q + 4j .. +3]: halves 0..3 or 4..7 of slot j >> 1
                        const uint4 xq = xv[j >> 1];
                        const uint32_t b0 = (j & 1) ? xq.z : xq.x, b1 = (j & 1) ? xq.w : xq.y;
                        const int ch = (j & 1) * 2;
                        mma_16816_pure(c[ch], a_ra, b0, b1, c[ch]);
                        mma_16816_pure(c[ch + 1], a_rb, b0, b1, c[ch + 1]);
                    }
                    // D of a row's MMA (lane q = 0): [0] high block 0, [1] high
                    // block 1, [2] low block 0, [3] low block 1
                    const float d00 = (c[0][0] + c[0][2]) + (c[2][0] + c[2][2]);   // row g, block 0
                    const float d01 = (c[0][1] + c[0][3]) + (c[2][1] + c[2][3]);   // row g, block 1
                    const float d10 = (c[1][0] + c[1][2]) + (c[3][0] + c[3][2]);   // row g+8, block 0
                    const float d11 = (c[1][1] + c[1][3]) + (c[3][1] + c[3][3]);   // row g+8, block 1
                    acc_a = fmaf(d00, ama[d].x, acc_a);
                    acc_a = fmaf(d01, ama[d].y, acc_a);
                    acc_b = fmaf(d10, amb[d].x, acc_b);
                    acc_b = fmaf(d11, amb[d].y, acc_b);
                }
            }
        }

        // rows r0+g and r0+g+8: lanes q = 0 hold them (columns 0 and 1 of D)
        if constexpr (P2P) {
            // push this block's partial rows to every rank; summed after the last block
            const int nrows = max(0, min(p.tr, out_f - r0));
            if (p.kw == 1) {
                // lane i < tr: row r0 + i, from lane (i & 7) * 4 (q = 0)
                const float va_i = __shfl_sync(0xffffffffu, acc_a, (lane & 7) * 4);
                const float vb_i = __shfl_sync(0xffffffffu, acc_b, (lane & 7) * 4);
                p2p_push(p.p2p, epoch, r0, nrows, lane < 8 ? va_i : vb_i);
            } else {
                float* mine = red + (grp * p.kw + ks) * 16;
                if (q == 0) {
                    mine[g] = acc_a;
                    mine[g + 8] = acc_b;
                }
                __syncthreads();
                if (ks == 0) {
                    float t = 0.0f;
                    if (lane < 16)
                        for (int k2 = 0; k2 < p.kw; ++k2) t += red[(grp * p.kw + k2) * 16 + lane];
                    p2p_push(p.p2p, epoch, r0, nrows, t);
                }
                __syncthreads();
            }
        } else if (p.kw == 1) {
            if (q == 0) {
                if (va) y[r0 + g] = acc_a;
                if (vb) y[r0 + g + 8] = acc_b;
            }
        } else {
            float* mine = red + (grp * p.kw + ks) * 16;
            if (q == 0) {
                mine[g] = acc_a;
                mine[g + 8] = acc_b;
            }
            __syncthreads();
            if (ks == 0 && lane < p.tr) {
                float t = 0.0f;
                for (int k2 = 0; k2 < p.kw; ++k2) t += red[(grp * p.kw + k2) * 16 + lane];
                if (r0 + lane < out_f) y[r0 + lane] = t;
            }
            __syncthreads();
        }
    }
    if constexpr (P2P) {
        // every rank's copy of this warp's blocks, summed in rank order (one segment)
        if (ks == 0) {
            for (int t = blockIdx.x; t < n_tiles; t += gridDim.x) {
                const int rr = t * rows_per_tile + grp * p.tr;
                p2p_reduce(p.p2p, epoch, rr, max(0, min(p.tr, p.seg[0].out_f - rr)), p.seg[0].y);
            }
        }
        __syncthreads();   // every warp of the CTA has read the epoch
        p2p_finish(p.p2p, epoch);
    }
}

void* gemv_kernel_nf4_mma(int depth);
void* gemv_kernel_nf4_mma_p2p(int depth);

}  // namespace b4
