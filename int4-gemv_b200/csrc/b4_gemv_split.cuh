// b4_gemv_split.cuh -- batch-1 GEMVs whose work is cut into equal pieces
// along the flattened (16-row block, k-step) space, for matrices with too few
// rows to give every SM the same whole-row work (q/o/down-shaped: 3584 rows
// are 224 MMA blocks for 296 resident CTAs).
//
// Why: the tile kernels (b4_gemv_lean.cuh, b4_gemv_nf4_mma.cuh) hand each CTA
// whole 16-row blocks and split a block's in_f over the CTA's warps.  With
// 224 blocks and 2 x 148 CTAs they either leave SMs with half the work of
// others or thin the blocks to 13 weight-carrying rows (3/16 of every MMA
// decodes nothing), and 148 groups do not split evenly over 8 warps; down_proj
// ran 35 % slower than gate_proj for the same bytes.  Here every warp of the
// grid takes `per` consecutive k-steps of the block-major sequence
//     unit u = block * nst + step,   warp w: [w * per, (w + 1) * per)
// so the decode work per warp differs by at most one step, whatever the shape.
//
// A warp's range covers the tail of one block, whole blocks, the head of
// another.  At each block boundary (and at its range end) the warp emits its
// partial sums of the block's 16 rows:
//   * a block covered by one warp is stored straight into y;
//   * otherwise each covering warp ("piece" p of the block, in k order)
//     stores its 16 partials into the workspace slot [block][p], fences and
//     counts itself in with one atomicAdd on the block's counter; the warp
//     that arrives last sums the block's pieces in piece order, stores y and
//     sets the counter back to zero.
// The pieces are fixed by the shape and the grid, and they are always summed
// in the same order, so y is deterministic (bit-identical run to run).  No
// warp ever waits for another: there is no spin, so no wait can hang.
//
// The workspace (caller-owned, or the library's static array for the
// no-allocation entry point) holds  float part[nblocks][maxp][16]  and
// uint32 cnt[nblocks].  Counters must be zero before a call and every call
// leaves them zero, so a zero-filled workspace stays valid across calls and
// CUDA-graph replays.  Two calls that run at the same time on one workspace
// race.
//
// The per-step decode is the tile kernels' own (lean_group for INT4, the
// byte -> (hi, lo) pair table for NF4); the weight stream runs through the
// same per-lane cp.async ring (INT4) or register pipeline (NF4), and it flows
// across block boundaries without draining.  The first stages are requested
// before griddepcontrol.wait; x is staged after it.
#pragma once

#include "b4_gemv_lean.cuh"
#include "b4_gemv_nf4_mma.cuh"

namespace b4 {

struct SplitParams {
    const uint32_t* qw;   // [out_f][in_f/8]
    const void* scale;    // INT4: fp16 [out_f][in_f/128]; NF4: fp32 [out_f][in_f/64]
    const __half* x;      // [in_f]
    float* y;             // [out_f]
    float* part;          // [nblocks][maxp][16] partial sums
    unsigned* cnt;        // [nblocks] arrivals, zero between calls
    long long total;      // nblocks * nst
    int in_f, out_f;
    int nst;              // k-steps per row
    int per;              // k-steps per warp
    int maxp;             // piece slots per block
    int x_vec;            // x is 16-byte aligned
};

// Lanes (g, q = 0) hold rows 16b + g and 16b + g + 8 of this warp's partial
// sum of block b over the warp's steps of it.  Called by a whole warp.
__device__ __forceinline__ void split_emit(const SplitParams& p, long long b, int warp_id, float acc_a, float acc_b)
{
    const int lane = threadIdx.x & 31;
    const int g = lane >> 2, q = lane & 3;
    const long long r0 = b * 16;
    const long long first = (b * p.nst) / p.per;
    const long long last = ((b + 1) * p.nst - 1) / p.per;
    const int np = (int)(last - first + 1);
    if (np == 1) {
        if (q == 0) {
            if (r0 + g < p.out_f) p.y[r0 + g] = acc_a;
            if (r0 + g + 8 < p.out_f) p.y[r0 + g + 8] = acc_b;
        }
        return;
    }
    const int piece = (int)(warp_id - first);
    float* slot = p.part + ((size_t)b * p.maxp + piece) * 16;
    if (q == 0) {
        __stcg(slot + g, acc_a);
        __stcg(slot + g + 8, acc_b);
    }
    __threadfence();
    __syncwarp();
    unsigned old = 0;
    if (lane == 0) old = atomicAdd(p.cnt + b, 1u);
    old = __shfl_sync(0xffffffffu, old, 0);
    if (old != (unsigned)(np - 1)) return;
    // the last piece: every other piece's stores are visible after its fence
    // and atomic, and ours after this fence
    __threadfence();
    if (lane < 16) {
        const float* col = p.part + (size_t)b * p.maxp * 16 + lane;
        float t = 0.0f;
        for (int k = 0; k < np; ++k) t += __ldcg(col + k * 16);
        if (r0 + lane < p.out_f) p.y[r0 + lane] = t;
    }
    if (lane == 0) p.cnt[b] = 0u;   // ready for the next call
}

// x (fp16, in_f columns) into shared memory, INT4 pair order (PAIR) or as is.
template <bool PAIR>
__device__ __forceinline__ void split_stage_x(const SplitParams& p, uint4* xs)
{
    stage_x_words<kXUnroll>(p.x, p.in_f >> 3, p.x_vec, [&](int w, uint4 v) { xs[w] = PAIR ? int4_pair_order(v) : v; });
}

// INT4 g128: a step is G consecutive 128-column groups (G divides in_f/128);
// the weight stream runs through the per-lane cp.async ring of the lean
// kernel (ring slot layout and decode as in b4_gemv_lean_kernel, ASYNC = 1).
template <int D, int G>   // D >= 2; G in {1, 2, 4}
__global__ void __launch_bounds__(256, 2) b4_gemv_split_int4_kernel(const SplitParams p)
{
    using ST = typename LeanScale<G>::T;
    extern __shared__ __align__(16) uint4 lsm[];
    const int lane = threadIdx.x & 31;
    const int g = lane >> 2, q = lane & 3;
    const int warp = threadIdx.x >> 5;
    const int words = p.in_f >> 3;
    const int ng = p.in_f >> 7;
    uint4* xs = lsm;                                      // one slot per word, pair order
    uint4* ring = xs + words + warp * (D * G * 64);       // D stages x G groups x 2 rows x 32 lanes
    const int warp_id = blockIdx.x * 8 + warp;
    const long long u0 = (long long)warp_id * p.per;
    const long long u1 = min(u0 + p.per, p.total);
    const int n_it = u1 > u0 ? (int)(u1 - u0) : 0;
    const __half* scale = static_cast<const __half*>(p.scale);

    // fetch cursor: block fb, step fs; rows past out_f are clamped to the
    // last row for loading and never stored
    long long fb = n_it ? u0 / p.nst : 0;
    int fs = n_it ? (int)(u0 % p.nst) : 0;
    const uint4 *pa = nullptr, *pb = nullptr;
    const ST *sa_p = nullptr, *sb_p = nullptr;
    ST bsa[D] = {}, bsb[D] = {};
    auto aim = [&]() {
        const long long last_row = p.out_f - 1;
        const long long ra = min(fb * 16 + g, last_row), rb = min(fb * 16 + g + 8, last_row);
        pa = reinterpret_cast<const uint4*>(p.qw + ra * words) + fs * 4 * G + q;
        pb = reinterpret_cast<const uint4*>(p.qw + rb * words) + fs * 4 * G + q;
        sa_p = reinterpret_cast<const ST*>(scale + ra * ng) + fs;
        sb_p = reinterpret_cast<const ST*>(scale + rb * ng) + fs;
    };
    auto fetch = [&](int slot) {
#pragma unroll
        for (int h = 0; h < G; ++h) {
            cp_async16(ring + ((slot * G + h) * 2) * 32 + lane, pa + 4 * h);
            cp_async16(ring + ((slot * G + h) * 2 + 1) * 32 + lane, pb + 4 * h);
        }
        bsa[slot] = __ldg(sa_p);
        bsb[slot] = __ldg(sb_p);
        pa += 4 * G;
        pb += 4 * G;
        ++sa_p;
        ++sb_p;
        if (++fs == p.nst) {
            ++fb;
            fs = 0;
            aim();
        }
    };

    if (n_it) aim();
#pragma unroll
    for (int d = 0; d < D - 1; ++d) {   // weights first: they do not depend on the preceding grid
        if (d < n_it) fetch(d);
        cp_async_commit();               // one group per stage, even if empty
    }
    asm volatile("griddepcontrol.launch_dependents;");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    split_stage_x<true>(p, xs);
    __syncthreads();
    if (!n_it) return;   // no barrier follows

    long long cb = u0 / p.nst;
    int cs = (int)(u0 % p.nst);
    const uint4* xp = xs + cs * 16 * G + q * 4;
    float acc_a = 0.0f, acc_b = 0.0f;
    // B fragments: column 0 holds x (lanes g = 0 load it per group), columns 1..7 zero
    uint4 xv[4] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
    for (int it0 = 0; it0 < n_it; it0 += D) {
#pragma unroll
        for (int d = 0; d < D; ++d) {
            const int it = it0 + d;
            if (it < n_it) {
                const int nxt = (d + D - 1) % D;
                if (it + D - 1 < n_it) fetch(nxt);
                cp_async_commit();
                cp_async_wait<D - 1>();   // this lane's copies of stage d landed
                float sa[G], sb[G];
                lean_scales_to_f32<G>(bsa[d], sa);
                lean_scales_to_f32<G>(bsb[d], sb);
#pragma unroll
                for (int h = 0; h < G; ++h) {
                    const uint4 wav = ring[((d * G + h) * 2) * 32 + lane];
                    const uint4 wbv = ring[((d * G + h) * 2 + 1) * 32 + lane];
                    if (g == 0) {   // B column 0 = x; the other lanes keep their zeros
#pragma unroll
                        for (int i = 0; i < 4; ++i) xv[i] = xp[16 * h + i];
                    }
                    float ua, ub;
                    lean_group(wav, wbv, xv, ua, ub);
                    acc_a = fmaf(ua, sa[h], acc_a);
                    acc_b = fmaf(ub, sb[h], acc_b);
                }
                xp += 16 * G;
                if (++cs == p.nst || it == n_it - 1) {
                    split_emit(p, cb, warp_id, acc_a, acc_b);
                    acc_a = acc_b = 0.0f;
                    if (cs == p.nst) {
                        ++cb;
                        cs = 0;
                        xp = xs + q * 4;
                    }
                }
            }
        }
    }
    cp_async_wait<0>();
}

// NF4 b64: a step is 128 columns (two NF4 blocks); codes and absmax through
// the register pipeline, the code book as the byte -> (hi, lo) pair table,
// decode and MMA as in b4_gemv_nf4_mma_kernel.
template <int D>   // D >= 2
__global__ void __launch_bounds__(256, 2) b4_gemv_split_nf4_kernel(const SplitParams p)
{
    extern __shared__ __align__(16) uint4 lsm[];
    unsigned char* base = reinterpret_cast<unsigned char*>(lsm);
    uint4* xs = reinterpret_cast<uint4*>(base + kNf4PairTableBytes);   // in_f / 8 slots of 8 halves
    const int lane = threadIdx.x & 31;
    const int g = lane >> 2, q = lane & 3;
    const int warp = threadIdx.x >> 5;
    const int words = p.in_f >> 3;
    const int nblk = p.in_f >> 6;
    const uint32_t lane8 = (uint32_t)lane * 8;
    const int warp_id = blockIdx.x * 8 + warp;
    const long long u0 = (long long)warp_id * p.per;
    const long long u1 = min(u0 + p.per, p.total);
    const int n_it = u1 > u0 ? (int)(u1 - u0) : 0;
    const float* absmax = static_cast<const float*>(p.scale);

    long long fb = n_it ? u0 / p.nst : 0;
    int fs = n_it ? (int)(u0 % p.nst) : 0;
    const uint4 *pa = nullptr, *pb = nullptr;
    const float2 *sa_p = nullptr, *sb_p = nullptr;
    uint4 bufa[D] = {}, bufb[D] = {};
    float2 ama[D] = {}, amb[D] = {};
    auto aim = [&]() {
        const long long last_row = p.out_f - 1;
        const long long ra = min(fb * 16 + g, last_row), rb = min(fb * 16 + g + 8, last_row);
        pa = reinterpret_cast<const uint4*>(p.qw + ra * words) + fs * 4 + q;
        pb = reinterpret_cast<const uint4*>(p.qw + rb * words) + fs * 4 + q;
        sa_p = reinterpret_cast<const float2*>(absmax + ra * nblk) + fs;
        sb_p = reinterpret_cast<const float2*>(absmax + rb * nblk) + fs;
    };
    auto fetch = [&](int slot) {
        const WordVec<4> va = ld_stream<4>(reinterpret_cast<const uint32_t*>(pa));
        const WordVec<4> vb = ld_stream<4>(reinterpret_cast<const uint32_t*>(pb));
        bufa[slot] = make_uint4(va.w[0], va.w[1], va.w[2], va.w[3]);
        bufb[slot] = make_uint4(vb.w[0], vb.w[1], vb.w[2], vb.w[3]);
        ama[slot] = __ldg(sa_p);
        amb[slot] = __ldg(sb_p);
        pa += 4;
        pb += 4;
        ++sa_p;
        ++sb_p;
        if (++fs == p.nst) {
            ++fb;
            fs = 0;
            aim();
        }
    };

    if (n_it) {   // weights first: they do not depend on the preceding grid
        aim();
#pragma unroll
        for (int d = 0; d < D - 1; ++d)
            if (d < n_it) fetch(d);
    }
    nf4_pair_table_fill(base);
    asm volatile("griddepcontrol.launch_dependents;");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    split_stage_x<false>(p, xs);
    __syncthreads();
    if (!n_it) return;   // no barrier follows

    // B carries x only on lanes (g, q) with g == q >> 1 (columns 0/1 = NF4 blocks 0/1)
    const bool x_lane = g == (q >> 1);
    const unsigned char* tb = base;
    long long cb = u0 / p.nst;
    int cs = (int)(u0 % p.nst);
    const uint4* xp = xs + cs * 16 + q * 4;
    float acc_a = 0.0f, acc_b = 0.0f;
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
                    for (int i = 0; i < 4; ++i) xv[i] = xp[i];
                }
                xp += 16;
                const uint32_t wa[4] = {bufa[d].x, bufa[d].y, bufa[d].z, bufa[d].w};
                const uint32_t wb[4] = {bufb[d].x, bufb[d].y, bufb[d].z, bufb[d].w};
                float c[4][4];
#pragma unroll
                for (int h = 0; h < 4; ++h) c[h][0] = c[h][1] = c[h][2] = c[h][3] = 0.0f;
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
                    const uint32_t a_hi[4] = {ea0.x, eb0.x, ea1.x, eb1.x};
                    const uint32_t a_lo[4] = {ea0.y, eb0.y, ea1.y, eb1.y};
                    const uint4 xq = xv[j >> 1];
                    const uint32_t b0 = (j & 1) ? xq.z : xq.x, b1 = (j & 1) ? xq.w : xq.y;
                    const int ch = (j & 1) * 2;
                    mma_16816_pure(c[ch], a_hi, b0, b1, c[ch]);
                    mma_16816_pure(c[ch + 1], a_lo, b0, b1, c[ch + 1]);
                }
                const float d00 = (c[0][0] + c[1][0]) + (c[2][0] + c[3][0]);   // row g, block 0
                const float d01 = (c[0][1] + c[1][1]) + (c[2][1] + c[3][1]);   // row g, block 1
                const float d10 = (c[0][2] + c[1][2]) + (c[2][2] + c[3][2]);   // row g+8, block 0
                const float d11 = (c[0][3] + c[1][3]) + (c[2][3] + c[3][3]);   // row g+8, block 1
                acc_a = fmaf(d00, ama[d].x, acc_a);
                acc_a = fmaf(d01, ama[d].y, acc_a);
                acc_b = fmaf(d10, amb[d].x, acc_b);
                acc_b = fmaf(d11, amb[d].y, acc_b);
                if (++cs == p.nst || it == n_it - 1) {
                    split_emit(p, cb, warp_id, acc_a, acc_b);
                    acc_a = acc_b = 0.0f;
                    if (cs == p.nst) {
                        ++cb;
                        cs = 0;
                        xp = xs + q * 4;
                    }
                }
            }
        }
    }
}

void* gemv_kernel_split_int4(int depth, int groups);
void* gemv_kernel_split_nf4(int depth);

}  // namespace b4
