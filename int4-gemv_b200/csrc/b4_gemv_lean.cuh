// b4_gemv_lean.cuh -- the batch-1 INT4 g128 GEMV with the least integer work
// per code: tensor-pipe multiply-accumulate (register-operand MMA, as in
// b4_gemv_mma.cuh) with every per-group cost other than the decode removed.
//
// Why: at 6.5 TB/s a B200 SM must decode ~45 codes per clock, and the decode
// alone (one SHF + four LOP3 per 8 codes) takes ~45% of the integer pipe at
// that rate, so address arithmetic, predicates and loop control must stay out
// of the inner loop.  Here:
//   * x is staged once per CTA in pair order at its natural word index: the
//     64 bytes lane q needs for group G are words 16*G + 4q .. 16*G + 4q + 3,
//     so one pointer bump per stage and four 16-byte loads with immediate
//     offsets per group fetch the B fragments.  m = 1: only column 0 of B
//     holds x (lanes g = 0 load it, the others hold zeros), since only
//     D[row][0] is used: a 16-byte x load then costs one shared-memory
//     wavefront instead of four, which took x from half of the kernel's
//     shared-memory traffic to a sixth;
//   * rows past out_f are clamped to a valid row for loading and never
//     stored, so the loop has no row predicates;
//   * codes and scales are addressed by running pointers, bumped once per
//     stage; a stage is G consecutive groups of the warp's rows (G = 1, 2, 4),
//     so the scales of a stage are one 2-, 4- or 8-byte load per row;
//   * a D-deep software pipeline, unrolled so every buffer index is a
//     compile-time constant, keeps D-1 stages per lane in flight;
//   * the group epilogue is two fp32 adds and two FMAs per lane: D[row][0]
//     (lanes q = 0) holds the row's partial sum.
// Work split as in the other kernels: warps_k warps share a 16-row MMA block
// and take stages ks, ks + warps_k, ...; CTAs loop over tiles of rg blocks.
// Only the first tr rows of a block carry weights (tr = 16 unless a matrix
// of few rows is spread thinner to give every SM the same number of rows);
// the other MMA rows load nothing and are never stored.  The
// tiles of up to four weight matrices that share x (q/k/v, gate/up) form one
// tile space, so a fused projection is one launch.
//
// The in-flight codes live in shared memory, not registers: each lane copies
// its own 16-byte pieces of every future stage with cp.async into private ring
// slots (((stage*G + group)*2 + row)*32 + lane: a warp's copies and reads of
// one slot are 512 contiguous bytes, conflict-free) and reads them back when
// the stage's turn comes.  Lanes only ever read what they copied themselves,
// so the per-thread cp.async.wait_group is the only ordering needed, and D
// stages in flight cost shared memory instead of registers.
//
// The first tile's first D-1 stages are requested before the kernel waits on
// the grid it depends on (griddepcontrol.wait): codes and scales are inputs
// that no preceding kernel of a decode step writes, so under programmatic
// dependent launch the weight stream starts while the previous kernel drains;
// only x is read after the wait.
#pragma once

#include "b4_gemv_mma.cuh"
#include "b4_p2p.cuh"

namespace b4 {

// One weight matrix of a launch.  Several matrices that share x (q/k/v, or
// gate/up) run as one launch: CTA tiles [tile_end[s-1], tile_end[s]) belong
// to segment s.
struct LeanSeg {
    const uint32_t* qw;
    const __half* scale;
    float* y;
    int out_f;
    int tile_end;
};

constexpr int kLeanMaxSeg = 4;

struct LeanParams {
    LeanSeg seg[kLeanMaxSeg];
    int nseg, n_tiles;
    const __half* x;
    int in_f;
    int kw, rg;
    int tr;      // rows of each warp's 16-row block that carry weights (1..16)
    int x_vec;
    P2pArgs p2p; // P2P kernels: the all-reduce of y over peer memory (b4_p2p.cuh)
};

// scales of one stage of G groups of one row
template <int G> struct LeanScale;
template <> struct LeanScale<1> { using T = unsigned short; };
template <> struct LeanScale<2> { using T = uint32_t; };
template <> struct LeanScale<4> { using T = uint2; };

template <int G>
__device__ __forceinline__ void lean_scales_to_f32(const typename LeanScale<G>::T& s, float (&f)[G])
{
    if constexpr (G == 1) {
        f[0] = __half2float(__ushort_as_half(s));
    } else if constexpr (G == 2) {
        const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&s));
        f[0] = a.x;
        f[1] = a.y;
    } else {
        const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&s.x));
        const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&s.y));
        f[0] = a.x;
        f[1] = a.y;
        f[2] = b.x;
        f[3] = b.y;
    }
}

// m16n8k16 f16 x f16 -> f32 with no side effects, so the compiler may
// schedule the MMAs of independent chains freely.
__device__ __forceinline__ void mma_16816_pure(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1,
                                               const float (&c)[4])
{
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%12,%13};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]), "f"(c[2]),
          "f"(c[3]));
}

// One 128-column group of rows (r0+g, r0+g+8): 8 MMAs in two interleaved
// chains (words 0,1 and 2,3 of this lane's 16 bytes per row).
__device__ __forceinline__ void lean_group(const uint4 wav, const uint4 wbv, const uint4 (&xv)[4], float& pa,
                                           float& pb)
{
    const uint32_t wa[4] = {wav.x, wav.y, wav.z, wav.w};
    const uint32_t wb[4] = {wbv.x, wbv.y, wbv.z, wbv.w};
    uint32_t ha[4][4], hb[4][4];
#pragma unroll
    for (int v = 0; v < 4; ++v) {
        int4_word_to_half2(wa[v], ha[v]);
        int4_word_to_half2(wb[v], hb[v]);
    }
    float c0[4] = {0.f, 0.f, 0.f, 0.f}, c1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int v0 = j >> 1, hf = j & 1, v1 = v0 + 2;
        const uint32_t a0[4] = {ha[v0][2 * hf], hb[v0][2 * hf], ha[v0][2 * hf + 1], hb[v0][2 * hf + 1]};
        mma_16816_pure(c0, a0, hf ? xv[v0].z : xv[v0].x, hf ? xv[v0].w : xv[v0].y, c0);
        const uint32_t a1[4] = {ha[v1][2 * hf], hb[v1][2 * hf], ha[v1][2 * hf + 1], hb[v1][2 * hf + 1]};
        mma_16816_pure(c1, a1, hf ? xv[v1].z : xv[v1].x, hf ? xv[v1].w : xv[v1].y, c1);
    }
    pa = c0[0] + c1[0];
    pb = c0[2] + c1[2];
}

// P2P = 1: a row-parallel shard of a tensor-parallel GEMV; y is all-reduced
// over the ranks through peer memory in the epilogue (b4_p2p.cuh), one warp
// block at a time, so the transfer of early blocks overlaps the math of later
// ones.  One segment only.
template <int D, int G, int P2P = 0>   // D >= 2; G in {1, 2, 4}
__global__ void __launch_bounds__(256, 2) b4_gemv_lean_kernel(const LeanParams p)
{
    using ST = typename LeanScale<G>::T;
    extern __shared__ __align__(16) uint4 lsm[];
    const int lane = threadIdx.x & 31;
    const int g = lane >> 2, q = lane & 3;
    const int warp = threadIdx.x >> 5;
    const int ks = warp % p.kw;
    const int grp = warp / p.kw;
    const int words = p.in_f >> 3;
    const int ng = p.in_f >> 7;
    const int nst = ng / G;                                  // stages per row (the host checks ng % G == 0)
    const int rows_per_tile = p.rg * p.tr;
    const int n_tiles = p.n_tiles;
    uint4* xs = lsm;                                         // one slot per word
    float* red = reinterpret_cast<float*>(xs + words);      // rg*kw*16
    // this warp's ring, D stages x G groups x 2 rows x 32 lanes x 16 bytes
    uint4* ring = xs + words + (p.rg * p.kw * 16 + 3) / 4 + warp * (D * G * 64);

    // stages of this warp: ks, ks + kw, ...; n_it is warp-uniform
    const int n_it = nst > ks ? (nst - ks + p.kw - 1) / p.kw : 0;
    const int wstep = 4 * G * p.kw;                          // uint4 per stage step

    // scales run SD - 1 stages ahead of their use (codes D - 1): a scale is
    // one small global load whose latency the codes' cp.async ring does not
    // hide, and a stage of 4 groups is only ~0.3 us of work
    constexpr int SD = 2 * D;
    const uint4 *pa = nullptr, *pb = nullptr;
    const ST *sa_p = nullptr, *sb_p = nullptr;
    ST bsa[SD] = {}, bsb[SD] = {};
    int r0 = 0, out_f = 0;
    bool va = false, vb = false;   // this lane's rows r0+g, r0+g+8 carry weights
    float* y = nullptr;
    auto setup = [&](int tile) {
        // the segment of this tile (constant indices only: no local-memory copy of the parameters)
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
        pa = reinterpret_cast<const uint4*>(qw + (long long)ra * words) + ks * 4 * G + q;
        pb = reinterpret_cast<const uint4*>(qw + (long long)rb * words) + ks * 4 * G + q;
        sa_p = reinterpret_cast<const ST*>(sc + (long long)ra * ng) + ks;
        sb_p = reinterpret_cast<const ST*>(sc + (long long)rb * ng) + ks;
    };
    auto fetch = [&](int slot) {
        // rows that carry no weights load nothing (their MMA rows are never stored)
#pragma unroll
        for (int h = 0; h < G; ++h) {
            if (va) cp_async16(ring + ((slot * G + h) * 2) * 32 + lane, pa + 4 * h);
            if (vb) cp_async16(ring + ((slot * G + h) * 2 + 1) * 32 + lane, pb + 4 * h);
        }
        pa += wstep;
        pb += wstep;
    };
    auto fetch_scales = [&](int slot) {
        if (va) bsa[slot] = __ldg(sa_p);
        if (vb) bsb[slot] = __ldg(sb_p);
        sa_p += p.kw;
        sb_p += p.kw;
    };
    auto prologue = [&]() {
#pragma unroll
        for (int d = 0; d < SD - 1; ++d)
            if (d < n_it) fetch_scales(d);
#pragma unroll
        for (int d = 0; d < D - 1; ++d) {
            if (d < n_it) fetch(d);
            cp_async_commit();   // one group per stage, even if empty
        }
    };

    int tile = blockIdx.x;
    if (tile < n_tiles) {   // weights first: they do not depend on the preceding grid
        setup(tile);
        prologue();
    }
    asm volatile("griddepcontrol.launch_dependents;");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (P2P && p.p2p.xgu)   // x = the SwiGLU of this rank's gate/up rows
        stage_x_swiglu<4>(p.p2p.xgu, words, [&](int w, uint4 v) { xs[w] = int4_pair_order(v); });
    else
        stage_x_words<kXUnroll>(p.x, words, p.x_vec, [&](int w, uint4 v) { xs[w] = int4_pair_order(v); });
    __syncthreads();
    const uint32_t epoch = P2P ? p2p_epoch(p.p2p) : 0u;

    for (; tile < n_tiles; tile += gridDim.x) {
        if (tile != (int)blockIdx.x) {
            setup(tile);
            prologue();
        }
        float acc_a = 0.0f, acc_b = 0.0f;
        const uint4* xp = xs + ks * 16 * G + q * 4;          // + 16*G*kw per stage step
        // B fragments: column 0 holds x (lanes g = 0 load it per group), columns 1..7 zero
        uint4 xv[4] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0),
                       make_uint4(0, 0, 0, 0)};

        for (int it0 = 0; it0 < n_it; it0 += SD) {   // SD is a multiple of D
#pragma unroll
            for (int d = 0; d < SD; ++d) {
                const int it = it0 + d;
                if (it < n_it) {
                    // refill the stage consumed in the previous step (constant slots once unrolled)
                    const int cs = d % D, nxt = (d + D - 1) % D;
                    if (it + D - 1 < n_it) fetch(nxt);
                    if (it + SD - 1 < n_it) fetch_scales((d + SD - 1) % SD);
                    cp_async_commit();
                    cp_async_wait<D - 1>();                // this lane's copies of stage it landed
                    float sa[G], sb[G];
                    lean_scales_to_f32<G>(bsa[d], sa);
                    lean_scales_to_f32<G>(bsb[d], sb);
#pragma unroll
                    for (int h = 0; h < G; ++h) {
                        const uint4 wav = ring[((cs * G + h) * 2) * 32 + lane];
                        const uint4 wbv = ring[((cs * G + h) * 2 + 1) * 32 + lane];
                        if (g == 0) {   // B column 0 = x; the other lanes keep their zeros
#pragma unroll
                            for (int i = 0; i < 4; ++i) xv[i] = xp[16 * h + i];
                        }
                        float ua, ub;
                        lean_group(wav, wbv, xv, ua, ub);
                        acc_a = fmaf(ua, sa[h], acc_a);
                        acc_b = fmaf(ub, sb[h], acc_b);
                    }
                    xp += 16 * G * p.kw;
                }
            }
        }
        cp_async_wait<0>();   // nothing of this tile left in flight

        // rows r0+g and r0+g+8; lanes q = 0..3 hold the same values
        if constexpr (P2P) {
            // push this block's partial rows to every rank; summed after the last block
            const int nrows = max(0, min(p.tr, out_f - r0));
            if (p.kw == 1) {
                // lane i < tr: row r0 + i
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

void* gemv_kernel_int4_lean(int depth, int groups);
void* gemv_kernel_int4_lean_p2p(int depth, int groups);

}  // namespace b4
