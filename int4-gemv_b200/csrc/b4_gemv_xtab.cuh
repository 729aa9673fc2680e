// b4_gemv_xtab.cuh -- the batch-1 NF4 b64 GEMV from tables of x-pair products.
//
// The code book is what bounds the other NF4 kernels: every code costs a
// shared-memory read of its value (4 bytes per code on the tensor-pipe kernel,
// fp16 high + low part), and the shared-memory data path (128 B/clk/SM) runs
// out before HBM does.  This kernel moves x into the table instead:
//
//   for a column pair (k, k+1) and a byte b of a packed word (codes c0 = b & 15
//   of column k, c1 = b >> 4 of column k+1):
//       P[b] = NF4[c0] * x[k] + NF4[c1] * x[k+1]          (fp32)
//
// so one 4-byte shared load per byte (two codes) returns the pair's share of
// the row's dot product, and one FADD accumulates it: 2 bytes of shared-memory
// reads per code instead of 4, and no multiply per code.  The row's NF4 block
// sums are scaled by their absmax afterwards (y = sum_b absmax_b * sum_k
// NF4[c_k] x_k, the dequantised weight NF4[c] * absmax of kernels.cuh:331
// factored per block).  Every product and sum is fp32, so y carries fp32
// rounding like an FMA chain over the fp32 dequantised weights.
//
// Geometry.  A table costs 1 KB per column pair, so a CTA (one per SM, its
// 128 KB of tables filling most of the SM's shared memory) covers a
// 256-column SLICE of in_f: 32 packed words, each word four column pairs
// (byte positions j = 0..3).  The table of pair (word w, byte j) is column w
// of the layout
//       float [j >> 1][b][j & 1][w]        (b = the byte value)
// so lookups of 32 different words hit the 32 banks once, whatever the bytes.
//
// Work.  The matrix is cut into (slice, 16-row batch) units.  With S =
// in_f/256 slices and G CTAs, slice s gets G/S or G/S + 1 CTAs that split its
// batches evenly (S > G: each CTA takes slices c, c + G, ... with every
// batch).  A warp takes the batches b0 + warp, b0 + warp + NW, ... of its CTA's
// range; each batch's codes (16 rows x 128 bytes) come through the warp's
// cp.async ring in shared memory, R stages deep.  Lane L works on rows L & 7
// and (L & 7) + 8 of a batch, in NF4 block L >> 3 of the slice (words
// 8 (L >> 3) .. + 7): at step k (0..7) it takes word 8 (L >> 3) + (k ^ (L & 7))
// of both rows -- its block's 8 words in an order permuted by the lane, so the
// 32 lanes of a step hold 32 different words and their lookups hit 32
// different table columns -- and adds the 4 + 4 looked-up pair sums to the
// two rows' block sums.  Each block sum is scaled by its absmax; two shuffles
// add the slice's four blocks; lanes 0..15 then add the slice's share of the
// batch's 16 rows into y.
//
// The slices' shares meet in y through fp32 atomic adds (reductions in L2,
// fire and forget: no cross-CTA wait at the end of the kernel).  y must be zero
// first: each CTA zeroes its share of y's rows right after the grid-dependency
// wait and counts itself in on a workspace counter (a release reduction); a
// warp keeps the results of its first kXtabHold batches in registers and
// waits (bounded) for all G arrivals before its first add, which by then has
// normally happened, so the count-in is off the critical path.  The last CTA to leave resets the two counters,
// so the workspace is zero between calls.  Summation order across slices
// therefore varies from run to run (within fp32 rounding); everything else is
// fixed.
//
// Waits: the arrival wait is the only one.  It is bounded (kXtabMaxPolls polls
// with a short sleep); when it runs out the kernel raises its device error
// flag and carries on, so it always ends.  It needs all G CTAs resident at
// once: the grid is sized to the device's SMs at one CTA each, and every CTA
// signals launch_dependents before waiting, so no programmatic dependent can
// take an SM that a CTA of this grid still needs.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>
#include <type_traits>

#include "b4_common.cuh"

namespace b4 {

constexpr int kXtabCols = 256;                          // columns per slice: 32 words
constexpr int kXtabBatch = 16;                          // rows per warp batch
constexpr int kXtabTableBytes = 4 * 256 * 32 * 4;       // 4 byte positions x 256 values x 32 lanes x fp32
constexpr int kXtabMaxSeg = 4;
constexpr unsigned kXtabMaxPolls = 1u << 22;
constexpr int kXtabHold = 2;   // batch results a warp keeps before its first add
constexpr int kErrXtabBarrier = 2;

// One weight matrix of a launch: 16-row batches [batch_end of the previous
// segment, batch_end) of the launch's batch space belong to it.
struct XtabSeg {
    const uint32_t* qw;
    const float* absmax;
    float* y;
    int out_f;
    int batch_end;
};

struct XtabParams {
    XtabSeg seg[kXtabMaxSeg];
    int nseg;
    int nbatch;          // total batches over the segments
    int in_f;
    int nslice;          // in_f / 256
    const __half* x;
    unsigned* bar;       // workspace: [0] arrivals, [1] departures; zero between calls
    uint32_t smem;       // dynamic shared memory of the launch (bytes)
};

// The device error flag of this translation unit (read by xtab_device_error).
static __device__ int g_xtab_error;

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p)
{
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void red_release_add_u32(unsigned* p, unsigned v)
{
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// fire-and-forget fp32 add in L2 (a generic-address atomicAdd compiles to a
// returning generic atomic)
__device__ __forceinline__ void red_add_f32(float* p, float v)
{
    asm volatile("red.relaxed.gpu.global.add.f32 [%0], %1;" ::"l"(p), "f"(v) : "memory");
}

// Shared loads the compiler may schedule freely (not volatile, no memory
// clobber): each load's address must therefore depend on a value produced
// after the barrier or wait that makes its data valid (opaque(), below), or
// the load could be hoisted above it or merged with another batch's.
__device__ __forceinline__ float lds_f32(uint32_t addr)
{
    float v;
    asm("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr));
    return v;
}

// `v` as a value the compiler cannot see through, defined here (after the
// preceding memory-clobbering asm in program order).
__device__ __forceinline__ uint32_t opaque(uint32_t v)
{
    asm volatile("" : "+r"(v)::"memory");
    return v;
}

// PRMT with the selector's sign-replicate bits honoured (a nibble with bit 3
// set gives the selected byte's sign bit in all 8 bits), written as PTX
template <uint32_t SEL>
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b)
{
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "n"(SEL));
    return r;
}

template <int OFF>
__device__ __forceinline__ uint32_t lds_u32(uint32_t addr)
{
    uint32_t v;
    asm("ld.shared.u32 %0, [%1+%2];" : "=r"(v) : "r"(addr), "n"(OFF));
    return v;
}

// f(integral_constant<int, D>) for D = D0 .. N - 1, each with a compile-time D
template <int D0, int N, typename F>
__device__ __forceinline__ void xtab_unroll(F&& f)
{
    if constexpr (D0 < N) {
        f(std::integral_constant<int, D0>{});
        xtab_unroll<D0 + 1, N>(f);
    }
}

__device__ __forceinline__ void sts_f32(uint32_t addr, float v)
{
    asm volatile("st.shared.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

// The k-th (slice, batch range) work item of CTA c; false when there is none.
__device__ __forceinline__ bool xtab_item(const XtabParams& p, int c, int k, int& s, int& b0, int& b1)
{
    const int G = gridDim.x;
    if (p.nslice <= G) {
        if (k > 0) return false;
        const int base = G / p.nslice, extra = G % p.nslice;
        int n, u;
        if (c < extra * (base + 1)) {
            s = c / (base + 1);
            u = c % (base + 1);
            n = base + 1;
        } else {
            const int c2 = c - extra * (base + 1);
            s = extra + c2 / base;
            u = c2 % base;
            n = base;
        }
        b0 = (int)((long long)u * p.nbatch / n);
        b1 = (int)((long long)(u + 1) * p.nbatch / n);
        return true;
    }
    s = c + k * G;
    b0 = 0;
    b1 = p.nbatch;
    return s < p.nslice;
}

// Segment of batch b and its first row.
__device__ __forceinline__ int xtab_seg_of(const XtabParams& p, int b, int& r0)
{
    int sg = 0, first = 0;
#pragma unroll
    for (int i = 1; i < kXtabMaxSeg; ++i) {
        if (i < p.nseg && b >= p.seg[i - 1].batch_end) {
            sg = i;
            first = p.seg[i - 1].batch_end;
        }
    }
    r0 = (b - first) * kXtabBatch;
    return sg;
}

// The shared-memory ring of one warp: R stages of a batch's codes (16 rows x
// 128 bytes).  absmax goes straight into registers.
constexpr int kXtabStageBytes = kXtabBatch * 128;
constexpr int kErrXtabLayout = 4;

// Shared-memory layout.  The two 64 KB halves of the tables (byte positions
// j = 0, 1 and j = 2, 3) start on 64 KB boundaries of the CTA's shared window,
// so one PRMT that drops a code byte into bits 8..15 of a lane register
// holding  half base + 128 * (j & 1) + 4 * w  yields the entry's complete
// shared address.  `base` is the window address where dynamic shared memory
// starts (after the reserved part); the warps' rings fill the space below
// the first boundary as far as whole rings fit, the rest go after the tables.
__host__ __device__ constexpr uint32_t xtab_align64k(uint32_t base) { return (base + 65535u) & ~65535u; }

__host__ __device__ constexpr uint32_t xtab_ring_bytes(int r) { return (uint32_t)(r * kXtabStageBytes); }

// warps whose rings fit below the tables
__host__ __device__ constexpr int xtab_low_warps(int nw, int r, uint32_t base)
{
    return (int)((xtab_align64k(base) - base) / xtab_ring_bytes(r)) < nw
               ? (int)((xtab_align64k(base) - base) / xtab_ring_bytes(r))
               : nw;
}

__host__ __device__ constexpr uint32_t xtab_smem_bytes(int nw, int r, uint32_t base)
{
    return (xtab_align64k(base) - base) + (uint32_t)kXtabTableBytes +
           (uint32_t)(nw - xtab_low_warps(nw, r, base)) * xtab_ring_bytes(r);
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}

template <int NW, int R>
__global__ void __launch_bounds__(32 * NW, 1) b4_gemv_xtab_kernel(const XtabParams p)
{
    static_assert(R >= 2, "ring stages: at least 2");
    extern __shared__ __align__(16) float xtab[];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int G = gridDim.x, c = blockIdx.x;
    const int nblk = p.in_f >> 6;
    const long long rowb = p.in_f >> 1;          // bytes of codes per row
    const int lr = lane & 7, lq = lane >> 3;     // this lane's rows (lr, lr + 8) and NF4 block of the slice

    const uint32_t base = static_cast<uint32_t>(__cvta_generic_to_shared(xtab));
    const uint32_t tab = xtab_align64k(base);
    if (xtab_smem_bytes(NW, R, base) > p.smem) {   // the launch did not size this layout: leave untouched
        if (threadIdx.x == 0) atomicOr(&g_xtab_error, kErrXtabLayout);
        return;
    }
    // table build: lane L writes its own column (word L) of the four pairs' tables
    const uint32_t lk0 = tab + (uint32_t)lane * 4, lk1 = lk0 + 128, lk2 = lk0 + 65536, lk3 = lk1 + 65536;

    // this warp's ring of codes; lane L copies 16-byte pieces L + 32 t (t = 0..3)
    // of a stage: rows L / 8 + 4 t, piece L % 8
    const int low = xtab_low_warps(NW, R, base);
    const uint32_t ring_s = warp < low ? base + (uint32_t)warp * xtab_ring_bytes(R)
                                       : tab + kXtabTableBytes + (uint32_t)(warp - low) * xtab_ring_bytes(R);
    const uint32_t wr_q = ring_s + lane * 16;
    // Step k (0..7): word w = 8 * (L >> 3) + (k ^ (L & 7)) of rows L & 7 and
    // (L & 7) + 8.  With w0 its step-0 word, 4w = 4 w0 ^ 4k (bits 2..4), so
    //   row address  = cr0 ^ 4k   (cr0 = the ring slot of row L & 7, word w0)
    //   lookup base  = lw0 ^ 0x404 k
    // where lw0 holds the bytes (4 w0, 4 w0 + 128, T, T + 1), T = the tables'
    // base >> 16, from which one PRMT per byte position j forms the address
    //     T*65536 + (j >> 1)*65536 + b*256 + (j & 1)*128 + 4w
    // (byte 3 is a sign-replicated copy of T: zero).
    const uint32_t T = tab >> 16;
    const uint32_t w0 = 8u * lq + (uint32_t)lr;
    const uint32_t cr0 = ring_s + lr * 128 + 4 * w0;
    const uint32_t lw0 = ((T + 1) << 24) | (T << 16) | ((4 * w0 + 128) << 8) | (4 * w0);

    int s = 0, b0 = 0, b1 = 0;
    // segment cursor (a warp's batches only increase) and the next batch's copy
    // sources: this lane's first code piece and its absmax (row L & 7, block L >> 3)
    int sg = -1, sg_first = 0, sg_end = 0, out_f = 0;
    float* yseg = nullptr;
    const unsigned char* qsrc = nullptr;
    const float* asrc = nullptr;
    int bnext = 0;
    const long long astep8 = 8LL * nblk;   // absmax floats between rows r and r + 8
    auto seek = [&](int b) {   // point the copy sources at batch b
        while (b >= sg_end) {
            sg_first = sg_end;
            ++sg;
            sg_end = p.seg[sg].batch_end;
        }
        const XtabSeg& g = p.seg[sg];
        out_f = g.out_f;
        yseg = g.y;
        const int r0 = (b - sg_first) * kXtabBatch;
        qsrc = reinterpret_cast<const unsigned char*>(g.qw) + s * 128 + (r0 + (lane >> 3)) * rowb + (lane & 7) * 16;
        asrc = g.absmax + (long long)(r0 + lr) * nblk + 4 * s + lq;
        bnext = b;
    };
    float* yb[R];
    int nvb[R];
    float aba[R], abb[R];
    // the next batch of this warp (bnext) into ring slot `slot`; rows past
    // out_f copy the segment's last row
    auto issue = [&](int slot) {
        if (bnext >= sg_end) seek(bnext);
        const int r0 = (bnext - sg_first) * kXtabBatch;
        const int nv = min(kXtabBatch, out_f - r0);
        const uint32_t st = (uint32_t)(slot * kXtabStageBytes);
        if (nv == kXtabBatch) {
#pragma unroll
            for (int t = 0; t < 4; ++t) cp_async16(wr_q + st + 512 * t, qsrc + 4 * t * rowb);
            aba[slot] = __ldg(asrc);
            abb[slot] = __ldg(asrc + astep8);
        } else {
            const unsigned char* q = qsrc - (lane >> 3) * rowb;
#pragma unroll
            for (int t = 0; t < 4; ++t) cp_async16(wr_q + st + 512 * t, q + min((lane >> 3) + 4 * t, nv - 1) * rowb);
            aba[slot] = __ldg(asrc + (long long)(min(lr, nv - 1) - lr) * nblk);
            abb[slot] = __ldg(asrc + (long long)(min(lr + 8, nv - 1) - lr) * nblk);
        }
        yb[slot] = yseg + r0;
        nvb[slot] = nv;
        bnext += NW;
        qsrc += NW * kXtabBatch * rowb;
        asrc += (long long)NW * kXtabBatch * nblk;
    };
    auto commit = [] { asm volatile("cp.async.commit_group;" ::: "memory"); };
    // This warp's adds into y wait until every CTA has counted in.  The count
    // is not awaited before the batches: the results of a warp's first
    // kHold batches are held in registers, and the wait comes before the
    // first add, by when the count is normally complete.
    bool counted_in = false;
    float hold_r[kXtabHold];
    float* hold_y[kXtabHold];
    int hold_n[kXtabHold];
    int held = 0;
    auto count_in = [&]() {
        if (lane == 0) {
            unsigned n = 0;
            while (ld_acquire_u32(&p.bar[0]) < (unsigned)G) {
                if (++n >= kXtabMaxPolls) {
                    atomicOr(&g_xtab_error, kErrXtabBarrier);
                    break;
                }
                __nanosleep(64);
            }
        }
        __syncwarp();
        counted_in = true;
#pragma unroll
        for (int i = 0; i < kXtabHold; ++i)
            if (i < held && lane < hold_n[i]) red_add_f32(hold_y[i] + lane, hold_r[i]);
        held = 0;
    };
    // batch `it` of this warp from ring slot D (it + R - 1 issued first if `more`)
    auto step = [&](auto dc, bool more) {
        constexpr int D = decltype(dc)::value;
        __syncwarp();   // every lane is done with the slot refilled next
        if (more) issue((D + R - 1) % R);
        commit();
        asm volatile("cp.async.wait_group %0;" ::"n"(R - 1) : "memory");
        __syncwarp();   // every lane's copies of this batch have landed
        // this batch's ring addresses: after the wait, and distinct per batch
        const uint32_t crb = opaque(cr0);
        float a0 = 0.0f, a1 = 0.0f, c0 = 0.0f, c1 = 0.0f;   // block sums of rows L & 7 and (L & 7) + 8
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const uint32_t ca = crb ^ (4u * k);
            const uint32_t lw = lw0 ^ (0x404u * k);
            const uint32_t wa = lds_u32<D * kXtabStageBytes>(ca);
            const uint32_t wb = lds_u32<D * kXtabStageBytes + 8 * 128>(ca);
            const float ea = (lds_f32(prmt<0xE604u>(wa, lw)) + lds_f32(prmt<0xE615u>(wa, lw))) +
                             (lds_f32(prmt<0xE724u>(wa, lw)) + lds_f32(prmt<0xE735u>(wa, lw)));
            const float eb = (lds_f32(prmt<0xE604u>(wb, lw)) + lds_f32(prmt<0xE615u>(wb, lw))) +
                             (lds_f32(prmt<0xE724u>(wb, lw)) + lds_f32(prmt<0xE735u>(wb, lw)));
            if (k & 1) {
                a1 += ea;
                c1 += eb;
            } else {
                a0 += ea;
                c0 += eb;
            }
        }
        float ra = (a0 + a1) * aba[D];                // row L & 7, block L >> 3
        float rb = (c0 + c1) * abb[D];                // row (L & 7) + 8
        ra += __shfl_xor_sync(0xffffffffu, ra, 8);    // + the slice's other blocks
        rb += __shfl_xor_sync(0xffffffffu, rb, 8);
        ra += __shfl_xor_sync(0xffffffffu, ra, 16);
        rb += __shfl_xor_sync(0xffffffffu, rb, 16);
        // lanes 0..7 hold rows 0..7 in ra, lanes 8..15 rows 8..15 in rb
        const float r = lane < 8 ? ra : rb;
        if (!counted_in) {
            if (held < kXtabHold) {   // keep it until the count-in (a compile-time slot per case)
#pragma unroll
                for (int i = 0; i < kXtabHold; ++i)
                    if (i == held) {
                        hold_r[i] = r;
                        hold_y[i] = yb[D];
                        hold_n[i] = nvb[D];
                    }
                ++held;
                return;
            }
            count_in();
        }
        if (lane < nvb[D]) red_add_f32(yb[D] + lane, r);
    };

    int k_item = 0;
    bool have = xtab_item(p, c, 0, s, b0, b1);
    int nb = have && b1 > b0 + warp ? (b1 - b0 - warp + NW - 1) / NW : 0;
    // weights first: they do not depend on the preceding grid
    if (nb > 0) seek(b0 + warp);
#pragma unroll
    for (int d = 0; d < R - 1; ++d) {
        if (d < nb) issue(d);
        commit();
    }
    asm volatile("griddepcontrol.launch_dependents;");
    asm volatile("griddepcontrol.wait;" ::: "memory");

    // the first item's x pieces (the table build below), requested before the zeroing
    __half2 xh[4];
    if (have) {
        const __half2* xp = reinterpret_cast<const __half2*>(p.x + s * kXtabCols + 8 * lane);
#pragma unroll
        for (int j = 0; j < 4; ++j) xh[j] = xp[j];
    }

    // ---- zero this CTA's share of y, then count in ----------------------------
    {
        const int z0 = (int)((long long)c * p.nbatch / G), z1 = (int)((long long)(c + 1) * p.nbatch / G);
        for (int i = z0 * kXtabBatch + (int)threadIdx.x; i < z1 * kXtabBatch; i += 32 * NW) {
            int r0;
            const XtabSeg& zs = p.seg[xtab_seg_of(p, i / kXtabBatch, r0)];
            const int r = r0 + (i % kXtabBatch);
            if (r < zs.out_f) zs.y[r] = 0.0f;
        }
        __syncthreads();
        // release: the CTA's zeroes (ordered before it by the barrier) are
        // visible to whoever sees the count; nothing here waits for it
        if (threadIdx.x == 0) red_release_add_u32(&p.bar[0], 1u);
    }

    while (have) {
        // ---- the slice's tables: warp w fills byte values w, w + NW, ...; lane L
        // its own column of each of its four pairs' tables (conflict-free stores);
        // the previous item's lookups are done (__syncthreads below the batches)
        {
            if (k_item > 0) {
                const __half2* xp = reinterpret_cast<const __half2*>(p.x + s * kXtabCols + 8 * lane);
#pragma unroll
                for (int j = 0; j < 4; ++j) xh[j] = xp[j];
            }
            float x0[4], x1[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                x0[j] = __low2float(xh[j]);
                x1[j] = __high2float(xh[j]);
            }
            for (int b = warp; b < 256; b += NW) {
                const float t0 = c_nf4_table[b & 15], t1 = c_nf4_table[b >> 4];
                const uint32_t o = (uint32_t)b << 8;
                sts_f32(lk0 + o, fmaf(t1, x1[0], t0 * x0[0]));
                sts_f32(lk1 + o, fmaf(t1, x1[1], t0 * x0[1]));
                sts_f32(lk2 + o, fmaf(t1, x1[2], t0 * x0[2]));
                sts_f32(lk3 + o, fmaf(t1, x1[3], t0 * x0[3]));
            }
        }
        __syncthreads();

        // ---- the batches, R per round so that ring slots are compile-time; the
        // steady rounds issue a batch per step, the last R - 1 steps do not
        int it = 0;
        for (; it + 2 * R - 1 <= nb; it += R)
            xtab_unroll<0, R>([&](auto dc) { step(dc, true); });
        for (; it < nb; it += R)
            xtab_unroll<0, R>([&](auto dc) {
                constexpr int D = decltype(dc)::value;
                if (it + D < nb) step(dc, it + D + R - 1 < nb);
            });
        asm volatile("cp.async.wait_group 0;" ::: "memory");
        if (held > 0) count_in();   // a warp with fewer batches than kHold
        ++k_item;
        have = xtab_item(p, c, k_item, s, b0, b1);
        __syncthreads();   // every warp is done with the tables and its ring
        nb = have && b1 > b0 + warp ? (b1 - b0 - warp + NW - 1) / NW : 0;
        if (nb > 0) {
            sg = -1;
            sg_first = 0;
            sg_end = 0;
            seek(b0 + warp);
        }
#pragma unroll
        for (int d = 0; d < R - 1; ++d) {
            if (d < nb) issue(d);
            commit();
        }
    }

    // ---- leave: the last CTA out resets the counters for the next call ------------
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned old = atomicAdd(&p.bar[1], 1u);
        if (old == (unsigned)G - 1) {
            atomicExch(&p.bar[0], 0u);
            atomicExch(&p.bar[1], 0u);
        }
    }
}

void* gemv_kernel_xtab(int warps, int stages);
int xtab_device_error(int clear);

}  // namespace b4
