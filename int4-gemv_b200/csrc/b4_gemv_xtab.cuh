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
// Geometry.  A table costs 1 KB per column pair, so a CTA (16 warps, one per
// SM: 128 KB of tables) covers a 256-column SLICE of in_f: lane L of every warp
// owns packed word L of the slice (bytes j = 0..3: column pairs 4L + j) and
// reads only its own copy of those four tables, laid out
//       float [j >> 1][b][j & 1][lane]
// so the 32 lanes of a lookup hit the 32 banks once, whatever the bytes.  PRMT
// builds a lookup's offset (byte b in bits 8..15, 4*lane (+128) in bits 0..7)
// from a packed word in one instruction.
//
// Work.  The matrix is cut into (slice, 8-row batch) units.  With S = in_f/256
// slices and G CTAs, slice s gets G/S or G/S + 1 CTAs that split its batches
// evenly (S > G: each CTA takes slices c, c + G, ... with every batch).  A warp
// takes the batches b0 + warp, + 16, ... of its CTA's range; per batch a lane
// loads its word of the 8 rows (one coalesced 128-byte row piece per warp and
// row) and one absmax, D batches ahead in registers.  The 8 rows' per-lane sums
// are reduced by a transposed butterfly over the lanes of each NF4 block (lanes
// 8q .. 8q+7 own block q of the slice): 7 shuffles leave lane L with row L & 7
// of block L >> 3, which its absmax scales; two more shuffles add the four
// blocks.  Lanes 0..7 then add the slice's share of rows r0 .. r0+7 into y.
//
// The slices' shares meet in y through fp32 atomic adds (reductions in L2,
// fire and forget: no cross-CTA wait at the end of the kernel).  y must be zero
// first: each CTA zeroes its share of y's rows right after the grid-dependency
// wait and counts itself in on a workspace counter; a warp waits (bounded) for
// all G arrivals before its first add, which in practice has long happened:
// the table build lies between.  The last CTA to leave resets the two counters,
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

#include "b4_common.cuh"

namespace b4 {

constexpr int kXtabCols = 256;                          // columns per slice: 32 words
constexpr int kXtabWarps = 16;
constexpr int kXtabThreads = 32 * kXtabWarps;
constexpr int kXtabBatch = 8;                           // rows per warp batch
constexpr int kXtabTableBytes = 4 * 256 * 32 * 4;       // 4 byte positions x 256 values x 32 lanes x fp32
constexpr int kXtabMaxSeg = 4;
constexpr unsigned kXtabMaxPolls = 1u << 22;
constexpr int kErrXtabBarrier = 2;

// One weight matrix of a launch: 8-row batches [batch_end of the previous
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
};

// The device error flag of this translation unit (read by xtab_device_error).
static __device__ int g_xtab_error;

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p)
{
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ float lds_f32(uint32_t addr)
{
    float v;
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr));
    return v;
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

template <int D>
__global__ void __launch_bounds__(kXtabThreads, 1) b4_gemv_xtab_kernel(const XtabParams p)
{
    extern __shared__ __align__(16) float xtab[];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int G = gridDim.x, c = blockIdx.x;
    const int words = p.in_f >> 3;
    const int nblk = p.in_f >> 6;
    const uint32_t tab0 = static_cast<uint32_t>(__cvta_generic_to_shared(xtab));
    const uint32_t lane4 = (uint32_t)lane * 4, lane4b = lane4 + 128;

    // ---- per-batch loads: this lane's word of 8 rows and one absmax ----------
    uint32_t wbuf[D][kXtabBatch];
    float abuf[D];
    int s = 0, b0 = 0, b1 = 0;
    auto fetch = [&](int b, int slot) {
        int r0;
        const XtabSeg& sg = p.seg[xtab_seg_of(p, b, r0)];
        const int last = sg.out_f - 1 - r0;   // rows past out_f load the last row
        const uint32_t* q = sg.qw + (long long)r0 * words + s * 32 + lane;
#pragma unroll
        for (int i = 0; i < kXtabBatch; ++i)
            wbuf[slot][i] = ld_stream<1>(q + (long long)min(i, last) * words).w[0];
        abuf[slot] = __ldg(sg.absmax + (long long)(r0 + min(lane & 7, last)) * nblk + 4 * s + (lane >> 3));
    };

    int k_item = 0;
    bool have = xtab_item(p, c, 0, s, b0, b1);
    // weights first: they do not depend on the preceding grid
    if (have) {
#pragma unroll
        for (int d = 0; d < D - 1; ++d) {
            const int b = b0 + warp + d * kXtabWarps;
            if (b < b1) fetch(b, d);
        }
    }
    asm volatile("griddepcontrol.launch_dependents;");
    asm volatile("griddepcontrol.wait;" ::: "memory");

    // ---- zero this CTA's share of y, then count in ----------------------------
    {
        const int z0 = (int)((long long)c * p.nbatch / G), z1 = (int)((long long)(c + 1) * p.nbatch / G);
        for (int i = z0 * kXtabBatch + (int)threadIdx.x; i < z1 * kXtabBatch; i += kXtabThreads) {
            int r0;
            const XtabSeg& sg = p.seg[xtab_seg_of(p, i / kXtabBatch, r0)];
            const int r = r0 + (i % kXtabBatch);
            if (r < sg.out_f) sg.y[r] = 0.0f;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            __threadfence();
            atomicAdd(&p.bar[0], 1u);
        }
    }
    bool counted_in = false;   // this warp has seen every CTA's zeroes

    while (have) {
        // ---- the slice's tables: warp w fills byte position j = w & 3, values
        // 64 * (w >> 2) .. +63, lane L its own column (conflict-free stores)
        {
            const int j = warp & 3, h = warp >> 2;
            const int k0 = s * kXtabCols + 8 * lane + 2 * j;
            const __half2 xp = *reinterpret_cast<const __half2*>(p.x + k0);
            const float x0 = __low2float(xp), x1 = __high2float(xp);
            float a[16];
#pragma unroll
            for (int c0 = 0; c0 < 16; ++c0) a[c0] = c_nf4_table[c0] * x0;
            const uint32_t wbase = tab0 + (uint32_t)((j >> 1) * 65536 + (j & 1) * 128) + lane4;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int c1 = 4 * h + q;
                const float t1 = c_nf4_table[c1];
#pragma unroll
                for (int c0 = 0; c0 < 16; ++c0) sts_f32(wbase + (uint32_t)(16 * c1 + c0) * 256, fmaf(t1, x1, a[c0]));
            }
        }
        __syncthreads();

        // ---- the batches ----------------------------------------------------------
        const int nb = b1 > b0 + warp ? (b1 - b0 - warp + kXtabWarps - 1) / kXtabWarps : 0;
        for (int it0 = 0; it0 < nb; it0 += D) {
#pragma unroll
            for (int d = 0; d < D; ++d) {
                const int it = it0 + d;
                if (it < nb) {
                    if (it + D - 1 < nb) fetch(b0 + warp + (it + D - 1) * kXtabWarps, (d + D - 1) % D);
                    float v[kXtabBatch];
#pragma unroll
                    for (int i = 0; i < kXtabBatch; ++i) {
                        const uint32_t w = wbuf[d][i];
                        const float e0 = lds_f32(tab0 + __byte_perm(w, lane4, 0x5504u));
                        const float e1 = lds_f32(tab0 + __byte_perm(w, lane4b, 0x5514u));
                        const float e2 = lds_f32(tab0 + 65536u + __byte_perm(w, lane4, 0x5524u));
                        const float e3 = lds_f32(tab0 + 65536u + __byte_perm(w, lane4b, 0x5534u));
                        v[i] = (e0 + e1) + (e2 + e3);
                    }
                    // transposed butterfly over the 8 lanes of this lane's NF4 block:
                    // lane L keeps row L & 7
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const bool hi = lane & 1;
                        const float send = hi ? v[2 * k] : v[2 * k + 1];
                        const float keep = hi ? v[2 * k + 1] : v[2 * k];
                        v[k] = keep + __shfl_xor_sync(0xffffffffu, send, 1);
                    }
#pragma unroll
                    for (int k = 0; k < 2; ++k) {
                        const bool hi = lane & 2;
                        const float send = hi ? v[2 * k] : v[2 * k + 1];
                        const float keep = hi ? v[2 * k + 1] : v[2 * k];
                        v[k] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
                    }
                    {
                        const bool hi = lane & 4;
                        const float send = hi ? v[0] : v[1];
                        const float keep = hi ? v[1] : v[0];
                        v[0] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
                    }
                    float r = v[0] * abuf[d];
                    r += __shfl_xor_sync(0xffffffffu, r, 8);
                    r += __shfl_xor_sync(0xffffffffu, r, 16);
                    if (!counted_in) {
                        // every CTA has zeroed its rows of y before any add (bounded wait)
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
                    }
                    int r0;
                    const XtabSeg& sg = p.seg[xtab_seg_of(p, b0 + warp + it * kXtabWarps, r0)];
                    if (lane < kXtabBatch && r0 + lane < sg.out_f) atomicAdd(sg.y + r0 + lane, r);
                }
            }
        }
        ++k_item;
        have = xtab_item(p, c, k_item, s, b0, b1);
        __syncthreads();   // every warp is done with the tables before they are refilled
        if (have) {
#pragma unroll
            for (int d = 0; d < D - 1; ++d) {
                const int b = b0 + warp + d * kXtabWarps;
                if (b < b1) fetch(b, d);
            }
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

void* gemv_kernel_xtab(int depth);
int xtab_device_error(int clear);

}  // namespace b4
