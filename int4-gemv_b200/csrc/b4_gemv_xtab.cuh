// b4_gemv_xtab.cuh -- the batch-1 NF4 b64 GEMV from tables of x-pair products.
//
// The code book is what bounds the other NF4 kernels: every code costs a
// shared-memory read of its value (4 bytes per code on the tensor-pipe kernel,
// fp16 high + low part), and the shared-memory path runs out before HBM does.
// This kernel moves x into the table instead:
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
// 256-column SLICE of in_f: 32 packed words of 4 byte positions each.  The
// matrix is cut into (slice, 16-row batch) units.  With S = in_f/256 slices
// and G CTAs, slice s gets G/S or G/S + 1 CTAs that split its batches evenly
// (S > G: each CTA takes slices c, c + G, ... with every batch), or, where the
// host finds that uneven (xtab_tail), G/S main CTAs per slice split all but
// its last `tail` batches and the other G % S CTAs share the S tails in equal
// runs, one item (table build) per slice a run touches.  A warp takes the
// batches b0 + warp, b0 + warp + NW, ... of its CTA's item; the next item's
// first batches and x are requested before the barrier that ends an item.
//
// Codes go straight from global memory into registers, P batches ahead, in
// whole 128-byte lines (the lookups are then the only shared-memory traffic
// of the steady state; staging the codes through shared memory cost 16 writes
// and 16 reads per batch next to the 64 lookups, and ran 10-15 % slower):
// lane L loads the 16-byte piece pc = L & 7 (words 4 pc .. 4 pc + 3 of the
// slice) of rows rq + 4t of a batch (rq = L >> 3, t = 0..3) and does that
// piece's lookups.  Registers cannot be indexed by a lane-dependent order, so
// at step (t, k) a lane uses word 4 pc + k of row rq + 4t, and the bank spread
// over the 32 lanes of a lookup comes from the table layout and a per-lane
// rotation: each code word is rotated right by 8 rq bits once, so byte
// position j of a lane is the word's byte jj = (j + rq) & 3.  The table of
// column pair (word w, byte jj) sits at
//     T*65536 + (w>>1 & 1)*65536 + b*256 + (w & 1)*128 + (w >> 2)*16 + jj*4
// (T = the tables' 64 KB-aligned base >> 16), so the bank (address bits 2..6)
// is (w >> 2 = pc, jj): different for the 32 lanes of every lookup, whatever
// the bytes.  The other bits depend only on k: a lane keeps per byte position
// j a register with the two possible low address bytes (k even, odd) and T,
// T + 1, and one PRMT with a constant selector forms a lookup's complete
// shared address from the code byte: one PRMT + one LDS + one FADD per two
// codes.
//
// A lane's four row sums (its piece of rows rq + 4t) are scaled by the
// absmax of its NF4 block (pc >> 1) and reduced over the 8 pieces of a row
// with four shuffles (a reduce-scatter), after which lanes with pc even hold
// row rq + 4 ((pc >> 1) & 3) and add it into y.
//
// The slices' shares meet in y through fp32 atomic adds (reductions in L2,
// fire and forget: no cross-CTA wait at the end of the kernel).  y must be zero
// first: each CTA zeroes its share of y's rows right after the grid-dependency
// wait and, once its first tables are built, counts itself in on a workspace
// counter; a warp keeps the results of its first kXtabHold batches in
// registers and waits (bounded) for all G arrivals of this call before its
// first add, which by then has normally happened, so the count-in is off the
// critical path.  The workspace holds two running counters, arrivals and
// base (the arrivals of all earlier calls): a call's CTAs read base after the
// grid-dependency wait and wait for arrivals to reach base + G (compared
// modulo 2^32); the CTA whose count-in completes the call (an acq_rel atomic
// that returns the old count) advances base by G.  Every CTA has read base
// before it counts in, so no read can see the advanced value, and nothing
// happens on the way out: no fence, no atomic, no reset.  Between calls the
// two counters are equal (zero-filled to start with).  Summation order across
// slices varies from run to run (within fp32 rounding); everything else is
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
    unsigned* bar;       // workspace: [0] arrivals, [1] base (equal between calls)
    uint32_t smem;       // dynamic shared memory of the launch (bytes)
    const float* xgu;    // non-null: x = fp16(silu(gate) * up) of fp32 gate = xgu[0 .. in_f), up = xgu[in_f ..)
    int mains, tail;     // tail > 0: mains CTAs per slice and tail batches per slice for the others (xtab_item)
};

// The device error flag of this translation unit (read by xtab_device_error).
static __device__ int g_xtab_error;

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p)
{
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ unsigned atom_acq_rel_add_u32(unsigned* p, unsigned v)
{
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

__device__ __forceinline__ void red_relaxed_add_u32(unsigned* p, unsigned v)
{
    asm volatile("red.relaxed.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned ld_relaxed_u32(const unsigned* p)
{
    unsigned v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
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

// The four lookups of a (rotated) code word at step k of its row: the sum of
// the word's four column-pair entries.  Selector bytes: the low address byte
// (lw byte 0 or 1 by k bit 0), code byte j, T or T + 1 (k bit 1), zero (the
// sign of T).
template <int K>
__device__ __forceinline__ float xtab_word(uint32_t w, const uint32_t (&lw)[4])
{
    constexpr uint32_t S = 0xE000u | ((6u + ((K >> 1) & 1)) << 8) | (4u + (K & 1));
    return (lds_f32(prmt<S>(w, lw[0])) + lds_f32(prmt<S | 0x10u>(w, lw[1]))) +
           (lds_f32(prmt<S | 0x20u>(w, lw[2])) + lds_f32(prmt<S | 0x30u>(w, lw[3])));
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
// tail > 0: CTAs c < mains * S are a slice's main CTAs (slice c / mains), which
// split its first nbatch - tail batches evenly, one item each; the other E
// CTAs split the S tails of tail batches (slice-major) into equal runs, one
// item per slice a run touches.  Otherwise slice s gets G/S or G/S + 1 CTAs
// that split its batches evenly (S > G: slices c, c + G, ... with every batch).
__device__ __forceinline__ bool xtab_item(const XtabParams& p, int c, int k, int& s, int& b0, int& b1)
{
    const int G = gridDim.x;
    if (p.tail > 0) {
        const int km = p.mains * p.nslice, head = p.nbatch - p.tail;
        if (c < km) {
            if (k > 0) return false;
            s = c / p.mains;
            const int u = c % p.mains;
            b0 = (int)((long long)u * head / p.mains);
            b1 = (int)((long long)(u + 1) * head / p.mains);
            return true;
        }
        const long long T = (long long)p.nslice * p.tail, E = G - km, e = c - km;
        const long long lo = e * T / E, hi = (e + 1) * T / E;
        s = (int)(lo / p.tail) + k;
        const long long first = (long long)s * p.tail;
        const long long a = lo > first ? lo : first, z = hi < first + p.tail ? hi : first + p.tail;
        if (s >= p.nslice || a >= z) return false;
        b0 = head + (int)(a - first);
        b1 = head + (int)(z - first);
        return true;
    }
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

// The tables' two 64 KB halves start on a 64 KB boundary of the CTA's shared
// window (`base` = where dynamic shared memory starts, after the reserved part),
// so a PRMT can place T and T + 1 in the address's third byte.
__host__ __device__ constexpr uint32_t xtab_align64k(uint32_t base) { return (base + 65535u) & ~65535u; }

constexpr int kErrXtabLayout = 4;

__host__ __device__ constexpr uint32_t xtab_smem_bytes(uint32_t base)
{
    return (xtab_align64k(base) - base) + (uint32_t)kXtabTableBytes;
}

__device__ __forceinline__ void ldg_v4_na(uint32_t& d0, uint32_t& d1, uint32_t& d2, uint32_t& d3, const void* p)
{
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(d0), "=r"(d1), "=r"(d2), "=r"(d3)
                 : "l"(p));
}

template <int NW, int P>
__global__ void __launch_bounds__(32 * NW, 1) b4_gemv_xtab_kernel(const XtabParams p)
{
    static_assert(P >= 1, "register stages: at least 1");
    extern __shared__ __align__(16) float xtab[];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int G = gridDim.x, c = blockIdx.x;
    const int nblk = p.in_f >> 6;
    const long long rowb = p.in_f >> 1;
    const int rq = lane >> 3, pc = lane & 7;
    const int myrow = rq + 4 * ((pc >> 1) & 3);   // the row this lane adds into y (pc even)
    const bool adder = (pc & 1) == 0;

    const uint32_t base = static_cast<uint32_t>(__cvta_generic_to_shared(xtab));
    const uint32_t tab = xtab_align64k(base);
    if (xtab_smem_bytes(base) > p.smem) {
        if (threadIdx.x == 0) atomicOr(&g_xtab_error, kErrXtabLayout);
        return;
    }
    const uint32_t T = tab >> 16;
    uint32_t lwr[4];   // per byte position j: (low byte for k even, for k odd, T, T + 1)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t jj = ((uint32_t)(j + rq)) & 3u;
        const uint32_t lo0 = ((uint32_t)pc << 4) | (jj << 2);
        lwr[j] = ((T + 1) << 24) | (T << 16) | ((lo0 | 128u) << 8) | lo0;
    }
    // table build: lane L writes word bits 2..4 = L >> 2, byte position L & 3,
    // the four words t = 0..3 of that group (w bit 0 -> +128, w bit 1 -> +64 KB)
    const uint32_t bl = tab + 4u * (uint32_t)lane;
    const int xcol = 32 * (lane >> 2) + 2 * (lane & 3);   // column of word t = 0's pair in the slice

    int s = 0, b0 = 0, b1 = 0;
    int sg = -1, sg_first = 0, sg_end = 0, out_f = 0;
    float* yseg = nullptr;
    const unsigned char* qsrc = nullptr;   // row rq of the next batch, this lane's piece
    const float* asrc = nullptr;           // absmax of row rq, this lane's block
    int bnext = 0;
    auto seek = [&](int b) {
        while (b >= sg_end) {
            sg_first = sg_end;
            ++sg;
            sg_end = p.seg[sg].batch_end;
        }
        const XtabSeg& g = p.seg[sg];
        out_f = g.out_f;
        yseg = g.y;
        const int r0 = (b - sg_first) * kXtabBatch;
        qsrc = reinterpret_cast<const unsigned char*>(g.qw) + s * 128 + (long long)(r0 + rq) * rowb + pc * 16;
        asrc = g.absmax + (long long)(r0 + rq) * nblk + 4 * s + (pc >> 1);
        bnext = b;
    };
    uint32_t cw[P][16];   // words 4 pc .. 4 pc + 3 of rows rq, rq + 4, rq + 8, rq + 12
    float ab[P][4];
    float* yb[P];
    int nvb[P];
    const uint32_t q4 = (uint32_t)(4 * rowb);   // bytes between a lane's rows rq + 4t and rq + 4t + 4
    const uint32_t q8 = 2 * q4, q12 = 3 * q4;
    const int a4 = 4 * nblk;                    // absmax floats between them
    auto issue = [&](auto dc) {
        constexpr int D = decltype(dc)::value;
        if (bnext >= sg_end) seek(bnext);
        const int r0 = (bnext - sg_first) * kXtabBatch;
        const int nv = min(kXtabBatch, out_f - r0);
        if (nv == kXtabBatch) {
            ldg_v4_na(cw[D][0], cw[D][1], cw[D][2], cw[D][3], qsrc);
            ldg_v4_na(cw[D][4], cw[D][5], cw[D][6], cw[D][7], qsrc + q4);
            ldg_v4_na(cw[D][8], cw[D][9], cw[D][10], cw[D][11], qsrc + q8);
            ldg_v4_na(cw[D][12], cw[D][13], cw[D][14], cw[D][15], qsrc + q12);
            ab[D][0] = __ldg(asrc);
            ab[D][1] = __ldg(asrc + a4);
            ab[D][2] = __ldg(asrc + 2 * a4);
            ab[D][3] = __ldg(asrc + 3 * a4);
        } else {   // rows past out_f read the segment's last row
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const int dr = min(rq + 4 * t, nv - 1) - rq;
                ldg_v4_na(cw[D][4 * t], cw[D][4 * t + 1], cw[D][4 * t + 2], cw[D][4 * t + 3], qsrc + dr * rowb);
                ab[D][t] = __ldg(asrc + (long long)dr * nblk);
            }
        }
        yb[D] = yseg + r0;
        nvb[D] = nv;
        bnext += NW;
        qsrc += NW * kXtabBatch * rowb;
        asrc += (long long)NW * kXtabBatch * nblk;
    };
    const bool h4 = (pc & 4) != 0, h2 = (pc & 2) != 0;
    // the lookups of register stage D and the lane's row sum; stage D takes the
    // warp's next batch (if `more`) once its codes are used
    auto compute = [&](auto dc, bool more) -> float {
        constexpr int D = decltype(dc)::value;
        const uint32_t sh = 8u * (uint32_t)rq;
        float v[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const uint32_t* wt = cw[D] + 4 * t;
            const float e0 = xtab_word<0>(__funnelshift_r(wt[0], wt[0], sh), lwr) +
                             xtab_word<2>(__funnelshift_r(wt[2], wt[2], sh), lwr);
            const float e1 = xtab_word<1>(__funnelshift_r(wt[1], wt[1], sh), lwr) +
                             xtab_word<3>(__funnelshift_r(wt[3], wt[3], sh), lwr);
            v[t] = (e0 + e1) * ab[D][t];
        }
        if (more) issue(dc);
        // reduce-scatter over the 8 pieces of each row: xor 4 keeps rows t = 2 h4 + {0, 1},
        // xor 2 keeps t = 2 h4 + h2, xor 1 completes it
        const float s0 = h4 ? v[0] : v[2], s1 = h4 ? v[1] : v[3];
        const float k0 = (h4 ? v[2] : v[0]) + __shfl_xor_sync(0xffffffffu, s0, 4);
        const float k1 = (h4 ? v[3] : v[1]) + __shfl_xor_sync(0xffffffffu, s1, 4);
        float r = (h2 ? k1 : k0) + __shfl_xor_sync(0xffffffffu, h2 ? k0 : k1, 2);
        r += __shfl_xor_sync(0xffffffffu, r, 1);
        return r;
    };
    auto add = [&](float* yd, int nd, float r) {
        if (adder && myrow < nd) red_add_f32(yd + myrow, r);
    };
    // This warp's adds into y wait until every CTA has counted in: the results
    // of an item's first kXtabHold batches are held in registers, and the
    // (first item's) wait comes after them, by when the count is normally
    // complete.
    bool counted_in = false;
    unsigned target = 0u;   // this call's arrivals end at base + G (set after the grid-dependency wait)
    auto wait_count = [&]() {
        if (lane == 0) {
            unsigned n = 0;
            while ((int)(ld_acquire_u32(&p.bar[0]) - target) < 0) {
                if (++n >= kXtabMaxPolls) {
                    atomicOr(&g_xtab_error, kErrXtabBarrier);
                    break;
                }
                __nanosleep(64);
            }
        }
        __syncwarp();
        counted_in = true;
    };
    constexpr int H = kXtabHold;

    int k_item = 0;
    bool have = xtab_item(p, c, 0, s, b0, b1);
    int nb = have && b1 > b0 + warp ? (b1 - b0 - warp + NW - 1) / NW : 0;
    // weights first: they do not depend on the preceding grid
    if (nb > 0) seek(b0 + warp);
    xtab_unroll<0, P>([&](auto dc) {
        constexpr int D = decltype(dc)::value;
        if (D < nb) issue(dc);
    });
    asm volatile("griddepcontrol.launch_dependents;");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // base is read before this CTA counts in
    target = ld_relaxed_u32(&p.bar[1]) + (unsigned)G;
    // the count-in: the CTA that completes the call advances base (old is
    // only looked at later, so the atomic's round trip is not waited for)
    auto count_in = [&]() { return atom_acq_rel_add_u32(&p.bar[0], 1u); };
    auto close_call = [&](unsigned old) {
        if (old == target - 1u) red_relaxed_add_u32(&p.bar[1], (unsigned)G);
    };

    // x of the tables' column pairs (columns xcol + 8t and the next, t = 0..3,
    // of slice sl): fp16 x, or fp16(silu(gate) * up) from fp32 gate/up rows
    __half2 xh[4];
    float2 xg[4], xu[4];
    auto load_x = [&](int sl) {
        if (p.xgu) {
            const float* g = p.xgu + sl * kXtabCols + xcol;
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                xg[t] = *reinterpret_cast<const float2*>(g + 8 * t);
                xu[t] = *reinterpret_cast<const float2*>(g + p.in_f + 8 * t);
            }
        } else {
#pragma unroll
            for (int t = 0; t < 4; ++t) xh[t] = *reinterpret_cast<const __half2*>(p.x + sl * kXtabCols + xcol + 8 * t);
        }
    };
    // the first item's x, requested before the zeroing
    if (have) load_x(s);

    // ---- zero this CTA's share of y (the count-in follows the table build) ---
    {
        const int z0 = (int)((long long)c * p.nbatch / G), z1 = (int)((long long)(c + 1) * p.nbatch / G);
        for (int i = z0 * kXtabBatch + (int)threadIdx.x; i < z1 * kXtabBatch; i += 32 * NW) {
            int r0;
            const XtabSeg& zs = p.seg[xtab_seg_of(p, i / kXtabBatch, r0)];
            const int r = r0 + (i % kXtabBatch);
            if (r < zs.out_f) zs.y[r] = 0.0f;
        }
        if (!have) {
            __syncthreads();
            if (threadIdx.x == 0) close_call(count_in());
        }
    }
    unsigned arrived = 0u;   // the count-in's old value (thread 32 (NW - 1) of a CTA with work)

    while (have) {
        // ---- the slice's tables: warp w fills byte values w, w + NW, ...
        {
            float x0[4], x1[4];
            if (p.xgu) {   // rounded as the SwiGLU glue kernel rounds it
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    x0[t] = __half2float(__float2half_rn(swiglu_silu(xg[t].x) * xu[t].x));
                    x1[t] = __half2float(__float2half_rn(swiglu_silu(xg[t].y) * xu[t].y));
                }
            } else {
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    x0[t] = __low2float(xh[t]);
                    x1[t] = __high2float(xh[t]);
                }
            }
            for (int b = warp; b < 256; b += NW) {
                const float t0 = c_nf4_table[b & 15], t1 = c_nf4_table[b >> 4];
                const uint32_t o = bl + ((uint32_t)b << 8);
                sts_f32(o, fmaf(t1, x1[0], t0 * x0[0]));
                sts_f32(o + 128, fmaf(t1, x1[1], t0 * x0[1]));
                sts_f32(o + 65536, fmaf(t1, x1[2], t0 * x0[2]));
                sts_f32(o + 65536 + 128, fmaf(t1, x1[3], t0 * x0[3]));
            }
        }
        __syncthreads();
        if (k_item == 0 && threadIdx.x == 32 * (NW - 1)) arrived = count_in();
        // the lookups' addresses, as values defined after the barrier (the shared
        // loads are not volatile and must not move above it)
#pragma unroll
        for (int j = 0; j < 4; ++j) lwr[j] = opaque(lwr[j]);

        // ---- the batches: batch i sits in register stage i % P (compile-time
        // below); the first H hold their results until the count-in
        float hr[H];
        float* hy[H];
        int hn[H];
        xtab_unroll<0, H>([&](auto hc) {
            constexpr int h = decltype(hc)::value;
            if (h < nb) {
                hy[h] = yb[h % P];
                hn[h] = nvb[h % P];
                hr[h] = compute(std::integral_constant<int, h % P>{}, h + P < nb);
            }
        });
        if (k_item == 0 && threadIdx.x == 32 * (NW - 1)) close_call(arrived);
        if (!counted_in) wait_count();
        xtab_unroll<0, H>([&](auto hc) {
            constexpr int h = decltype(hc)::value;
            if (h < nb) add(hy[h], hn[h], hr[h]);
        });
        int it = H;
        for (; it + 2 * P <= nb; it += P)   // every batch of the round refills its stage
            xtab_unroll<0, P>([&](auto ec) {
                constexpr int D = (H + decltype(ec)::value) % P;
                float* const yd = yb[D];
                const int nd = nvb[D];
                add(yd, nd, compute(std::integral_constant<int, D>{}, true));
            });
        for (; it < nb; it += P)
            xtab_unroll<0, P>([&](auto ec) {
                constexpr int E = decltype(ec)::value;
                constexpr int D = (H + E) % P;
                if (it + E < nb) {
                    float* const yd = yb[D];
                    const int nd = nvb[D];
                    add(yd, nd, compute(std::integral_constant<int, D>{}, it + E + P < nb));
                }
            });
        // the next item's first batches and its x are requested before the
        // barrier (registers only), so they are in flight while the slower
        // warps finish and the tables are rebuilt
        ++k_item;
        have = xtab_item(p, c, k_item, s, b0, b1);
        nb = have && b1 > b0 + warp ? (b1 - b0 - warp + NW - 1) / NW : 0;
        if (nb > 0) {
            sg = -1;
            sg_first = 0;
            sg_end = 0;
            seek(b0 + warp);
        }
        xtab_unroll<0, P>([&](auto dc) {
            constexpr int D = decltype(dc)::value;
            if (D < nb) issue(dc);
        });
        if (have) load_x(s);
        __syncthreads();   // every warp is done with the tables
    }
}

void* gemv_kernel_xtab(int warps, int stages);
int xtab_device_error(int clear);

}  // namespace b4
