// b4_p2p.cuh -- the all-reduce of a row-parallel GEMV over NVLink peer
// memory, fused into the GEMV's epilogue.
//
// Each rank holds one device allocation (exported through CUDA IPC and mapped
// by every peer):
//   recv    uint64 [2][world][max_rows]   (epoch << 32) | fp32 bits of a partial row
//   error   uint32
//   epochs  uint32 [kP2pEpochSlots]       the call counter, one copy per CTA index
// indexed first by the call's parity (epoch & 1), so a rank may start call
// e+1 while a peer still reads call e's slots (call e+2 can only start after
// every peer has finished call e: it needs their call e+1 rows, which they
// store after their call e kernel has completed).
//
// The value and the call's epoch travel in ONE naturally aligned 64-bit store,
// which is single-copy atomic: a reader that sees the epoch also sees the
// value, with no flag, no fence and no second round trip.  Stale slots hold
// an older epoch (e - 2 or earlier), so they never match.
//
// A warp that has finished a block of rows stores them into slot
// [parity][rank] of every rank's recv (peer stores over NVLink, its own by a
// local store) and goes on to its next block; only after its last block does
// it read back, for each of its blocks, every rank's copy from its own memory
// (bounded polls: after kP2pMaxSpins polls, or as soon as another wait of the
// call has given up, it records kP2pErrTimeout in the error word and stores
// NaN for that row), sums the ranks in rank order and stores y.  Every rank
// adds the same numbers in the same order: y is bit-identical on all ranks.
// The call counter lives in device memory, one copy per CTA index: CTA c
// reads copy c after griddepcontrol.wait (every earlier call has completed,
// so a plain load sees its value) and, as it leaves, writes the advanced
// value into copies c, c + G, c + 2G, ... (G = the grid), so every call
// advances all copies and calls of different grid sizes agree, with no
// atomic and no fence on the way out.  Only CTA c reads copy c during a
// call.  A call captured in a CUDA graph stays correct when it is replayed.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>

namespace b4 {

constexpr int kP2pMaxRanks = 8;
constexpr uint32_t kP2pErrTimeout = 1u;
constexpr long long kP2pMaxSpins = 1ll << 22;   // x ~0.2-1 us per poll: one to a few seconds
constexpr int kP2pEpochSlots = 4096;            // copies of the call counter: the largest grid of a P2P launch

struct P2pArgs {
    unsigned long long* recv[kP2pMaxRanks];   // every rank's slots (this rank's own at [rank])
    uint32_t* epochs;                         // this rank's call counter, kP2pEpochSlots copies
    uint32_t* error;                          // this rank's error word
    int rank, world;
    int max_rows;
    __half* y16;         // optional: y rounded to fp16 as well (the next GEMV's x)
    const float* xgu;    // optional: x = fp16(silu(gate) * up) of fp32 gate = xgu[0 .. in_f),
                         // up = xgu[in_f .. 2 in_f), computed while x is staged
};

__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v)
{
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* p)
{
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// The epoch of this call (read by the CTA's threads after griddepcontrol.wait).
__device__ __forceinline__ uint32_t p2p_epoch(const P2pArgs& a)
{
    return *(volatile const uint32_t*)(a.epochs + blockIdx.x) + 1u;
}

// Lane i < nrows holds row r0 + i of this rank's partial y in v: store it into
// slot [parity][rank][r0 + i] of every rank.  Called by a whole warp.
__device__ __forceinline__ void p2p_push(const P2pArgs& a, uint32_t epoch, int r0, int nrows, float v)
{
    const int lane = threadIdx.x & 31;
    if (lane < nrows) {
        const unsigned long long w = ((unsigned long long)epoch << 32) | __float_as_uint(v);
        const size_t off = ((size_t)(epoch & 1u) * a.world + a.rank) * a.max_rows + r0 + lane;
        for (int k = 1; k <= a.world; ++k) {
            const int r = (a.rank + k) % a.world;   // peers first, this rank's own slot last
            st_relaxed_sys_u64(a.recv[r] + off, w);
        }
    }
}

// Lane i < nrows waits for row r0 + i from every rank in this rank's own slots
// and stores their sum, in rank order, into y[r0 + i].  Called by a whole warp.
// Every rank's slot is read at once (one memory round trip when the rows are
// there, not one per rank); only the ranks not yet arrived are polled again.
__device__ __forceinline__ void p2p_reduce(const P2pArgs& a, uint32_t epoch, int r0, int nrows, float* y)
{
    const int lane = threadIdx.x & 31;
    if (lane < nrows) {
        const unsigned long long* mine = a.recv[a.rank] + (size_t)(epoch & 1u) * a.world * a.max_rows + r0 + lane;
        unsigned long long w[kP2pMaxRanks];
#pragma unroll
        for (int r = 0; r < kP2pMaxRanks; ++r)
            if (r < a.world) w[r] = ld_relaxed_sys_u64(mine + (size_t)r * a.max_rows);
        float s = 0.0f;
        bool ok = true;
#pragma unroll
        for (int r = 0; r < kP2pMaxRanks; ++r) {
            if (r >= a.world || !ok) continue;
            long long n = 0;
            while ((uint32_t)(w[r] >> 32) != epoch) {
                // give up after kP2pMaxSpins polls, or at once when another wait
                // of this call already gave up (a missing peer costs one timeout)
                if (++n >= kP2pMaxSpins || ((n & 63) == 0 && *(volatile const uint32_t*)a.error)) {
                    atomicOr(a.error, kP2pErrTimeout);
                    ok = false;
                    break;
                }
                __nanosleep(64);
                w[r] = ld_relaxed_sys_u64(mine + (size_t)r * a.max_rows);
            }
            if (ok) s += __uint_as_float((uint32_t)w[r]);
        }
        if (!ok) s = __int_as_float(0x7fffffff);   // a row with a missing rank is NaN, never a partial sum
        y[r0 + lane] = s;
        if (a.y16) a.y16[r0 + lane] = __float2half_rn(s);
    }
}

// The CTA advances its copies of the call counter (called by every thread of
// the CTA, after a barrier that follows every thread's p2p_epoch).
__device__ __forceinline__ void p2p_finish(const P2pArgs& a, uint32_t epoch)
{
    for (int i = blockIdx.x + threadIdx.x * gridDim.x; i < kP2pEpochSlots; i += blockDim.x * gridDim.x)
        a.epochs[i] = epoch;
}

}  // namespace b4
