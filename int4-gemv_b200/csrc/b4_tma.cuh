// b4_tma.cuh -- bulk-copy (TMA) and mbarrier helpers for the streaming GEMV
// kernels, plus the device error flag that bounded waits report through.
//
// Only the untiled cp.async.bulk global -> shared copy is used, and every copy
// lands in the issuing CTA's own shared memory.
#pragma once

#include <cstdint>

namespace b4 {

// Set (atomicOr) by a kernel whose bounded wait ran out; read and cleared by
// b4_device_error() through the reader of the translation unit that holds the
// streaming kernels (gemv_tma.cu).  No relocatable device code, so the flag is
// per translation unit; only that one includes this header.
static __device__ int g_device_error;

constexpr int kErrMbarrierTimeout = 1;

__device__ __forceinline__ uint32_t smem_addr(const void* p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

// Makes mbarrier initialisation visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_mbar_init()
{
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Orders this thread's earlier generic-proxy shared-memory accesses before its
// later async-proxy (bulk copy) writes to shared memory.
__device__ __forceinline__ void fence_proxy_async()
{
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}

// 1-D bulk copy of `bytes` (a multiple of 16, both addresses 16-byte aligned)
// from global memory into this CTA's shared memory; completion is counted on
// `bar` in bytes.  The source is streamed once: evict-first in L2.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy)
{
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
        "%4;" ::"r"(smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ uint64_t evict_first_policy()
{
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t phase)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(phase)
        : "memory");
    return ok != 0;
}

// Bounded wait for phase `phase` of `bar`.  Each try_wait suspends the thread
// for up to a hardware time limit; after kMaxTries unsuccessful tries (far
// beyond any real copy time) the wait gives up, raises the device error flag
// and returns false so that the kernel can leave instead of hanging.
constexpr uint32_t kMaxTries = 1u << 22;

__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t phase)
{
    for (uint32_t i = 0; i < kMaxTries; ++i)
        if (mbar_try_wait(bar, phase)) return true;
    atomicOr(&g_device_error, kErrMbarrierTimeout);
    return false;
}

}  // namespace b4
