// b4_p2p.cu -- host side of the peer-memory all-reduce fused into the
// row-parallel GEMV (device side: b4_p2p.cuh, b4_gemv_lean.cuh P2P = 1).
//
// One cudaMalloc per rank holds the receive slots and the call counter; its CUDA IPC handle travels to the peers over whatever channel
// the caller has (the Python layer uses torch.distributed), and each peer
// maps it with cudaIpcOpenMemHandle.  Kernels only ever store to peers and
// read their own memory; every wait in them is bounded.
#include <algorithm>
#include <cstring>
#include <new>

#include "b4_internal.h"

using namespace b4;

struct b4_p2p {
    int device = 0;
    int rank = 0, world = 0;
    int max_rows = 0;
    char* base = nullptr;                 // this rank's allocation
    char* peers[kP2pMaxRanks] = {};      // every rank's allocation as mapped here (own at [rank])
    size_t recv_bytes = 0, bytes = 0;
    // after the receive slots: 256 bytes holding the error word, the call
    // counter's kP2pEpochSlots copies, 256 bytes of x-pair table kernel
    // counters, then max_rows floats of this rank's partial y (the NF4
    // shard's GEMV before the all-reduce)
    static constexpr size_t kEpochBytes = kP2pEpochSlots * sizeof(uint32_t);
    uint32_t* error_word() const { return reinterpret_cast<uint32_t*>(base + recv_bytes); }
    uint32_t* epochs() const { return reinterpret_cast<uint32_t*>(base + recv_bytes + 256); }
    void* xtab_ws() const { return base + recv_bytes + 256 + kEpochBytes; }
    float* partial() const { return reinterpret_cast<float*>(base + recv_bytes + 512 + kEpochBytes); }
};

namespace {

P2pArgs args_of(const b4_p2p* h)
{
    P2pArgs a = {};
    for (int r = 0; r < h->world; ++r) a.recv[r] = reinterpret_cast<unsigned long long*>(h->peers[r]);
    a.epochs = h->epochs();
    a.error = h->error_word();
    a.rank = h->rank;
    a.world = h->world;
    a.max_rows = h->max_rows;
    return a;
}

// The all-reduce of a row-parallel shard's partial y (part) over the ranks'
// peer memory, as its own launch (after a GEMV that cannot carry it in its
// epilogue): warp w of CTA c pushes rows 32 (8c + w) + 32 * 8 * gridDim.x * i
// of this rank to every rank's slots, then sums every rank's copy of them in
// rank order into y (and y16).  A programmatic dependent of the GEMV: it waits
// for the GEMV's grid before it reads part.  A CTA waits only for the CTA of
// the same index on the peers, and the grid (rows / 256 CTAs of 8 warps) is
// small enough to be resident at once.
__global__ void __launch_bounds__(256) p2p_allreduce_kernel(const P2pArgs a, const float* __restrict__ part,
                                                             float* __restrict__ y, int rows)
{
    asm volatile("griddepcontrol.launch_dependents;");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const uint32_t epoch = p2p_epoch(a);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int step = 32 * 8 * (int)gridDim.x;
    for (int r0 = 32 * (8 * (int)blockIdx.x + warp); r0 < rows; r0 += step) {
        const int n = min(32, rows - r0);
        p2p_push(a, epoch, r0, n, lane < n ? part[r0 + lane] : 0.0f);
    }
    for (int r0 = 32 * (8 * (int)blockIdx.x + warp); r0 < rows; r0 += step) p2p_reduce(a, epoch, r0, min(32, rows - r0), y);
    __syncthreads();   // every warp of the CTA has read the epoch
    p2p_finish(a, epoch);
}

}  // namespace

extern "C" {

int b4_p2p_create(int rank, int world, int max_rows, b4_p2p** out)
{
    if (!out || world < 1 || world > kP2pMaxRanks || rank < 0 || rank >= world || max_rows < 1)
        return cudaErrorInvalidValue;
    b4_p2p* h = new (std::nothrow) b4_p2p;
    if (!h) return cudaErrorMemoryAllocation;
    cudaError_t e = cudaGetDevice(&h->device);
    if (e != cudaSuccess) {
        delete h;
        return e;
    }
    h->rank = rank;
    h->world = world;
    h->max_rows = max_rows;
    h->recv_bytes = (size_t)2 * world * max_rows * sizeof(unsigned long long);
    h->bytes = h->recv_bytes + 512 + b4_p2p::kEpochBytes + (size_t)max_rows * sizeof(float);
    e = cudaMalloc(&h->base, h->bytes);
    if (e == cudaSuccess) e = cudaMemset(h->base, 0, h->bytes);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        if (h->base) cudaFree(h->base);
        delete h;
        return e;
    }
    h->peers[rank] = h->base;
    *out = h;
    return cudaSuccess;
}

int b4_p2p_ipc_handle(const b4_p2p* h, void* handle64)
{
    if (!h || !handle64) return cudaErrorInvalidValue;
    cudaIpcMemHandle_t ipc;
    const cudaError_t e = cudaIpcGetMemHandle(&ipc, h->base);
    if (e != cudaSuccess) return e;
    static_assert(sizeof(ipc) == 64, "CUDA IPC handles are 64 bytes");
    std::memcpy(handle64, &ipc, sizeof(ipc));
    return cudaSuccess;
}

int b4_p2p_open_peer(b4_p2p* h, int peer, const void* handle64)
{
    if (!h || !handle64 || peer < 0 || peer >= h->world || peer == h->rank || h->peers[peer])
        return cudaErrorInvalidValue;
    cudaIpcMemHandle_t ipc;
    std::memcpy(&ipc, handle64, sizeof(ipc));
    void* p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, ipc, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return e;
    h->peers[peer] = static_cast<char*>(p);
    return cudaSuccess;
}

int b4_p2p_status(b4_p2p* h, int clear)
{
    if (!h) return cudaErrorInvalidValue;
    uint32_t* err = h->error_word();
    uint32_t v = 0;
    cudaError_t e = cudaMemcpy(&v, err, sizeof(v), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return e;
    if (clear && v) {
        e = cudaMemset(err, 0, sizeof(v));
        if (e != cudaSuccess) return e;
    }
    return v ? B4_STATUS_TIMEOUT : cudaSuccess;
}

int b4_p2p_destroy(b4_p2p* h)
{
    if (!h) return cudaErrorInvalidValue;
    cudaError_t first = cudaSuccess;
    for (int r = 0; r < h->world; ++r) {
        if (r != h->rank && h->peers[r]) {
            const cudaError_t e = cudaIpcCloseMemHandle(h->peers[r]);
            if (first == cudaSuccess) first = e;
        }
    }
    const cudaError_t e = cudaFree(h->base);
    if (first == cudaSuccess) first = e;
    delete h;
    return first;
}

int b4_tp_gemv_p2p_ex(int fmt, const uint32_t* qw_shard, const void* scale_shard, const void* x_shard, float* y,
                      void* y16, int in_shard, int out_f, b4_p2p* h, int flags, b4_stream_t stream)
{
    if (!h) return cudaErrorInvalidValue;
    for (int r = 0; r < h->world; ++r)
        if (!h->peers[r]) return cudaErrorInvalidValue;   // every peer must be mapped first
    if (flags & ~(B4_FLAG_PDL | B4_FLAG_X_SWIGLU)) return cudaErrorInvalidValue;
    const bool swiglu = flags & B4_FLAG_X_SWIGLU;
    // the checks see an fp16 x of in_shard columns; an fp32 gate/up pair needs 16-byte alignment
    if (swiglu && (!x_shard || reinterpret_cast<uintptr_t>(x_shard) % 16)) return cudaErrorInvalidValue;
    if (y16 && reinterpret_cast<uintptr_t>(y16) % 2) return cudaErrorInvalidValue;
    const GemvProblem p{fmt, qw_shard, scale_shard, x_shard, y, in_shard, out_f, 1, in_shard, out_f};
    int e = check_problem(p);
    if (e != cudaSuccess) return e;
    P2pArgs a = args_of(h);
    a.y16 = static_cast<__half*>(y16);
    a.xgu = swiglu ? static_cast<const float*>(x_shard) : nullptr;
    const int lf = flags & B4_FLAG_PDL;
    const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (fmt == B4_FMT_NF4_B64) {
        // shards the x-pair table kernel takes: that GEMV into this rank's
        // partial y, then the all-reduce as its own launch (the kernel adds
        // its slices' shares with atomics, so no CTA of it holds a finished
        // row to push)
        if (out_f <= h->max_rows) {
            GemvProblem q = p;
            q.y = h->partial();
            e = launch_xtab_shard(q, a.xgu, lf, h->xtab_ws(), st);
            if (e == cudaSuccess) {
                a.xgu = nullptr;
                cudaLaunchConfig_t lc = {};
                lc.gridDim = dim3((unsigned)std::min((out_f + 255) / 256, kP2pEpochSlots));
                lc.blockDim = dim3(256);
                lc.stream = st;
                cudaLaunchAttribute attr[1];
                attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
                attr[0].val.programmaticStreamSerializationAllowed = 1;
                lc.attrs = attr;
                lc.numAttrs = 1;
                return cudaLaunchKernelEx(&lc, p2p_allreduce_kernel, a, static_cast<const float*>(h->partial()), y,
                                          out_f);
            }
            if (e != cudaErrorNotSupported) return e;
        }
        return launch_nf4_mma_p2p(p, a, lf, st);
    }
    b4_gemv_config c;
    default_config(p, &c);
    c.flags = lf;
    return launch_lean_int4_p2p(p, c, a, reinterpret_cast<cudaStream_t>(stream));
}

int b4_tp_gemv_p2p(int fmt, const uint32_t* qw_shard, const void* scale_shard, const void* x_shard, float* y,
                   int in_shard, int out_f, b4_p2p* h, int flags, b4_stream_t stream)
{
    if (flags & ~B4_FLAG_PDL) return cudaErrorInvalidValue;
    return b4_tp_gemv_p2p_ex(fmt, qw_shard, scale_shard, x_shard, y, nullptr, in_shard, out_f, h, flags, stream);
}

}  // extern "C"
