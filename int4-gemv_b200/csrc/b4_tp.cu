// b4_tp.cu -- tensor-parallel pieces of the decode layer: column sharding of
// packed weights for row-parallel projections, the row-parallel GEMV followed
// by an NCCL all-reduce of fp32 y, the SwiGLU activation between gate/up and
// down, and NCCL communicator management.  The reference has no multi-GPU
// code ("One GPU, one architecture", README.md:175); this is new.
//
// NCCL is resolved at run time (the process's already-loaded libnccl.so.2,
// e.g. PyTorch's, else dlopen), so loading this library never pins an NCCL
// version for the rest of the process.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <mutex>
#include <thread>

#include "b4_common.cuh"
#include "b4_internal.h"

namespace b4 {
namespace {

struct NcclApi {
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
    ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
    bool ok = false;
};

const NcclApi& nccl()
{
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = nullptr;
        void* probe = dlsym(RTLD_DEFAULT, "ncclAllReduce");
        if (!probe) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        auto sym = [&](const char* n) { return h ? dlsym(h, n) : dlsym(RTLD_DEFAULT, n); };
        api.GetUniqueId = reinterpret_cast<decltype(api.GetUniqueId)>(sym("ncclGetUniqueId"));
        api.CommInitRank = reinterpret_cast<decltype(api.CommInitRank)>(sym("ncclCommInitRank"));
        api.CommDestroy = reinterpret_cast<decltype(api.CommDestroy)>(sym("ncclCommDestroy"));
        api.CommAbort = reinterpret_cast<decltype(api.CommAbort)>(sym("ncclCommAbort"));
        api.CommGetAsyncError = reinterpret_cast<decltype(api.CommGetAsyncError)>(sym("ncclCommGetAsyncError"));
        api.AllReduce = reinterpret_cast<decltype(api.AllReduce)>(sym("ncclAllReduce"));
        api.GetErrorString = reinterpret_cast<decltype(api.GetErrorString)>(sym("ncclGetErrorString"));
        api.ok = api.GetUniqueId && api.CommInitRank && api.CommDestroy && api.CommAbort &&
                 api.CommGetAsyncError && api.AllReduce && api.GetErrorString;
    });
    return api;
}

int nccl_status(ncclResult_t r) { return r == ncclSuccess ? 0 : B4_STATUS_NCCL_BASE + (int)r; }


// The glue kernels run as programmatic dependents (launch_glue): they let the
// next kernel (a GEMV, whose weight stream does not depend on them) launch
// at once, then wait for the grid that produced their input.
__global__ void swiglu_kernel(const float* __restrict__ gate, const float* __restrict__ up,
                              __half* __restrict__ out, long long n)
{
    asm volatile("griddepcontrol.launch_dependents;");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x)
        out[i] = __float2half_rn(swiglu_silu(gate[i]) * up[i]);
}

__global__ void cast_f16_kernel(const float* __restrict__ in, __half* __restrict__ out, long long n)
{
    asm volatile("griddepcontrol.launch_dependents;");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x)
        out[i] = __float2half_rn(in[i]);
}

int grid_for(long long n) { long long g = (n + 255) / 256; return (int)(g > 148 * 8 ? 148 * 8 : (g < 1 ? 1 : g)); }

// Launches a glue kernel as a programmatic dependent of the previous kernel
// in the stream.  Safe after any kernel: the glue waits (griddepcontrol.wait)
// for the preceding grid's completion and memory before it reads.
template <typename... Args>
cudaError_t launch_glue(void (*fn)(Args...), long long n, cudaStream_t st, Args... args)
{
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3((unsigned)grid_for(n));
    lc.blockDim = dim3(256);
    lc.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    lc.attrs = attr;
    lc.numAttrs = 1;
    return cudaLaunchKernelEx(&lc, fn, args...);
}

}  // namespace
}  // namespace b4

using namespace b4;

extern "C" {

int b4_nccl_get_unique_id(b4_nccl_id* id)
{
    const NcclApi& n = nccl();
    if (!n.ok) return B4_STATUS_NCCL_MISSING;
    if (!id) return cudaErrorInvalidValue;
    static_assert(sizeof(ncclUniqueId) == sizeof(b4_nccl_id), "ncclUniqueId size");
    return nccl_status(n.GetUniqueId(reinterpret_cast<ncclUniqueId*>(id)));
}

int b4_nccl_comm_init(void** comm, int nranks, const b4_nccl_id* id, int rank)
{
    const NcclApi& n = nccl();
    if (!n.ok) return B4_STATUS_NCCL_MISSING;
    if (!comm || !id || nranks < 1 || rank < 0 || rank >= nranks) return cudaErrorInvalidValue;
    ncclUniqueId uid;
    memcpy(&uid, id, sizeof(uid));
    ncclComm_t c = nullptr;
    const int st = nccl_status(n.CommInitRank(&c, nranks, uid, rank));
    *comm = st == 0 ? c : nullptr;
    return st;
}

int b4_nccl_comm_destroy(void* comm)
{
    const NcclApi& n = nccl();
    if (!n.ok) return B4_STATUS_NCCL_MISSING;
    if (!comm) return cudaErrorInvalidValue;
    return nccl_status(n.CommDestroy(static_cast<ncclComm_t>(comm)));
}

int b4_nccl_wait(void* comm, b4_stream_t stream, int timeout_ms)
{
    const NcclApi& n = nccl();
    if (!n.ok) return B4_STATUS_NCCL_MISSING;
    if (!comm) return cudaErrorInvalidValue;
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(timeout_ms);
    for (;;) {
        const cudaError_t q = cudaStreamQuery(reinterpret_cast<cudaStream_t>(stream));
        if (q == cudaSuccess) return 0;
        if (q != cudaErrorNotReady) return q;
        ncclResult_t ar = ncclSuccess;
        n.CommGetAsyncError(static_cast<ncclComm_t>(comm), &ar);
        if (ar != ncclSuccess && ar != ncclInProgress) {
            n.CommAbort(static_cast<ncclComm_t>(comm));
            return nccl_status(ar);
        }
        if (std::chrono::steady_clock::now() > deadline) {
            n.CommAbort(static_cast<ncclComm_t>(comm));
            return B4_STATUS_TIMEOUT;
        }
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

int b4_shard_columns(int fmt, const uint32_t* qw, const void* scale, int in_f, int out_f, int col0,
                     int ncols, uint32_t* qw_out, void* scale_out, b4_stream_t stream)
{
    const int unit = fmt == kInt4 ? kGroup : (fmt == kNf4 ? kNf4Block : 0);
    if (!unit || !qw || !scale || !qw_out || !scale_out || in_f <= 0 || out_f <= 0) return cudaErrorInvalidValue;
    if (col0 < 0 || ncols <= 0 || col0 % unit || ncols % unit || col0 + ncols > in_f || in_f % unit)
        return cudaErrorInvalidValue;
    const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemcpy2DAsync(qw_out, (size_t)ncols / 2, qw + col0 / 8, (size_t)in_f / 2,
                                      (size_t)ncols / 2, out_f, cudaMemcpyDeviceToDevice, st);
    if (e != cudaSuccess) return e;
    const size_t sb = fmt == kInt4 ? 2 : 4;
    e = cudaMemcpy2DAsync(scale_out, (size_t)(ncols / unit) * sb,
                          static_cast<const char*>(scale) + (size_t)(col0 / unit) * sb, (size_t)(in_f / unit) * sb,
                          (size_t)(ncols / unit) * sb, out_f, cudaMemcpyDeviceToDevice, st);
    return e;
}

int b4_tp_gemv_allreduce(int fmt, const uint32_t* qw_shard, const void* scale_shard, const void* x_shard,
                         float* y, int in_shard, int out_f, int m, void* comm, b4_stream_t stream)
{
    const NcclApi& n = nccl();
    if (!n.ok) return B4_STATUS_NCCL_MISSING;
    if (!comm) return cudaErrorInvalidValue;
    const int e = b4_gemv_ex(fmt, qw_shard, scale_shard, x_shard, y, in_shard, out_f, m, nullptr, stream);
    if (e != 0) return e;
    return nccl_status(n.AllReduce(y, y, (size_t)m * out_f, ncclFloat32, ncclSum, static_cast<ncclComm_t>(comm),
                                   reinterpret_cast<cudaStream_t>(stream)));
}

int b4_tp_gemv_allreduce_ws(int fmt, const uint32_t* qw_shard, const void* scale_shard, const void* x_shard,
                            float* y, int in_shard, int out_f, int m, void* ws, size_t ws_bytes, void* comm,
                            b4_stream_t stream)
{
    const NcclApi& n = nccl();
    if (!n.ok) return B4_STATUS_NCCL_MISSING;
    if (!comm) return cudaErrorInvalidValue;
    const int e = b4_gemv_ws(fmt, qw_shard, scale_shard, x_shard, y, in_shard, out_f, m, nullptr, ws, ws_bytes, stream);
    if (e != 0) return e;
    return nccl_status(n.AllReduce(y, y, (size_t)m * out_f, ncclFloat32, ncclSum, static_cast<ncclComm_t>(comm),
                                   reinterpret_cast<cudaStream_t>(stream)));
}

int b4_swiglu_f16(const float* gate, const float* up, void* out, long long n, b4_stream_t stream)
{
    if (!gate || !up || !out || n <= 0) return cudaErrorInvalidValue;
    return launch_glue(swiglu_kernel, n, reinterpret_cast<cudaStream_t>(stream), gate, up, static_cast<__half*>(out),
                       n);
}

int b4_cast_f16(const float* in, void* out, long long n, b4_stream_t stream)
{
    if (!in || !out || n <= 0) return cudaErrorInvalidValue;
    return launch_glue(cast_f16_kernel, n, reinterpret_cast<cudaStream_t>(stream), in, static_cast<__half*>(out), n);
}

const char* b4_nccl_error_string(int status)
{
    if (status == B4_STATUS_NCCL_MISSING) return "libnccl.so.2 not found";
    if (status == B4_STATUS_TIMEOUT) return "timed out (b4_nccl_wait: communicator aborted; b4_p2p: a peer did not arrive)";
    if (status == B4_STATUS_SCRATCH_TOO_SMALL)
        return "the split needs more scratch than the static array holds (B4_STATIC_SCRATCH_BYTES): use b4_gemv_ws";
    const NcclApi& n = nccl();
    if (status > B4_STATUS_NCCL_BASE && status < B4_STATUS_NCCL_BASE + 100 && n.ok)
        return n.GetErrorString((ncclResult_t)(status - B4_STATUS_NCCL_BASE));
    return "unknown status";
}

}  // extern "C"
