// b4_split_static.cu -- the split batch-1 GEMV (b4_gemv_split.cuh) for callers
// that cannot allocate device memory: its workspace is this file's static
// device array instead of a caller-owned buffer.
//
// Who needs it: code that runs where cudaMalloc is unavailable or forbidden
// -- a plugin handed only its input and output buffers by a host framework
// that owns every allocation (and may forbid cudaMalloc so its own pool and
// memory accounting stay exact), or a caller with a fixed memory budget
// decided before the first call.  The split kernels need scratch (per
// 16-row block: an arrival counter and the pieces' partial sums); here it
// is B4_STATIC_SCRATCH_BYTES of module memory, which every GPU that loads
// the library holds until the process exits.
//
// In host code the array's name is a host-side stand-in, not a device
// address: the entry point looks up the device address with
// cudaGetSymbolAddress once per device (with that device current) and passes
// that pointer to the kernel.  That first call per device should come before
// any stream capture; the cached address belongs to the device's context as
// it was then, so the entry point must not be used across cudaDeviceReset.
// Every call clears the counters it uses (cudaMemsetAsync on its own stream,
// so the clear is ordered before its kernel whatever kind of stream it is)
// and writes every partial sum before reading it, so nothing else needs
// clearing.  It allocates nothing and shares the one array with every other
// call on the device, so calls that may overlap on the GPU (different
// streams, or threads without ordering between them) race.
#include <mutex>

#include "b4_internal.h"

namespace {

static __device__ __align__(256) unsigned char g_split_scratch[B4_STATIC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;

// The array's device address on `dev` (the current device), looked up on the
// first call per device.  No whole-array clear: a synchronous cudaMemset runs
// on the legacy default stream, which a caller's non-blocking stream is not
// ordered after, so it could overlap the first kernel.
cudaError_t scratch_address(int dev, void** out)
{
    static std::mutex mu;
    static void* addr[kMaxDevices] = {};
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_split_scratch);
        if (e != cudaSuccess) return e;
        addr[dev] = p;
    }
    *out = addr[dev];
    return cudaSuccess;
}

// The split config used when the caller passes none: the dispatch rule's
// split config for INT4 (2 stages of 4 groups; 3 of 2 or 6 of 1 where 4 or 2
// groups do not divide the row or the scales' alignment), the register
// pipeline of depth 3 for NF4.
void noalloc_default_config(const b4::GemvProblem& p, b4_gemv_config* c)
{
    *c = b4_gemv_config{};
    c->vec_words = 4;
    c->rows_per_warp = 16;
    c->warps_k = 1;
    c->row_groups = 8;
    c->batch_tile = 1;
    c->flags = B4_FLAG_SPLIT;
    if (p.fmt == B4_FMT_INT4_G128) {
        const int ng = p.in_f / B4_GROUP;
        const uintptr_t sa = reinterpret_cast<uintptr_t>(p.scale);
        c->engine = B4_ENGINE_MMA_LEAN_ASYNC;
        if (ng % 4 == 0 && sa % 8 == 0) {
            c->stages = 2;
            c->stage_groups = 4;
        } else if (ng % 2 == 0 && sa % 4 == 0) {
            c->stages = 3;
            c->stage_groups = 2;
        } else {
            c->stages = 6;
            c->stage_groups = 1;
        }
    } else {
        c->engine = B4_ENGINE_MMA_NF4;
        c->stages = 3;
    }
}

}  // namespace

extern "C" int b4_gemv_split_noalloc(int fmt, const uint32_t* qw, const void* scale, const void* x, float* y,
                                     int in_f, int out_f, const b4_gemv_config* cfg, b4_stream_t stream)
{
    const b4::GemvProblem p{fmt, qw, scale, x, y, in_f, out_f, 1, in_f, out_f};
    int e = b4::check_problem(p);
    if (e != cudaSuccess) return e;
    b4_gemv_config c;
    if (cfg) c = *cfg;
    else noalloc_default_config(p, &c);
    if (!(c.flags & B4_FLAG_SPLIT)) return cudaErrorInvalidValue;
    b4::SplitPlan s;
    e = b4::split_plan(p, c, &s);
    if (e != cudaSuccess) return e;
    if (s.ws_bytes > B4_STATIC_SCRATCH_BYTES) return B4_STATUS_SCRATCH_TOO_SMALL;
    int dev = 0;
    cudaError_t ce = cudaGetDevice(&dev);
    if (ce != cudaSuccess) return ce;
    void* ws = nullptr;
    ce = scratch_address(dev, &ws);
    if (ce != cudaSuccess) return ce;
    const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    // the counters start at zero whatever an earlier (possibly overlapping) call left
    ce = cudaMemsetAsync(ws, 0, s.cnt_bytes, st);
    if (ce != cudaSuccess) return ce;
    return b4::launch_split(p, c, ws, B4_STATIC_SCRATCH_BYTES, st);
}
