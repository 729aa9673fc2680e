// b4_internal.h -- host-side interfaces between the C-ABI layer and the kernels.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "../../include/b4gemv.h"
#include "b4_p2p.cuh"

namespace b4 {

// Everything one GEMV launch needs.  Pointers are device (or managed) memory.
struct GemvProblem {
    int fmt;              // kInt4 / kNf4
    const uint32_t* qw;   // [out_f][in_f/8]
    const void* scale;    // INT4: __half [out_f][in_f/128]; NF4: float [out_f][in_f/64]
    const void* x;        // __half [m][x_ld]
    float* y;             // float [m][y_ld]
    int in_f, out_f, m;
    long long x_ld, y_ld; // leading dimensions (elements) of the batch rows
};

// Shape checks shared by every entry point: returns cudaSuccess or
// cudaErrorInvalidValue.
int check_problem(const GemvProblem& p);

// Fills cfg with the dispatch rule's choice for this problem.
void default_config(const GemvProblem& p, b4_gemv_config* cfg);

// Validates cfg against p (and the pointer alignment it needs) and launches.
int launch_gemv(const GemvProblem& p, const b4_gemv_config& cfg, cudaStream_t st);

// A row-parallel INT4 shard at batch 1 whose epilogue all-reduces y over the
// ranks' peer memory (b4_p2p.cuh); cfg must be a lean INT4 config.
int launch_lean_int4_p2p(const GemvProblem& p, const b4_gemv_config& cfg, const P2pArgs& a, cudaStream_t st);
// ... and an NF4 shard (in_f a multiple of 128) on the tensor-pipe NF4 kernel.
int launch_nf4_mma_p2p(const GemvProblem& p, const P2pArgs& a, int flags, cudaStream_t st);

// Several weight matrices over one x (b4_gemv_multi): the dispatch rule over
// their total rows, and the launch (one kernel for the lean engines at m = 1).
void default_config_multi(int fmt, const b4_gemv_segment* segs, int nseg, int in_f, int m, b4_gemv_config* cfg);
int launch_gemv_multi(int fmt, const b4_gemv_segment* segs, int nseg, const void* x, int in_f, int m,
                      const b4_gemv_config& cfg, cudaStream_t st);

// A split launch (b4_gemv_split.cuh) on the current device: kernel, grid,
// k-steps per row and per warp, piece slots per 16-row block, shared memory
// and the workspace it needs ([cnt_bytes of counters][partial sums]).
struct SplitPlan {
    void* fn;
    long long nblocks, total;
    int nst, per, maxp, grid;
    size_t smem, cnt_bytes, ws_bytes;
};
int split_plan(const GemvProblem& p, const b4_gemv_config& cfg, SplitPlan* plan);

// Launches the split kernel of cfg (B4_FLAG_SPLIT) with the caller's workspace
// (16-byte aligned, at least the plan's ws_bytes, counters zero).
int launch_split(const GemvProblem& p, const b4_gemv_config& cfg, void* ws, size_t ws_bytes, cudaStream_t st);

// The workspace rule: default_config, switched to the x-pair table kernel for
// large NF4 matrices at batch 1 and to column slices (B4_FLAG_KSLICE) for
// small batches of long rows.
void default_config_ws(const GemvProblem& p, b4_gemv_config* cfg);

// An NF4 shard at batch 1 on the x-pair table kernel when the workspace rule
// takes its shape: y = the shard's partial GEMV (x fp16, or fp16(silu(gate) *
// up) of fp32 gate/up rows when xgu is set), ws = the kernel's 256-byte
// counters.  cudaErrorNotSupported when the rule does not take the shape.
int launch_xtab_shard(const GemvProblem& p, const float* xgu, int flags, void* ws, cudaStream_t st);

}  // namespace b4
