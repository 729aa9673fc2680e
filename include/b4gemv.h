/*
 * b4gemv.h -- C ABI of the B200 (sm_100a) fused 4-bit dequantisation GEMV.
 *
 * Drop-in for the GEMV path of QuantumDrizzy/int4-gemv.  The reference has no
 * library: callers include src/kernels.cuh and launch its __global__ functions
 * with <<<>>> on the legacy default stream (src/int4_gemv.cu:56-68).  Each
 * entry point below replaces one of those kernels or host functions, named in
 * its comment, over the SAME buffers: packed codes, fp16 scales / fp32 absmax,
 * fp16 x and fp32 y have identical layouts, so reference-quantised weights drop
 * straight in.
 *
 * Conventions
 *   - Every buffer is owned by the caller.  Device pointers for the GEMV,
 *     dequant and *_device entry points, host pointers for the host quantisers.
 *   - Return value: a cudaError_t value (0 = cudaSuccess).  Bad shapes, null
 *     pointers or an unusable config return cudaErrorInvalidValue (1) before
 *     anything is launched; launch failures return the CUDA error.  Nothing
 *     exits the process (the reference's CUDA_CHECK does, kernels.cuh:13-21).
 *   - in_f must be a positive multiple of 128 (INT4) or 64 (NF4); the
 *     reference silently drops a ragged tail (kernels.cuh:36,101), this ABI
 *     rejects it.
 *   - Work is enqueued on `stream` (NULL = legacy default stream) and returns
 *     without synchronising.  The only host-global state is mutex-guarded
 *     caches of per-device facts (SM count, kernels whose shared-memory limit
 *     was already raised, resident CTAs per kernel, the device address of the
 *     static scratch array of b4_gemv_split_noalloc): any host thread may call
 *     on its own stream concurrently (b4_gemv_split_noalloc's scratch and a
 *     b4_gemv_ws workspace excepted: calls sharing them must not overlap).
 *   - Vector paths need 16-byte (or 8-byte) aligned codes and x; other
 *     alignments fall back to 4-byte loads, never to the CPU.
 */
#ifndef B4GEMV_H
#define B4GEMV_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B4_GROUP 128     /* INT4 columns per fp16 scale   (kernels.cuh:12) */
#define B4_NF4_BLOCK 64  /* NF4 columns per fp32 absmax   (kernels.cuh:85) */

#define B4_FMT_INT4_G128 0
#define B4_FMT_NF4_B64 1

/* 8: a b4_gemv_ws workspace keeps the x-pair table kernel's running counters
 *    in its first 256 bytes (equal, not zero, between calls), and the split
 *    and k-slice workspace sizes include them; the b4_p2p allocation holds
 *    one copy of the call counter per CTA index. */
#define B4_ABI_VERSION 8

/* Same type as cudaStream_t, spelled without the CUDA headers. */
typedef struct CUstream_st* b4_stream_t;

/* Launch geometry of the GEMV kernel.  b4_gemv_default_config() fills it with
 * the dispatch rule's choice; b4_gemv_ex() takes any valid one (the sweeps
 * that fit the rule use it).  One CTA holds warps_k * row_groups warps; warps
 * that share a row group split in_f and reduce through shared memory. */
typedef struct b4_gemv_config {
    int vec_words;     /* packed words per lane load: 1, 2 or 4                */
    int rows_per_warp; /* rows a warp accumulates at once: 1, 2, 4 or 8        */
    int warps_k;       /* warps sharing one row group along in_f: 1..16        */
    int row_groups;    /* row groups per CTA; warps_k * row_groups <= 16       */
    int batch_tile;    /* batch rows per pass over the weights: 1, 2 or 4      */
    int nf4_lut;       /* NF4 code book: 0 warp shuffle, 1 shared memory, 2 pair table */
    int x_tile;        /* columns of x staged in shared memory per pass, 0 = auto */
    int flags;         /* B4_FLAG_* */
    int engine;        /* B4_ENGINE_*: which pipe does the multiply-accumulates   */
    int stages;        /* *_TMA engines: ring stages per warp (3, 4, 6 or 8)      */
    int stage_groups;  /* B4_ENGINE_MMA_TMA: 128-column groups per stage (2, 4, 8) */
    int tile_rows;     /* engines 4, 5, 7: rows of each warp's 16-row MMA block that
                        * carry weights (1..16, 0 = 16); fewer rows per CTA spread
                        * a matrix of few rows evenly over the SMs */
} b4_gemv_config;

/* The dispatch rule picks the launch, as with cfg NULL; only `flags` is read
 * (so a caller can ask for B4_FLAG_PDL without choosing a geometry).  With the
 * rule, a batch whose x does not fit next to the tensor-pipe engines' buffers
 * in shared memory (m * in_f too large, e.g. 18944 columns at m >= 8) runs as
 * launches over chunks of 8, 4 or 2 batch rows, each a full pass over the
 * weights, instead of on the engines that re-read them per batch row. */
#define B4_ENGINE_AUTO (-1)
/* CUDA cores: fp32 FMA (INT4 and NF4).  rows_per_warp 1/2/4/8, batch_tile 1/2/4. */
#define B4_ENGINE_FMA 0
/* Tensor pipe (INT4 only): register-operand MMA, exact fp16 (code-8) and x,
 * fp32 accumulate.  rows_per_warp 16 or 32, batch_tile 8 or 16 (the MMA's N:
 * batch rows ride along for free), vec_words 4, x_tile a multiple of 128. */
#define B4_ENGINE_MMA 1
/* Tensor pipe fed by a per-warp ring of bulk copies (TMA) in shared memory:
 * rows_per_warp 16, batch_tile 8 (m <= 8) or 16 (m <= 16), vec_words 4; the
 * whole of x must fit in shared memory next to the rings.  Persistent grid. */
#define B4_ENGINE_MMA_TMA 2
/* Engine numbers 3 (a CUDA-core NF4 kernel fed by bulk copies) and 4 (the lean
 * INT4 kernel with its codes in registers) are retired: no shape's rule picked
 * them; configs naming them return cudaErrorInvalidValue. */
#define B4_ENGINE_FMA_TMA 3
#define B4_ENGINE_MMA_LEAN 4
/* Tensor pipe, INT4, lean inner loop (batch 1; m = 2..16 with batch rows in
 * the MMA's N): rows_per_warp 16, vec_words 4; the in-flight codes in a
 * per-lane cp.async ring in shared memory; a stage holds `stage_groups`
 * consecutive 128-column groups ((stages, stage_groups) = (4,1), (6,1), (8,1),
 * (3,2), (4,2), (6,2), (2,4) or (3,4); stage_groups must divide in_f/128). */
#define B4_ENGINE_MMA_LEAN_ASYNC 5
/* CUDA cores, NF4, batch 1, lean inner loop fed by a per-lane cp.async ring:
 * rows_per_warp 4 or 8, vec_words 2 or 4, `stages` 4, 6 or 8, nf4_lut 0
 * (warp-shuffle code book) or 2 (replicated pair table in shared memory). */
#define B4_ENGINE_FMA_LEAN 6
/* Tensor pipe, NF4, batch 1, in_f a multiple of 128: the code book as a
 * 32-way replicated table of byte -> (fp16 hi, fp16 lo) pairs, one PRMT and
 * one 8-byte shared load per two codes, MMA on hi and lo into one fp32
 * accumulator, the two NF4 blocks of a 128-column step kept apart by the
 * MMA's N columns; codes and absmax through a register pipeline of depth
 * `stages` (2, 3, 4).  rows_per_warp 16, vec_words 4. */
#define B4_ENGINE_MMA_NF4 7
/* CUDA cores, NF4, batch 1, in_f a multiple of 256, x 4-byte aligned: tables
 * of x-pair products.  A CTA (one per SM) builds, for each column pair
 * (k, k+1) of a 256-column slice of in_f, the 256 fp32 sums
 * NF4[b & 15]*x[k] + NF4[b >> 4]*x[k+1] (one per byte value b), so one 4-byte
 * shared load and one add take a byte (two codes) of a packed row; codes come
 * straight into registers in whole 128-byte lines; the NF4 blocks' sums are
 * scaled by their absmax, and the slices' shares of y are added in y with
 * fp32 atomics after every CTA has zeroed its rows (order of the slice
 * additions varies from run to run).  Needs a workspace (b4_gemv_ws,
 * b4_gemv_multi_ws) of B4_XTAB_WORKSPACE_BYTES: two running counters (the
 * call's arrivals and their running base), equal between calls.  Codes and absmax 16-byte aligned.  row_groups = warps per CTA and
 * stages = batches of 16 rows each warp keeps in flight: (8, 4), (12, 2),
 * (12, 3), (16, 2), (20, 1) or (24, 1); the other fields are ignored. */
#define B4_ENGINE_NF4_XTAB 8
#define B4_XTAB_WORKSPACE_BYTES 256

/* Launch as a programmatic dependent of the previous kernel in the stream:
 * the weight stream starts before the producer of x has finished.  Only x is
 * ordered after the previous kernel; codes and scales may be read while it
 * still runs, so do not set the flag on a launch whose immediately preceding
 * kernel writes this launch's weights. */
#define B4_FLAG_PDL 1
/* Split the work into equal runs of (16-row block, k-step) units per warp,
 * with a deterministic cross-CTA reduction through a workspace; engines
 * B4_ENGINE_MMA_LEAN_ASYNC (INT4: stages x stage_groups ring) and
 * B4_ENGINE_MMA_NF4 (NF4: register pipeline of `stages`), batch 1.  Only
 * b4_gemv_ws takes it (the other entry points reject it). */
#define B4_FLAG_SPLIT 2
/* Batches of 2..16 rows: split the columns into in_f / x_tile slices of
 * x_tile columns (2..4 slices, each a whole number of the engine's k-steps:
 * 128 * stage_groups columns for INT4 on B4_ENGINE_MMA_LEAN_ASYNC, 128 for NF4
 * on B4_ENGINE_MMA_NF4), run them as the segments of one small-batch launch
 * (x staged per slice, so long rows of a whole batch fit in shared memory and
 * row blocks x slices spread over every SM), and sum the slices' partial y in
 * a fixed order in a second launch, which clears them.  Needs a workspace of
 * 256 + slices * m * out_f * 4 bytes; only b4_gemv_ws takes it. */
#define B4_FLAG_KSLICE 8

/* ---- GEMV: y[b][r] = sum_k dequant(W)[r][k] * x[b][k], b < m ----------------
 * qw     : uint32 [out_f][in_f/8] packed codes
 * scales : fp16   [out_f][in_f/128]        absmax : fp32 [out_f][in_f/64]
 * x      : fp16   [m][in_f]                y      : fp32 [m][out_f]
 * fp32 accumulation; y is within 1e-3 max relative error of a double GEMV
 * over the dequantised weights (order of summation differs from the
 * reference's, so y is not bit-identical to it). */

/* Replaces int4_gemv_warp_per_row (kernels.cuh:26-30) and its launch
 * (int4_gemv.cu:40-41,65-67); m > 1 is new. */
int b4_gemv_int4_g128(const uint32_t* qw, const void* scales, const void* x, float* y,
                      int in_f, int out_f, int m, b4_stream_t stream);

/* Replaces nf4_gemv_warp_per_row (kernels.cuh:87-91), nf4_gemv_block_per_row
 * (kernels.cuh:211-215) and the dispatch rule choosing between them
 * (int4_gemv.cu:52-63); m > 1 is new. */
int b4_gemv_nf4_b64(const uint32_t* qw, const float* absmax, const void* x, float* y,
                    int in_f, int out_f, int m, b4_stream_t stream);

/* The dispatch rule (int4_gemv.cu:52-53, refitted for 148 SMs): the config
 * b4_gemv_int4_g128 / b4_gemv_nf4_b64 would use for this shape. */
int b4_gemv_default_config(int fmt, int in_f, int out_f, int m, b4_gemv_config* cfg);

/* Any format with an explicit config: the launch the reference's sweeps make
 * by hand (diag_aspect.cu:54-56,253-256,262-266). */
int b4_gemv_ex(int fmt, const uint32_t* qw, const void* scale, const void* x, float* y,
               int in_f, int out_f, int m, const b4_gemv_config* cfg, b4_stream_t stream);

/* ---- GEMV with a caller-owned workspace --------------------------------------
 * Two kernels need device scratch, which the caller owns:
 *   - at batch 1, NF4 with in_f a multiple of 256 (x 4-byte aligned, codes
 *     and absmax 16-byte aligned) and at least 17.5 MB of weights (5 MB for
 *     rows of 8192 columns or more) runs on the
 *     x-pair table kernel (B4_ENGINE_NF4_XTAB): its CTAs each cover a
 *     256-column slice of in_f, add their shares into y with atomics and
 *     count themselves in on two counters in `ws` first
 *     (B4_XTAB_WORKSPACE_BYTES); smaller NF4 matrices keep the plain rule
 *     (the kernel's ~4 us start-up costs more than it saves there);
 *   - the split path (B4_FLAG_SPLIT) gives every warp of the grid an equal
 *     run of (16-row block, k-step) units and adds a block's pieces through
 *     `ws` (per 16-row block, one arrival counter and the pieces' partial
 *     sums), the warp that completes a block summing its pieces in k order.
 *     Its cross-CTA sum costs ~2 us, and no batch-1 shape measured faster
 *     split than on the tile rule, so the rule never splits; split configs
 *     are taken when passed explicitly.
 * The rule of b4_gemv_ws (b4_gemv_default_config_ws) is the x-pair table
 * kernel where it applies and b4_gemv_default_config's choice elsewhere.
 * Same operands and semantics as b4_gemv_ex; a replacement for
 * b4_gemv_int4_g128 / b4_gemv_nf4_b64 (kernels.cuh:26-30, 87-91).
 *
 * b4_gemv_workspace_size: bytes of workspace the call with these arguments
 * needs on the current device (0 when the config needs none; cfg NULL or
 * B4_ENGINE_AUTO = the rule of b4_gemv_ws).  ws: device memory, 16-byte aligned, at least that
 * size, ZERO-FILLED before its first use (cudaMemset).  Its first
 * B4_XTAB_WORKSPACE_BYTES hold the x-pair table kernel's running counters
 * (left equal by every call); the split and k-slice paths use the bytes after
 * them and leave zero what a later call expects zero (the split path's
 * arrival counters; the k-slice partials are cleared once summed).  So one
 * workspace serves every path, later
 * calls and CUDA-graph replays, as long as it is not cleared or written
 * between calls other than by zero-filling all of it.  Calls that may run at
 * the same time (different streams) need different workspaces.  A workspace that is too small returns
 * cudaErrorInvalidValue before anything is launched. */
int b4_gemv_workspace_size(int fmt, int in_f, int out_f, int m, const b4_gemv_config* cfg, size_t* bytes);
/* The dispatch rule of b4_gemv_ws (cfg NULL): the x-pair table kernel for NF4
 * at batch 1 with in_f % 256 == 0 and at least 17.5 MB of weights (5 MB for
 * in_f >= 8192), b4_gemv_default_config's choice otherwise. */
int b4_gemv_default_config_ws(int fmt, int in_f, int out_f, int m, b4_gemv_config* cfg);
int b4_gemv_ws(int fmt, const uint32_t* qw, const void* scale, const void* x, float* y, int in_f, int out_f,
               int m, const b4_gemv_config* cfg, void* ws, size_t ws_bytes, b4_stream_t stream);

/* ---- Split GEMV without allocation -------------------------------------------
 * No counterpart in the reference (its kernels need no scratch).  For callers
 * that cannot allocate device memory -- a plugin given only its input and
 * output buffers by a framework that owns every allocation, or code whose
 * memory budget is fixed before its first call -- this is b4_gemv_ws's split
 * path (B4_FLAG_SPLIT, batch 1) with the workspace held in the library's own
 * static device array of B4_STATIC_SCRATCH_BYTES (1 MiB), which every GPU that
 * loads the library keeps until the process exits.  It calls no cudaMalloc or
 * cudaFree.  cfg NULL = a split config for the format (INT4: stages x groups
 * chosen by divisibility; NF4: depth 3); a cfg without B4_FLAG_SPLIT is
 * rejected, and so is NF4 with in_f not a multiple of 128 (the NF4 split
 * kernel's k-step; cudaErrorInvalidValue: use b4_gemv_nf4_b64 there).  A
 * shape whose split needs more than the array holds returns
 * B4_STATUS_SCRATCH_TOO_SMALL before anything is launched (b4_gemv_ws and a
 * workspace of b4_gemv_workspace_size bytes handle it).  The first call on a
 * device looks up the array's device address (cudaGetSymbolAddress): make it
 * before any stream capture, and do not use the entry point across
 * cudaDeviceReset (the address is kept for the device's first context).
 * Every call clears the counters it uses with cudaMemsetAsync on `stream`
 * before its kernel.  All calls on a device share the one array: calls that
 * may overlap on the GPU (different streams, unordered threads) race, so
 * serialise them. */
#define B4_STATIC_SCRATCH_BYTES (1u << 20)
#define B4_STATUS_SCRATCH_TOO_SMALL 10902
int b4_gemv_split_noalloc(int fmt, const uint32_t* qw, const void* scale, const void* x, float* y, int in_f,
                          int out_f, const b4_gemv_config* cfg, b4_stream_t stream);

/* ---- Several projections that share x, as one launch ----------------------
 * y_s[b][r] = sum_k dequant(W_s)[r][k] * x[b][k] for every segment s < nseg
 * (1..B4_MAX_SEGMENTS), all with the same in_f: q/k/v of an attention block,
 * or gate/up of an MLP.  At batch 1 with the lean engines this is ONE kernel
 * launch whose row tiles span all segments, so narrow projections (k/v) ride
 * along with a wide one instead of paying their own launch.  No counterpart
 * in the reference, which names fused QKV as the fix for dispatch-bound k/v
 * and leaves it unimplemented (README.md:177-179); it replaces nseg
 * consecutive b4_gemv_int4_g128 / b4_gemv_nf4_b64 calls over the same
 * buffers.  Other engines and m > 1 run one launch per segment.  cfg may be
 * NULL (the dispatch rule over the segments' total rows, which
 * b4_gemv_multi_default_config returns; it reads only qw, scale and out_f of
 * each segment). */
#define B4_MAX_SEGMENTS 4
typedef struct b4_gemv_segment {
    const uint32_t* qw;   /* uint32 [out_f][in_f/8] */
    const void* scale;    /* INT4: fp16 [out_f][in_f/128]; NF4: fp32 [out_f][in_f/64] */
    float* y;             /* fp32 [m][out_f] */
    int out_f;
} b4_gemv_segment;
int b4_gemv_multi(int fmt, const b4_gemv_segment* segs, int nseg, const void* x, int in_f, int m,
                  const b4_gemv_config* cfg, b4_stream_t stream);
int b4_gemv_multi_default_config(int fmt, const b4_gemv_segment* segs, int nseg, int in_f, int m,
                                 b4_gemv_config* cfg);
/* b4_gemv_multi with a caller-owned workspace (conventions of b4_gemv_ws): the
 * same one-launch fusion, and at batch 1 for NF4 with in_f % 256 == 0 and at
 * least 17.5 MB of weights over all segments (5 MB for in_f >= 8192) the
 * x-pair table kernel (ws of B4_XTAB_WORKSPACE_BYTES).  cfg
 * NULL or B4_ENGINE_AUTO = that rule (only cfg->flags' B4_FLAG_PDL is read). */
int b4_gemv_multi_default_config_ws(int fmt, const b4_gemv_segment* segs, int nseg, int in_f, int m,
                                    b4_gemv_config* cfg);
int b4_gemv_multi_ws(int fmt, const b4_gemv_segment* segs, int nseg, const void* x, int in_f, int m,
                     const b4_gemv_config* cfg, void* ws, size_t ws_bytes, b4_stream_t stream);

/* nf4_gemv_block_per_row (kernels.cuh:211-215) with its launch geometry
 * <<<out_f, warps_per_block*32>>> (int4_gemv.cu:56-58): one CTA per row,
 * warps_per_block (1..16) warps split in_f and reduce in shared memory. */
int b4_gemv_nf4_b64_block_per_row(const uint32_t* qw, const float* absmax, const void* x,
                                  float* y, int in_f, int out_f, int warps_per_block,
                                  b4_stream_t stream);

/* ---- Dequantisation: the W_dequant reconstruction, bit-exact --------------
 * w_out fp32 [out_f][in_f] = (code-8)*float(scale) or NF4[code]*absmax: the
 * `deq` output of quantise()/quantise_nf4() (kernels.cuh:290,331). */
int b4_dequant_int4_g128(const uint32_t* qw, const void* scales, float* w_out,
                         int in_f, int out_f, b4_stream_t stream);
int b4_dequant_nf4_b64(const uint32_t* qw, const float* absmax, float* w_out,
                       int in_f, int out_f, b4_stream_t stream);

/* Unpacked codes, one byte per column: codes[r][k] = nibble k%8 of
 * qw[r][k/8] (the packing of kernels.cuh:289,329).  in_f % 8 == 0. */
int b4_unpack_codes(const uint32_t* qw, uint8_t* codes, int in_f, int out_f,
                    b4_stream_t stream);

/* bitsandbytes-layout NF4 codes (two per byte, the lower column in the HIGH
 * nibble, row-major [out_f][in_f/2] bytes) -> this library's packed words
 * (lower column in the LOW nibble, kernels.cuh:329); the swap of the two
 * nibbles of every byte, its own inverse, so the same call converts back.
 * No counterpart in the reference, which packs its own layout on purpose
 * (README.md:180-181).  A non-nested bitsandbytes fp32 absmax ([out_f][in_f/64]
 * for a row-major weight with in_f % 64 == 0) is already this library's absmax
 * layout, and bitsandbytes' NF4 code indices are the same 16 values in the same
 * order (kernels.cuh:64-83), so repacked codes + absmax go straight into
 * b4_gemv_nf4_b64.  Nested (double-quantised) absmax is not handled.
 * in_f % 64 == 0; 4-byte aligned buffers (16-byte for the vector path). */
int b4_repack_bnb_nf4(const void* bnb_packed, uint32_t* qw, int in_f, int out_f, b4_stream_t stream);

/* ---- Quantisers -------------------------------------------------------------
 * Host: quantise() (kernels.cuh:268-297) and quantise_nf4() (kernels.cuh:
 * 308-339), byte-identical output, spread over `nthreads` host threads
 * (<= 0: all online cores).  W fp32 [out_f][in_f]; scales fp16 bits; deq may
 * be NULL. */
int b4_quantise_int4_g128(const float* W, int out_f, int in_f, uint32_t* packed,
                          uint16_t* scales, float* deq, int nthreads);
int b4_quantise_nf4_b64(const float* W, int out_f, int in_f, uint32_t* packed,
                        float* absmax, float* deq, int nthreads);

/* Device: the same two quantisers on the GPU (IEEE division and rounding,
 * byte-identical to the host ones).  Device pointers; deq may be NULL. */
int b4_quantise_int4_g128_device(const float* W, int out_f, int in_f, uint32_t* packed,
                                 void* scales, float* deq, b4_stream_t stream);
int b4_quantise_nf4_b64_device(const float* W, int out_f, int in_f, uint32_t* packed,
                               float* absmax, float* deq, b4_stream_t stream);

/* ---- Tensor-parallel decode layer -------------------------------------------
 * New (the reference has no multi-GPU code, README.md:175).  Column-parallel
 * projections (q/k/v/gate/up) need no entry point: a rank's rows are a
 * contiguous slice of qw/scales, passed to the GEMV as is.  Row-parallel
 * projections (o/down) hold a column shard (b4_shard_columns) and finish with
 * an all-reduce of fp32 y (b4_tp_gemv_allreduce).  NCCL is loaded at run time.
 * Statuses >= B4_STATUS_NCCL_BASE are NCCL results (base + ncclResult_t). */
#define B4_STATUS_NCCL_BASE 10000
#define B4_STATUS_NCCL_MISSING 10900 /* no libnccl.so.2 in the process or on the path */
#define B4_STATUS_TIMEOUT 10901      /* b4_nccl_wait deadline passed (communicator aborted), or a b4_p2p wait gave up */

typedef struct b4_nccl_id { char internal[128]; } b4_nccl_id; /* = ncclUniqueId */

int b4_nccl_get_unique_id(b4_nccl_id* id);
/* ncclCommInitRank; *comm receives the ncclComm_t. */
int b4_nccl_comm_init(void** comm, int nranks, const b4_nccl_id* id, int rank);
int b4_nccl_comm_destroy(void* comm);
/* Host-side failure detection: waits for `stream` with a deadline, polling
 * ncclCommGetAsyncError; on an NCCL error or the deadline it aborts the
 * communicator (ncclCommAbort) and returns the error / B4_STATUS_TIMEOUT. */
int b4_nccl_wait(void* comm, b4_stream_t stream, int timeout_ms);

/* Columns [col0, col0+ncols) of every row of a packed weight (and the matching
 * scales / absmax) into contiguous buffers: qw_out [out_f][ncols/8],
 * scale_out [out_f][ncols/unit], unit = 128 (INT4) or 64 (NF4); col0 and ncols
 * multiples of unit.  Device pointers. */
int b4_shard_columns(int fmt, const uint32_t* qw, const void* scale, int in_f, int out_f, int col0,
                     int ncols, uint32_t* qw_out, void* scale_out, b4_stream_t stream);

/* Row-parallel GEMV: y = this rank's partial (column shard . x_shard), then
 * ncclAllReduce(y, y, m*out_f, fp32, sum) on the same stream. */
int b4_tp_gemv_allreduce(int fmt, const uint32_t* qw_shard, const void* scale_shard, const void* x_shard,
                         float* y, int in_shard, int out_f, int m, void* nccl_comm, b4_stream_t stream);
/* The same with the GEMV through b4_gemv_ws (the rule of b4_gemv_ws, a
 * caller-owned workspace as b4_gemv_ws takes it): NF4 shards with in_shard a
 * multiple of 256 run on the x-pair table kernel. */
int b4_tp_gemv_allreduce_ws(int fmt, const uint32_t* qw_shard, const void* scale_shard, const void* x_shard,
                            float* y, int in_shard, int out_f, int m, void* ws, size_t ws_bytes, void* nccl_comm,
                            b4_stream_t stream);

/* Row-parallel GEMV with the all-reduce fused into its epilogue over NVLink
 * peer memory, no collective library: each warp stores its finished rows into
 * every rank's receive slots (one 64-bit word per row: the call's epoch and
 * the fp32 partial), goes on to its next rows, and after its last rows sums
 * every rank's copy in rank order.  y is bit-identical on every rank.  Waits
 * are bounded: a rank that never arrives makes the others' calls time out,
 * their rows of y are NaN, b4_p2p_status reports B4_STATUS_TIMEOUT, and the
 * GPU stays usable (then destroy and re-create the b4_p2p on every rank: the
 * call counters disagree).  Set-up, once per rank and device: b4_p2p_create
 * (one device allocation of 16 * world * max_rows + 4 * max_rows + 16896 bytes, max_rows >=
 * the out_f of every call), b4_p2p_ipc_handle -> send the 64-byte handle to
 * every peer -> b4_p2p_open_peer for each peer's handle.  One process per GPU
 * (CUDA IPC).  Every rank must make the same sequence of calls; the call
 * counter lives on the device, so calls captured in a CUDA graph may be
 * replayed.  flags: B4_FLAG_PDL (or 0).  Batch 1; INT4, or NF4 with in_shard
 * a multiple of 128 (the NF4 kernel's MMA k-step).  NF4 shards that the
 * x-pair table kernel takes (b4_gemv_default_config_ws) run it into a partial
 * y in the b4_p2p allocation and the same all-reduce as a second launch (y
 * then varies from call to call within fp32 rounding, identically on every
 * rank).  No counterpart in the reference (it has no multi-GPU code). */
typedef struct b4_p2p b4_p2p;
int b4_p2p_create(int rank, int world, int max_rows, b4_p2p** out);
int b4_p2p_ipc_handle(const b4_p2p* p2p, void* handle64);
int b4_p2p_open_peer(b4_p2p* p2p, int peer, const void* handle64);
int b4_p2p_status(b4_p2p* p2p, int clear);   /* B4_STATUS_TIMEOUT if a wait gave up */
int b4_p2p_destroy(b4_p2p* p2p);
int b4_tp_gemv_p2p(int fmt, const uint32_t* qw_shard, const void* scale_shard, const void* x_shard, float* y,
                   int in_shard, int out_f, b4_p2p* p2p, int flags, b4_stream_t stream);
/* b4_tp_gemv_p2p with the decode layer's elementwise glue folded in, so that a
 * layer needs no glue launches on this path:
 *   y16 (optional, NULL = none): y is also written rounded to fp16, as
 *     b4_cast_f16 would write it (the o projection's output, the next GEMV's x);
 *   flags B4_FLAG_X_SWIGLU: x_shard is fp32 [2][in_shard], this rank's gate
 *     rows then its up rows (16-byte aligned), and the GEMV's x is
 *     fp16(silu(gate) * up), computed while x is staged, rounded as
 *     b4_swiglu_f16 rounds it (the down projection after gate/up).
 * y is then bit-identical to the glue launches followed by b4_tp_gemv_p2p. */
#define B4_FLAG_X_SWIGLU 4
int b4_tp_gemv_p2p_ex(int fmt, const uint32_t* qw_shard, const void* scale_shard, const void* x_shard, float* y,
                      void* y16, int in_shard, int out_f, b4_p2p* p2p, int flags, b4_stream_t stream);

/* Elementwise glue of the decode layer: out = fp16(silu(gate) * up) (the MLP
 * activation between gate/up and down) and out = fp16(in).  Launched as
 * programmatic dependents: each waits for the preceding kernel's completion
 * before it reads, and lets the next kernel launch at once. */
int b4_swiglu_f16(const float* gate, const float* up, void* out, long long n, b4_stream_t stream);
int b4_cast_f16(const float* in, void* out, long long n, b4_stream_t stream);
const char* b4_nccl_error_string(int status);

/* Reads (and with clear != 0 resets) the current device's error flags: non-zero
 * after a bounded wait ran out -- 1: a streaming kernel's wait on its copy
 * ring (the kernel then ended early), 2: the x-pair table kernel's count-in
 * (it then carried on without it) -- and that launch's y is not valid.
 * Returns the flags, or -1 if they could not be read. */
int b4_device_error(int clear);

/* ---- Misc -------------------------------------------------------------------
 * One empty kernel launch: the empty-launch floor that bench/baseline.py:71-76
 * measures (there with a 1x1 fp16 matmul) and that bounds the narrow shapes. */
int b4_empty_launch(b4_stream_t stream);

const char* b4_status_string(int status);
int b4_abi_version(void);

#ifdef __cplusplus
}
#endif
#endif /* B4GEMV_H */
