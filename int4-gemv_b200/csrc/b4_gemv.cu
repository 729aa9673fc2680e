// b4_gemv.cu -- host side of the GEMV: shape checks, the dispatch rule and the
// launch of b4_gemv_kernel, behind the extern "C" entry points of b4gemv.h.
#include <algorithm>
#include <atomic>
#include <map>
#include <mutex>
#include <utility>

#include "b4_gemv_kernel.cuh"
#include "b4_gemv_mma.cuh"
#include "b4_gemv_tma.cuh"
#include "b4_gemv_lean.cuh"
#include "b4_gemv_lean_mb.cuh"
#include "b4_gemv_lean_nf4.cuh"
#include "b4_gemv_nf4_mma.cuh"
#include "b4_gemv_nf4_mma_mb.cuh"
#include "b4_gemv_split.cuh"
#include "b4_gemv_xtab.cuh"
#include "b4_internal.h"

namespace b4 {

namespace {

constexpr int kMaxWarps = 16;

bool aligned(const void* p, unsigned a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

void* pick_kernel(int fmt, int vw, int rw, int mb, int lut)
{
    if (fmt == kInt4) {
        if (lut != 0) return nullptr;
        switch (vw) {
            case 1: return gemv_kernel_int4_v1(rw, mb, 0);
            case 2: return gemv_kernel_int4_v2(rw, mb, 0);
            case 4: return gemv_kernel_int4_v4(rw, mb, 0);
        }
    } else {
        switch (vw) {
            case 1: return gemv_kernel_nf4_v1(rw, mb, lut);
            case 2: return gemv_kernel_nf4_v2(rw, mb, lut);
            case 4: return gemv_kernel_nf4_v4(rw, mb, lut);
        }
    }
    return nullptr;
}

// Raises a kernel's dynamic shared-memory limit on the current device once
// per (kernel, device, size).  The cache is the only host-side state of the
// library; it is guarded by a mutex and changes no result, so concurrent
// callers stay safe, and a launch inside stream capture makes no attribute
// call after the first eager launch of the same kernel and size.
cudaError_t ensure_smem(const void* fn, int dev, size_t smem)
{
    static std::mutex mu;
    static std::map<std::pair<const void*, int>, size_t> done;
    std::lock_guard<std::mutex> lock(mu);
    size_t& have = done[{fn, dev}];
    if (have >= smem) return cudaSuccess;
    const cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess) have = smem;
    return e;
}

__global__ void empty_kernel() {}

// Largest shared-memory footprint the dispatch rule aims for, so that two
// CTAs fit on one SM.
constexpr int kSmemBudget = 96 * 1024;

}  // namespace

// Shared memory of the streaming kernel: x (whole of in_f, nb batch rows),
// the warps_k reduction scratch, then per-warp rings and mbarriers.
struct TmaLayout {
    size_t ring_offset, bar_offset, total;
};

TmaLayout tma_layout(int nb, int ng, int kw, int rg, int nt, int stages, int kcg)
{
    const size_t x_bytes = (size_t)nb * ng * 256;
    const size_t red_bytes = kw > 1 ? (size_t)rg * kw * nt * 4 * 32 * 4 : 0;
    TmaLayout l;
    l.ring_offset = (x_bytes + red_bytes + 127) / 128 * 128;
    const size_t stage_bytes = 16 * (size_t)(kcg * 64 + 64);
    l.bar_offset = l.ring_offset + (size_t)kw * rg * stages * stage_bytes;
    l.total = l.bar_offset + (size_t)kw * rg * stages * 8;
    return l;
}

// Opt-in shared memory per CTA on B200 (227 KB).
constexpr size_t kTmaSmemLimit = 227 * 1024;

// Shared memory of the lean NF4 kernel: [pair table][x chunks][reduction][rings].
size_t lean_nf4_smem(int in_f, int kw, int rg, int rw, int vw, int depth, int lut)
{
    const int nchunks = in_f / 8 / vw, nsteps = (nchunks + 31) / 32;
    size_t s = lut == 2 ? 256 * 16 * 8 : 0;
    s += (size_t)nsteps * 32 * 2 * vw * 16;
    s += (size_t)((rg * kw * rw * 4 + 15) / 16) * 16;
    s += (size_t)kw * rg * depth * rw * 32 * (4 * vw + 4);
    return s;
}

// Shared memory of the lean INT4 kernel: [x][reduction][rings].
size_t lean_int4_smem(int in_f, int kw, int rg, int stages, int groups)
{
    size_t smem = (size_t)in_f * 2 + (size_t)(rg * kw * 16 + 3) / 4 * 16;
    // per warp: stages x groups x 2 rows x 32 lanes x 16 B
    smem += (size_t)kw * rg * stages * groups * 64 * 16;
    return smem;
}

// Shared memory of the small-batch lean INT4 kernel: [x, m rows][reduction][rings].
size_t lean_int4_mb_smem(int in_f, int m, int kw, int rg, int stages, int groups)
{
    const int nc = m > 8 ? 16 : 8;
    return (size_t)m * xmb_stride(in_f / 8) * 16 + (size_t)rg * kw * 16 * nc * 4 +
           (size_t)kw * rg * stages * groups * 64 * 16;
}

// Shared memory of the NF4 tensor-pipe kernel: [pair table][x][reduction].
size_t nf4_mma_smem(int in_f, int kw, int rg)
{
    return (size_t)kNf4PairTableBytes + (size_t)in_f * 2 + (size_t)(rg * kw * 16 + 3) / 4 * 16;
}

// ... and of its small-batch form: [pair table][x, m rows][reduction].
size_t nf4_mma_mb_smem(int in_f, int m, int kw, int rg)
{
    const int nr = (m + 3) / 4 > 2 ? 16 : ((m + 3) / 4) * 4;
    return (size_t)kNf4PairTableBytes + (size_t)m * xmb_stride(in_f / 8) * 16 + (size_t)rg * kw * 16 * nr * 4;
}

// Rows per 16-row MMA block for the tensor-pipe batch-1 engines: when a
// matrix has fewer than 2*SMs full tiles (rg = 1), spread its rows over just
// under 2*SMs tiles, so no SM carries two tiles while another has one; k/v-
// sized matrices (< 2048 rows) keep full blocks (they are launch-bound).
int even_tile_rows(int out_f, int rg, int sms)
{
    if (rg != 1 || out_f < 2048) return 0;
    const int tr = (out_f + 2 * sms - 1) / (2 * sms);
    return tr >= 16 ? 0 : tr;
}

int check_problem(const GemvProblem& p)
{
    if (p.fmt != kInt4 && p.fmt != kNf4) return cudaErrorInvalidValue;
    if (!p.qw || !p.scale || !p.x || !p.y) return cudaErrorInvalidValue;
    if (p.in_f <= 0 || p.out_f <= 0 || p.m <= 0) return cudaErrorInvalidValue;
    const int unit = p.fmt == kInt4 ? kGroup : kNf4Block;
    if (p.in_f % unit) return cudaErrorInvalidValue;
    if (p.x_ld < p.in_f || p.y_ld < p.out_f) return cudaErrorInvalidValue;
    if (!aligned(p.qw, 4) || !aligned(p.y, 4) || !aligned(p.x, 2)) return cudaErrorInvalidValue;
    if (!aligned(p.scale, p.fmt == kInt4 ? 2 : 4)) return cudaErrorInvalidValue;
    return cudaSuccess;
}

namespace {
int sm_count_cached(int dev);
}

// SMs of the current device (148 on a B200; a partitioned or MPS-limited
// device reports fewer), 148 when no device can be queried (the rule asked for
// on a machine without a GPU).
int current_sms()
{
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        return 148;
    }
    return sm_count_cached(dev);
}

void default_config(const GemvProblem& p, b4_gemv_config* cfg)
{
    const int words = p.in_f / 8;
    const int sms = current_sms();   // the rule's tile counts were fitted on B200 (148 SMs)
    cfg->nf4_lut = 0;
    cfg->x_tile = 0;
    cfg->flags = 0;
    cfg->stages = 4;
    cfg->stage_groups = 4;
    cfg->tile_rows = 0;

    // Batch 1 (fitted on B200 with `b4gemv.diag sweep --pdl` over the Qwen2.5-7B,
    // Llama-3-70B and tensor-parallel shard shapes; the reference's rule was
    // fitted on a 36-SM part, int4_gemv.cu:52-53): the lean kernel with the
    // cp.async ring, CTAs of 8 warps, and the fewest row groups per CTA (a
    // power of two, so warps_k * row_groups = 8) that still gives one tile per
    // CTA with every CTA resident at once (2 per SM).  A tile count just above
    // the resident CTAs costs a second wave for a handful of tiles (Llama-3-70B
    // gate/up had 299 tiles: 34.9 us, now 27.6 us), and several tiles per CTA
    // restart the ring per tile.  Rows longer than 8192 columns on fewer 16-row
    // blocks than resident CTAs use thinner tiles instead (down_proj).
    if (p.m == 1 && p.fmt == kInt4 && aligned(p.qw, 16)) {
        const int ng = p.in_f / kGroup;
        const long long blocks = (p.out_f + 15) / 16;
        int rg = 1;
        while (rg < 8 && (blocks + rg - 1) / rg > 2LL * sms) rg *= 2;
        cfg->vec_words = 4;
        cfg->rows_per_warp = 16;
        cfg->batch_tile = 1;
        cfg->warps_k = 8 / rg;
        cfg->row_groups = rg;
        cfg->tile_rows = p.in_f > 8192 ? even_tile_rows(p.out_f, rg, sms) : 0;
        // two stages of four groups where two CTAs still fit in shared memory
        // (within 2 % of the best ring on every swept shape), else fewer groups
        const int variants[3][2] = {{2, 4}, {3, 2}, {4, 1}};   // (stages, groups per stage)
        for (int pass = 0; pass < 2; ++pass) {
            for (const auto& v : variants) {
                if (ng % v[1] || (v[1] > 1 && !aligned(p.scale, 2u * v[1]))) continue;
                const size_t smem = lean_int4_smem(p.in_f, cfg->warps_k, rg, v[0], v[1]);
                if (smem > (pass == 0 ? kTmaSmemLimit / 2 - 1024 : kTmaSmemLimit)) continue;
                cfg->engine = B4_ENGINE_MMA_LEAN_ASYNC;
                cfg->stages = v[0];
                cfg->stage_groups = v[1];
                return;
            }
        }
    }
    // INT4 at small batch (2..16 rows): the same lean kernel with the batch rows
    // in the MMA's N columns, when x for all rows fits next to the rings.
    // (fitted on B200 for m = 2..16 on gate/down: one CTA per SM's worth of
    // rows per tile, 2 stages of 4 groups up to m = 4, 3 of 2 beyond)
    if (p.m >= 2 && p.m <= 16 && p.fmt == kInt4 && aligned(p.qw, 16)) {
        const int ng = p.in_f / kGroup;
        const int row_groups = (p.out_f + 15) / 16;
        const int rg = std::max(1, std::min(8, (row_groups + sms - 1) / sms));
        const int variants[3][2] = {{p.m <= 4 ? 2 : 3, p.m <= 4 ? 4 : 2}, {3, 2}, {4, 1}};
        for (const auto& v : variants) {
            if (ng % v[1] || (v[1] > 1 && !aligned(p.scale, 2u * v[1]))) continue;
            if (lean_int4_mb_smem(p.in_f, p.m, 8 / rg, rg, v[0], v[1]) > kTmaSmemLimit) continue;
            cfg->engine = B4_ENGINE_MMA_LEAN_ASYNC;
            cfg->vec_words = 4;
            cfg->rows_per_warp = 16;
            cfg->batch_tile = 1;
            cfg->warps_k = 8 / rg;
            cfg->row_groups = rg;
            cfg->tile_rows = even_tile_rows(p.out_f, rg, sms);
            cfg->stages = v[0];
            cfg->stage_groups = v[1];
            return;
        }
    }
    // NF4 at small batch (2..16 rows): the tensor-pipe engine with the batch
    // rows in the MMA's N columns, when x for all rows fits next to the table.
    if (p.m >= 2 && p.m <= 16 && p.fmt == kNf4 && p.in_f % 128 == 0 && aligned(p.qw, 16) && aligned(p.scale, 8)) {
        const int row_groups = (p.out_f + 15) / 16;
        int rg = std::max(1, std::min(8, (row_groups + sms - 1) / sms));
        if (p.m <= 4 && rg == 8) rg = 4;
        if (nf4_mma_mb_smem(p.in_f, p.m, 8 / rg, rg) <= kTmaSmemLimit) {
            cfg->engine = B4_ENGINE_MMA_NF4;
            cfg->vec_words = 4;
            cfg->rows_per_warp = 16;
            cfg->batch_tile = 1;
            cfg->warps_k = 8 / rg;
            cfg->row_groups = rg;
            cfg->tile_rows = 0;
            cfg->stages = p.m <= 4 ? 2 : 3;
            return;
        }
    }
    // NF4 at batch 1, q/o/gate/up-like (in_f < 8192, or 8192 on at most one
    // resident tile per CTA: the tensor-parallel q and gate/up shards, 5 %
    // faster there; at least 2048 rows): the tensor-pipe engine; its 64 KB
    // code-book table costs more than it saves on narrow (k/v) or long-row
    // (down) matrices.
    const bool nf4_mma_shape = p.in_f < 8192 || (p.in_f == 8192 && (p.out_f + 15) / 16 <= 2 * sms);
    if (p.m == 1 && p.fmt == kNf4 && p.in_f % 128 == 0 && nf4_mma_shape && p.out_f >= 2048 && aligned(p.qw, 16) &&
        aligned(p.scale, 8) && nf4_mma_smem(p.in_f, 8, 1) <= kTmaSmemLimit) {
        // the fewest row groups (a power of two) that give one resident tile per CTA
        const long long blocks = (p.out_f + 15) / 16;
        int rg = 1;
        while (rg < 8 && (blocks + rg - 1) / rg > 2LL * sms) rg *= 2;
        cfg->engine = B4_ENGINE_MMA_NF4;
        cfg->vec_words = 4;
        cfg->rows_per_warp = 16;
        cfg->batch_tile = 1;
        cfg->warps_k = 8 / rg;
        cfg->row_groups = rg;
        cfg->tile_rows = 0;   // full 16-row blocks (q_proj 5.3 us with 13-row tiles, 5.2 us without)
        // four row groups (two warps per block): a depth-4 pipeline (gate_proj
        // 14.05 -> 13.75 us); depth 3 otherwise (eight row groups, the fused
        // gate+up launch: the step 59.3 -> 59.8 us at depth 4)
        cfg->stages = rg == 4 ? 4 : 3;
        return;
    }
    if (p.m == 1 && p.fmt == kNf4 && aligned(p.qw, 16) && aligned(p.scale, 4) && words % 4 == 0) {
        // many rows or rows longer than 8192 columns: bigger tiles; rows longer
        // than 8192 columns: the replicated pair-table code book, else the
        // shuffle code book (refitted on B200 PDL chains: Llama-3-70B k/v
        // 1024x8192 7.1 -> 5.2 us and q/o 8192x8192 18.0 -> 17.0 us; Qwen down
        // 3584x18944 and 8192x28672 keep the pair table)
        const bool big = p.out_f >= 8192 || p.in_f > 8192;
        const int vw = p.in_f >= 8192 ? 4 : 2;
        const int lut = p.in_f > 8192 ? 2 : 0;
        const int quads = (p.out_f + 3) / 4;
        const int rg = std::max(1, std::min(8, quads / (big ? sms / 2 : 224)));
        const size_t smem = lean_nf4_smem(p.in_f, 8 / rg, rg, 4, vw, 4, lut);
        if (smem <= kTmaSmemLimit) {
            cfg->engine = B4_ENGINE_FMA_LEAN;
            cfg->vec_words = vw;
            cfg->rows_per_warp = 4;
            cfg->batch_tile = 1;
            cfg->nf4_lut = lut;
            cfg->warps_k = 8 / rg;
            cfg->row_groups = rg;
            cfg->stages = 4;
            return;
        }
    }

    // INT4 with 16-byte aligned codes: multiply-accumulates on the tensor pipe,
    // codes streamed through per-warp bulk-copy rings when x fits next to them.
    if (p.fmt == kInt4 && aligned(p.qw, 16)) {
        const int groups = p.in_f / kGroup;
        const int row_groups = (p.out_f + 15) / 16;
        const int nb = std::min(p.m, 16);
        cfg->vec_words = 4;
        cfg->rows_per_warp = 16;
        cfg->batch_tile = p.m > 8 ? 16 : 8;
        if (p.m <= 16) {
            const int rg = std::max(1, std::min(8, row_groups / sms));
            // largest CTA (8, 4 or 2 warps) whose x + rings fit in shared memory
            for (int warps = 8; warps >= 2; warps /= 2) {
                const int rgw = std::min(rg, warps);
                const int kw = std::max(1, warps / rgw);
                const TmaLayout l = tma_layout(nb, groups, kw, rgw, cfg->batch_tile / 8, 4, 4);
                if (l.total <= kTmaSmemLimit) {
                    cfg->engine = B4_ENGINE_MMA_TMA;
                    cfg->warps_k = kw;
                    cfg->row_groups = rgw;
                    return;
                }
            }
        }
        int kw = 1;
        while (kw < 8 && (long long)row_groups * kw < sms * 16LL && groups >= 2 * (2 * kw)) kw *= 2;
        cfg->engine = B4_ENGINE_MMA;
        cfg->warps_k = kw;
        cfg->row_groups = std::max(1, std::min(8 / kw, row_groups / (2 * sms)));
        return;
    }

    int vw = 1;
    if (aligned(p.qw, 16) && words % 4 == 0) vw = 4;
    else if (aligned(p.qw, 8) && words % 2 == 0) vw = 2;
    const int chunks = words / vw;

    int mb = p.m >= 4 ? 4 : (p.m >= 2 ? 2 : 1);
    if (vw == 1) mb = 1;

    int rw = 4;
    if ((p.out_f + rw - 1) / rw < sms * 8) rw = 2;
    if ((p.out_f + rw - 1) / rw < sms * 8) rw = 1;
    if (vw == 1) rw = rw >= 4 ? 4 : 1;
    if (mb == 4 && rw == 8) rw = 4;

    const int grps = (p.out_f + rw - 1) / rw;
    int kw = 1;
    while (kw < 8 && (long long)grps * kw < sms * 16LL && chunks >= 32 * kw * 2) kw *= 2;
    int rg = std::max(1, 8 / kw);

    cfg->engine = B4_ENGINE_FMA;
    cfg->vec_words = vw;
    cfg->rows_per_warp = rw;
    cfg->warps_k = kw;
    cfg->row_groups = rg;
    cfg->batch_tile = mb;
}

int launch_gemv_mma(const GemvProblem& p, const b4_gemv_config& c, cudaStream_t st);
int launch_gemv_tma(const GemvProblem& p, const b4_gemv_config& c, cudaStream_t st);
int launch_gemv_lean(const GemvProblem& p, const b4_gemv_config& c, cudaStream_t st);
int launch_gemv_lean_nf4(const GemvProblem& p, const b4_gemv_config& c, cudaStream_t st);
int launch_gemv_nf4_mma(const GemvProblem& p, const b4_gemv_config& c, cudaStream_t st);

int launch_gemv(const GemvProblem& p, const b4_gemv_config& c, cudaStream_t st)
{
    if (c.engine == B4_ENGINE_MMA) return launch_gemv_mma(p, c, st);
    if (c.engine == B4_ENGINE_MMA_TMA) return launch_gemv_tma(p, c, st);
    if (c.engine == B4_ENGINE_MMA_LEAN_ASYNC) return launch_gemv_lean(p, c, st);
    if (c.engine == B4_ENGINE_FMA_LEAN) return launch_gemv_lean_nf4(p, c, st);
    if (c.engine == B4_ENGINE_MMA_NF4) return launch_gemv_nf4_mma(p, c, st);
    if (c.engine != B4_ENGINE_FMA) return cudaErrorInvalidValue;
    const int vw = c.vec_words, rw = c.rows_per_warp, kw = c.warps_k, rg = c.row_groups;
    const int mb = c.batch_tile, lut = c.nf4_lut;
    if (kw < 1 || kw > kMaxWarps || rg < 1 || kw * rg > kMaxWarps) return cudaErrorInvalidValue;
    // 16-warp CTAs exist only for the single-row, single-batch variants
    // (MaxThreads in b4_gemv_kernel.cuh).
    if ((rw > 1 || mb > 1) && kw * rg > 8) return cudaErrorInvalidValue;
    const int words = p.in_f / 8;
    if (vw != 1 && vw != 2 && vw != 4) return cudaErrorInvalidValue;
    if (words % vw) return cudaErrorInvalidValue;
    if (!aligned(p.qw, 4u * vw)) return cudaErrorInvalidValue;
    void* fn = pick_kernel(p.fmt, vw, rw, mb, lut);
    if (!fn) return cudaErrorInvalidValue;

    const int chunks = words / vw;
    const int S = x_slots_per_chunk(vw);
    const int cols_per_chunk = 8 * vw;
    int tile_chunks;
    if (c.x_tile > 0) {
        if (c.x_tile % cols_per_chunk) return cudaErrorInvalidValue;
        tile_chunks = std::min(chunks, c.x_tile / cols_per_chunk);
    } else {
        const int budget_chunks = kSmemBudget / (mb * S * 16);
        tile_chunks = std::min(chunks, std::max(32 * kw, budget_chunks / (32 * kw) * (32 * kw)));
    }
    if (tile_chunks < 1) return cudaErrorInvalidValue;

    const size_t smem = (size_t)mb * tile_chunks * S * 16 + (size_t)rg * kw * mb * rw * 4 + 64;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    int smem_max = 0;
    e = cudaDeviceGetAttribute(&smem_max, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e != cudaSuccess) return e;
    if (smem > (size_t)smem_max) return cudaErrorInvalidValue;
    if (smem > 48 * 1024) {
        e = ensure_smem(fn, dev, smem);
        if (e != cudaSuccess) return e;
    }

    KParams kp;
    kp.qw = p.qw;
    kp.scale = p.scale;
    kp.x = static_cast<const __half*>(p.x);
    kp.y = p.y;
    kp.in_f = p.in_f;
    kp.out_f = p.out_f;
    kp.m = p.m;
    kp.x_ld = p.x_ld;
    kp.y_ld = p.y_ld;
    kp.kw = kw;
    kp.rg = rg;
    kp.tile_chunks = tile_chunks;
    const unsigned xa = p.fmt == kInt4 ? 16u : 8u;
    kp.x_vec = aligned(p.x, xa) && ((p.x_ld * 2) % xa == 0);

    const long long rows_per_cta = (long long)rg * rw;
    long long grid = (p.out_f + rows_per_cta - 1) / rows_per_cta;
    if (grid > 0x7fffffffLL) return cudaErrorInvalidValue;

    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3((unsigned)grid);
    lc.blockDim = dim3(32 * kw * rg);
    lc.dynamicSmemBytes = smem;
    lc.stream = st;
    cudaLaunchAttribute attr[1];
    if (c.flags & B4_FLAG_PDL) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        lc.attrs = attr;
        lc.numAttrs = 1;
    }
    void* args[] = {&kp};
    e = cudaLaunchKernelExC(&lc, fn, args);
    return e;
}

namespace {

cudaError_t launch_common(void* fn, const GemvProblem& p, KParams& kp, long long grid, int threads, size_t smem,
                          int flags, cudaStream_t st)
{
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    int smem_max = 0;
    e = cudaDeviceGetAttribute(&smem_max, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e != cudaSuccess) return e;
    if (smem > (size_t)smem_max) return cudaErrorInvalidValue;
    if (smem > 48 * 1024) {
        e = ensure_smem(fn, dev, smem);
        if (e != cudaSuccess) return e;
    }
    if (grid < 1 || grid > 0x7fffffffLL) return cudaErrorInvalidValue;
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3((unsigned)grid);
    lc.blockDim = dim3(threads);
    lc.dynamicSmemBytes = smem;
    lc.stream = st;
    cudaLaunchAttribute attr[1];
    if (flags & B4_FLAG_PDL) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        lc.attrs = attr;
        lc.numAttrs = 1;
    }
    void* args[] = {&kp};
    return cudaLaunchKernelExC(&lc, fn, args);
}

}  // namespace

int launch_gemv_mma(const GemvProblem& p, const b4_gemv_config& c, cudaStream_t st)
{
    if (p.fmt != kInt4) return cudaErrorInvalidValue;
    if (c.vec_words != 4 || (c.rows_per_warp != 16 && c.rows_per_warp != 32)) return cudaErrorInvalidValue;
    if (c.batch_tile != 8 && c.batch_tile != 16) return cudaErrorInvalidValue;
    const int kw = c.warps_k, rg = c.row_groups;
    if (kw < 1 || rg < 1 || kw * rg > 8) return cudaErrorInvalidValue;
    if (!aligned(p.qw, 16)) return cudaErrorInvalidValue;
    const int rt = c.rows_per_warp / 16, nt = c.batch_tile / 8;
    void* fn = gemv_kernel_int4_mma(rt, nt);
    if (!fn) return cudaErrorInvalidValue;
    const int groups = p.in_f / kGroup;
    const int nb_max = std::min(p.m, c.batch_tile);
    int tile_groups;
    if (c.x_tile > 0) {
        if (c.x_tile % kGroup) return cudaErrorInvalidValue;
        tile_groups = std::min(groups, c.x_tile / kGroup);
    } else {
        tile_groups = std::min(groups, std::max(kw, kSmemBudget / (nb_max * 256) / kw * kw));
    }
    if (tile_groups < 1) return cudaErrorInvalidValue;
    const size_t smem = (size_t)nb_max * tile_groups * 256 + (kw > 1 ? (size_t)rg * kw * rt * nt * 4 * 32 * 4 : 0);
    KParams kp;
    kp.qw = p.qw;
    kp.scale = p.scale;
    kp.x = static_cast<const __half*>(p.x);
    kp.y = p.y;
    kp.in_f = p.in_f;
    kp.out_f = p.out_f;
    kp.m = p.m;
    kp.x_ld = p.x_ld;
    kp.y_ld = p.y_ld;
    kp.kw = kw;
    kp.rg = rg;
    kp.tile_chunks = tile_groups;
    kp.x_vec = aligned(p.x, 16) && ((p.x_ld * 2) % 16 == 0);
    const long long rows_per_cta = (long long)rg * c.rows_per_warp;
    const long long grid = (p.out_f + rows_per_cta - 1) / rows_per_cta;
    return launch_common(fn, p, kp, grid, 32 * kw * rg, smem, c.flags, st);
}

namespace {

// Resident CTAs per SM of a kernel at a block size and shared-memory size,
// queried once per (kernel, device, size) under a mutex (the split launches
// size their grid with it on every call).
cudaError_t occupancy_cached(const void* fn, int dev, int threads, size_t smem, int* occ)
{
    static std::mutex mu;
    static std::map<std::pair<std::pair<const void*, int>, std::pair<int, size_t>>, int> done;
    std::lock_guard<std::mutex> lock(mu);
    const auto key = std::make_pair(std::make_pair(fn, dev), std::make_pair(threads, smem));
    const auto it = done.find(key);
    if (it != done.end()) {
        *occ = it->second;
        return cudaSuccess;
    }
    int n = 0;
    const cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, fn, threads, smem);
    if (e != cudaSuccess) return e;
    done[key] = n;
    *occ = n;
    return cudaSuccess;
}

int sm_count_cached(int dev)
{
    static std::atomic<int> cache[64];
    if (dev < 0 || dev >= 64) return 148;
    int n = cache[dev].load(std::memory_order_relaxed);
    if (n == 0) {
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
            cudaGetLastError();   // no device: the rule keeps B200's count
            n = 148;
        }
        cache[dev].store(n, std::memory_order_relaxed);
    }
    return n;
}

}  // namespace

int launch_gemv_tma(const GemvProblem& p, const b4_gemv_config& c, cudaStream_t st)
{
    if (p.fmt != kInt4 || c.vec_words != 4 || c.rows_per_warp != 16) return cudaErrorInvalidValue;
    if (c.batch_tile != 8 && c.batch_tile != 16) return cudaErrorInvalidValue;
    if (p.m > c.batch_tile) return cudaErrorInvalidValue;
    const int kw = c.warps_k, rg = c.row_groups;
    if (kw < 1 || rg < 1 || kw * rg > 8) return cudaErrorInvalidValue;
    if (!aligned(p.qw, 16)) return cudaErrorInvalidValue;
    const int nt = c.batch_tile / 8;
    void* fn = gemv_kernel_int4_tma(nt, c.stages, c.stage_groups);
    if (!fn) return cudaErrorInvalidValue;
    const int ng = p.in_f / kGroup;
    const int nb = std::min(p.m, c.batch_tile);
    const TmaLayout l = tma_layout(nb, ng, kw, rg, nt, c.stages, c.stage_groups);
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    TmaParams tp;
    KParams& kp = tp.k;
    kp.qw = p.qw;
    kp.scale = p.scale;
    kp.x = static_cast<const __half*>(p.x);
    kp.y = p.y;
    kp.in_f = p.in_f;
    kp.out_f = p.out_f;
    kp.m = p.m;
    kp.x_ld = p.x_ld;
    kp.y_ld = p.y_ld;
    kp.kw = kw;
    kp.rg = rg;
    kp.tile_chunks = ng;
    kp.x_vec = aligned(p.x, 16) && ((p.x_ld * 2) % 16 == 0);
    tp.stages_dummy = c.stages;
    tp.ring_offset = (int)l.ring_offset;
    tp.bar_offset = (int)l.bar_offset;
    const long long rows_per_cta = (long long)rg * 16;
    const long long tiles = (p.out_f + rows_per_cta - 1) / rows_per_cta;
    const int per_sm = std::max<int>(1, (int)((228 * 1024) / (l.total + 1024)));
    const long long grid = std::min<long long>(tiles, (long long)sm_count_cached(dev) * per_sm);
    // launch_common takes KParams; the streaming kernel's parameter block is larger
    int smem_max = 0;
    e = cudaDeviceGetAttribute(&smem_max, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e != cudaSuccess) return e;
    if (l.total > (size_t)smem_max) return cudaErrorInvalidValue;
    if (l.total > 48 * 1024) {
        e = ensure_smem(fn, dev, l.total);
        if (e != cudaSuccess) return e;
    }
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3((unsigned)grid);
    lc.blockDim = dim3(32 * kw * rg);
    lc.dynamicSmemBytes = l.total;
    lc.stream = st;
    cudaLaunchAttribute attr[1];
    if (c.flags & B4_FLAG_PDL) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        lc.attrs = attr;
        lc.numAttrs = 1;
    }
    void* args[] = {&tp};
    return cudaLaunchKernelExC(&lc, fn, args);
}

namespace {

// One launch of a streaming kernel whose parameter block is `params`.
cudaError_t launch_persistent(void* fn, void* params, long long tiles, int threads, size_t smem, int flags,
                              cudaStream_t st, bool resident_only = false)
{
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    int smem_max = 0;
    e = cudaDeviceGetAttribute(&smem_max, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e != cudaSuccess) return e;
    if (smem > (size_t)smem_max) return cudaErrorInvalidValue;
    if (smem > 48 * 1024) {
        e = ensure_smem(fn, dev, smem);
        if (e != cudaSuccess) return e;
    }
    const int per_sm = std::max<int>(1, (int)((228 * 1024) / (smem + 1024)));
    long long grid = std::min<long long>(tiles, (long long)sm_count_cached(dev) * per_sm);
    if (resident_only) {
        // every CTA resident at once (registers and threads counted too)
        int occ = 0;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, fn, threads, smem);
        if (e != cudaSuccess) return e;
        grid = std::min<long long>(grid, (long long)sm_count_cached(dev) * occ);
        if (grid > kP2pEpochSlots) return cudaErrorInvalidValue;   // one call-counter copy per CTA
    }
    if (grid < 1) return cudaErrorInvalidValue;
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3((unsigned)grid);
    lc.blockDim = dim3(threads);
    lc.dynamicSmemBytes = smem;
    lc.stream = st;
    cudaLaunchAttribute attr[1];
    if (flags & B4_FLAG_PDL) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        lc.attrs = attr;
        lc.numAttrs = 1;
    }
    void* args[] = {params};
    return cudaLaunchKernelExC(&lc, fn, args);
}

}  // namespace

namespace {

bool lean_geometry_ok(const b4_gemv_config& c) { return c.warps_k >= 1 && c.row_groups >= 1 && c.warps_k * c.row_groups <= 8; }

// Row strides and column slices of a small-batch launch whose segments are
// k slices of one matrix (launch_ksliced); nullptr: segments are whole
// matrices sharing x.
struct MbSlices {
    int ld_words, ld_scales, x_ld;
    int xoff[kLeanMaxSeg];
};

template <typename MP>
void set_mb_slices(MP& mp, const MbSlices* sl, int in_f, int scales_per_row)
{
    mp.ld_words = sl ? sl->ld_words : in_f / 8;
    mp.ld_scales = sl ? sl->ld_scales : scales_per_row;
    mp.x_ld = sl ? sl->x_ld : in_f;
    for (int s = 0; s < kLeanMaxSeg; ++s) mp.xoff[s] = sl ? sl->xoff[s] : 0;
}

// One launch of the lean INT4 kernel over nseg weight matrices sharing x
// (m = 1; m = 2..16 with the cp.async ring: the small-batch kernel).
int launch_lean_int4_segs(const b4_gemv_segment* segs, int nseg, const void* x, int in_f, int m,
                          const b4_gemv_config& c, cudaStream_t st, const MbSlices* sl = nullptr)
{
    // CTAs of 16 warps: batches of 9..16 rows on the 4-stage single-group ring
    const bool wide = c.warps_k >= 1 && c.row_groups >= 1 && c.warps_k * c.row_groups == 16;
    if (wide && (m < 9 || c.stages != 4 || c.stage_groups != 1)) return cudaErrorInvalidValue;
    if (m < 1 || m > 16 || c.vec_words != 4 || c.rows_per_warp != 16 || (!wide && !lean_geometry_ok(c)))
        return cudaErrorInvalidValue;
    if (m > 1 && c.engine != B4_ENGINE_MMA_LEAN_ASYNC) return cudaErrorInvalidValue;
    if (nseg < 1 || nseg > kLeanMaxSeg) return cudaErrorInvalidValue;
    const int kw = c.warps_k, rg = c.row_groups;
    if (c.engine != B4_ENGINE_MMA_LEAN_ASYNC) return cudaErrorInvalidValue;
    const int groups = c.stage_groups;
    if (groups != 1 && groups != 2 && groups != 4) return cudaErrorInvalidValue;
    if ((in_f / kGroup) % groups) return cudaErrorInvalidValue;   // a stage of `groups` groups tiles the row
    const int nb = m > 8 ? 2 : 1;
    void* fn = m == 1 ? gemv_kernel_int4_lean(c.stages, groups)
                      : gemv_kernel_int4_lean_mb(c.stages, groups, nb, wide, sl ? 1 : 0);
    if (!fn) return cudaErrorInvalidValue;
    const int tr = c.tile_rows ? c.tile_rows : 16;
    if (tr < 1 || tr > 16) return cudaErrorInvalidValue;
    LeanParams lp = {};
    const long long rows_per_cta = (long long)rg * tr;
    long long tiles = 0;
    for (int s = 0; s < nseg; ++s) {
        // a stage's scales are one load of `groups` fp16 per row
        if (!aligned(segs[s].qw, 16) || !aligned(segs[s].scale, 2u * groups)) return cudaErrorInvalidValue;
        tiles += (segs[s].out_f + rows_per_cta - 1) / rows_per_cta;
        if (tiles > INT32_MAX) return cudaErrorInvalidValue;
        lp.seg[s].qw = segs[s].qw;
        lp.seg[s].scale = static_cast<const __half*>(segs[s].scale);
        lp.seg[s].y = segs[s].y;
        lp.seg[s].out_f = segs[s].out_f;
        lp.seg[s].tile_end = (int)tiles;
    }
    lp.nseg = nseg;
    lp.n_tiles = (int)tiles;
    lp.x = static_cast<const __half*>(x);
    lp.in_f = in_f;
    lp.kw = kw;
    lp.rg = rg;
    lp.tr = tr;
    lp.x_vec = aligned(x, 16);
    if (m > 1) {
        LeanMbParams mp;
        mp.base = lp;
        mp.m = m;
        set_mb_slices(mp, sl, in_f, in_f / kGroup);
        const size_t smem = lean_int4_mb_smem(in_f, m, kw, rg, c.stages, groups);
        return launch_persistent(fn, &mp, tiles, 32 * kw * rg, smem, c.flags, st);
    }
    if (sl) return cudaErrorInvalidValue;
    const size_t smem = lean_int4_smem(in_f, kw, rg, c.stages, groups);
    return launch_persistent(fn, &lp, tiles, 32 * kw * rg, smem, c.flags, st);
}

// One launch of the lean NF4 kernel over nseg weight matrices sharing x.
int launch_lean_nf4_segs(const b4_gemv_segment* segs, int nseg, const void* x, int in_f, int m,
                         const b4_gemv_config& c, cudaStream_t st)
{
    if (m != 1 || !lean_geometry_ok(c)) return cudaErrorInvalidValue;
    if (nseg < 1 || nseg > kLeanMaxSeg) return cudaErrorInvalidValue;
    const int kw = c.warps_k, rg = c.row_groups, rw = c.rows_per_warp, vw = c.vec_words;
    if ((vw != 2 && vw != 4) || (in_f / 8) % vw) return cudaErrorInvalidValue;
    void* fn = gemv_kernel_nf4_lean(c.stages, rw, vw, c.nf4_lut);
    if (!fn) return cudaErrorInvalidValue;
    LeanNf4Params lp = {};
    const long long rows_per_cta = (long long)rg * rw;
    long long tiles = 0;
    for (int s = 0; s < nseg; ++s) {
        if (!aligned(segs[s].qw, 4u * vw) || !aligned(segs[s].scale, 4)) return cudaErrorInvalidValue;
        tiles += (segs[s].out_f + rows_per_cta - 1) / rows_per_cta;
        if (tiles > INT32_MAX) return cudaErrorInvalidValue;
        lp.seg[s].qw = segs[s].qw;
        lp.seg[s].absmax = static_cast<const float*>(segs[s].scale);
        lp.seg[s].y = segs[s].y;
        lp.seg[s].out_f = segs[s].out_f;
        lp.seg[s].tile_end = (int)tiles;
    }
    lp.nseg = nseg;
    lp.n_tiles = (int)tiles;
    lp.x = static_cast<const __half*>(x);
    lp.in_f = in_f;
    lp.kw = kw;
    lp.rg = rg;
    lp.x_vec = aligned(x, 8);
    const size_t smem = lean_nf4_smem(in_f, kw, rg, rw, vw, c.stages, c.nf4_lut);
    return launch_persistent(fn, &lp, tiles, 32 * kw * rg, smem, c.flags, st);
}

// One launch of the NF4 tensor-pipe kernel over nseg weight matrices sharing x.
int launch_nf4_mma_segs(const b4_gemv_segment* segs, int nseg, const void* x, int in_f, int m,
                        const b4_gemv_config& c, cudaStream_t st, const MbSlices* sl = nullptr)
{
    if (m < 1 || m > 16 || c.vec_words != 4 || c.rows_per_warp != 16 || !lean_geometry_ok(c))
        return cudaErrorInvalidValue;
    if (nseg < 1 || nseg > kLeanMaxSeg || in_f % 128) return cudaErrorInvalidValue;
    const int nb = (m + 3) / 4 > 2 ? 4 : (m + 3) / 4;   // 8-column MMA blocks of 4 batch rows
    void* fn = m == 1 ? gemv_kernel_nf4_mma(c.stages) : gemv_kernel_nf4_mma_mb(c.stages, nb, sl ? 1 : 0);
    if (!fn) return cudaErrorInvalidValue;
    const int kw = c.warps_k, rg = c.row_groups;
    const int tr = c.tile_rows ? c.tile_rows : 16;
    if (tr < 1 || tr > 16) return cudaErrorInvalidValue;
    LeanNf4Params lp = {};
    const long long rows_per_cta = (long long)rg * tr;
    long long tiles = 0;
    for (int s = 0; s < nseg; ++s) {
        // 16-byte code loads, 8-byte absmax loads (two blocks per step)
        if (!aligned(segs[s].qw, 16) || !aligned(segs[s].scale, 8)) return cudaErrorInvalidValue;
        tiles += (segs[s].out_f + rows_per_cta - 1) / rows_per_cta;
        if (tiles > INT32_MAX) return cudaErrorInvalidValue;
        lp.seg[s].qw = segs[s].qw;
        lp.seg[s].absmax = static_cast<const float*>(segs[s].scale);
        lp.seg[s].y = segs[s].y;
        lp.seg[s].out_f = segs[s].out_f;
        lp.seg[s].tile_end = (int)tiles;
    }
    lp.nseg = nseg;
    lp.n_tiles = (int)tiles;
    lp.x = static_cast<const __half*>(x);
    lp.in_f = in_f;
    lp.kw = kw;
    lp.rg = rg;
    lp.tr = tr;
    lp.x_vec = aligned(x, 16);
    if (m > 1) {
        Nf4MmaMbParams mp;
        mp.base = lp;
        mp.m = m;
        set_mb_slices(mp, sl, in_f, in_f / kNf4Block);
        const size_t smem = nf4_mma_mb_smem(in_f, m, kw, rg);
        return launch_persistent(fn, &mp, tiles, 32 * kw * rg, smem, c.flags, st);
    }
    if (sl) return cudaErrorInvalidValue;
    const size_t smem = nf4_mma_smem(in_f, kw, rg);
    return launch_persistent(fn, &lp, tiles, 32 * kw * rg, smem, c.flags, st);
}

}  // namespace

// A row-parallel INT4 shard at batch 1 with the peer-memory all-reduce fused
// into the epilogue (b4_p2p.cuh): the lean kernel's P2P variant.
int launch_lean_int4_p2p(const GemvProblem& p, const b4_gemv_config& c, const P2pArgs& a, cudaStream_t st)
{
    if (p.fmt != kInt4 || p.m != 1 || c.vec_words != 4 || c.rows_per_warp != 16 || !lean_geometry_ok(c))
        return cudaErrorInvalidValue;
    if (c.engine != B4_ENGINE_MMA_LEAN_ASYNC) return cudaErrorInvalidValue;
    const int kw = c.warps_k, rg = c.row_groups;
    const int groups = c.stage_groups;
    if (groups != 1 && groups != 2 && groups != 4) return cudaErrorInvalidValue;
    if ((p.in_f / kGroup) % groups) return cudaErrorInvalidValue;
    if (!aligned(p.qw, 16) || !aligned(p.scale, 2u * groups)) return cudaErrorInvalidValue;
    void* fn = gemv_kernel_int4_lean_p2p(c.stages, groups);
    if (!fn) return cudaErrorInvalidValue;
    const int tr = c.tile_rows ? c.tile_rows : 16;
    if (tr < 1 || tr > 16) return cudaErrorInvalidValue;
    const long long rows_per_cta = (long long)rg * tr;
    const long long tiles = (p.out_f + rows_per_cta - 1) / rows_per_cta;
    if (p.out_f > a.max_rows) return cudaErrorInvalidValue;
    LeanParams lp = {};
    lp.seg[0].qw = p.qw;
    lp.seg[0].scale = static_cast<const __half*>(p.scale);
    lp.seg[0].y = p.y;
    lp.seg[0].out_f = p.out_f;
    lp.seg[0].tile_end = (int)tiles;
    lp.nseg = 1;
    lp.n_tiles = (int)tiles;
    lp.x = static_cast<const __half*>(p.x);
    lp.in_f = p.in_f;
    lp.kw = kw;
    lp.rg = rg;
    lp.tr = tr;
    lp.x_vec = aligned(p.x, 16);
    lp.p2p = a;
    const size_t smem = lean_int4_smem(p.in_f, kw, rg, c.stages, groups);
    // a CTA waits only for the CTA of the same index on every peer, so with
    // every CTA resident no wait can depend on a CTA that is not running
    return launch_persistent(fn, &lp, tiles, 32 * kw * rg, smem, c.flags, st, true);
}

// A row-parallel NF4 shard at batch 1 with the peer-memory all-reduce fused
// into the epilogue: the tensor-pipe NF4 kernel's P2P variant.  Geometry: the
// dispatch rule's when it picks this kernel (so each rank's partial sums are
// the plain GEMV's, bit for bit), else 8 warps per CTA, the fewest
// power-of-two row groups whose tiles fit two resident CTAs per SM, depth 3.
int launch_nf4_mma_p2p(const GemvProblem& p, const P2pArgs& a, int flags, cudaStream_t st)
{
    if (p.fmt != kNf4 || p.m != 1 || p.in_f % 128) return cudaErrorInvalidValue;
    if (!aligned(p.qw, 16) || !aligned(p.scale, 8)) return cudaErrorInvalidValue;
    if (p.out_f > a.max_rows) return cudaErrorInvalidValue;
    int dev = 0;
    const cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    b4_gemv_config c;
    default_config(p, &c);
    int kw, rg, tr, depth;
    if (c.engine == B4_ENGINE_MMA_NF4 && gemv_kernel_nf4_mma_p2p(c.stages)) {
        kw = c.warps_k;
        rg = c.row_groups;
        tr = c.tile_rows ? c.tile_rows : 16;
        depth = c.stages;
    } else {
        const long long blocks = (p.out_f + 15) / 16, cap = 2LL * sm_count_cached(dev);
        rg = 1;
        while (rg < 8 && (blocks + rg - 1) / rg > cap) rg *= 2;
        kw = 8 / rg;
        tr = 16;
        depth = 3;
    }
    if (kw * rg > 8 || tr < 1 || tr > 16) return cudaErrorInvalidValue;
    if (nf4_mma_smem(p.in_f, kw, rg) > kTmaSmemLimit) return cudaErrorInvalidValue;
    void* fn = gemv_kernel_nf4_mma_p2p(depth);
    if (!fn) return cudaErrorInvalidValue;
    const long long rows_per_cta = (long long)rg * tr;
    const long long tiles = (p.out_f + rows_per_cta - 1) / rows_per_cta;
    LeanNf4Params lp = {};
    lp.seg[0].qw = p.qw;
    lp.seg[0].absmax = static_cast<const float*>(p.scale);
    lp.seg[0].y = p.y;
    lp.seg[0].out_f = p.out_f;
    lp.seg[0].tile_end = (int)tiles;
    lp.nseg = 1;
    lp.n_tiles = (int)tiles;
    lp.x = static_cast<const __half*>(p.x);
    lp.in_f = p.in_f;
    lp.kw = kw;
    lp.rg = rg;
    lp.tr = tr;
    lp.x_vec = aligned(p.x, 16);
    lp.p2p = a;
    // every CTA resident at once: a CTA waits only for the CTA of the same index on the peers
    return launch_persistent(fn, &lp, tiles, 32 * kw * rg, nf4_mma_smem(p.in_f, kw, rg), flags, st, true);
}

int launch_gemv_nf4_mma(const GemvProblem& p, const b4_gemv_config& c, cudaStream_t st)
{
    if (p.fmt != kNf4) return cudaErrorInvalidValue;
    const b4_gemv_segment s{p.qw, p.scale, p.y, p.out_f};
    return launch_nf4_mma_segs(&s, 1, p.x, p.in_f, p.m, c, st);
}

int launch_gemv_lean(const GemvProblem& p, const b4_gemv_config& c, cudaStream_t st)
{
    if (p.fmt != kInt4) return cudaErrorInvalidValue;
    const b4_gemv_segment s{p.qw, p.scale, p.y, p.out_f};
    return launch_lean_int4_segs(&s, 1, p.x, p.in_f, p.m, c, st);
}

int launch_gemv_lean_nf4(const GemvProblem& p, const b4_gemv_config& c, cudaStream_t st)
{
    if (p.fmt != kNf4) return cudaErrorInvalidValue;
    const b4_gemv_segment s{p.qw, p.scale, p.y, p.out_f};
    return launch_lean_nf4_segs(&s, 1, p.x, p.in_f, p.m, c, st);
}

void default_config_multi(int fmt, const b4_gemv_segment* segs, int nseg, int in_f, int m, b4_gemv_config* cfg)
{
    // the rule over the total rows, with the alignment every segment offers
    long long rows = 0;
    bool qw16 = true, sc4 = true;
    for (int s = 0; s < nseg; ++s) {
        rows += segs[s].out_f;
        qw16 = qw16 && aligned(segs[s].qw, 16);
        sc4 = sc4 && aligned(segs[s].scale, 4);
    }
    const int total = (int)std::min<long long>(rows, INT32_MAX);
    GemvProblem p{fmt, reinterpret_cast<const uint32_t*>(qw16 ? 256 : 4),
                  reinterpret_cast<const void*>(sc4 ? 256 : 2), reinterpret_cast<const void*>(256),
                  reinterpret_cast<float*>(256), in_f, total, m, in_f, total};
    default_config(p, cfg);
}

int launch_gemv_multi(int fmt, const b4_gemv_segment* segs, int nseg, const void* x, int in_f, int m,
                      const b4_gemv_config& c, cudaStream_t st)
{
    if (fmt == kInt4 && m <= 16 && c.engine == B4_ENGINE_MMA_LEAN_ASYNC)
        return launch_lean_int4_segs(segs, nseg, x, in_f, m, c, st);
    if (m == 1 && fmt == kNf4 && c.engine == B4_ENGINE_FMA_LEAN)
        return launch_lean_nf4_segs(segs, nseg, x, in_f, m, c, st);
    if (m <= 16 && fmt == kNf4 && c.engine == B4_ENGINE_MMA_NF4)
        return launch_nf4_mma_segs(segs, nseg, x, in_f, m, c, st);
    // the other engines: one launch per segment with this config
    for (int s = 0; s < nseg; ++s) {
        const GemvProblem p{fmt, segs[s].qw, segs[s].scale, x, segs[s].y, in_f, segs[s].out_f, m, in_f,
                            segs[s].out_f};
        const int e = launch_gemv(p, c, st);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

// ---- k-sliced small batches ----------------------------------------------------

// y[i] = part[0][i] + ... + part[S - 1][i] (fixed order), as a programmatic
// dependent of the sliced GEMV; the partials are zeroed once read, so the
// workspace is left as b4_gemv_ws found it.
__global__ void slice_sum_kernel(float* __restrict__ part, float* __restrict__ y, long long n, int S)
{
    asm volatile("griddepcontrol.launch_dependents;");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        float t = part[i];
        for (int s = 1; s < S; ++s) t += part[(long long)s * n + i];
        y[i] = t;
        for (int s = 0; s < S; ++s) part[(long long)s * n + i] = 0.0f;
    }
}

bool ksliced_shape(const GemvProblem& p, const b4_gemv_config& c, int* slices)
{
    const int sw = c.x_tile;
    if (p.m < 2 || p.m > 16 || sw <= 0 || p.in_f % sw) return false;
    const int S = p.in_f / sw;
    if (S < 2 || S > kLeanMaxSeg) return false;
    if (p.fmt == kInt4) {
        if (c.engine != B4_ENGINE_MMA_LEAN_ASYNC || c.stage_groups < 1 || sw % (kGroup * c.stage_groups)) return false;
    } else if (c.engine != B4_ENGINE_MMA_NF4 || sw % 128) {
        return false;
    }
    *slices = S;
    return true;
}

size_t ksliced_ws_bytes(const GemvProblem& p, int slices) { return (size_t)slices * p.m * p.out_f * sizeof(float); }

// The batch's GEMV as `slices` column slices of x_tile columns, one segment
// each in one launch of the small-batch kernel (x staged per slice, so a
// batch of long rows fits in shared memory and the row blocks times slices
// spread over every SM), each slice's partial y in the workspace; a second
// launch sums the slices in order into y.
int launch_ksliced(const GemvProblem& p, const b4_gemv_config& c, void* ws, size_t ws_bytes, cudaStream_t st)
{
    int S = 0;
    if (!ksliced_shape(p, c, &S)) return cudaErrorInvalidValue;
    if (!ws || !aligned(ws, 16) || ws_bytes < ksliced_ws_bytes(p, S)) return cudaErrorInvalidValue;
    const int sw = c.x_tile;
    float* part = static_cast<float*>(ws);
    const long long n = (long long)p.m * p.out_f;
    b4_gemv_segment segs[kLeanMaxSeg];
    MbSlices sl = {};
    sl.ld_words = p.in_f / 8;
    if (p.x_ld % 8) return cudaErrorInvalidValue;
    sl.x_ld = (int)p.x_ld;
    for (int s = 0; s < S; ++s) {
        segs[s].qw = p.qw + (size_t)s * sw / 8;
        segs[s].scale = p.fmt == kInt4
                            ? static_cast<const void*>(static_cast<const __half*>(p.scale) + (size_t)s * sw / kGroup)
                            : static_cast<const void*>(static_cast<const float*>(p.scale) + (size_t)s * sw / kNf4Block);
        segs[s].y = part + (size_t)s * n;
        segs[s].out_f = p.out_f;
        sl.xoff[s] = s * sw;
    }
    b4_gemv_config k = c;
    k.flags &= B4_FLAG_PDL;
    int e;
    if (p.fmt == kInt4) {
        sl.ld_scales = p.in_f / kGroup;
        e = launch_lean_int4_segs(segs, S, p.x, sw, p.m, k, st, &sl);
    } else {
        sl.ld_scales = p.in_f / kNf4Block;
        e = launch_nf4_mma_segs(segs, S, p.x, sw, p.m, k, st, &sl);
    }
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3((unsigned)std::min<long long>((n + 255) / 256, 1184));
    lc.blockDim = dim3(256);
    lc.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    lc.attrs = attr;
    lc.numAttrs = 1;
    return cudaLaunchKernelEx(&lc, slice_sum_kernel, part, p.y, n, S);
}

// ---- x-pair table NF4 launches (b4_gemv_xtab.cuh) --------------------------------

bool xtab_shape(int fmt, int in_f, int m, const void* x)
{
    return fmt == kNf4 && m == 1 && in_f % kXtabCols == 0 && aligned(x, 4);
}

// codes and absmax are copied in 16-byte pieces
bool xtab_buffers(const b4_gemv_segment* segs, int nseg)
{
    for (int s = 0; s < nseg; ++s)
        if (!aligned(segs[s].qw, 16) || !aligned(segs[s].scale, 16)) return false;
    return true;
}

// The work split of the x-pair table kernel (xtab_item) for S slices of nb
// batches over G CTAs.  The even split gives G % S slices one CTA more than
// the others, whose CTAs then carry up to nb / (G / S) batches; the split into
// G / S main CTAs per slice (one item each) and G % S tail CTAs that share
// every slice's last `tail` batches in equal runs evens that out, at the cost
// of a barrier, an x load and a table build for each further slice a tail
// CTA's run touches (item_cost batches each).  The busiest CTA is counted
// exactly for every tail; the tail split is taken where it beats the even
// split by 3 %.  Returns tail (0: the even split), cached per shape.
// A further item's cost in batches, fitted on B200 over the Qwen2.5-7B and
// Llama-3-70B (tp 1, 2, 4, 8) NF4 shapes with values from 15 to 90: 45 was
// the best overall, 40 and 50 each lost up to 5 % on some shape (with 45:
// Llama-3-70B gate/up 59.4 -> 53.4 us, down 35.9 -> 31.0, tp 2 gate/up
// 32.0 -> 29.1, tp 2 down 20.4 -> 18.6).
constexpr int kXtabItemCost = 45;

int xtab_tail(int S, int nb, int G, int item_cost)
{
    if (S > G || G % S == 0 || nb < 2) return 0;
    static std::mutex mu;
    static std::map<std::pair<std::pair<int, int>, std::pair<int, int>>, int> done;
    const auto key = std::make_pair(std::make_pair(S, nb), std::make_pair(G, item_cost));
    std::lock_guard<std::mutex> lock(mu);
    const auto it = done.find(key);
    if (it != done.end()) return it->second;
    const int k = G / S, E = G - k * S;
    const long long even = (nb + k - 1) / k;
    long long best = even;
    int best_r = 0;
    for (int r = 1; r <= nb - k; ++r) {
        long long worst = (nb - r + k - 1) / k;   // a main CTA
        const long long T = (long long)S * r;
        for (int e = 0; e < E && worst < best; ++e) {
            const long long lo = e * T / E, hi = (e + 1) * T / E;
            if (hi <= lo) continue;
            const long long items = (hi - 1) / r - lo / r + 1;
            worst = std::max(worst, hi - lo + item_cost * (items - 1));
        }
        if (worst < best) {
            best = worst;
            best_r = r;
        }
    }
    const int tail = 100 * best < 97 * even ? best_r : 0;
    done[key] = tail;
    return tail;
}

// One launch of the x-pair table NF4 kernel over nseg weight matrices sharing
// x (batch 1): one CTA per SM, all resident at once (the start-of-kernel
// count-in waits for every CTA), the workspace's first 8 bytes as its two
// running counters (equal between calls; zero-filled before the first).
int launch_xtab_segs(const b4_gemv_segment* segs, int nseg, const void* x, int in_f, const b4_gemv_config& c,
                     void* ws, size_t ws_bytes, cudaStream_t st, const float* xgu)
{
    if (nseg < 1 || nseg > kXtabMaxSeg || !xtab_shape(kNf4, in_f, 1, x) || !xtab_buffers(segs, nseg))
        return cudaErrorInvalidValue;
    if (!ws || !aligned(ws, 16) || ws_bytes < B4_XTAB_WORKSPACE_BYTES) return cudaErrorInvalidValue;
    const int nw = c.row_groups;   // warps per CTA; c.stages = batches each warp keeps in flight
    void* fn = gemv_kernel_xtab(nw, c.stages);
    if (!fn) return cudaErrorInvalidValue;
    XtabParams xp = {};
    long long nb = 0;
    for (int s = 0; s < nseg; ++s) {
        nb += (segs[s].out_f + kXtabBatch - 1) / kXtabBatch;
        if (nb > INT32_MAX / kXtabBatch) return cudaErrorInvalidValue;
        xp.seg[s].qw = segs[s].qw;
        xp.seg[s].absmax = static_cast<const float*>(segs[s].scale);
        xp.seg[s].y = segs[s].y;
        xp.seg[s].out_f = segs[s].out_f;
        xp.seg[s].batch_end = (int)nb;
    }
    xp.nseg = nseg;
    xp.nbatch = (int)nb;
    xp.in_f = in_f;
    xp.nslice = in_f / kXtabCols;
    xp.x = static_cast<const __half*>(x);
    xp.bar = static_cast<unsigned*>(ws);
    xp.xgu = xgu;
    if (xgu && !aligned(xgu, 16)) return cudaErrorInvalidValue;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    int reserved = 0;   // dynamic shared memory starts after the reserved part of the window
    e = cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev);
    if (e != cudaSuccess) return e;
    const size_t smem = xtab_smem_bytes((uint32_t)reserved);
    int smem_max = 0;
    e = cudaDeviceGetAttribute(&smem_max, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e != cudaSuccess) return e;
    if (smem > (size_t)smem_max) return cudaErrorInvalidValue;
    xp.smem = (uint32_t)smem;
    e = ensure_smem(fn, dev, smem);
    if (e != cudaSuccess) return e;
    int occ = 0;
    e = occupancy_cached(fn, dev, 32 * nw, smem, &occ);
    if (e != cudaSuccess) return e;
    if (occ < 1) return cudaErrorInvalidValue;
    const long long grid = (long long)sm_count_cached(dev) * occ;
    xp.tail = xtab_tail(xp.nslice, xp.nbatch, (int)grid, kXtabItemCost);
    xp.mains = (int)(grid / xp.nslice);
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3((unsigned)grid);
    lc.blockDim = dim3(32 * nw);
    lc.dynamicSmemBytes = smem;
    lc.stream = st;
    cudaLaunchAttribute attr[1];
    if (c.flags & B4_FLAG_PDL) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        lc.attrs = attr;
        lc.numAttrs = 1;
    }
    void* args[] = {&xp};
    return cudaLaunchKernelExC(&lc, fn, args);
}

int launch_gemv_xtab(const GemvProblem& p, const b4_gemv_config& c, void* ws, size_t ws_bytes, cudaStream_t st)
{
    if (!xtab_shape(p.fmt, p.in_f, p.m, p.x)) return cudaErrorInvalidValue;
    const b4_gemv_segment s{p.qw, p.scale, p.y, p.out_f};
    return launch_xtab_segs(&s, 1, p.x, p.in_f, c, ws, ws_bytes, st, nullptr);
}

// The x-pair table kernel pays ~4 us per launch before it streams (the tables,
// the zeroing of y, the previous launch's drain: it holds one CTA per SM) and
// then streams faster than the tensor-pipe and CUDA-core NF4 kernels, which
// start in ~3 us (B200, PDL chains over every Qwen2.5-7B, Llama-3-70B and
// tensor-parallel shard shape and the fused q/k/v and gate/up launches).  It
// is taken from 17.5 MB of weights up, and from 5 MB where rows are 8192
// columns or longer (the other kernels are slowest there): Qwen gate/up 12.4
// us against 13.8, fused gate+up 19.1 against 25.0, down 11.6 against 22.3,
// Llama-3-70B q/o 12.9 against 17.0, tp4 q 6.6 against 8.8, tp8 gate/up 8.6
// against 9.3, tp8 q/k/v (5.9 MB) 6.0 against 6.9; below, e.g. Qwen q/o (7.2
// MB) 5.9 against 5.0.  16 warps with two batches in flight each from 9 MB,
// 12 warps with three below.
bool xtab_pays(long long weight_bytes, int in_f)
{
    return weight_bytes >= 17500LL * 1000 || (in_f >= 8192 && weight_bytes >= 5000LL * 1000);
}

void xtab_config(b4_gemv_config* cfg, long long weight_bytes, int in_f)
{
    (void)in_f;
    *cfg = b4_gemv_config{};
    cfg->engine = B4_ENGINE_NF4_XTAB;
    cfg->vec_words = 4;
    cfg->rows_per_warp = kXtabBatch;
    cfg->warps_k = 1;
    const bool big = weight_bytes >= 9LL * 1000 * 1000;
    cfg->row_groups = big ? 16 : 12;   // warps per CTA
    cfg->batch_tile = 1;
    cfg->stages = big ? 2 : 3;         // batches in flight per warp
}

long long nf4_weight_bytes(long long rows, int in_f)
{
    return rows * in_f / 2 + rows * (in_f / kNf4Block) * 4;
}

int launch_xtab_shard(const GemvProblem& p, const float* xgu, int flags, void* ws, cudaStream_t st)
{
    const b4_gemv_segment s{p.qw, p.scale, p.y, p.out_f};
    const long long wb = nf4_weight_bytes(p.out_f, p.in_f);
    if (!xtab_shape(p.fmt, p.in_f, p.m, xgu ? static_cast<const void*>(xgu) : p.x) || !xtab_buffers(&s, 1) ||
        !xtab_pays(wb, p.in_f))
        return cudaErrorNotSupported;
    b4_gemv_config c;
    xtab_config(&c, wb, p.in_f);
    c.flags = flags & B4_FLAG_PDL;
    return launch_xtab_segs(&s, 1, p.x, p.in_f, c, ws, B4_XTAB_WORKSPACE_BYTES, st, xgu);
}

// ---- split launches (b4_gemv_split.cuh) ---------------------------------------

int split_plan(const GemvProblem& p, const b4_gemv_config& c, SplitPlan* plan)
{
    if (p.m != 1 || !(c.flags & B4_FLAG_SPLIT)) return cudaErrorInvalidValue;
    SplitPlan s = {};
    if (p.fmt == kInt4) {
        const int G = c.stage_groups, ng = p.in_f / kGroup;
        if (c.engine != B4_ENGINE_MMA_LEAN_ASYNC || (G != 1 && G != 2 && G != 4) || ng % G) return cudaErrorInvalidValue;
        if (!aligned(p.qw, 16) || !aligned(p.scale, 2u * G)) return cudaErrorInvalidValue;
        s.fn = gemv_kernel_split_int4(c.stages, G);
        s.nst = ng / G;
        s.smem = (size_t)p.in_f * 2 + (size_t)8 * c.stages * G * 64 * 16;
    } else {
        if (c.engine != B4_ENGINE_MMA_NF4 || p.in_f % 128) return cudaErrorInvalidValue;
        if (!aligned(p.qw, 16) || !aligned(p.scale, 8)) return cudaErrorInvalidValue;
        s.fn = gemv_kernel_split_nf4(c.stages);
        s.nst = p.in_f / 128;
        s.smem = (size_t)kNf4PairTableBytes + (size_t)p.in_f * 2;
    }
    if (!s.fn) return cudaErrorInvalidValue;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    int smem_max = 0;
    e = cudaDeviceGetAttribute(&smem_max, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e != cudaSuccess) return e;
    if (s.smem > (size_t)smem_max) return cudaErrorInvalidValue;
    if (s.smem > 48 * 1024) {
        e = ensure_smem(s.fn, dev, s.smem);
        if (e != cudaSuccess) return e;
    }
    int occ = 0;
    e = occupancy_cached(s.fn, dev, 256, s.smem, &occ);
    if (e != cudaSuccess) return e;
    if (occ < 1) return cudaErrorInvalidValue;
    s.nblocks = (p.out_f + 15) / 16;
    s.total = s.nblocks * s.nst;
    // every resident warp takes an equal run of k-steps; CTAs left without
    // work are not launched
    const long long warps = (long long)sm_count_cached(dev) * occ * 8;
    s.per = (int)std::min<long long>((s.total + warps - 1) / warps, INT32_MAX);
    const long long used = (s.total + s.per - 1) / s.per;
    s.grid = (int)((used + 7) / 8);
    s.maxp = (s.nst - 1) / s.per + 2;
    s.cnt_bytes = ((size_t)s.nblocks * 4 + 255) / 256 * 256;
    s.ws_bytes = s.cnt_bytes + (size_t)s.nblocks * s.maxp * 16 * sizeof(float);
    *plan = s;
    return cudaSuccess;
}

int launch_split(const GemvProblem& p, const b4_gemv_config& c, void* ws, size_t ws_bytes, cudaStream_t st)
{
    SplitPlan s;
    int e = split_plan(p, c, &s);
    if (e != cudaSuccess) return e;
    if (!ws || !aligned(ws, 16) || ws_bytes < s.ws_bytes) return cudaErrorInvalidValue;
    SplitParams sp;
    sp.qw = p.qw;
    sp.scale = p.scale;
    sp.x = static_cast<const __half*>(p.x);
    sp.y = p.y;
    sp.cnt = static_cast<unsigned*>(ws);
    sp.part = reinterpret_cast<float*>(static_cast<char*>(ws) + s.cnt_bytes);
    sp.total = s.total;
    sp.in_f = p.in_f;
    sp.out_f = p.out_f;
    sp.nst = s.nst;
    sp.per = s.per;
    sp.maxp = s.maxp;
    sp.x_vec = aligned(p.x, 16);
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3((unsigned)s.grid);
    lc.blockDim = dim3(256);
    lc.dynamicSmemBytes = s.smem;
    lc.stream = st;
    cudaLaunchAttribute attr[1];
    if (c.flags & B4_FLAG_PDL) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        lc.attrs = attr;
        lc.numAttrs = 1;
    }
    void* args[] = {&sp};
    return cudaLaunchKernelExC(&lc, s.fn, args);
}

// The dispatch rule's launch for cfg NULL.  A batch whose x does not fit
// next to the tensor-pipe engines' buffers in shared memory (m * in_f too
// large: down_proj at m >= 8) would fall back to the generic CUDA-core or
// register-operand engines, which re-read or re-decode the weights per batch
// row (NF4 down_proj, m = 8: 292 us).  It runs instead as launches of the
// largest chunk of batch rows that the tensor-pipe engines take (8, 4 or 2
// rows), each a full pass over the weights (m = 8 as two passes of 4 rows:
// 2 x 31 us).
int launch_default(const GemvProblem& p, int flags, cudaStream_t st)
{
    b4_gemv_config c;
    default_config(p, &c);
    c.flags = flags;
    const bool tensor_pipe = c.engine == B4_ENGINE_MMA_LEAN_ASYNC || c.engine == B4_ENGINE_MMA_NF4;
    if (p.m > 1 && !tensor_pipe) {
        for (int mc = 8; mc >= 2; mc /= 2) {
            if (mc >= p.m) continue;
            GemvProblem q = p;
            q.m = mc;
            b4_gemv_config cc;
            default_config(q, &cc);
            if (cc.engine != B4_ENGINE_MMA_LEAN_ASYNC && cc.engine != B4_ENGINE_MMA_NF4) continue;
            for (int b0 = 0; b0 < p.m; b0 += mc) {
                GemvProblem part = p;
                part.m = std::min(mc, p.m - b0);
                part.x = static_cast<const __half*>(p.x) + (long long)b0 * p.x_ld;
                part.y = p.y + (long long)b0 * p.y_ld;
                b4_gemv_config pc;
                default_config(part, &pc);
                pc.flags = flags;
                const int e = launch_gemv(part, pc, st);
                if (e != cudaSuccess) return e;
            }
            return cudaSuccess;
        }
    }
    return launch_gemv(p, c, st);
}

// Batches of 2..16 rows whose x does not fit beside the small-batch kernels'
// buffers (long rows: down_proj from 8 rows): the fewest column slices whose
// x does (B4_FLAG_KSLICE), instead of the batch chunks of the plain entry
// points, which stream the weights once per chunk.  Measured on B200 (PDL
// chains, us): INT4 down 3584x18944 m = 8 19.3 against 32.8, m = 16 31.7
// against 66.4; NF4 down m = 8 36.6 against 67.2, m = 16 53.2 against 134.1.
// Where the whole batch fits, slicing measured slower (the second launch and
// the per-slice x): gate_proj and down_proj at m = 2, 4.
bool ksliced_rule(const GemvProblem& p, b4_gemv_config* cfg)
{
    if (p.m < 2 || p.m > 16 || p.in_f % 128) return false;
    const int want = p.fmt == kInt4 ? B4_ENGINE_MMA_LEAN_ASYNC : B4_ENGINE_MMA_NF4;
    b4_gemv_config plain;
    default_config(p, &plain);
    if (plain.engine == want) return false;
    const int ng = p.in_f / 128;
    for (int S = 2; S <= kLeanMaxSeg; ++S) {
        if (ng % S) continue;
        GemvProblem q = p;
        q.in_f = p.in_f / S;
        b4_gemv_config c;
        default_config(q, &c);
        if (c.engine != want) continue;
        if (p.fmt == kInt4)
            while (c.stage_groups > 1 && (q.in_f / kGroup) % c.stage_groups) c.stage_groups /= 2;
        c.flags = B4_FLAG_KSLICE;
        c.x_tile = q.in_f;
        *cfg = c;
        return true;
    }
    return false;
}

void default_config_ws(const GemvProblem& p, b4_gemv_config* cfg)
{
    // NF4 at batch 1 with in_f a multiple of 256: the x-pair table kernel,
    // which needs the workspace for its count-in.  Otherwise the plain rule:
    // measured on B200 (`b4gemv.diag sweep --split-only --pdl`), the split's
    // cross-CTA sum costs ~2 us at the kernel's end (store, fence, atomic, then
    // the last arriver's L2 reads), and once the tile rule gives every CTA one
    // resident tile no batch-1 shape ran faster split (INT4 8192x8192: 11.3 us
    // split, 8.8 us with two 16-row blocks per CTA; Qwen q/o 6.4 vs 3.4 us,
    // down 13.2 vs 10.5 us; NF4 gate 16.8 vs 14.2 us); split configs are taken
    // when passed explicitly.
    const b4_gemv_segment seg{p.qw, p.scale, p.y, p.out_f};
    const long long wb = nf4_weight_bytes(p.out_f, p.in_f);
    if (xtab_shape(p.fmt, p.in_f, p.m, p.x) && xtab_buffers(&seg, 1) && xtab_pays(wb, p.in_f)) {
        xtab_config(cfg, wb, p.in_f);
        return;
    }
    if (aligned(p.qw, 16) && aligned(p.scale, 16) && aligned(p.x, 16) && ksliced_rule(p, cfg)) return;
    default_config(p, cfg);
}

bool needs_workspace(const b4_gemv_config& c)
{
    return (c.flags & (B4_FLAG_SPLIT | B4_FLAG_KSLICE)) || c.engine == B4_ENGINE_NF4_XTAB;
}

}  // namespace b4

using namespace b4;

extern "C" {

int b4_gemv_default_config(int fmt, int in_f, int out_f, int m, b4_gemv_config* cfg)
{
    if (!cfg) return cudaErrorInvalidValue;
    GemvProblem p{fmt, reinterpret_cast<const uint32_t*>(256), reinterpret_cast<const void*>(256),
                  reinterpret_cast<const void*>(256), reinterpret_cast<float*>(256),
                  in_f, out_f, m, in_f, out_f};
    const int e = check_problem(p);
    if (e != cudaSuccess) return e;
    default_config(p, cfg);
    return cudaSuccess;
}

int b4_gemv_ex(int fmt, const uint32_t* qw, const void* scale, const void* x, float* y,
               int in_f, int out_f, int m, const b4_gemv_config* cfg, b4_stream_t stream)
{
    GemvProblem p{fmt, qw, scale, x, y, in_f, out_f, m, in_f, out_f};
    int e = check_problem(p);
    if (e != cudaSuccess) return e;
    if (!cfg || cfg->engine == B4_ENGINE_AUTO)
        return launch_default(p, cfg ? cfg->flags & B4_FLAG_PDL : 0, reinterpret_cast<cudaStream_t>(stream));
    if (needs_workspace(*cfg)) return cudaErrorInvalidValue;   // b4_gemv_ws
    return launch_gemv(p, *cfg, reinterpret_cast<cudaStream_t>(stream));
}

int b4_gemv_default_config_ws(int fmt, int in_f, int out_f, int m, b4_gemv_config* cfg)
{
    if (!cfg) return cudaErrorInvalidValue;
    GemvProblem p{fmt, reinterpret_cast<const uint32_t*>(256), reinterpret_cast<const void*>(256),
                  reinterpret_cast<const void*>(256), reinterpret_cast<float*>(256), in_f, out_f, m, in_f, out_f};
    const int e = check_problem(p);
    if (e != cudaSuccess) return e;
    default_config_ws(p, cfg);
    return cudaSuccess;
}

// The workspace of b4_gemv_ws: its first B4_XTAB_WORKSPACE_BYTES hold the
// x-pair table kernel's running counters, the split and k-slice paths use
// what follows (the split path's arrival counters are zero between calls,
// its partial sums are written before they are read, and the k-slice sum
// clears its partials), so one workspace may serve every path.
void* ws_past_counters(void* ws, size_t ws_bytes, size_t* rest)
{
    if (!ws || ws_bytes < B4_XTAB_WORKSPACE_BYTES) {
        *rest = 0;
        return nullptr;
    }
    *rest = ws_bytes - B4_XTAB_WORKSPACE_BYTES;
    return static_cast<char*>(ws) + B4_XTAB_WORKSPACE_BYTES;
}

int b4_gemv_workspace_size(int fmt, int in_f, int out_f, int m, const b4_gemv_config* cfg, size_t* bytes)
{
    if (!bytes) return cudaErrorInvalidValue;
    // the rule sees 256-byte aligned buffers, as every cudaMalloc gives
    GemvProblem p{fmt, reinterpret_cast<const uint32_t*>(256), reinterpret_cast<const void*>(256),
                  reinterpret_cast<const void*>(256), reinterpret_cast<float*>(256), in_f, out_f, m, in_f, out_f};
    int e = check_problem(p);
    if (e != cudaSuccess) return e;
    b4_gemv_config c;
    if (cfg && cfg->engine != B4_ENGINE_AUTO) c = *cfg;
    else default_config_ws(p, &c);   // the rule, as b4_gemv_ws runs it for cfg NULL or B4_ENGINE_AUTO
    *bytes = 0;
    if (c.engine == B4_ENGINE_NF4_XTAB) {
        *bytes = B4_XTAB_WORKSPACE_BYTES;
        return cudaSuccess;
    }
    if (c.flags & B4_FLAG_KSLICE) {
        int S = 0;
        if (!ksliced_shape(p, c, &S)) return cudaErrorInvalidValue;
        *bytes = B4_XTAB_WORKSPACE_BYTES + ksliced_ws_bytes(p, S);
        return cudaSuccess;
    }
    if (!(c.flags & B4_FLAG_SPLIT)) return cudaSuccess;
    SplitPlan s;
    e = split_plan(p, c, &s);
    if (e != cudaSuccess) return e;
    *bytes = B4_XTAB_WORKSPACE_BYTES + s.ws_bytes;
    return cudaSuccess;
}

int b4_gemv_ws(int fmt, const uint32_t* qw, const void* scale, const void* x, float* y, int in_f, int out_f,
               int m, const b4_gemv_config* cfg, void* ws, size_t ws_bytes, b4_stream_t stream)
{
    GemvProblem p{fmt, qw, scale, x, y, in_f, out_f, m, in_f, out_f};
    int e = check_problem(p);
    if (e != cudaSuccess) return e;
    const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    size_t rest = 0;
    void* const tail = ws_past_counters(ws, ws_bytes, &rest);
    if (!cfg || cfg->engine == B4_ENGINE_AUTO) {
        b4_gemv_config c;
        default_config_ws(p, &c);
        const int pdl = cfg ? cfg->flags & B4_FLAG_PDL : 0;
        if (c.flags & B4_FLAG_KSLICE) {
            c.flags |= pdl;
            return launch_ksliced(p, c, tail, rest, st);
        }
        if (c.engine != B4_ENGINE_NF4_XTAB)   // the rule of b4_gemv_ws never splits
            return launch_default(p, pdl, st);
        c.flags = pdl;
        return launch_gemv_xtab(p, c, ws, ws_bytes, st);
    }
    if (cfg->engine == B4_ENGINE_NF4_XTAB) return launch_gemv_xtab(p, *cfg, ws, ws_bytes, st);
    if (cfg->flags & B4_FLAG_SPLIT) return launch_split(p, *cfg, tail, rest, st);
    if (cfg->flags & B4_FLAG_KSLICE) return launch_ksliced(p, *cfg, tail, rest, st);
    return launch_gemv(p, *cfg, st);
}

int b4_gemv_int4_g128(const uint32_t* qw, const void* scales, const void* x, float* y,
                      int in_f, int out_f, int m, b4_stream_t stream)
{
    return b4_gemv_ex(kInt4, qw, scales, x, y, in_f, out_f, m, nullptr, stream);
}

int b4_gemv_nf4_b64(const uint32_t* qw, const float* absmax, const void* x, float* y,
                    int in_f, int out_f, int m, b4_stream_t stream)
{
    return b4_gemv_ex(kNf4, qw, absmax, x, y, in_f, out_f, m, nullptr, stream);
}

int b4_gemv_nf4_b64_block_per_row(const uint32_t* qw, const float* absmax, const void* x,
                                  float* y, int in_f, int out_f, int warps_per_block,
                                  b4_stream_t stream)
{
    if (warps_per_block < 1 || warps_per_block > kMaxWarps) return cudaErrorInvalidValue;
    GemvProblem p{kNf4, qw, absmax, x, y, in_f, out_f, 1, in_f, out_f};
    int e = check_problem(p);
    if (e != cudaSuccess) return e;
    // the CUDA-core kernel with one row per CTA: warps_per_block warps split
    // in_f, 16-, 8- or 4-byte loads as the alignment allows
    b4_gemv_config c;
    default_config(p, &c);
    const int words = in_f / 8;
    c.engine = B4_ENGINE_FMA;
    c.vec_words = (words % 4 == 0 && aligned(qw, 16)) ? 4 : (words % 2 == 0 && aligned(qw, 8)) ? 2 : 1;
    c.rows_per_warp = 1;
    c.warps_k = warps_per_block;
    c.row_groups = 1;
    c.batch_tile = 1;
    c.nf4_lut = 0;
    c.x_tile = 0;
    c.flags = 0;
    return launch_gemv(p, c, reinterpret_cast<cudaStream_t>(stream));
}

namespace {

// Shape and pointer checks of every segment (check_problem per segment).
int check_segments(int fmt, const b4_gemv_segment* segs, int nseg, const void* x, int in_f, int m, bool need_y)
{
    if (!segs || nseg < 1 || nseg > B4_MAX_SEGMENTS) return cudaErrorInvalidValue;
    for (int s = 0; s < nseg; ++s) {
        float* y = need_y ? segs[s].y : reinterpret_cast<float*>(256);
        const GemvProblem p{fmt, segs[s].qw, segs[s].scale, x, y, in_f, segs[s].out_f, m, in_f, segs[s].out_f};
        const int e = check_problem(p);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace

int b4_gemv_multi_default_config(int fmt, const b4_gemv_segment* segs, int nseg, int in_f, int m,
                                 b4_gemv_config* cfg)
{
    if (!cfg) return cudaErrorInvalidValue;
    const int e = check_segments(fmt, segs, nseg, reinterpret_cast<const void*>(256), in_f, m, false);
    if (e != cudaSuccess) return e;
    default_config_multi(fmt, segs, nseg, in_f, m, cfg);
    return cudaSuccess;
}

int b4_gemv_multi(int fmt, const b4_gemv_segment* segs, int nseg, const void* x, int in_f, int m,
                  const b4_gemv_config* cfg, b4_stream_t stream)
{
    const int e = check_segments(fmt, segs, nseg, x, in_f, m, true);
    if (e != cudaSuccess) return e;
    b4_gemv_config c;
    if (cfg) c = *cfg;
    else default_config_multi(fmt, segs, nseg, in_f, m, &c);
    if (needs_workspace(c)) return cudaErrorInvalidValue;   // b4_gemv_multi_ws
    return launch_gemv_multi(fmt, segs, nseg, x, in_f, m, c, reinterpret_cast<cudaStream_t>(stream));
}

int b4_gemv_multi_default_config_ws(int fmt, const b4_gemv_segment* segs, int nseg, int in_f, int m,
                                    b4_gemv_config* cfg)
{
    if (!cfg) return cudaErrorInvalidValue;
    const int e = check_segments(fmt, segs, nseg, reinterpret_cast<const void*>(256), in_f, m, false);
    if (e != cudaSuccess) return e;
    long long rows = 0;
    for (int s = 0; s < nseg; ++s) rows += segs[s].out_f;
    const long long wb = nf4_weight_bytes(rows, in_f);
    if (xtab_shape(fmt, in_f, m, reinterpret_cast<const void*>(256)) && xtab_buffers(segs, nseg) && xtab_pays(wb, in_f))
        xtab_config(cfg, wb, in_f);
    else default_config_multi(fmt, segs, nseg, in_f, m, cfg);
    return cudaSuccess;
}

int b4_gemv_multi_ws(int fmt, const b4_gemv_segment* segs, int nseg, const void* x, int in_f, int m,
                     const b4_gemv_config* cfg, void* ws, size_t ws_bytes, b4_stream_t stream)
{
    const int e = check_segments(fmt, segs, nseg, x, in_f, m, true);
    if (e != cudaSuccess) return e;
    const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    b4_gemv_config c;
    if (!cfg || cfg->engine == B4_ENGINE_AUTO) {
        long long rows = 0;
        for (int s = 0; s < nseg; ++s) rows += segs[s].out_f;
        const long long wb = nf4_weight_bytes(rows, in_f);
        if (xtab_shape(fmt, in_f, m, x) && xtab_buffers(segs, nseg) && xtab_pays(wb, in_f)) xtab_config(&c, wb, in_f);
        else default_config_multi(fmt, segs, nseg, in_f, m, &c);
        c.flags = cfg ? cfg->flags & B4_FLAG_PDL : 0;
    } else {
        c = *cfg;
    }
    if (c.engine == B4_ENGINE_NF4_XTAB) return launch_xtab_segs(segs, nseg, x, in_f, c, ws, ws_bytes, st, nullptr);
    if (c.flags & B4_FLAG_SPLIT) return cudaErrorInvalidValue;
    return launch_gemv_multi(fmt, segs, nseg, x, in_f, m, c, st);
}

int b4_device_error(int clear)
{
    const int a = gemv_tma_device_error(clear), b = xtab_device_error(clear);
    if (a < 0 || b < 0) return -1;
    return a | b;
}

int b4_empty_launch(b4_stream_t stream)
{
    empty_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>();
    return cudaGetLastError();
}

const char* b4_status_string(int status)
{
    if (status >= B4_STATUS_NCCL_BASE) return b4_nccl_error_string(status);
    return cudaGetErrorString(static_cast<cudaError_t>(status));
}

int b4_abi_version(void) { return B4_ABI_VERSION; }

}  // extern "C"
