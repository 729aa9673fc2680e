// b4_gemv_tma.cuh -- the streaming INT4 GEMV: packed codes arrive through a
// per-warp ring of bulk copies (TMA) in shared memory, the multiply-
// accumulates run on the tensor pipe (register-operand MMA, as in
// b4_gemv_mma.cuh).
//
// Why: at batch 1 the kernel must keep ~6.5 TB/s x ~1 us of loads in flight,
// about 45 KB per SM.  Register prefetch ties that to occupancy; here each
// warp keeps STAGES-1 stages of 16 rows x KCG groups (KCG*64 bytes per row)
// in flight, issued by its own lanes (one cp.async.bulk per row segment) and
// tracked by one mbarrier per stage, so in-flight bytes cost no registers.
//
// Work split: a CTA holds rg row groups of 16 rows; warps_k warps share a row
// group and each takes a contiguous range of its 128-column groups, cut into
// chunks of KCG groups (one ring stage each).  CTAs loop over row tiles
// (blockIdx.x, + gridDim.x, ...); a warp's stage sequence runs across row
// tiles, so the next tile's copies are in flight while the current one
// finishes.  x is staged once per CTA (the whole of in_f, pair order).
//
// Shared-memory ring rows are padded to KCG*64 + 64 bytes: the 8 lanes of a
// quarter warp read 16 bytes from each of two adjacent rows at 4 consecutive
// 16-byte offsets, and the padding puts the two rows on disjoint bank groups.
//
// Every mbarrier wait is bounded (mbar_wait_bounded); a wait that runs out
// sets the device error flag, and the warp stops issuing and waiting so the
// kernel ends (with a wrong y) instead of hanging.
#pragma once

#include "b4_gemv_mma.cuh"
#include "b4_tma.cuh"

namespace b4 {

struct TmaParams {
    KParams k;
    int stages_dummy;   // keeps the struct layout explicit; stages are a template parameter
    int ring_offset;    // byte offset of the rings in dynamic shared memory
    int bar_offset;     // byte offset of the mbarriers
};

template <int KCG>
struct RingGeom {
    static constexpr int kRowBytes = KCG * 64 + 64;   // padded row slot
    static constexpr int kStageBytes = 16 * kRowBytes;
};

template <int NT, int STAGES, int KCG>
__global__ void __launch_bounds__(256, 1) b4_gemv_tma_mma_kernel(const TmaParams tp)
{
    const KParams& p = tp.k;
    constexpr int NB = 8 * NT;
    constexpr int ROWB = RingGeom<KCG>::kRowBytes;
    constexpr int STB = RingGeom<KCG>::kStageBytes;
    extern __shared__ __align__(128) unsigned char smem[];
    const int lane = threadIdx.x & 31;
    const int g = lane >> 2, q = lane & 3;
    const int warp = threadIdx.x >> 5;
    const int nwarps = blockDim.x >> 5;
    const int ks = warp % p.kw;
    const int grp = warp / p.kw;
    const int words = p.in_f >> 3;
    const int ng = p.in_f / kGroup;
    const int rows_per_tile = p.rg * 16;
    const int n_row_tiles = (p.out_f + rows_per_tile - 1) / rows_per_tile;
    const int nb = min(p.m, NB);

    uint4* xs = reinterpret_cast<uint4*>(smem);
    float* red = reinterpret_cast<float*>(smem + (size_t)nb * ng * 256);
    unsigned char* ring = smem + tp.ring_offset + (size_t)warp * STAGES * STB;
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + tp.bar_offset) + warp * STAGES;

    if (lane == 0) {
        for (int i = 0; i < STAGES; ++i) mbar_init(&bar[i], 1);
        fence_mbar_init();
    }
    __syncwarp();

    // this warp's groups [gs, ge) and its chunks (uniform count over warps)
    const int gs = ks * ng / p.kw, ge = (ks + 1) * ng / p.kw;
    const int per_warp_max = (ng + p.kw - 1) / p.kw;
    const int n_chunks = (per_warp_max + KCG - 1) / KCG;
    const int my_tiles = blockIdx.x < n_row_tiles ? (n_row_tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
    const int total = my_tiles * n_chunks;
    const uint64_t policy = evict_first_policy();
    bool aborted = false;   // warp-uniform: set once any lane's bounded wait ran out
    int issued = 0;         // stages whose copies were issued

    auto tile_row0 = [&](int j) { return (blockIdx.x + j * gridDim.x) * rows_per_tile + grp * 16; };

    auto issue = [&](int s) {
        if (s >= total || aborted) return;
        issued = s + 1;
        const int j = s / n_chunks, c = s - j * n_chunks;
        const int row0 = tile_row0(j);
        const int G0 = gs + c * KCG, G1 = min(G0 + KCG, ge);
        const int rows = max(0, min(16, p.out_f - row0));
        const uint32_t bytes = G1 > G0 ? (uint32_t)(G1 - G0) * 64u : 0u;
        unsigned char* buf = ring + (s % STAGES) * STB;
        uint64_t* b = &bar[s % STAGES];
        __syncwarp();
        if (lane == 0) mbar_arrive_expect_tx(b, bytes * (uint32_t)rows);
        __syncwarp();
        if (lane < rows && bytes) {
            fence_proxy_async();
            bulk_g2s(buf + lane * ROWB, p.qw + (long long)(row0 + lane) * words + G0 * 16, bytes, b, policy);
        }
    };

    // scales of one stage: rows g and g+8, groups G0 .. G0+KCG-1
    auto load_scales = [&](int s, float (&sa)[KCG], float (&sb)[KCG]) {
#pragma unroll
        for (int i = 0; i < KCG; ++i) sa[i] = sb[i] = 0.0f;
        if (s >= total) return;
        const int j = s / n_chunks, c = s - j * n_chunks;
        const int row0 = tile_row0(j);
        const int G0 = gs + c * KCG, G1 = min(G0 + KCG, ge);
        const __half* sc = static_cast<const __half*>(p.scale);
        const int ra = row0 + g, rb = ra + 8;
#pragma unroll
        for (int i = 0; i < KCG; ++i) {
            if (G0 + i < G1) {
                if (ra < p.out_f) sa[i] = __half2float(__ldg(sc + (long long)ra * ng + G0 + i));
                if (rb < p.out_f) sb[i] = __half2float(__ldg(sc + (long long)rb * ng + G0 + i));
            }
        }
    };

    // prologue: the first STAGES-1 stages go out before waiting on x's producer
    for (int s = 0; s < STAGES - 1; ++s) issue(s);
    asm volatile("griddepcontrol.launch_dependents;");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    mma_stage_x(p, xs, 0, nb, 0, ng * 16);
    __syncthreads();

    float sa[KCG], sb[KCG], na[KCG], nbs[KCG];
    load_scales(0, sa, sb);
    float acc[NT][4];
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[n][j] = 0.0f;

    for (int s = 0; s < total; ++s) {
        issue(s + STAGES - 1);
        load_scales(s + 1, na, nbs);
        const bool ok = aborted || mbar_wait_bounded(&bar[s % STAGES], (uint32_t)(s / STAGES) & 1u);
        if (__any_sync(0xffffffffu, !ok)) aborted = true;

        const int j = s / n_chunks, c = s - j * n_chunks;
        const int row0 = tile_row0(j);
        const int G0 = gs + c * KCG, G1 = min(G0 + KCG, ge);
        const unsigned char* buf = ring + (s % STAGES) * STB;
#pragma unroll
        for (int i = 0; i < KCG; ++i) {
            if (G0 + i < G1) {
                const uint4 wa = *reinterpret_cast<const uint4*>(buf + g * ROWB + i * 64 + q * 16);
                const uint4 wb = *reinterpret_cast<const uint4*>(buf + (g + 8) * ROWB + i * 64 + q * 16);
                uint4 xb[NT][4];
#pragma unroll
                for (int n = 0; n < NT; ++n) {
                    const int bb = 8 * n + g;
#pragma unroll
                    for (int v = 0; v < 4; ++v)
                        xb[n][v] = bb < nb ? xs[mma_xslot(bb, (G0 + i) * 16 + 4 * q + v, ng * 16)]
                                           : make_uint4(0u, 0u, 0u, 0u);
                }
                const uint32_t wav[4] = {wa.x, wa.y, wa.z, wa.w};
                const uint32_t wbv[4] = {wb.x, wb.y, wb.z, wb.w};
                float d0[NT][4], d1[NT][4];
#pragma unroll
                for (int v = 0; v < 4; ++v) {
                    uint32_t ha[4], hb[4];
                    int4_word_to_half2(wav[v], ha);
                    int4_word_to_half2(wbv[v], hb);
#pragma unroll
                    for (int pp = 0; pp < 2; ++pp) {
                        const uint32_t a[4] = {ha[2 * pp], hb[2 * pp], ha[2 * pp + 1], hb[2 * pp + 1]};
#pragma unroll
                        for (int n = 0; n < NT; ++n) {
                            const uint32_t b0 = pp ? xb[n][v].z : xb[n][v].x;
                            const uint32_t b1 = pp ? xb[n][v].w : xb[n][v].y;
                            float (&d)[4] = (v & 1) ? d1[n] : d0[n];
                            if (v < 2 && pp == 0) {
                                const float z[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                                mma_16816(d, a, b0, b1, z);
                            } else {
                                mma_16816(d, a, b0, b1, d);
                            }
                        }
                    }
                }
#pragma unroll
                for (int n = 0; n < NT; ++n) {
                    acc[n][0] = fmaf(d0[n][0] + d1[n][0], sa[i], acc[n][0]);
                    acc[n][1] = fmaf(d0[n][1] + d1[n][1], sa[i], acc[n][1]);
                    acc[n][2] = fmaf(d0[n][2] + d1[n][2], sb[i], acc[n][2]);
                    acc[n][3] = fmaf(d0[n][3] + d1[n][3], sb[i], acc[n][3]);
                }
            }
        }
#pragma unroll
        for (int i = 0; i < KCG; ++i) {
            sa[i] = na[i];
            sb[i] = nbs[i];
        }

        if (c == n_chunks - 1) {
            // row tile done: y for rows g, g+8 and batch rows 2q, 2q+1 (+8n)
            auto store = [&](int n, int jj, float v) {
                const int row = row0 + g + ((jj & 2) ? 8 : 0);
                const int bb = 8 * n + 2 * q + (jj & 1);
                if (row < p.out_f && bb < p.m) p.y[(long long)bb * p.y_ld + row] = v;
            };
            if (p.kw == 1) {
#pragma unroll
                for (int n = 0; n < NT; ++n)
#pragma unroll
                    for (int jj = 0; jj < 4; ++jj) store(n, jj, acc[n][jj]);
            } else {
                constexpr int PER = NT * 4;
                float* mine = red + ((grp * p.kw + ks) * PER) * 32;
#pragma unroll
                for (int n = 0; n < NT; ++n)
#pragma unroll
                    for (int jj = 0; jj < 4; ++jj) mine[(n * 4 + jj) * 32 + lane] = acc[n][jj];
                __syncthreads();
                if (ks == 0) {
#pragma unroll
                    for (int n = 0; n < NT; ++n)
#pragma unroll
                        for (int jj = 0; jj < 4; ++jj) {
                            float t = 0.0f;
                            for (int k2 = 0; k2 < p.kw; ++k2)
                                t += red[((grp * p.kw + k2) * PER + n * 4 + jj) * 32 + lane];
                            store(n, jj, t);
                        }
                }
                __syncthreads();
            }
#pragma unroll
            for (int n = 0; n < NT; ++n)
#pragma unroll
                for (int jj = 0; jj < 4; ++jj) acc[n][jj] = 0.0f;
        }
    }
    // After a failed wait, copies issued earlier may still land: wait for them
    // (each wait bounded again) before the CTA's shared memory is released.
    if (aborted) {
        for (int s = max(0, issued - (STAGES - 1)); s < issued; ++s)
            mbar_wait_bounded(&bar[s % STAGES], (uint32_t)(s / STAGES) & 1u);
    }
    (void)nwarps;
}

void* gemv_kernel_int4_tma(int nt, int stages, int kcg);
int gemv_tma_device_error(int clear);

}  // namespace b4
