// b4_gemv_tma_nf4.cuh -- the streaming NF4 b64 GEMV: packed codes and their
// fp32 absmax arrive through a per-warp ring of bulk copies (TMA) in shared
// memory; CUDA cores decode with the warp-register code book (a shuffle per
// code, as kernels.cuh:64-76 does) and accumulate in fp32.
//
// Work split: a warp owns RW consecutive rows and a contiguous range of
// chunks of in_f, a chunk being 32 lanes x VW packed words (256*VW columns);
// warps_k warps share the RW rows and reduce through shared memory.  A ring
// stage holds RW rows x one chunk of codes (128*VW bytes per row) plus the
// chunk's 4*VW absmax values (16*VW bytes per row); one lane per row issues
// the two bulk copies.  Lane l reads the 4*VW bytes at offset 4*VW*l of each
// row: the 32 lanes cover one contiguous row segment, so shared-memory reads
// are conflict-free without padding.  x is staged once per CTA as fp32.
//
// in_f must be a multiple of 256*VW (whole chunks; this also makes the absmax
// segments 16-byte aligned); other shapes use the register-fed kernel.
#pragma once

#include "b4_gemv_kernel.cuh"
#include "b4_tma.cuh"

namespace b4 {

struct TmaNf4Params {
    KParams k;
    int ring_offset;
    int bar_offset;
};

template <int RW, int VW>
struct Nf4RingGeom {
    static constexpr int kCols = 256 * VW;                    // columns per chunk
    static constexpr int kCodeBytes = 128 * VW;               // one chunk of one row
    static constexpr int kAbsBytes = 16 * VW;                 // its absmax values
    static constexpr int kStageBytes = RW * (kCodeBytes + kAbsBytes);
};

template <int RW, int VW, int STAGES>
__global__ void __launch_bounds__(256, 1) b4_gemv_tma_nf4_kernel(const TmaNf4Params tp)
{
    const KParams& p = tp.k;
    constexpr int STB = Nf4RingGeom<RW, VW>::kStageBytes;
    constexpr int CB = Nf4RingGeom<RW, VW>::kCodeBytes;
    constexpr int AB = Nf4RingGeom<RW, VW>::kAbsBytes;
    constexpr int COLS = Nf4RingGeom<RW, VW>::kCols;
    extern __shared__ __align__(128) unsigned char smem[];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int ks = warp % p.kw;
    const int grp = warp / p.kw;
    const int words = p.in_f >> 3;
    const int nblk = p.in_f / kNf4Block;
    const int nchunk = p.in_f / COLS;
    const int rows_per_tile = p.rg * RW;
    const int n_row_tiles = (p.out_f + rows_per_tile - 1) / rows_per_tile;

    float* xs = reinterpret_cast<float*>(smem);                       // in_f fp32
    float* red = xs + p.in_f;                                          // rg*kw*RW
    unsigned char* ring = smem + tp.ring_offset + (size_t)warp * STAGES * STB;
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + tp.bar_offset) + warp * STAGES;

    if (lane == 0) {
        for (int i = 0; i < STAGES; ++i) mbar_init(&bar[i], 1);
        fence_mbar_init();
    }
    __syncwarp();

    const int cs = ks * nchunk / p.kw, ce = (ks + 1) * nchunk / p.kw;
    const int n_steps = (nchunk + p.kw - 1) / p.kw;     // uniform over warps
    const int my_tiles = blockIdx.x < n_row_tiles ? (n_row_tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
    const int total = my_tiles * n_steps;
    const uint64_t policy = evict_first_policy();
    const float lut = nf4_lane_value(lane);
    bool aborted = false;
    int issued = 0;

    auto tile_row0 = [&](int j) { return (blockIdx.x + j * gridDim.x) * rows_per_tile + grp * RW; };

    auto issue = [&](int s) {
        if (s >= total || aborted) return;
        issued = s + 1;
        const int j = s / n_steps, c = cs + (s - j * n_steps);
        const int row0 = tile_row0(j);
        const int rows = (c < ce) ? max(0, min(RW, p.out_f - row0)) : 0;
        unsigned char* buf = ring + (s % STAGES) * STB;
        uint64_t* b = &bar[s % STAGES];
        __syncwarp();
        if (lane == 0) mbar_arrive_expect_tx(b, (uint32_t)rows * (CB + AB));
        __syncwarp();
        if (lane < rows) {
            fence_proxy_async();
            const long long r = row0 + lane;
            bulk_g2s(buf + lane * CB, p.qw + r * words + (long long)c * (CB / 4), CB, b, policy);
            bulk_g2s(buf + RW * CB + lane * AB, static_cast<const float*>(p.scale) + r * nblk + c * (AB / 4), AB, b,
                     policy);
        }
    };

    for (int s = 0; s < STAGES - 1; ++s) issue(s);
    asm volatile("griddepcontrol.launch_dependents;");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    for (int i = threadIdx.x; i < p.in_f / 4; i += blockDim.x) {
        float4 v;
        if (p.x_vec) {
            const uint2 raw = __ldg(reinterpret_cast<const uint2*>(p.x) + i);
            const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
            const float2 d = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
            v = make_float4(a.x, a.y, d.x, d.y);
        } else {
            v = make_float4(__half2float(p.x[4 * i]), __half2float(p.x[4 * i + 1]), __half2float(p.x[4 * i + 2]),
                            __half2float(p.x[4 * i + 3]));
        }
        reinterpret_cast<float4*>(xs)[i] = v;
    }
    __syncthreads();

    float acc[RW];
#pragma unroll
    for (int i = 0; i < RW; ++i) acc[i] = 0.0f;

    for (int s = 0; s < total; ++s) {
        issue(s + STAGES - 1);
        const bool ok = aborted || mbar_wait_bounded(&bar[s % STAGES], (uint32_t)(s / STAGES) & 1u);
        if (__any_sync(0xffffffffu, !ok)) aborted = true;
        const int j = s / n_steps, c = cs + (s - j * n_steps);
        const int row0 = tile_row0(j);
        if (c < ce) {
            const unsigned char* buf = ring + (s % STAGES) * STB;
            // x for this lane's 8*VW columns: COLS*c + 8*VW*lane ...
            const float4* xp = reinterpret_cast<const float4*>(xs + (long long)c * COLS + lane * 8 * VW);
            float4 xv[2 * VW];
#pragma unroll
            for (int t = 0; t < 2 * VW; ++t) xv[t] = xp[t];
#pragma unroll
            for (int i = 0; i < RW; ++i) {
                uint32_t w4[VW];
                if constexpr (VW == 4) {
                    const uint4 wv = *reinterpret_cast<const uint4*>(buf + i * CB + lane * 16);
                    w4[0] = wv.x; w4[1] = wv.y; w4[2] = wv.z; w4[3] = wv.w;
                } else {
                    const uint2 wv = *reinterpret_cast<const uint2*>(buf + i * CB + lane * 8);
                    w4[0] = wv.x; w4[1] = wv.y;
                }
                // lane's columns lie in one 64-column block: block (8*VW*lane)/64
                const float am = reinterpret_cast<const float*>(buf + RW * CB + i * AB)[(lane * VW) >> 3];
                float pa = 0.0f, pb = 0.0f;
#pragma unroll
                for (int v = 0; v < VW; ++v) {
                    const float xa[8] = {xv[2 * v].x, xv[2 * v].y, xv[2 * v].z, xv[2 * v].w,
                                         xv[2 * v + 1].x, xv[2 * v + 1].y, xv[2 * v + 1].z, xv[2 * v + 1].w};
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        const float t = nf4_lookup_shfl(lut, w4[v] >> (4 * k));
                        if (k & 1)
                            pb = fmaf(t, xa[k], pb);
                        else
                            pa = fmaf(t, xa[k], pa);
                    }
                }
                acc[i] = fmaf(pa + pb, am, acc[i]);
            }
        }
        if (s - j * n_steps == n_steps - 1) {
            // row tile done: butterfly over lanes, then warps_k partials in order
#pragma unroll
            for (int i = 0; i < RW; ++i) {
                float v = acc[i];
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
                acc[i] = v;
            }
            if (p.kw == 1) {
                if (lane < RW && row0 + lane < p.out_f) {
                    float v = acc[0];
#pragma unroll
                    for (int i = 1; i < RW; ++i)
                        if (lane == i) v = acc[i];
                    p.y[row0 + lane] = v;
                }
            } else {
                if (lane == 0) {
#pragma unroll
                    for (int i = 0; i < RW; ++i) red[(grp * p.kw + ks) * RW + i] = acc[i];
                }
                __syncthreads();
                if (ks == 0 && lane < RW) {
                    float t = 0.0f;
                    for (int q = 0; q < p.kw; ++q) t += red[(grp * p.kw + q) * RW + lane];
                    if (row0 + lane < p.out_f) p.y[row0 + lane] = t;
                }
                __syncthreads();
            }
#pragma unroll
            for (int i = 0; i < RW; ++i) acc[i] = 0.0f;
        }
    }
    if (aborted) {
        for (int s = max(0, issued - (STAGES - 1)); s < issued; ++s)
            mbar_wait_bounded(&bar[s % STAGES], (uint32_t)(s / STAGES) & 1u);
    }
}

void* gemv_kernel_nf4_tma(int rw, int vw, int stages);

}  // namespace b4
