// b4_gemv_lean_nf4.cuh -- the batch-1 NF4 b64 GEMV with a lean inner loop.
//
// Mapping: a warp owns RW consecutive rows; a step is 32 lanes x VW packed
// words of each of those rows (256*VW columns), lane l taking words
// VW*(32*step + l) ...; warps_k warps share the rows and take steps ks,
// ks + warps_k, ...  The x values of a lane's columns are read once per step
// (fp32, staged per CTA, XOR-swizzled so 8 consecutive lanes hit 8 distinct
// 16-byte bank groups) and serve all RW rows.
//
// Up to four weight matrices that share x form one tile space (LeanNf4Seg),
// and the first tile's first stages are requested before griddepcontrol.wait
// (codes and absmax do not depend on the preceding grid; x does).
//
// In flight: each lane copies its own codes (4*VW bytes per row) and the
// absmax of its columns (4 bytes per row) for future steps with cp.async into
// private ring slots in shared memory, D steps deep; it reads back only what
// it copied, so the per-thread cp.async.wait_group is the only ordering.
//
// Code book, exact fp32 NF4 values (kernels.cuh:78-83):
//   LUT = 0: lane L holds NF4[L & 15], one shuffle per code (the reference's
//            register table, kernels.cuh:64-76);
//   LUT = 2: a 256-entry table of value pairs (NF4[b & 15], NF4[b >> 4]) for
//            each byte b of a packed word, so one 8-byte shared load decodes
//            two codes straight into an fp32 pair for a packed FMA.  The table
//            is replicated 16 times (copy k at 8*k within every 128-byte
//            entry row) and lane l reads copy l & 15: the 16 lanes of a
//            half-warp always hit 16 distinct bank pairs.
#pragma once

#include "b4_gemv_kernel.cuh"
#include "b4_gemv_lean.cuh"

namespace b4 {

// One weight matrix of a launch (see LeanSeg): tiles [tile_end[s-1],
// tile_end[s]) belong to segment s.
struct LeanNf4Seg {
    const uint32_t* qw;
    const float* absmax;
    float* y;
    int out_f;
    int tile_end;
};

struct LeanNf4Params {
    LeanNf4Seg seg[kLeanMaxSeg];
    int nseg, n_tiles;
    const __half* x;
    int in_f;
    int kw, rg;
    int tr;      // engine 7: rows of each warp's 16-row block that carry weights (1..16)
    int x_vec;
    P2pArgs p2p; // engine 7 P2P kernel: the all-reduce of y over peer memory (b4_p2p.cuh)
};

template <int BYTES>
__device__ __forceinline__ void cp_async_bytes(void* smem_dst, const void* gsrc)
{
    if constexpr (BYTES == 16)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr_u32(smem_dst)), "l"(gsrc)
                     : "memory");
    else
        asm volatile("cp.async.ca.shared.global [%0], [%1], %2;" ::"r"(smem_addr_u32(smem_dst)), "l"(gsrc),
                     "n"(BYTES)
                     : "memory");
}

template <int D, int RW, int VW, int LUT>
__global__ void __launch_bounds__(256, 2) b4_gemv_lean_nf4_kernel(const LeanNf4Params p)
{
    constexpr int S = 2 * VW;                 // 16-byte x slots per lane chunk
    constexpr int CB = 4 * VW;                // code bytes per lane per row
    extern __shared__ __align__(16) uint4 lsm[];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int nwarps = blockDim.x >> 5;
    const int ks = warp % p.kw;
    const int grp = warp / p.kw;
    const int words = p.in_f >> 3;
    const int nblk = p.in_f >> 6;
    const int nchunks = words / VW;           // lane chunks per row
    const int nsteps = (nchunks + 31) / 32;
    const int rows_per_tile = p.rg * RW;
    const int n_tiles = p.n_tiles;

    // shared memory: [pair table 32 KB if LUT=2][x][red][rings]
    unsigned char* base = reinterpret_cast<unsigned char*>(lsm);
    float2* ptab = reinterpret_cast<float2*>(base);
    const int tab_bytes = LUT == 2 ? 256 * 16 * 8 : 0;
    uint4* xs = reinterpret_cast<uint4*>(base + tab_bytes);                    // nsteps*32*S slots
    float* red = reinterpret_cast<float*>(xs + nsteps * 32 * S);              // rg*kw*RW
    unsigned char* rings = reinterpret_cast<unsigned char*>(red) + ((p.rg * p.kw * RW * 4 + 15) / 16) * 16;
    unsigned char* ring_c = rings + (size_t)warp * D * RW * 32 * CB;          // codes
    float* ring_a = reinterpret_cast<float*>(rings + (size_t)nwarps * D * RW * 32 * CB) + warp * D * RW * 32;

    if constexpr (LUT == 2) {
        for (int i = threadIdx.x; i < 256 * 16; i += blockDim.x) {
            const int e = i >> 4;
            ptab[i] = make_float2(c_nf4_table[e & 15], c_nf4_table[e >> 4]);
        }
    }
    const float lut = nf4_lane_value(lane);
    const int n_it = nsteps > ks ? (nsteps - ks + p.kw - 1) / p.kw : 0;

    int r0 = 0, out_f = 0, rlast = 0;
    const uint32_t* qw = nullptr;
    const float* absmax = nullptr;
    float* y = nullptr;
    int c_next = 0;                                       // chunk of the next fetch
    // this lane's chunk in step `it`: c = 32*(ks + it*kw) + lane
    auto fetch = [&](int slot) {
        const bool ok = c_next < nchunks;
        const int cc = ok ? c_next : 0;
#pragma unroll
        for (int i = 0; i < RW; ++i) {
            const long long r = min(r0 + i, rlast);
            cp_async_bytes<CB>(ring_c + ((slot * RW + i) * 32 + lane) * CB, qw + r * words + (long long)cc * VW);
            cp_async_bytes<4>(ring_a + (slot * RW + i) * 32 + lane, absmax + r * nblk + (cc * VW) / 8);
        }
        c_next += 32 * p.kw;
    };
    auto start_tile = [&](int tile) {
        // the segment of this tile (constant indices only)
        qw = p.seg[0].qw;
        absmax = p.seg[0].absmax;
        y = p.seg[0].y;
        out_f = p.seg[0].out_f;
        int t0 = 0;
#pragma unroll
        for (int s = 1; s < kLeanMaxSeg; ++s) {
            if (s < p.nseg && tile >= p.seg[s - 1].tile_end) {
                qw = p.seg[s].qw;
                absmax = p.seg[s].absmax;
                y = p.seg[s].y;
                out_f = p.seg[s].out_f;
                t0 = p.seg[s - 1].tile_end;
            }
        }
        rlast = out_f - 1;
        r0 = (tile - t0) * rows_per_tile + grp * RW;
        c_next = 32 * ks + lane;
#pragma unroll
        for (int d = 0; d < D - 1; ++d) {
            if (d < n_it) fetch(d);
            cp_async_commit();
        }
    };

    // codes and absmax first: they do not depend on the preceding grid
    int tile = blockIdx.x;
    if (tile < n_tiles) start_tile(tile);

    asm volatile("griddepcontrol.launch_dependents;");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // x: lane chunk c (VW words, 8*VW columns) -> S swizzled 16-byte slots;
    // kXUnroll slots' loads in flight per thread before any is stored (one
    // memory round trip per kXUnroll slots on this critical path)
    const int nslots = nsteps * 32 * S;
    for (int i0 = threadIdx.x; i0 < nslots; i0 += kXUnroll * blockDim.x) {
        float4 v[kXUnroll];
#pragma unroll
        for (int u = 0; u < kXUnroll; ++u) {
            const int i = i0 + u * (int)blockDim.x;
            const int c = i / S, sl = i - c * S;
            v[u] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (i < nslots && c < nchunks) {
                const long long col = (long long)c * VW * 8 + sl * 4;
                if (p.x_vec) {
                    const uint2 raw = __ldg(reinterpret_cast<const uint2*>(p.x + col));
                    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
                    const float2 d = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
                    v[u] = make_float4(a.x, a.y, d.x, d.y);
                } else {
                    v[u] = make_float4(__half2float(p.x[col]), __half2float(p.x[col + 1]),
                                       __half2float(p.x[col + 2]), __half2float(p.x[col + 3]));
                }
            }
        }
#pragma unroll
        for (int u = 0; u < kXUnroll; ++u) {
            const int i = i0 + u * (int)blockDim.x;
            const int c = i / S, sl = i - c * S;
            if (i < nslots) reinterpret_cast<float4*>(xs)[swz<S>(c, sl)] = v[u];
        }
    }
    __syncthreads();

    const int lx = S >= 8 ? (lane & 7) : ((lane / (8 / S)) & (S - 1));   // the swizzle of this lane's chunks
    const int tabk = (lane & 15) * 8;

    for (; tile < n_tiles; tile += gridDim.x) {
        if (tile != (int)blockIdx.x) start_tile(tile);
        float acc[RW];
#pragma unroll
        for (int i = 0; i < RW; ++i) acc[i] = 0.0f;
        int c_cur = 32 * ks + lane;

        for (int it0 = 0; it0 < n_it; it0 += D) {
#pragma unroll
            for (int d = 0; d < D; ++d) {
                const int it = it0 + d;
                if (it < n_it) {
                    const int nxt = (d + D - 1) % D;
                    if (it + D - 1 < n_it) fetch(nxt);
                    cp_async_commit();
                    cp_async_wait<D - 1>();
                    const bool active = c_cur < nchunks;
                    // x of this lane's columns (zero for a lane past the row end)
                    float4 xv[S];
                    const float4* xc = reinterpret_cast<const float4*>(xs) + (long long)(active ? c_cur : 0) * S;
#pragma unroll
                    for (int t = 0; t < S; ++t) xv[t] = active ? xc[t ^ lx] : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                    for (int i = 0; i < RW; ++i) {
                        uint32_t w[VW];
                        if constexpr (VW == 4) {
                            const uint4 v4 = *reinterpret_cast<const uint4*>(ring_c + ((d * RW + i) * 32 + lane) * CB);
                            w[0] = v4.x; w[1] = v4.y; w[2] = v4.z; w[3] = v4.w;
                        } else {
                            const uint2 v2 = *reinterpret_cast<const uint2*>(ring_c + ((d * RW + i) * 32 + lane) * CB);
                            w[0] = v2.x; w[1] = v2.y;
                        }
                        const float am = ring_a[(d * RW + i) * 32 + lane];
                        float2 pacc = make_float2(0.0f, 0.0f);
#pragma unroll
                        for (int v = 0; v < VW; ++v) {
                            const float4 xa = xv[2 * v], xb = xv[2 * v + 1];
                            const float2 xp[4] = {make_float2(xa.x, xa.y), make_float2(xa.z, xa.w),
                                                  make_float2(xb.x, xb.y), make_float2(xb.z, xb.w)};
                            if constexpr (LUT == 2) {
                                // byte b holds the codes of columns 2b, 2b+1: entry row b*128
                                const uint32_t o0 = ((w[v] << 7) & 0x7f80u) | tabk;
                                const uint32_t o1 = ((w[v] >> 1) & 0x7f80u) | tabk;
                                const uint32_t o2 = ((w[v] >> 9) & 0x7f80u) | tabk;
                                const uint32_t o3 = ((w[v] >> 17) & 0x7f80u) | tabk;
                                const unsigned char* tb = reinterpret_cast<const unsigned char*>(ptab);
                                pacc = __ffma2_rn(*reinterpret_cast<const float2*>(tb + o0), xp[0], pacc);
                                pacc = __ffma2_rn(*reinterpret_cast<const float2*>(tb + o1), xp[1], pacc);
                                pacc = __ffma2_rn(*reinterpret_cast<const float2*>(tb + o2), xp[2], pacc);
                                pacc = __ffma2_rn(*reinterpret_cast<const float2*>(tb + o3), xp[3], pacc);
                            } else {
#pragma unroll
                                for (int k = 0; k < 8; ++k) {
                                    const float t = nf4_lookup_shfl(lut, w[v] >> (4 * k));
                                    const float xk = (k & 1) ? xp[k >> 1].y : xp[k >> 1].x;
                                    if (k & 1)
                                        pacc.y = fmaf(t, xk, pacc.y);
                                    else
                                        pacc.x = fmaf(t, xk, pacc.x);
                                }
                            }
                        }
                        acc[i] = fmaf(pacc.x + pacc.y, active ? am : 0.0f, acc[i]);
                    }
                    c_cur += 32 * p.kw;
                }
            }
        }
        cp_async_wait<0>();

        // close the rows: butterfly over lanes, then warps_k partials in order
#pragma unroll
        for (int i = 0; i < RW; ++i) {
            float v = acc[i];
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
            acc[i] = v;
        }
        float mine = acc[0];
#pragma unroll
        for (int i = 1; i < RW; ++i)
            if (lane == i) mine = acc[i];
        if (p.kw == 1) {
            if (lane < RW && r0 + lane < out_f) y[r0 + lane] = mine;
        } else {
            if (lane < RW) red[(grp * p.kw + ks) * RW + lane] = mine;
            __syncthreads();
            if (ks == 0 && lane < RW) {
                float t = 0.0f;
                for (int k2 = 0; k2 < p.kw; ++k2) t += red[(grp * p.kw + k2) * RW + lane];
                if (r0 + lane < out_f) y[r0 + lane] = t;
            }
            __syncthreads();
        }
    }
}

void* gemv_kernel_nf4_lean(int depth, int rw, int vw, int lut);

}  // namespace b4
