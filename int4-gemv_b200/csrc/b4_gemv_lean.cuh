// b4_gemv_lean.cuh -- the batch-1 INT4 g128 GEMV with the least integer work
// per code: tensor-pipe multiply-accumulate (register-operand MMA, as in
// b4_gemv_mma.cuh) with every per-group cost other than the decode removed.
//
// Why: at 6.5 TB/s a B200 SM must decode ~45 codes per clock, and the decode
// alone (one SHF + four LOP3 per 8 codes) takes ~45% of the integer pipe at
// that rate, so address arithmetic, predicates and loop control must stay out
// of the inner loop.  Here:
//   * x is staged once per CTA in pair order at its natural word index: the
//     64 bytes lane q needs for group G are words 16*G + 4q .. 16*G + 4q + 3,
//     so one pointer bump per group and four 16-byte loads with immediate
//     offsets fetch all B fragments (m = 1: every batch column of B holds x,
//     all lanes read; the 8 lanes with the same q read the same address);
//   * rows past out_f are clamped to a valid row for loading and never
//     stored, so the loop has no row predicates;
//   * codes and scales are addressed by running pointers, bumped once per
//     group step;
//   * a D-deep software pipeline of register buffers, unrolled so every
//     buffer index is a compile-time constant, keeps 2*(D-1) 16-byte loads
//     per lane in flight;
//   * the group epilogue is two fp32 adds and two FMAs: with all B columns
//     equal, D[row][0] holds the row's partial sum.
// Work split as in the other kernels: warps_k warps share a 16-row tile and
// take groups ks, ks + warps_k, ...; CTAs loop over tiles of rg*16 rows.
//
// ASYNC = 1 moves the in-flight codes out of registers: each lane copies its
// own two 16-byte pieces of every future group with cp.async into a private
// ring slot in shared memory ((stage*2 + row)*32 + lane: a warp's copies and
// reads of one slot are 512 contiguous bytes, conflict-free) and reads them
// back when the group's turn comes.  Lanes only ever read what they copied
// themselves, so the per-thread cp.async.wait_group is the only ordering
// needed, and D stages in flight cost shared memory instead of registers.
#pragma once

#include "b4_gemv_mma.cuh"

namespace b4 {

struct LeanParams {
    const uint32_t* qw;
    const __half* scale;
    const __half* x;
    float* y;
    int in_f, out_f;
    int kw, rg;
    int x_vec;
};

template <int D, int ASYNC>   // D >= 2
__global__ void __launch_bounds__(256, 2) b4_gemv_lean_kernel(const LeanParams p)
{
    extern __shared__ __align__(16) uint4 lsm[];
    const int lane = threadIdx.x & 31;
    const int g = lane >> 2, q = lane & 3;
    const int warp = threadIdx.x >> 5;
    const int ks = warp % p.kw;
    const int grp = warp / p.kw;
    const int words = p.in_f >> 3;
    const int ng = p.in_f >> 7;
    const int rows_per_tile = p.rg * 16;
    const int n_tiles = (p.out_f + rows_per_tile - 1) / rows_per_tile;
    uint4* xs = lsm;                                         // one slot per word
    float* red = reinterpret_cast<float*>(xs + words);      // rg*kw*16
    // ASYNC: this warp's ring, D stages x 2 rows x 32 lanes x 16 bytes
    uint4* ring = xs + words + (p.rg * p.kw * 16 + 3) / 4 + warp * (D * 64);

    asm volatile("griddepcontrol.launch_dependents;");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    for (int w = threadIdx.x; w < words; w += blockDim.x) {
        const __half* src = p.x + (long long)w * 8;
        uint4 raw;
        if (p.x_vec) {
            raw = __ldg(reinterpret_cast<const uint4*>(src));
        } else {
            const unsigned short* h = reinterpret_cast<const unsigned short*>(src);
            raw.x = (uint32_t)__ldg(h + 0) | ((uint32_t)__ldg(h + 1) << 16);
            raw.y = (uint32_t)__ldg(h + 2) | ((uint32_t)__ldg(h + 3) << 16);
            raw.z = (uint32_t)__ldg(h + 4) | ((uint32_t)__ldg(h + 5) << 16);
            raw.w = (uint32_t)__ldg(h + 6) | ((uint32_t)__ldg(h + 7) << 16);
        }
        xs[w] = int4_pair_order(raw);
    }
    __syncthreads();

    // groups of this warp: ks, ks + kw, ...; n_it is warp-uniform
    const int n_it = ng > ks ? (ng - ks + p.kw - 1) / p.kw : 0;
    const int wstep = 4 * p.kw;                              // uint4 per group step

    for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
        const int r0 = tile * rows_per_tile + grp * 16;
        const int ra = min(r0 + g, p.out_f - 1);
        const int rb = min(r0 + g + 8, p.out_f - 1);
        const uint4* pa = reinterpret_cast<const uint4*>(p.qw + (long long)ra * words) + ks * 4 + q;
        const uint4* pb = reinterpret_cast<const uint4*>(p.qw + (long long)rb * words) + ks * 4 + q;
        const __half* sa_p = p.scale + (long long)ra * ng + ks;
        const __half* sb_p = p.scale + (long long)rb * ng + ks;

        uint4 bufa[D], bufb[D];
        __half bsa[D], bsb[D];
        auto fetch = [&](int slot) {
            if constexpr (ASYNC) {
                cp_async16(ring + (slot * 2) * 32 + lane, pa);
                cp_async16(ring + (slot * 2 + 1) * 32 + lane, pb);
            } else {
                const WordVec<4> va = ld_stream<4>(reinterpret_cast<const uint32_t*>(pa));
                const WordVec<4> vb = ld_stream<4>(reinterpret_cast<const uint32_t*>(pb));
                bufa[slot] = make_uint4(va.w[0], va.w[1], va.w[2], va.w[3]);
                bufb[slot] = make_uint4(vb.w[0], vb.w[1], vb.w[2], vb.w[3]);
            }
            bsa[slot] = __ldg(sa_p);
            bsb[slot] = __ldg(sb_p);
            pa += wstep;
            pb += wstep;
            sa_p += p.kw;
            sb_p += p.kw;
        };
#pragma unroll
        for (int d = 0; d < D - 1; ++d) {
            if (d < n_it) fetch(d);
            if constexpr (ASYNC) cp_async_commit();   // one group per stage, even if empty
        }
        float acc_a = 0.0f, acc_b = 0.0f;
        const uint4* xp = xs + ks * 16 + q * 4;              // + 16*kw per group step

        for (int it0 = 0; it0 < n_it; it0 += D) {
#pragma unroll
            for (int d = 0; d < D; ++d) {
                const int it = it0 + d;
                if (it < n_it) {
                    // refill the stage consumed in the previous step
                    const int nxt = (d + D - 1) % D;   // a constant once unrolled
                    if (it + D - 1 < n_it) fetch(nxt);
                    uint4 wav, wbv;
                    if constexpr (ASYNC) {
                        cp_async_commit();
                        cp_async_wait<D - 1>();            // this lane's copies of stage d landed
                        wav = ring[(d * 2) * 32 + lane];
                        wbv = ring[(d * 2 + 1) * 32 + lane];
                    } else {
                        wav = bufa[d];
                        wbv = bufb[d];
                    }
                    const uint4 xv[4] = {xp[0], xp[1], xp[2], xp[3]};
                    xp += 16 * p.kw;
                    const uint32_t wa[4] = {wav.x, wav.y, wav.z, wav.w};
                    const uint32_t wb[4] = {wbv.x, wbv.y, wbv.z, wbv.w};
                    float c0[4] = {0.0f, 0.0f, 0.0f, 0.0f}, c1[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
                    for (int v = 0; v < 4; ++v) {
                        uint32_t ha[4], hb[4];
                        int4_word_to_half2(wa[v], ha);
                        int4_word_to_half2(wb[v], hb);
                        const uint32_t a0[4] = {ha[0], hb[0], ha[1], hb[1]};
                        const uint32_t a1[4] = {ha[2], hb[2], ha[3], hb[3]};
                        float (&c)[4] = (v & 1) ? c1 : c0;
                        mma_16816(c, a0, xv[v].x, xv[v].y, c);
                        mma_16816(c, a1, xv[v].z, xv[v].w, c);
                    }
                    acc_a = fmaf(c0[0] + c1[0], __half2float(bsa[d]), acc_a);
                    acc_b = fmaf(c0[2] + c1[2], __half2float(bsb[d]), acc_b);
                }
            }
        }
        if constexpr (ASYNC) cp_async_wait<0>();   // nothing of this tile left in flight

        // rows r0+g and r0+g+8; lanes q = 0..3 hold the same values
        if (p.kw == 1) {
            if (q == 0) {
                if (r0 + g < p.out_f) p.y[r0 + g] = acc_a;
                if (r0 + g + 8 < p.out_f) p.y[r0 + g + 8] = acc_b;
            }
        } else {
            float* mine = red + (grp * p.kw + ks) * 16;
            if (q == 0) {
                mine[g] = acc_a;
                mine[g + 8] = acc_b;
            }
            __syncthreads();
            if (ks == 0 && lane < 16) {
                float t = 0.0f;
                for (int k2 = 0; k2 < p.kw; ++k2) t += red[(grp * p.kw + k2) * 16 + lane];
                if (r0 + lane < p.out_f) p.y[r0 + lane] = t;
            }
            __syncthreads();
        }
    }
}

void* gemv_kernel_int4_lean(int depth, int async_ring);

}  // namespace b4
