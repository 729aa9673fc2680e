// ref_shim.cu -- C entry points over the reference's own header, compiled in
// place from the reference checkout (never copied into this repository).
//
// TEST INFRASTRUCTURE ONLY.  Built by oracle/ref/Makefile into oracle/_ref/,
// it lets the tests pin the oracle against the reference's real host code
// (quantise / quantise_nf4, kernels.cuh:268-339) and lets the measurement
// legs run the reference's kernels (kernels.cuh:26-266), rebuilt for sm_100a,
// on the same device buffers as this library.
#include "kernels.cuh"

#include <cstdint>
#include <cstring>
#include <vector>

extern "C" {

// quantise(), kernels.cuh:270.  deq may be null.
void ref_quantise(const float* W, int out_f, int in_f, uint32_t* packed,
                  uint16_t* scales, float* deq)
{
    std::vector<float> w(W, W + (size_t)out_f * in_f);
    std::vector<uint32_t> p; std::vector<half> s; std::vector<float> d;
    quantise(w, out_f, in_f, p, s, d);
    std::memcpy(packed, p.data(), p.size() * sizeof(uint32_t));
    std::memcpy(scales, s.data(), s.size() * sizeof(uint16_t));
    if (deq) std::memcpy(deq, d.data(), d.size() * sizeof(float));
}

// quantise_nf4(), kernels.cuh:308.  deq may be null.
void ref_quantise_nf4(const float* W, int out_f, int in_f, uint32_t* packed,
                      float* absmax, float* deq)
{
    std::vector<float> w(W, W + (size_t)out_f * in_f);
    std::vector<uint32_t> p; std::vector<float> a, d;
    quantise_nf4(w, out_f, in_f, p, a, d);
    std::memcpy(packed, p.data(), p.size() * sizeof(uint32_t));
    std::memcpy(absmax, a.data(), a.size() * sizeof(float));
    if (deq) std::memcpy(deq, d.data(), d.size() * sizeof(float));
}

// The reference launches, with the geometry of int4_gemv.cu:40-41 and
// diag_aspect.cu:154-160,262-266.  Device pointers; returns cudaGetLastError().
int ref_launch_int4_warp_per_row(const uint32_t* qw, const void* scales, const void* x,
                                 float* y, int in_f, int out_f, cudaStream_t st)
{
    const int block = 256, grid = (out_f + 7) / 8;
    int4_gemv_warp_per_row<<<grid, block, 0, st>>>(qw, (const half*)scales,
                                                   (const half*)x, y, in_f, out_f);
    return (int)cudaGetLastError();
}

int ref_launch_nf4_warp_per_row(const uint32_t* qw, const float* absmax, const void* x,
                                float* y, int in_f, int out_f, cudaStream_t st)
{
    const int block = 256, grid = (out_f + 7) / 8;
    nf4_gemv_warp_per_row<<<grid, block, 0, st>>>(qw, absmax, (const half*)x, y, in_f, out_f);
    return (int)cudaGetLastError();
}

int ref_launch_nf4_block_per_row(const uint32_t* qw, const float* absmax, const void* x,
                                 float* y, int in_f, int out_f, int wpb, cudaStream_t st)
{
    nf4_gemv_block_per_row<<<out_f, wpb * 32, wpb * sizeof(float), st>>>(
        qw, absmax, (const half*)x, y, in_f, out_f);
    return (int)cudaGetLastError();
}

// y must be zeroed first (kernels.cuh:145); this launch does not do it.
int ref_launch_nf4_split_k(const uint32_t* qw, const float* absmax, const void* x,
                           float* y, int in_f, int out_f, int splits, cudaStream_t st)
{
    const int block = 256, warps = out_f * splits, grid = (warps + 7) / 8;
    nf4_gemv_split_k<<<grid, block, 0, st>>>(qw, absmax, (const half*)x, y, in_f, out_f, splits);
    return (int)cudaGetLastError();
}

// The benchmark's dispatch rule, int4_gemv.cu:52-68: block-per-row with 2 warps
// iff NF4 && out_f < 8192 && in_f/8 >= 1024, else one warp per row.
int ref_launch_dispatch(int nf4, const uint32_t* qw, const void* scale, const void* x,
                        float* y, int in_f, int out_f, cudaStream_t st)
{
    const bool block_per_row = nf4 && out_f < 8192 && (in_f >> 3) >= 1024;
    if (block_per_row)
        return ref_launch_nf4_block_per_row(qw, (const float*)scale, x, y, in_f, out_f, 2, st);
    if (nf4) return ref_launch_nf4_warp_per_row(qw, (const float*)scale, x, y, in_f, out_f, st);
    return ref_launch_int4_warp_per_row(qw, scale, x, y, in_f, out_f, st);
}

}  // extern "C"
