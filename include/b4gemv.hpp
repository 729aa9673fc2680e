// b4gemv.hpp -- C++ host API over the C ABI, shaped like the reference's
// header (QuantumDrizzy/int4-gemv, src/kernels.cuh) so that its callers switch
// by changing one #include:
//
//   reference (kernels.cuh)                      here (namespace b4gemv)
//   #define GROUP 128              :12           GROUP            (constexpr)
//   #define NF4_BLOCK 64           :85           NF4_BLOCK        (constexpr)
//   quantise(W, out, in, packed, scales, deq)    quantise(...)    same arguments
//                                  :270-272
//   quantise_nf4(W, out, in, packed, absmax, deq)quantise_nf4(...) same arguments
//                                  :308-310
//   median(std::vector<float>&)    :341-345      median(...)
//   int4_gemv_warp_per_row<<<g,b>>>(qw, scales,  int4_gemv(qw, scales, x, y, in_f,
//       x, y, in_f, out_f)         :26-30            out_f[, m, stream])
//   nf4_gemv_warp_per_row / _block_per_row       nf4_gemv(qw, absmax, x, y, in_f,
//       <<<...>>>(qw, absmax, x, y, in_f, out_f)      out_f[, m, stream])
//                                  :87-91, :211-215
//   CUDA_CHECK(call) -> exit(1)    :13-21        check(status) -> throws b4gemv::error
//
// Defining B4GEMV_GLOBAL_NAMES before the include also brings quantise,
// quantise_nf4 and median into the global namespace, where the reference's
// drivers call them unqualified.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

#include "b4gemv.h"

namespace b4gemv {

constexpr int GROUP = B4_GROUP;
constexpr int NF4_BLOCK = B4_NF4_BLOCK;

struct error : std::runtime_error {
    int status;
    error(const std::string& what, int s) : std::runtime_error(what), status(s) {}
};

inline void check(int status, const char* what = "b4gemv")
{
    if (status != 0)
        throw error(std::string(what) + ": " + b4_status_string(status), status);
}

// Symmetric group-wise INT4 (kernels.cuh:268-297): byte-identical packed codes,
// fp16 scales and dequantised weights.
inline void quantise(const std::vector<float>& W, int out_f, int in_f, std::vector<uint32_t>& packed,
                     std::vector<half>& scales, std::vector<float>& deq, int nthreads = 0)
{
    packed.assign((size_t)out_f * (in_f / 8), 0u);
    scales.resize((size_t)out_f * (in_f / GROUP));
    deq.resize((size_t)out_f * in_f);
    check(b4_quantise_int4_g128(W.data(), out_f, in_f, packed.data(),
                                reinterpret_cast<uint16_t*>(scales.data()), deq.data(), nthreads),
          "quantise");
}

// NF4, block 64, fp32 absmax, canonical NormalFloat table (kernels.cuh:308-339).
inline void quantise_nf4(const std::vector<float>& W, int out_f, int in_f, std::vector<uint32_t>& packed,
                         std::vector<float>& absmax, std::vector<float>& deq, int nthreads = 0)
{
    packed.assign((size_t)out_f * (in_f / 8), 0u);
    absmax.resize((size_t)out_f * (in_f / NF4_BLOCK));
    deq.resize((size_t)out_f * in_f);
    check(b4_quantise_nf4_b64(W.data(), out_f, in_f, packed.data(), absmax.data(), deq.data(), nthreads),
          "quantise_nf4");
}

// kernels.cuh:341-345: sorts v and returns element size/2.
inline float median(std::vector<float>& v)
{
    std::sort(v.begin(), v.end());
    return v[v.size() / 2];
}

// y[b][r] = sum_k dequant(W)[r][k] * x[b][k] for b < m, device pointers,
// enqueued on `stream` (the reference launches on the legacy default stream).
inline int int4_gemv(const uint32_t* qw, const half* scales, const half* x, float* y, int in_f, int out_f,
                     int m = 1, cudaStream_t stream = nullptr)
{
    return b4_gemv_int4_g128(qw, scales, x, y, in_f, out_f, m, reinterpret_cast<b4_stream_t>(stream));
}

inline int nf4_gemv(const uint32_t* qw, const float* absmax, const half* x, float* y, int in_f, int out_f,
                    int m = 1, cudaStream_t stream = nullptr)
{
    return b4_gemv_nf4_b64(qw, absmax, x, y, in_f, out_f, m, reinterpret_cast<b4_stream_t>(stream));
}

// W_dequant reconstruction on the device, bit-exact with quantise()'s deq.
inline int int4_dequant(const uint32_t* qw, const half* scales, float* w, int in_f, int out_f,
                        cudaStream_t stream = nullptr)
{
    return b4_dequant_int4_g128(qw, scales, w, in_f, out_f, reinterpret_cast<b4_stream_t>(stream));
}

inline int nf4_dequant(const uint32_t* qw, const float* absmax, float* w, int in_f, int out_f,
                       cudaStream_t stream = nullptr)
{
    return b4_dequant_nf4_b64(qw, absmax, w, in_f, out_f, reinterpret_cast<b4_stream_t>(stream));
}

}  // namespace b4gemv

#ifdef B4GEMV_GLOBAL_NAMES
using b4gemv::median;
using b4gemv::quantise;
using b4gemv::quantise_nf4;
#endif
