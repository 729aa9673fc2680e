// b4_quant.cu -- bit-exact format kernels: dequantisation (W_dequant), code
// unpacking and the on-GPU quantisers.
//
// Compiled with --fmad=false: every value here is defined by a single IEEE
// rounding (division, multiplication, fp16 conversion) and must not be fused.
#include <cmath>

#include "b4_common.cuh"
#include "b4_internal.h"

namespace b4 {
namespace {

bool aligned(const void* p, unsigned a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// (int)std::lround(q) as kernels.cuh:286 computes it on glibc x86-64: a NaN, an
// infinity or a magnitude beyond long gives LONG_MIN, whose low 32 bits (kept
// by the (int) cast) are 0.  Finite values round half away from zero.
__device__ __forceinline__ int lround_int(float q)
{
    if (!(fabsf(q) < 0x1p63f)) return 0;
    const long long l = llroundf(q);
    return (int)(uint32_t)(unsigned long long)l;
}

// x86 SSE arithmetic turns an invalid operation on non-NaN operands (here
// only 0 * inf, when a group's fp16 scale overflowed) into the "default NaN"
// 0xffc00000; the GPU produces 0x7fffffff.  Dequantised values are rewritten to
// the x86 bits so the device output is byte-identical to the reference's
// host-computed `deq` (kernels.cuh:290,331).  No operand here is ever NaN:
// scales and absmax come from a max that skips NaN.
__device__ __forceinline__ float host_nan(float v)
{
    return isnan(v) ? __uint_as_float(0xffc00000u) : v;
}

// One thread per packed word: 8 dequantised columns.
template <int F>
__global__ void dequant_kernel(const uint32_t* __restrict__ qw, const void* __restrict__ scale,
                               float* __restrict__ out, int in_f, long long n_words, int vec_out)
{
    const int words = in_f >> 3;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n_words;
         i += (long long)gridDim.x * blockDim.x) {
        const long long r = i / words;
        const int wi = (int)(i - r * words);
        const uint32_t w = __ldg(qw + i);
        float s;
        if (F == kInt4)
            s = __half2float(__ldg(static_cast<const __half*>(scale) + r * (in_f / kGroup) + (wi * 8) / kGroup));
        else
            s = __ldg(static_cast<const float*>(scale) + r * (in_f / kNf4Block) + (wi * 8) / kNf4Block);
        float v[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int code = (w >> (4 * k)) & 0xf;
            v[k] = host_nan((F == kInt4) ? __fmul_rn((float)(code - 8), s) : __fmul_rn(c_nf4_table[code], s));
        }
        float* o = out + i * 8;
        if (vec_out) {
            reinterpret_cast<float4*>(o)[0] = make_float4(v[0], v[1], v[2], v[3]);
            reinterpret_cast<float4*>(o)[1] = make_float4(v[4], v[5], v[6], v[7]);
        } else {
#pragma unroll
            for (int k = 0; k < 8; ++k) o[k] = v[k];
        }
    }
}

__global__ void unpack_kernel(const uint32_t* __restrict__ qw, uint8_t* __restrict__ codes,
                              long long n_words, int vec_out)
{
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n_words;
         i += (long long)gridDim.x * blockDim.x) {
        const uint32_t w = __ldg(qw + i);
        uint32_t lo = 0, hi = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            lo |= ((w >> (4 * k)) & 0xfu) << (8 * k);
            hi |= ((w >> (4 * (k + 4))) & 0xfu) << (8 * k);
        }
        if (vec_out) {
            reinterpret_cast<uint2*>(codes)[i] = make_uint2(lo, hi);
        } else {
            uint8_t* o = codes + i * 8;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                o[k] = (lo >> (8 * k)) & 0xff;
                o[k + 4] = (hi >> (8 * k)) & 0xff;
            }
        }
    }
}

// bitsandbytes' 4-bit packing holds two codes per byte with the lower column
// in the HIGH nibble; this library's (the reference's, kernels.cuh:289,329)
// holds the lower column in the LOW nibble, bytes in the same order.  The
// repack swaps the two nibbles of every byte (its own inverse).
__global__ void repack_nibbles_kernel(const uint32_t* __restrict__ src, uint32_t* __restrict__ dst,
                                      long long n_words, int vec)
{
    const long long n = vec ? n_words / 4 : n_words;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        if (vec) {
            uint4 w = __ldg(reinterpret_cast<const uint4*>(src) + i);
            w.x = ((w.x & 0x0f0f0f0fu) << 4) | ((w.x >> 4) & 0x0f0f0f0fu);
            w.y = ((w.y & 0x0f0f0f0fu) << 4) | ((w.y >> 4) & 0x0f0f0f0fu);
            w.z = ((w.z & 0x0f0f0f0fu) << 4) | ((w.z >> 4) & 0x0f0f0f0fu);
            w.w = ((w.w & 0x0f0f0f0fu) << 4) | ((w.w >> 4) & 0x0f0f0f0fu);
            reinterpret_cast<uint4*>(dst)[i] = w;
        } else {
            const uint32_t w = __ldg(src + i);
            dst[i] = ((w & 0x0f0f0f0fu) << 4) | ((w >> 4) & 0x0f0f0f0fu);
        }
    }
}

// INT4 g128 (kernels.cuh:268-297): one warp per (row, group); lane l holds
// columns 4l..4l+3 of the group.
__global__ void quant_int4_kernel(const float* __restrict__ W, int out_f, int in_f,
                                  uint32_t* __restrict__ packed, __half* __restrict__ scales,
                                  float* __restrict__ deq)
{
    const int groups = in_f / kGroup;
    const long long gw = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (gw >= (long long)out_f * groups) return;
    const long long r = gw / groups;
    const int g = (int)(gw - r * groups);
    const long long off = r * in_f + (long long)g * kGroup + lane * 4;
    float w[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) w[k] = W[off + k];

    float amax = 0.0f;  // std::max(amax, |w|) never takes a NaN
#pragma unroll
    for (int k = 0; k < 4; ++k) amax = fmaxf(amax, fabsf(w[k]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));

    const float s = (amax > 0.0f) ? __fdiv_rn(amax, 7.0f) : 1.0f;
    const __half sh = __float2half_rn(s);
    const float s_used = __half2float(sh);
    if (lane == 0) scales[r * groups + g] = sh;

    uint32_t nib = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        int code = lround_int(__fdiv_rn(w[k], s_used)) + 8;
        code = min(15, max(0, code));
        nib |= (uint32_t)code << (4 * k);
        if (deq) deq[off + k] = host_nan(__fmul_rn((float)(code - 8), s_used));
    }
    const uint32_t other = __shfl_down_sync(0xffffffffu, nib, 1);
    if ((lane & 1) == 0) packed[(off >> 3)] = nib | (other << 16);
}

// NF4 b64 (kernels.cuh:308-339): one warp per (row, block); lane l holds
// columns 2l, 2l+1 of the block.
__global__ void quant_nf4_kernel(const float* __restrict__ W, int out_f, int in_f,
                                 uint32_t* __restrict__ packed, float* __restrict__ absmax,
                                 float* __restrict__ deq)
{
    const int blocks = in_f / kNf4Block;
    const long long gw = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (gw >= (long long)out_f * blocks) return;
    const long long r = gw / blocks;
    const int b = (int)(gw - r * blocks);
    const long long off = r * in_f + (long long)b * kNf4Block + lane * 2;
    const float w0 = W[off], w1 = W[off + 1];

    float amax = fmaxf(fmaxf(0.0f, fabsf(w0)), fabsf(w1));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (amax == 0.0f) amax = 1.0f;
    if (lane == 0) absmax[r * blocks + b] = amax;

    uint32_t byte = 0;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const float norm = __fdiv_rn(k ? w1 : w0, amax);
        int best = 0;
        float bd = fabsf(__fsub_rn(norm, c_nf4_table[0]));
        for (int c = 1; c < 16; ++c) {
            const float d = fabsf(__fsub_rn(norm, c_nf4_table[c]));
            if (d < bd) { bd = d; best = c; }
        }
        byte |= (uint32_t)best << (4 * k);
        if (deq) deq[off + k] = host_nan(__fmul_rn(c_nf4_table[best], amax));
    }
    const uint32_t b1 = __shfl_down_sync(0xffffffffu, byte, 1);
    const uint32_t b2 = __shfl_down_sync(0xffffffffu, byte, 2);
    const uint32_t b3 = __shfl_down_sync(0xffffffffu, byte, 3);
    if ((lane & 3) == 0) packed[off >> 3] = byte | (b1 << 8) | (b2 << 16) | (b3 << 24);
}

int grid_for(long long n, int block)
{
    long long g = (n + block - 1) / block;
    if (g > 148LL * 32) g = 148LL * 32;
    return (int)(g < 1 ? 1 : g);
}

}  // namespace
}  // namespace b4

using namespace b4;

extern "C" {

int b4_dequant_int4_g128(const uint32_t* qw, const void* scales, float* w_out, int in_f,
                         int out_f, b4_stream_t stream)
{
    if (!qw || !scales || !w_out || in_f <= 0 || out_f <= 0 || in_f % kGroup) return cudaErrorInvalidValue;
    const long long n = (long long)out_f * (in_f / 8);
    dequant_kernel<kInt4><<<grid_for(n, 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        qw, scales, w_out, in_f, n, aligned(w_out, 16));
    return cudaGetLastError();
}

int b4_dequant_nf4_b64(const uint32_t* qw, const float* absmax, float* w_out, int in_f,
                       int out_f, b4_stream_t stream)
{
    if (!qw || !absmax || !w_out || in_f <= 0 || out_f <= 0 || in_f % kNf4Block) return cudaErrorInvalidValue;
    const long long n = (long long)out_f * (in_f / 8);
    dequant_kernel<kNf4><<<grid_for(n, 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        qw, absmax, w_out, in_f, n, aligned(w_out, 16));
    return cudaGetLastError();
}

int b4_unpack_codes(const uint32_t* qw, uint8_t* codes, int in_f, int out_f, b4_stream_t stream)
{
    if (!qw || !codes || in_f <= 0 || out_f <= 0 || in_f % 8) return cudaErrorInvalidValue;
    const long long n = (long long)out_f * (in_f / 8);
    unpack_kernel<<<grid_for(n, 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        qw, codes, n, aligned(codes, 8));
    return cudaGetLastError();
}

int b4_repack_bnb_nf4(const void* bnb_packed, uint32_t* qw, int in_f, int out_f, b4_stream_t stream)
{
    if (!bnb_packed || !qw || in_f <= 0 || out_f <= 0 || in_f % 64) return cudaErrorInvalidValue;
    if (!aligned(bnb_packed, 4) || !aligned(qw, 4)) return cudaErrorInvalidValue;
    const long long n = (long long)out_f * (in_f / 8);
    const int vec = aligned(bnb_packed, 16) && aligned(qw, 16) && n % 4 == 0;
    repack_nibbles_kernel<<<grid_for(vec ? n / 4 : n, 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint32_t*>(bnb_packed), qw, n, vec);
    return cudaGetLastError();
}

int b4_quantise_int4_g128_device(const float* W, int out_f, int in_f, uint32_t* packed,
                                 void* scales, float* deq, b4_stream_t stream)
{
    if (!W || !packed || !scales || in_f <= 0 || out_f <= 0 || in_f % kGroup) return cudaErrorInvalidValue;
    const long long warps = (long long)out_f * (in_f / kGroup);
    const long long blocks = (warps + 7) / 8;
    if (blocks > 0x7fffffffLL) return cudaErrorInvalidValue;
    quant_int4_kernel<<<(unsigned)blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        W, out_f, in_f, packed, static_cast<__half*>(scales), deq);
    return cudaGetLastError();
}

int b4_quantise_nf4_b64_device(const float* W, int out_f, int in_f, uint32_t* packed,
                               float* absmax, float* deq, b4_stream_t stream)
{
    if (!W || !packed || !absmax || in_f <= 0 || out_f <= 0 || in_f % kNf4Block) return cudaErrorInvalidValue;
    const long long warps = (long long)out_f * (in_f / kNf4Block);
    const long long blocks = (warps + 7) / 8;
    if (blocks > 0x7fffffffLL) return cudaErrorInvalidValue;
    quant_nf4_kernel<<<(unsigned)blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        W, out_f, in_f, packed, absmax, deq);
    return cudaGetLastError();
}

}  // extern "C"
