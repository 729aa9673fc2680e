/*
 * b4_oracle.h -- CPU oracle for the fused 4-bit dequantisation GEMV.
 *
 * TEST INFRASTRUCTURE ONLY.  This is a plain-C restatement of the reference's
 * host-side format definitions and CPU GEMV (QuantumDrizzy/int4-gemv,
 * src/kernels.cuh and src/int4_gemv.cu).  Only tests/, the smoke check in
 * __graft_entry__.py and the cpu_baseline / reference legs of bench.py may
 * load it.  The shipped library (int4-gemv_b200/) never links or calls it.
 *
 * Parity pin: tests/test_oracle.py checks every function here bit-exactly
 * against the reference's own host code compiled in place (oracle/_ref/,
 * built by oracle/ref/Makefile) and against the committed fixtures in
 * tests/golden/, which that compiled reference generated.
 *
 * Formats (identical bytes to the reference):
 *   packed : uint32 [out_f][in_f/8], code of column k sits in word k/8 at
 *            nibble k%8 (low nibble first)                 kernels.cuh:289
 *   INT4   : fp16 scale per (row, group of 128 columns)     kernels.cuh:12,282
 *   NF4    : fp32 absmax per (row, block of 64 columns)     kernels.cuh:85,322
 */
#ifndef B4_ORACLE_H
#define B4_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B4O_GROUP 128     /* INT4 group size, kernels.cuh:12      */
#define B4O_NF4_BLOCK 64  /* NF4 block size,  kernels.cuh:85      */

/* The 16-entry NormalFloat code table, kernels.cuh:78-83 / :301-306. */
extern const float b4o_nf4_table[16];

/* IEEE binary16 conversions with round-to-nearest-even (the semantics of
 * __float2half / __half2float used by kernels.cuh:282-283). */
uint16_t b4o_half_from_float(float f);
float b4o_float_from_half(uint16_t h);

/* INT4 g128 quantiser, kernels.cuh:268-297.  deq may be NULL. */
void b4o_quantise_int4(const float* W, int out_f, int in_f, uint32_t* packed,
                       uint16_t* scales, float* deq);

/* NF4 b64 quantiser, kernels.cuh:308-339.  deq may be NULL. */
void b4o_quantise_nf4(const float* W, int out_f, int in_f, uint32_t* packed,
                      float* absmax, float* deq);

/* Codes as one byte per column, [out_f][in_f]. */
void b4o_unpack_codes(const uint32_t* packed, int out_f, int in_f, uint8_t* codes);

/* W_dequant reconstruction from packed buffers (the values the reference's
 * quantisers return in `deq`, and that its kernels form in registers,
 * kernels.cuh:50 and :121). */
void b4o_dequant_int4(const uint32_t* packed, const uint16_t* scales, int out_f,
                      int in_f, float* deq);
void b4o_dequant_nf4(const uint32_t* packed, const float* absmax, int out_f,
                     int in_f, float* deq);

/* The reference's CPU GEMV: fp32 accumulation in column order over the
 * dequantised matrix, int4_gemv.cu:33-38.  x is fp32. */
void b4o_gemv_deq_f32(const float* deq, const float* x, int out_f, int in_f, float* y);

/* The same loop with rows spread over nthreads host threads (<= 0: all online
 * cores); each row's sum is still the reference's sequential fp32 sum.
 * Returns the number of threads used. */
int b4o_gemv_deq_f32_mt(const float* deq, const float* x, int out_f, int in_f, float* y,
                        int nthreads);

/* Double-precision GEMV over the dequantised weights and fp16 x, the parity
 * reference for y.  X is [m][in_f] binary16 bits, Y is [m][out_f]. */
void b4o_gemv_int4_f64(const uint32_t* packed, const uint16_t* scales, const uint16_t* X,
                       int out_f, int in_f, int m, double* Y);
void b4o_gemv_nf4_f64(const uint32_t* packed, const float* absmax, const uint16_t* X,
                      int out_f, int in_f, int m, double* Y);

/* Fused CPU GEMV straight from the packed codes with the reference kernels'
 * per-lane arithmetic (kernels.cuh:44-59 INT4, :108-129 NF4): lane L of 32
 * accumulates words L, L+32, ... with fmaf in column order, then the 16/8/4/
 * 2/1 shuffle tree.  Rows are spread over nthreads host threads (<=0: all
 * online cores).  X is [m][in_f] binary16 bits, Y is [m][out_f].  Returns the
 * number of threads used. */
int b4o_gemv_int4_fused(const uint32_t* packed, const uint16_t* scales, const uint16_t* X,
                        int out_f, int in_f, int m, float* Y, int nthreads);
int b4o_gemv_nf4_fused(const uint32_t* packed, const float* absmax, const uint16_t* X,
                       int out_f, int in_f, int m, float* Y, int nthreads);

/* max_r |got - ref| / max_r |ref|, int4_gemv.cu:74-81 (computed in double). */
double b4o_rel_err(const float* got, const double* ref, int n);

#ifdef __cplusplus
}
#endif
#endif
