/*
 * b4_oracle.c -- CPU oracle for the fused 4-bit dequantisation GEMV.
 *
 * TEST INFRASTRUCTURE ONLY (see b4_oracle.h).  A restatement in plain C of the
 * reference's host-side semantics, written from its documented behaviour;
 * each function names the reference lines it follows.  Never linked into the
 * shipped library.
 */
#define _GNU_SOURCE
#include "b4_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

/* kernels.cuh:78-83 and :301-306 (the same 16 literals on both sides). */
const float b4o_nf4_table[16] = {
    -1.0f,                 -0.6961928009986877f,  -0.5250730514526367f,
    -0.39491748809814453f, -0.28444138169288635f, -0.18477343022823334f,
    -0.09105003625154495f, 0.0f,                  0.07958029955625534f,
    0.16093020141124725f,  0.24611230194568634f,  0.33791524171829224f,
    0.44070982933044434f,  0.5626170039176941f,   0.7229568362236023f,
    1.0f};

static uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* binary32 -> binary16, round to nearest even, overflow to infinity, NaN to
 * the canonical 0x7fff with the input's sign dropped.  The quantiser only ever
 * converts amax/7 >= 0 (kernels.cuh:281-282), so NaN never reaches it. */
uint16_t b4o_half_from_float(float f)
{
    const uint32_t x = f2u(f);
    const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    const uint32_t a = x & 0x7fffffffu;
    if (a > 0x7f800000u) return 0x7fffu;                  /* NaN            */
    if (a >= 0x477ff000u) return sign | 0x7c00u;          /* >= 65520 -> inf */
    if (a >= 0x38800000u) {                               /* normal half     */
        const uint32_t r = a + 0xfffu + ((a >> 13) & 1u);
        return (uint16_t)(sign | ((r - 0x38000000u) >> 13));
    }
    const int e = (int)(a >> 23);
    if (e < 102) return sign;                             /* < 2^-25 -> 0    */
    const uint32_t m = (a & 0x7fffffu) | 0x800000u;       /* 24-bit significand */
    const int shift = 126 - e;                            /* 14..24          */
    uint32_t h = m >> shift;
    const uint32_t rem = m & ((1u << shift) - 1u);
    const uint32_t halfway = 1u << (shift - 1);
    if (rem > halfway || (rem == halfway && (h & 1u))) ++h;
    return (uint16_t)(sign | h);
}

float b4o_float_from_half(uint16_t h)
{
    const uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1fu;
    uint32_t m = h & 0x3ffu;
    if (e == 0x1f) return u2f(sign | 0x7f800000u | (m << 13));
    if (e == 0) {
        if (m == 0) return u2f(sign);
        int ee = 113;                       /* normalise the subnormal */
        while (!(m & 0x400u)) { m <<= 1; --ee; }
        return u2f(sign | ((uint32_t)ee << 23) | ((m & 0x3ffu) << 13));
    }
    return u2f(sign | ((e + 112u) << 23) | (m << 13));
}

/* (int)std::lround(q) as the reference writes it (kernels.cuh:286).  lround of
 * a float rounds half away from zero; glibc on x86-64 returns LONG_MIN for a
 * NaN, an infinity or a value beyond the range of long, and the (int) cast
 * keeps the low 32 bits, which for LONG_MIN are 0.  A quotient is non-finite
 * only when the fp16 scale rounded to 0 or to infinity. */
static int lround_int(float q)
{
    if (!(fabsf(q) < 0x1p63f)) return 0;
    const long l = lroundf(q);
    return (int)(int32_t)(uint32_t)(unsigned long)l;
}

/* kernels.cuh:268-297 */
void b4o_quantise_int4(const float* W, int out_f, int in_f, uint32_t* packed,
                       uint16_t* scales, float* deq)
{
    const int groups = in_f / B4O_GROUP;
    const int words = in_f / 8;
    memset(packed, 0, (size_t)out_f * words * sizeof(uint32_t));
    for (int r = 0; r < out_f; ++r) {
        for (int g = 0; g < groups; ++g) {
            const size_t off = (size_t)r * in_f + (size_t)g * B4O_GROUP;
            float amax = 0.0f;
            for (int i = 0; i < B4O_GROUP; ++i) {
                const float a = fabsf(W[off + i]);
                amax = (amax < a) ? a : amax;             /* std::max(amax, a) */
            }
            const float s = (amax > 0.0f) ? amax / 7.0f : 1.0f;
            const uint16_t sh = b4o_half_from_float(s);
            scales[(size_t)r * groups + g] = sh;
            const float s_used = b4o_float_from_half(sh);
            for (int i = 0; i < B4O_GROUP; ++i) {
                int code = lround_int(W[off + i] / s_used) + 8;
                code = code < 0 ? 0 : (code > 15 ? 15 : code);
                const int idx = g * B4O_GROUP + i;
                packed[(size_t)r * words + idx / 8] |= (uint32_t)code << ((idx % 8) * 4);
                if (deq) deq[off + i] = (float)(code - 8) * s_used;
            }
        }
    }
}

/* kernels.cuh:308-339 */
void b4o_quantise_nf4(const float* W, int out_f, int in_f, uint32_t* packed,
                      float* absmax, float* deq)
{
    const int blocks = in_f / B4O_NF4_BLOCK;
    const int words = in_f / 8;
    memset(packed, 0, (size_t)out_f * words * sizeof(uint32_t));
    for (int r = 0; r < out_f; ++r) {
        for (int b = 0; b < blocks; ++b) {
            const size_t off = (size_t)r * in_f + (size_t)b * B4O_NF4_BLOCK;
            float amax = 0.0f;
            for (int i = 0; i < B4O_NF4_BLOCK; ++i) {
                const float a = fabsf(W[off + i]);
                amax = (amax < a) ? a : amax;
            }
            if (amax == 0.0f) amax = 1.0f;
            absmax[(size_t)r * blocks + b] = amax;
            for (int i = 0; i < B4O_NF4_BLOCK; ++i) {
                const float norm = W[off + i] / amax;
                int best = 0;
                float bd = fabsf(norm - b4o_nf4_table[0]);
                for (int c = 1; c < 16; ++c) {              /* strict <: ties keep the lower code */
                    const float d = fabsf(norm - b4o_nf4_table[c]);
                    if (d < bd) { bd = d; best = c; }
                }
                const int idx = b * B4O_NF4_BLOCK + i;
                packed[(size_t)r * words + idx / 8] |= (uint32_t)best << ((idx % 8) * 4);
                if (deq) deq[off + i] = b4o_nf4_table[best] * amax;
            }
        }
    }
}

void b4o_unpack_codes(const uint32_t* packed, int out_f, int in_f, uint8_t* codes)
{
    const int words = in_f / 8;
    for (int r = 0; r < out_f; ++r)
        for (int k = 0; k < in_f; ++k)
            codes[(size_t)r * in_f + k] =
                (uint8_t)((packed[(size_t)r * words + k / 8] >> ((k % 8) * 4)) & 0xfu);
}

/* (code - 8) * float(half(s)), kernels.cuh:50 and :290 */
void b4o_dequant_int4(const uint32_t* packed, const uint16_t* scales, int out_f,
                      int in_f, float* deq)
{
    const int words = in_f / 8, groups = in_f / B4O_GROUP;
    for (int r = 0; r < out_f; ++r)
        for (int k = 0; k < in_f; ++k) {
            const int code = (packed[(size_t)r * words + k / 8] >> ((k % 8) * 4)) & 0xf;
            const float s = b4o_float_from_half(scales[(size_t)r * groups + k / B4O_GROUP]);
            deq[(size_t)r * in_f + k] = (float)(code - 8) * s;
        }
}

/* NF4[code] * absmax, kernels.cuh:121 and :331 */
void b4o_dequant_nf4(const uint32_t* packed, const float* absmax, int out_f,
                     int in_f, float* deq)
{
    const int words = in_f / 8, blocks = in_f / B4O_NF4_BLOCK;
    for (int r = 0; r < out_f; ++r)
        for (int k = 0; k < in_f; ++k) {
            const int code = (packed[(size_t)r * words + k / 8] >> ((k % 8) * 4)) & 0xf;
            deq[(size_t)r * in_f + k] =
                b4o_nf4_table[code] * absmax[(size_t)r * blocks + k / B4O_NF4_BLOCK];
        }
}

/* int4_gemv.cu:33-38: a float accumulator, a += deq * x in column order. */
void b4o_gemv_deq_f32(const float* deq, const float* x, int out_f, int in_f, float* y)
{
    for (int r = 0; r < out_f; ++r) {
        float a = 0.0f;
        for (int i = 0; i < in_f; ++i) a += deq[(size_t)r * in_f + i] * x[i];
        y[r] = a;
    }
}

typedef struct {
    const float* deq; const float* x; int in_f; int r0, r1; float* y;
} deq_job;

static void* deq_worker(void* arg)
{
    const deq_job* j = (const deq_job*)arg;
    for (int r = j->r0; r < j->r1; ++r) {
        float a = 0.0f;
        const float* row = j->deq + (size_t)r * j->in_f;
        for (int i = 0; i < j->in_f; ++i) a += row[i] * j->x[i];
        j->y[r] = a;
    }
    return NULL;
}

int b4o_gemv_deq_f32_mt(const float* deq, const float* x, int out_f, int in_f, float* y,
                        int nthreads)
{
    if (nthreads <= 0) {
        const long n = sysconf(_SC_NPROCESSORS_ONLN);
        nthreads = n > 0 ? (int)n : 1;
    }
    if (nthreads > out_f) nthreads = out_f > 0 ? out_f : 1;
    deq_job* jobs = (deq_job*)calloc((size_t)nthreads, sizeof(deq_job));
    pthread_t* th = (pthread_t*)calloc((size_t)nthreads, sizeof(pthread_t));
    for (int t = 0; t < nthreads; ++t) {
        jobs[t].deq = deq; jobs[t].x = x; jobs[t].in_f = in_f; jobs[t].y = y;
        jobs[t].r0 = (int)((long long)out_f * t / nthreads);
        jobs[t].r1 = (int)((long long)out_f * (t + 1) / nthreads);
    }
    for (int t = 1; t < nthreads; ++t) pthread_create(&th[t], NULL, deq_worker, &jobs[t]);
    deq_worker(&jobs[0]);
    for (int t = 1; t < nthreads; ++t) pthread_join(th[t], NULL);
    free(th); free(jobs);
    return nthreads;
}

void b4o_gemv_int4_f64(const uint32_t* packed, const uint16_t* scales, const uint16_t* X,
                       int out_f, int in_f, int m, double* Y)
{
    const int words = in_f / 8, groups = in_f / B4O_GROUP;
    double* xd = (double*)malloc(sizeof(double) * (size_t)in_f);
    for (int b = 0; b < m; ++b) {
        for (int k = 0; k < in_f; ++k) xd[k] = b4o_float_from_half(X[(size_t)b * in_f + k]);
        for (int r = 0; r < out_f; ++r) {
            double acc = 0.0;
            for (int k = 0; k < in_f; ++k) {
                const int code = (packed[(size_t)r * words + k / 8] >> ((k % 8) * 4)) & 0xf;
                const float s = b4o_float_from_half(scales[(size_t)r * groups + k / B4O_GROUP]);
                acc += (double)((float)(code - 8) * s) * xd[k];
            }
            Y[(size_t)b * out_f + r] = acc;
        }
    }
    free(xd);
}

void b4o_gemv_nf4_f64(const uint32_t* packed, const float* absmax, const uint16_t* X,
                      int out_f, int in_f, int m, double* Y)
{
    const int words = in_f / 8, blocks = in_f / B4O_NF4_BLOCK;
    double* xd = (double*)malloc(sizeof(double) * (size_t)in_f);
    for (int b = 0; b < m; ++b) {
        for (int k = 0; k < in_f; ++k) xd[k] = b4o_float_from_half(X[(size_t)b * in_f + k]);
        for (int r = 0; r < out_f; ++r) {
            double acc = 0.0;
            for (int k = 0; k < in_f; ++k) {
                const int code = (packed[(size_t)r * words + k / 8] >> ((k % 8) * 4)) & 0xf;
                acc += (double)(b4o_nf4_table[code] * absmax[(size_t)r * blocks + k / B4O_NF4_BLOCK]) * xd[k];
            }
            Y[(size_t)b * out_f + r] = acc;
        }
    }
    free(xd);
}

/* ---- fused CPU GEMV with the reference kernels' per-lane arithmetic ------ */

/* Lane sums closed by __shfl_down_sync with offsets 16, 8, 4, 2, 1
 * (kernels.cuh:57-59): only lane 0's result is kept. */
static float shuffle_tree(float* lane)
{
    for (int off = 16; off > 0; off >>= 1)
        for (int l = 0; l < off; ++l) lane[l] = lane[l] + lane[l + off];
    return lane[0];
}

typedef struct {
    int nf4;
    const uint32_t* packed;
    const void* scale;              /* uint16_t* (INT4) or float* (NF4) */
    const float* xf;                /* [m][in_f] fp32 copies of the fp16 x */
    int out_f, in_f, m;
    int r0, r1;
    float* Y;
} fused_job;

static void* fused_worker(void* arg)
{
    const fused_job* j = (const fused_job*)arg;
    const int words = j->in_f / 8;
    float lane[32];
    for (int b = 0; b < j->m; ++b) {
        const float* x = j->xf + (size_t)b * j->in_f;
        for (int r = j->r0; r < j->r1; ++r) {
            const uint32_t* wrow = j->packed + (size_t)r * words;
            for (int l = 0; l < 32; ++l) {
                float acc = 0.0f;
                for (int w = l; w < words; w += 32) {
                    const uint32_t p = wrow[w];
                    const int base = w * 8;
                    if (!j->nf4) {        /* kernels.cuh:44-55 */
                        const uint16_t* srow = (const uint16_t*)j->scale + (size_t)r * (j->in_f / B4O_GROUP);
                        const float s = b4o_float_from_half(srow[base / B4O_GROUP]);
                        for (int k = 0; k < 8; ++k) {
                            const int code = (p >> (k * 4)) & 0xf;
                            acc = fmaf((float)(code - 8) * s, x[base + k], acc);
                        }
                    } else {              /* kernels.cuh:111-125 */
                        const float* arow = (const float*)j->scale + (size_t)r * (j->in_f / B4O_NF4_BLOCK);
                        const float s = arow[w >> 3];
                        for (int k = 0; k < 8; ++k) {
                            const int code = (p >> (k * 4)) & 0xf;
                            acc = fmaf(b4o_nf4_table[code] * s, x[base + k], acc);
                        }
                    }
                }
                lane[l] = acc;
            }
            j->Y[(size_t)b * j->out_f + r] = shuffle_tree(lane);
        }
    }
    return NULL;
}

static int fused_run(int nf4, const uint32_t* packed, const void* scale, const uint16_t* X,
                     int out_f, int in_f, int m, float* Y, int nthreads)
{
    if (nthreads <= 0) {
        const long n = sysconf(_SC_NPROCESSORS_ONLN);
        nthreads = n > 0 ? (int)n : 1;
    }
    if (nthreads > out_f) nthreads = out_f > 0 ? out_f : 1;
    float* xf = (float*)malloc(sizeof(float) * (size_t)m * in_f + 1);
    for (size_t i = 0; i < (size_t)m * in_f; ++i) xf[i] = b4o_float_from_half(X[i]);
    fused_job* jobs = (fused_job*)calloc((size_t)nthreads, sizeof(fused_job));
    pthread_t* th = (pthread_t*)calloc((size_t)nthreads, sizeof(pthread_t));
    for (int t = 0; t < nthreads; ++t) {
        fused_job* j = &jobs[t];
        j->nf4 = nf4; j->packed = packed; j->scale = scale; j->xf = xf;
        j->out_f = out_f; j->in_f = in_f; j->m = m; j->Y = Y;
        j->r0 = (int)((long long)out_f * t / nthreads);
        j->r1 = (int)((long long)out_f * (t + 1) / nthreads);
    }
    for (int t = 1; t < nthreads; ++t) pthread_create(&th[t], NULL, fused_worker, &jobs[t]);
    fused_worker(&jobs[0]);
    for (int t = 1; t < nthreads; ++t) pthread_join(th[t], NULL);
    free(th); free(jobs); free(xf);
    return nthreads;
}

int b4o_gemv_int4_fused(const uint32_t* packed, const uint16_t* scales, const uint16_t* X,
                        int out_f, int in_f, int m, float* Y, int nthreads)
{
    return fused_run(0, packed, scales, X, out_f, in_f, m, Y, nthreads);
}

int b4o_gemv_nf4_fused(const uint32_t* packed, const float* absmax, const uint16_t* X,
                       int out_f, int in_f, int m, float* Y, int nthreads)
{
    return fused_run(1, packed, absmax, X, out_f, in_f, m, Y, nthreads);
}

double b4o_rel_err(const float* got, const double* ref, int n)
{
    double max_err = 0.0, scale = 0.0;
    for (int i = 0; i < n; ++i) {
        const double e = fabs((double)got[i] - ref[i]);
        if (e > max_err || e != e) max_err = e;
        const double a = fabs(ref[i]);
        if (a > scale) scale = a;
    }
    return scale > 0.0 ? max_err / scale : max_err;
}
