/*
 * smk_oracle.c — TEST INFRASTRUCTURE ONLY: CPU restatement of the reference's
 * decode-GEMV path. See smk_oracle.h for what each function restates and
 * where. Built by oracle/Makefile with -ffp-contract=off (every FP step
 * rounds on its own, as in the reference's scalar unit) and OpenMP over rows
 * (rows are independent, so results do not depend on the thread count).
 */
#include "smk_oracle.h"

#include <float.h>
#include <math.h>
#include <stdint.h>
#include <string.h>

#define QK 32 /* values per block, q4_0.hpp:44 / q8_0.hpp:29 */
#define Q4_BYTES 18
#define Q8_BYTES 34

static uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static int is_finite_bits(float f) { return (f2u(f) & 0x7f800000u) != 0x7f800000u; }

/* binary16 by integer rounding: the float is m·2^(e−150) (e the biased
 * exponent, 1 for subnormals); the half with unbiased exponent Eh >= −14 has
 * ulp 2^(Eh−10), so the value is m·2^−s half ulps with s = 140 + Eh − e,
 * rounded to nearest even. ((Eh+15) << 10) + q − 1024 is then the half's bit
 * pattern for every q (a carry to 2048 moves into the exponent, and Eh = −14
 * gives the subnormals), and patterns at or past 0x7c00 overflowed. */
uint16_t smko_fp32_to_fp16(float f) {
    const uint32_t u = f2u(f);
    const uint16_t sign = (uint16_t)((u >> 16) & 0x8000u);
    const uint32_t a = u & 0x7fffffffu;
    if (a > 0x7f800000u) return sign | 0x7e00u;
    if (a == 0x7f800000u) return sign | 0x7c00u;
    int e = (int)(a >> 23);
    uint32_t m = a & 0x7fffffu;
    if (e == 0) e = 1; else m |= 0x800000u;
    const int E = e - 127;
    const int Eh = E < -14 ? -14 : E;
    const int s = 140 + Eh - e;
    uint32_t q;
    if (s > 31) {
        q = 0;
    } else {
        q = m >> s;
        const uint32_t rem = m & ((1u << s) - 1u), half = 1u << (s - 1);
        if (rem > half || (rem == half && (q & 1u))) ++q;
    }
    const int64_t bits = ((int64_t)(Eh + 15) << 10) + (int64_t)q - 1024;
    if (bits >= 0x7c00) return sign | 0x7c00u;
    return sign | (uint16_t)bits;
}

float smko_fp16_to_fp32(uint16_t h) {
    const int exp = (h >> 10) & 0x1f, man = h & 0x3ff;
    const int neg = (h & 0x8000) != 0;
    float v;
    if (exp == 0x1f) v = man ? u2f(0x7fc00000u | ((uint32_t)man << 13)) : INFINITY;
    else if (exp == 0) v = ldexpf((float)man, -24);
    else v = ldexpf((float)(1024 + man), exp - 25);
    return neg ? -v : v;
}

void smko_fp32_to_fp16_n(const float* in, uint16_t* out, int64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) out[i] = smko_fp32_to_fp16(in[i]);
}

/* ---- quantizers ----------------------------------------------------------- */

/* One Q4_0 block (q4_0_scalar.cpp:33-60): the first value of largest
 * magnitude keeps its sign, d = max / −8, id = 1/d (0 when d == 0 or 1/d
 * overflows), q = min(15, trunc(w·id + 8.5)); byte j = q[j] | q[16+j] << 4. */
static int q4_block(const float* w, uint8_t* blk) {
    float amax = 0.0f, mx = 0.0f;
    int finite = 1;
    for (int j = 0; j < QK; ++j) {
        finite &= is_finite_bits(w[j]);
        if (amax < fabsf(w[j])) { amax = fabsf(w[j]); mx = w[j]; }
    }
    if (!finite) return 0;
    const float d = mx / -8.0f;
    float id = d != 0.0f ? 1.0f / d : 0.0f;
    if (!(fabsf(id) <= FLT_MAX)) id = 0.0f;
    const uint16_t h = smko_fp32_to_fp16(d);
    if ((h & 0x7fffu) == 0x7c00u) return 0;
    blk[0] = (uint8_t)(h & 0xff);
    blk[1] = (uint8_t)(h >> 8);
    for (int j = 0; j < QK / 2; ++j) {
        const float t0 = w[j] * id + 8.5f, t1 = w[QK / 2 + j] * id + 8.5f;   /* two roundings each */
        int q0 = (int)t0, q1 = (int)t1;
        if (q0 > 15) q0 = 15;
        if (q1 > 15) q1 = 15;
        blk[2 + j] = (uint8_t)(q0 | (q1 << 4));
    }
    return 1;
}

/* One Q8 block (q8_0_scalar.cpp:45-61): d = amax / 127, id = 1/d (0 when
 * d == 0 or 1/d overflows), q = roundf(w·id), half away from zero. */
static int q8_block(const float* w, int8_t* q, float* d_out) {
    float amax = 0.0f;
    int finite = 1;
    for (int j = 0; j < QK; ++j) {
        finite &= is_finite_bits(w[j]);
        if (fabsf(w[j]) > amax) amax = fabsf(w[j]);
    }
    if (!finite) return 0;
    const float d = amax / 127.0f;
    float id = d != 0.0f ? 1.0f / d : 0.0f;
    if (!(id <= FLT_MAX)) id = 0.0f;
    for (int j = 0; j < QK; ++j) q[j] = (int8_t)roundf(w[j] * id);
    *d_out = d;
    return 1;
}

int smko_quantize_q4_0(const float* W, int64_t N, int K, uint8_t* out) {
    const int nb = K / QK;
    int ok = 1;
#pragma omp parallel for schedule(static) reduction(& : ok)
    for (int64_t n = 0; n < N; ++n)
        for (int b = 0; b < nb; ++b)
            ok &= q4_block(W + n * K + (int64_t)QK * b, out + (n * nb + b) * Q4_BYTES);
    return ok;
}

int smko_quantize_q8_0(const float* W, int64_t N, int K, uint8_t* out) {
    const int nb = K / QK;
    int ok = 1;
#pragma omp parallel for schedule(static) reduction(& : ok)
    for (int64_t n = 0; n < N; ++n)
        for (int b = 0; b < nb; ++b) {
            uint8_t* blk = out + (n * nb + b) * Q8_BYTES;
            float d = 0.0f;
            if (!q8_block(W + n * K + (int64_t)QK * b, (int8_t*)(blk + 2), &d)) { ok = 0; continue; }
            const uint16_t h = smko_fp32_to_fp16(d);
            if ((h & 0x7fffu) == 0x7c00u) { ok = 0; continue; }
            blk[0] = (uint8_t)(h & 0xff);
            blk[1] = (uint8_t)(h >> 8);
        }
    return ok;
}

int smko_quantize_x_q8(const float* x, int K, int8_t* qs, float* dx) {
    for (int b = 0; b < K / QK; ++b)
        if (!q8_block(x + QK * b, qs + QK * b, dx + b)) return 0;
    return 1;
}

/* ---- integer block sums --------------------------------------------------- */

static int32_t q4_isum(const uint8_t* blk, const int8_t* p) {
    int32_t s = 0;
    for (int j = 0; j < QK / 2; ++j)
        s += ((blk[2 + j] & 0x0f) - 8) * p[j] + ((blk[2 + j] >> 4) - 8) * p[QK / 2 + j];
    return s;
}

static int32_t q8_isum(const uint8_t* blk, const int8_t* p) {
    const int8_t* q = (const int8_t*)(blk + 2);
    int32_t s = 0;
    for (int i = 0; i < QK; ++i) s += q[i] * p[i];
    return s;
}

static float blk_scale(const uint8_t* blk) { return smko_fp16_to_fp32((uint16_t)(blk[0] | (blk[1] << 8))); }

void smko_block_sums_q4_0(int N, int K, const int8_t* xq, const uint8_t* Wq, int32_t* out) {
    const int nb = K / QK;
#pragma omp parallel for schedule(static)
    for (int n = 0; n < N; ++n)
        for (int b = 0; b < nb; ++b)
            out[(int64_t)n * nb + b] = q4_isum(Wq + ((int64_t)n * nb + b) * Q4_BYTES, xq + QK * b);
}

void smko_block_sums_q8_0(int N, int K, const int8_t* xq, const uint8_t* Wq, int32_t* out) {
    const int nb = K / QK;
#pragma omp parallel for schedule(static)
    for (int n = 0; n < N; ++n)
        for (int b = 0; b < nb; ++b)
            out[(int64_t)n * nb + b] = q8_isum(Wq + ((int64_t)n * nb + b) * Q8_BYTES, xq + QK * b);
}

/* ---- GEMV, scalar-table order ----------------------------------------------- */

typedef int32_t (*isum_fn)(const uint8_t*, const int8_t*);

/* The driver (q8_0_scalar.cpp:120-166) around the scalar rows
 * (q4_0_scalar.cpp:82-99, q8_0_scalar.cpp:170-186). */
static void gemv_scalar(int N, int K, const float* x, const uint8_t* Wq, float* y, int bytes, isum_fn isum) {
    if (N <= 0) return;
    if (K <= 0) { for (int n = 0; n < N; ++n) y[n] = 0.0f; return; }
    const int nb = K / QK;
    int8_t qs[K];
    float dx[nb];
    if (!smko_quantize_x_q8(x, K, qs, dx)) {
        for (int n = 0; n < N; ++n) y[n] = NAN;
        return;
    }
#pragma omp parallel for schedule(static)
    for (int n = 0; n < N; ++n) {
        const uint8_t* blk = Wq + (int64_t)n * nb * bytes;
        float acc = 0.0f;
        for (int b = 0; b < nb; ++b, blk += bytes) {
            const float s = blk_scale(blk) * dx[b];
            acc = acc + (float)isum(blk, qs + QK * b) * s;
        }
        y[n] = acc;
    }
}

void smko_gemv_q4_0(int N, int K, const float* x, const uint8_t* Wq, float* y) {
    gemv_scalar(N, K, x, Wq, y, Q4_BYTES, q4_isum);
}

void smko_gemv_q8_0(int N, int K, const float* x, const uint8_t* Wq, float* y) {
    gemv_scalar(N, K, x, Wq, y, Q8_BYTES, q8_isum);
}

/* ---- float64 references --------------------------------------------------- */

static void ref64(int N, int K, const int8_t* xq, const float* dx, const uint8_t* Wq, double* y64, double* mag,
                  int bytes, int q4) {
    const int nb = K / QK;
#pragma omp parallel for schedule(static)
    for (int n = 0; n < N; ++n) {
        double r = 0.0, m = 0.0;
        for (int b = 0; b < nb; ++b) {
            const uint8_t* blk = Wq + ((int64_t)n * nb + b) * bytes;
            const int8_t* p = xq + QK * b;
            int64_t s = 0, a = 0;
            for (int i = 0; i < QK; ++i) {
                int w;
                if (q4) w = (i < QK / 2 ? (blk[2 + i] & 0x0f) : (blk[2 + i - QK / 2] >> 4)) - 8;
                else w = ((const int8_t*)(blk + 2))[i];
                const int64_t pr = (int64_t)w * p[i];
                s += pr;
                a += pr < 0 ? -pr : pr;
            }
            const double sc = (double)blk_scale(blk) * (double)dx[b];   /* exact: 11 × 24 bits */
            r += sc * (double)s;
            m += fabs(sc) * (double)a;
        }
        y64[n] = r;
        mag[n] = m;
    }
}

void smko_ref64_q4_0(int N, int K, const int8_t* xq, const float* dx, const uint8_t* Wq, double* y64,
                     double* mag) {
    ref64(N, K, xq, dx, Wq, y64, mag, Q4_BYTES, 1);
}

void smko_ref64_q8_0(int N, int K, const int8_t* xq, const float* dx, const uint8_t* Wq, double* y64,
                     double* mag) {
    ref64(N, K, xq, dx, Wq, y64, mag, Q8_BYTES, 0);
}

/* ---- dense ---------------------------------------------------------------- */

static float load_kind(const void* base, int kind, int64_t i) {
    if (kind == 0) return ((const float*)base)[i];
    const uint16_t h = ((const uint16_t*)base)[i];
    if (kind == 1) return smko_fp16_to_fp32(h);
    return u2f((uint32_t)h << 16);
}

void smko_dense_ref64(int M, int N, int K, const void* A, int a_kind, const void* B, int b_kind, double* y64,
                      double* mag) {
#pragma omp parallel for schedule(static) collapse(2)
    for (int i = 0; i < M; ++i)
        for (int j = 0; j < N; ++j) {
            double r = 0.0, m = 0.0;
            for (int p = 0; p < K; ++p) {
                const double t = (double)load_kind(A, a_kind, (int64_t)i * K + p) *
                                 (double)load_kind(B, b_kind, (int64_t)j * K + p);   /* exact */
                r += t;
                m += fabs(t);
            }
            y64[(int64_t)i * N + j] = r;
            mag[(int64_t)i * N + j] = m;
        }
}

void smko_dense_scalar(int M, int N, int K, float alpha, const void* A, int a_kind, const void* B, int b_kind,
                       float beta, float* C) {
    if (M <= 0 || N <= 0 || K < 0) return;
    for (int64_t i = 0; i < (int64_t)M * N; ++i) C[i] = beta == 0.0f ? 0.0f : (beta == 1.0f ? C[i] : beta * C[i]);
    if (K == 0) return;
#pragma omp parallel for schedule(static) collapse(2)
    for (int i = 0; i < M; ++i)
        for (int j = 0; j < N; ++j) {
            float acc = 0.0f;
            for (int p = 0; p < K; ++p)
                acc = acc + load_kind(A, a_kind, (int64_t)i * K + p) * load_kind(B, b_kind, (int64_t)j * K + p);
            C[(int64_t)i * N + j] = C[(int64_t)i * N + j] + alpha * acc;
        }
}

void smko_gemv_slice(int N, int t, int parts, int* lo, int* hi) {
    const int64_t groups = ((int64_t)N + 7) / 8;
    int64_t a = groups * t / parts * 8, b = groups * (t + 1) / parts * 8;
    *lo = (int)(a < N ? a : N);
    *hi = (int)(b < N ? b : N);
}

/* B element (row k, column j) of op(B). */
static int64_t u8s8_b(int trans_b, const int8_t* B, int ldb, int k, int j) {
    return trans_b ? (int64_t)B[(int64_t)j * ldb + k] : (int64_t)B[(int64_t)k * ldb + j];
}

void smko_sgemm_u8s8(int trans_b, int M, int N, int K, const uint8_t* A, int lda, int a_zero_point,
                     const int8_t* B, int ldb, float a_scale, const float* b_scales, float* C, int ldc) {
    if (M <= 0 || N <= 0 || K < 0) return;
#pragma omp parallel for schedule(static) collapse(2)
    for (int i = 0; i < M; ++i)
        for (int j = 0; j < N; ++j) {
            int64_t acc = 0;
            for (int k = 0; k < K; ++k)
                acc += ((int64_t)A[(int64_t)i * lda + k] - a_zero_point) * u8s8_b(trans_b, B, ldb, k, j);
            const double s = (double)a_scale * (double)b_scales[j];   /* exact: two 24-bit significands */
            C[(int64_t)i * ldc + j] = (float)(s * (double)acc);
        }
}

void smko_u8s8_ref64(int trans_b, int M, int N, int K, const uint8_t* A, int a_zero_point, const int8_t* B,
                     double* sum64, double* mag) {
    const int ldb = trans_b ? K : N;
#pragma omp parallel for schedule(static) collapse(2)
    for (int i = 0; i < M; ++i)
        for (int j = 0; j < N; ++j) {
            int64_t acc = 0, m = 0;
            for (int k = 0; k < K; ++k) {
                const int64_t a = (int64_t)A[(int64_t)i * K + k] - a_zero_point, b = u8s8_b(trans_b, B, ldb, k, j);
                acc += a * b;
                m += (a < 0 ? -a : a) * (b < 0 ? -b : b);
            }
            sum64[(int64_t)i * N + j] = (double)acc;
            mag[(int64_t)i * N + j] = (double)m;
        }
}
