/*
 * smk_oracle.h — TEST INFRASTRUCTURE ONLY: the CPU restatement of the
 * reference's decode-GEMV path (Mattral/simd-ml-kernels 0.3.0), used as the
 * checker of the parity tests (tests/), of __graft_entry__.smoke() and as the
 * "port" CPU baseline of bench.py. The shipped package never links, loads or
 * calls it.
 *
 * Pinned against the reference itself: tests/golden/make_golden.py runs the
 * reference (oracle/_ref, compiled from its sources) on seeded inputs and the
 * llama.cpp fixture the reference's tests hold; tests/test_oracle_golden.py
 * checks this restatement against those vectors byte for byte (quantizers,
 * x-quantization) and bit for bit (scalar-order GEMV outputs).
 *
 * File:line citations are into the reference tree.
 */
#ifndef SMK_ORACLE_H
#define SMK_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* binary32 -> binary16, round to nearest even; NaN -> 0x7e00 | sign
 * (src/kernels/quant/q8_0_scalar.cpp:65-83). */
uint16_t smko_fp32_to_fp16(float f);
/* binary16 -> binary32, exact (q8_0_scalar.cpp:85-94). */
float smko_fp16_to_fp32(uint16_t h);
/* Round-trip helpers over arrays (for the exhaustive conversion test). */
void smko_fp32_to_fp16_n(const float* in, uint16_t* out, int64_t n);

/* ggml quantize_row_q4_0_ref per row, W [N, K] -> N·K/32 blocks of 18 bytes.
 * Returns 1, or 0 on NaN/Inf input or a binary16-overflowing scale
 * (q4_0_scalar.cpp:26-78, q4_0.hpp:54-60). */
int smko_quantize_q4_0(const float* W, int64_t N, int K, uint8_t* out);
/* ggml quantize_row_q8_0_ref per row, 34-byte blocks (q8_0_scalar.cpp:36-61,96-111). */
int smko_quantize_q8_0(const float* W, int64_t N, int K, uint8_t* out);
/* x [K] -> K int8 quants + K/32 fp32 scales; 0 on NaN/Inf (q8_0_scalar.cpp:113-118). */
int smko_quantize_x_q8(const float* x, int K, int8_t* qs, float* dx);

/* The reference's scalar table, same FP32 operation order
 * (q4_0_scalar.cpp:82-105, q8_0_scalar.cpp:170-192, driver q8_0_scalar.cpp:120-166):
 * y[n] = ((0 + p_0) + p_1) + ..., p_b = float(isum_b) · (fp16(dw_b) · dx_b). */
void smko_gemv_q4_0(int N, int K, const float* x, const uint8_t* Wq, float* y);
void smko_gemv_q8_0(int N, int K, const float* x, const uint8_t* Wq, float* y);

/* Per-block exact integer sums isum[n][b] of the quantized operands
 * (q4_0_scalar.cpp:91-95: Σ (q − 8)·qx; q8_0_scalar.cpp:179-183: Σ qw·qx). */
void smko_block_sums_q4_0(int N, int K, const int8_t* xq, const uint8_t* Wq, int32_t* out);
void smko_block_sums_q8_0(int N, int K, const int8_t* xq, const uint8_t* Wq, int32_t* out);

/* The float64 result of the same quantized operands and the magnitude of the
 * reference's error bound, Σ_b |dw_b·dx_b|·Σ_i |qw·qx| (python/simd_ml_kernels/
 * _cli.py:157-189, q4_0.hpp:23-30). Row sums in int64. */
void smko_ref64_q4_0(int N, int K, const int8_t* xq, const float* dx, const uint8_t* Wq, double* y64,
                     double* mag);
void smko_ref64_q8_0(int N, int K, const int8_t* xq, const float* dx, const uint8_t* Wq, double* y64,
                     double* mag);

/* Dense x·Wᵀ: element kinds 0 = float32, 1 = IEEE binary16, 2 = bfloat16.
 * y64 = Σ_k x·w in float64 and mag = Σ_k |x·w| (the bound's |A||W|ᵀ,
 * tests/test_precision.py:212-221). A [M, K], B [N, K], y [M, N]. */
void smko_dense_ref64(int M, int N, int K, const void* A, int a_kind, const void* B, int b_kind, double* y64,
                      double* mag);
/* The scalar table's trans_b GEMM order (src/kernels/scalar_kernels.cpp:69-84):
 * C = fl(beta·C) (C zeroed when beta == 0) then c += alpha·(sequential fp32 sum). */
void smko_dense_scalar(int M, int N, int K, float alpha, const void* A, int a_kind, const void* B, int b_kind,
                       float beta, float* C);

/* sgemm_u8s8 as the reference's scalar table (src/kernels/scalar_kernels.cpp:148-170,
 * contract src/kernels/gemm/int8_gemm.hpp:5-26): acc[i][j] = Σ_k (A[i][k] − zp)·op(B)[k][j]
 * exactly in int64, then C[i][j] = float(double(a_scale)·b_scales[j]·double(acc)).
 * trans_b: B [N, ldb] (ldb ≥ K); else B [K, ldb] (ldb ≥ N). A [M, lda], C [M, ldc]. */
void smko_sgemm_u8s8(int trans_b, int M, int N, int K, const uint8_t* A, int lda, int a_zero_point,
                     const int8_t* B, int ldb, float a_scale, const float* b_scales, float* C, int ldc);
/* The exact sums and the magnitude of the documented bound,
 * Σ_k |A − zp|·|op(B)| (int8_gemm.hpp:23-24), both in float64 (exact below 2^53). */
void smko_u8s8_ref64(int trans_b, int M, int N, int K, const uint8_t* A, int a_zero_point, const int8_t* B,
                     double* sum64, double* mag);

/* Row slice [lo, hi) of part t of `parts` in whole 8-row groups
 * (src/dispatch/dispatch.cpp:373-379, kGemvRowGroup = 8). */
void smko_gemv_slice(int N, int t, int parts, int* lo, int* hi);

#ifdef __cplusplus
}
#endif

#endif
