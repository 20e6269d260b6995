// ref_glue.cpp — TEST INFRASTRUCTURE ONLY (never linked into the product).
//
// A C ABI over the reference library (Mattral/simd-ml-kernels), which the
// Makefile in this directory compiles from its own sources into
// oracle/_ref/libsmk_ref.so. Python (tests/golden/make_golden.py, bench.py's
// reference arm and cpu_baseline leg) loads it with ctypes; nothing in the
// shipped package does.
//
// Every function forwards to the reference's public C++ entry point of the
// decode-GEMV path:
//   kernels().gemv_q4_0 / gemv_q8_0      src/dispatch/kernels.hpp:70-71
//   quant::quantize_q4_0_rows            src/kernels/quant/q4_0.hpp:60
//   quant::quantize_q8_0_rows            src/kernels/quant/q8_0.hpp:58
//   quant::quantize_x_q8                 src/kernels/quant/q8_0.hpp:64
//   kernels().sgemm / sgemm_f16 / _bf16  src/dispatch/kernels.hpp:66-68 (trans_b, x·Wᵀ)
//   kernels().sgemm_u8s8, gemm::u8s8_path src/dispatch/kernels.hpp:47,69, src/kernels/gemm/int8_gemm.hpp:41
//   gemm::set_num_threads                src/kernels/gemm/avx2_gemm_packed.hpp:94
//   use_kernels / kernels_for            src/dispatch/kernels.hpp:91,98

#include "dispatch/kernels.hpp"
#include "kernels/gemm/avx2_gemm_packed.hpp"
#include "kernels/gemm/int8_gemm.hpp"
#include "kernels/quant/q4_0.hpp"
#include "kernels/quant/q8_0.hpp"

#include <cstdint>

using simd_ml::Isa;

namespace {
const simd_ml::KernelTable& table(int isa) {
    if (isa >= 0 && isa < simd_ml::kNumIsa)
        if (const simd_ml::KernelTable* t = simd_ml::kernels_for(static_cast<Isa>(isa))) return *t;
    return simd_ml::kernels();
}
}  // namespace

extern "C" {

// isa: -1 = the table the reference picks for this CPU; 0 scalar, 1 avx2, 2 avx512.
int smkref_isa_usable(int isa) { return simd_ml::kernels_for(static_cast<Isa>(isa)) != nullptr; }
const char* smkref_active_isa(void) { return simd_ml::kernels().name; }
const char* smkref_q8_0_path(void) { return simd_ml::quant::q8_0_path(); }

void smkref_set_num_threads(int n) { simd_ml::gemm::set_num_threads(n); }
int smkref_get_num_threads(void) { return simd_ml::gemm::get_num_threads(); }

void smkref_gemv_q4_0(int isa, int N, int K, const float* x, const std::uint8_t* Wq, float* y) {
    table(isa).gemv_q4_0(N, K, x, Wq, y);
}
void smkref_gemv_q8_0(int isa, int N, int K, const float* x, const std::uint8_t* Wq, float* y) {
    table(isa).gemv_q8_0(N, K, x, Wq, y);
}
int smkref_quantize_q4_0(const float* W, int N, int K, std::uint8_t* out) {
    return simd_ml::quant::quantize_q4_0_rows(W, N, K, out) ? 1 : 0;
}
int smkref_quantize_q8_0(const float* W, int N, int K, std::uint8_t* out) {
    return simd_ml::quant::quantize_q8_0_rows(W, N, K, out) ? 1 : 0;
}
int smkref_quantize_x_q8(const float* x, int K, std::int8_t* qs, float* dx) {
    return simd_ml::quant::quantize_x_q8(x, K, qs, dx) ? 1 : 0;
}
// C [M, N] = alpha · A [M, K] · B[N, K]ᵀ + beta · C, the decode path of sgemm(trans_b=True).
void smkref_sgemm_tb(int isa, int M, int N, int K, float alpha, const float* A, const float* B, float beta,
                     float* C) {
    table(isa).sgemm(false, true, M, N, K, alpha, A, K, B, K, beta, C, N);
}
void smkref_sgemm_f16_tb(int isa, int M, int N, int K, float alpha, const std::uint16_t* A,
                         const std::uint16_t* B, float beta, float* C) {
    table(isa).sgemm_f16(true, M, N, K, alpha, A, K, B, K, beta, C, N);
}
void smkref_sgemm_bf16_tb(int isa, int M, int N, int K, float alpha, const std::uint16_t* A,
                          const std::uint16_t* B, float beta, float* C) {
    table(isa).sgemm_bf16(true, M, N, K, alpha, A, K, B, K, beta, C, N);
}

// C [M, N] = a_scale·b_scales[j]·Σ_k (A − zp)·op(B); A [M, K]; B [N, K] (trans_b) or [K, N].
void smkref_sgemm_u8s8(int isa, int trans_b, int M, int N, int K, const std::uint8_t* A, int a_zero_point,
                       const std::int8_t* B, float a_scale, const float* b_scales, float* C) {
    table(isa).sgemm_u8s8(trans_b != 0, M, N, K, A, K, a_zero_point, B, trans_b ? K : N, a_scale, b_scales, C, N);
}
const char* smkref_u8s8_path(void) { return simd_ml::gemm::u8s8_path(); }

}  // extern "C"
