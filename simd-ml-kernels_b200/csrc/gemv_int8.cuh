// gemv_int8.cuh — launch parameters of the INT8 decode GEMV (gemv_int8.cu):
// the reference's sgemm_u8s8 with trans_b for M ≤ 8 rows of A,
//   C[i][j] = a_scale · b_scales[j] · Σ_k (A[i][k] − zp) · W[j][k],
// A uint8 [M, lda] (per-tensor scale and zero point), W int8 [N, ldw]
// (symmetric, one scale per output row j), C float32 [M, ldc]
// (src/kernels/gemm/int8_gemm.hpp:5-26; the M = 1 row path
// src/kernels/gemm/int8_rows.hpp:1-26; scalar table
// src/kernels/scalar_kernels.cpp:148-170).
//
// The integer sums are exact; C is the scalar table's epilogue,
// float(double(a_scale) · b_scales[j] · double(sum)), so every output is
// bitwise the reference's scalar result.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace smk {

struct U8S8Params {
    const uint8_t* a;      // [M, lda]
    long long lda;
    const int8_t* w;       // [N, ldw]
    long long ldw;
    const float* scales;   // [N]
    float* y;              // [M, ldy]
    long long ldy;
    int M, N, K;
    int zp;                // a_zero_point, 0..255
    float a_scale;
    unsigned* err;         // device error word (bounded waits), may be null
};

// Rows of A from which the tensor-core kernel is used (dp4a kernel below).
// B200, K = 4096: at M = 8 it takes 12.95 against 19.6 us (N = 14336), at
// M = 4 12.9 against 13.9 us (N = 14336) and 6.8 against 6.3 us (N = 4096).
constexpr int kU8S8MmaMinRows = 4;

cudaError_t launch_gemv_u8s8(cudaStream_t s, bool pdl, int num_sms, const U8S8Params& p);

}  // namespace smk
