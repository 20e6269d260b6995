// gemv_dense.cuh — launch parameters of the dense decode GEMV (gemv_dense.cu):
// C = alpha · X · Wᵀ + beta · C with W [N, K] in float32 / binary16 /
// bfloat16, X [M, K] (M ≤ 8) in float32 or the weights' 16-bit type, FP32
// accumulation and output (reference sgemm / sgemm_f16 / sgemm_bf16 with
// trans_b=True, the dot_rows path: src/kernels/gemm/avx2_gemm_packed.cpp:358-448,
// 686-711; scalar order src/kernels/scalar_kernels.cpp:69-84).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace smk {

enum DKind : int { kF32 = 0, kF16 = 1, kBF16 = 2 };

struct DenseParams {
    const void* x;     // [M, ldx] elements of x_kind
    long long ldx;
    const void* w;     // [N, ldw] elements of w_kind
    long long ldw;
    float* y;          // [M, ldy]
    long long ldy;
    int M, N, K;
    float alpha, beta;
    unsigned* err;     // device error word (bounded waits), may be null
    void* xfrag;       // tensor-core path: scratch of dense_mma_scratch bytes for x's bf16 parts, or null
};

cudaError_t launch_gemv_dense(cudaStream_t s, bool pdl, int num_sms, int w_kind, int x_kind, const DenseParams& p);

// Tensor-core path (gemv_dense_mma.cu): bfloat16 W with float32 or bfloat16 x,
// or float16 W with float32 x, kDenseMmaMinRows..8 rows, K a multiple of 128,
// W 16-byte aligned with
// a 16-byte row stride. dense_mma_scratch gives the scratch bytes it needs for
// the call (0: the call does not take it); launch_gemv_dense_mma runs it with
// p.xfrag pointing at that scratch (two kernels: the split of x, the GEMV).
constexpr int kDenseMmaMinRows = 4, kDenseMmaMinRowsF16 = 6;
size_t dense_mma_scratch(int w_kind, int x_kind, int M, int K, long long ldw, const void* w);
cudaError_t launch_gemv_dense_mma(cudaStream_t s, bool pdl, int num_sms, int w_kind, int x_kind, const DenseParams& p);

}  // namespace smk
