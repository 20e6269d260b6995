// dequant.cuh — launch of the Q4_0 / Q8_0 row dequantization (dequant.cu).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace smk {

// out[r][k] (row stride ldo floats) = value k of row rows[r] of the N-row
// matrix w (K/32 blocks per row; fmt 0 = Q4_0, 1 = Q8_0). Rows outside
// [0, N) become NaN and set kErrBadLaunch in *err.
cudaError_t launch_dequantize_rows(cudaStream_t s, int fmt, const uint8_t* w, int N, int K, const int32_t* rows,
                                   int nrows, float* out, long long ldo, unsigned* err, int num_sms);

}  // namespace smk
