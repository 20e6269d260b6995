// dequant.cu — rows of a Q4_0 / Q8_0 matrix as float32 on the device: the
// embedding lookup of a decode step whose token table is stored as ggml
// blocks (the reference's examples/llama/gguf_reader.py:113-129,
// dequantize_rows, for its quantized types).
//
// Value j of a block is fp16(d)·(q_j − 8) for Q4_0 (q_j in the low nibble of
// byte j for j < 16, the high nibble of byte j − 16 otherwise) and
// fp16(d)·q_j for Q8_0 (q_j signed). Each product is exact in float32: an
// 11-bit significand times an integer of at most 8 bits. So every output is
// bitwise the reference's value.
//
// One thread per 32-value block: it reads the block's 18 or 34 bytes (blocks
// start at any byte offset, so byte loads) and writes its 32 floats as eight
// 16-byte stores when the output row is 16-byte aligned. A row index outside
// [0, N) gives a row of NaN and sets kErrBadLaunch in the error word; nothing
// outside the matrix is read.

#include "dequant.cuh"
#include "smk_device.cuh"

#include <algorithm>

namespace smk {

namespace {

template <int F>
__global__ void __launch_bounds__(256) dequantize_rows_kernel(const uint8_t* __restrict__ w, int N, int K,
                                                              const int32_t* __restrict__ rows, int nrows,
                                                              float* __restrict__ out, long long ldo, unsigned* err) {
    constexpr int BB = F == 0 ? 18 : 34;
    const int nb = K / 32;
    const long long total = (long long)nrows * nb;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int r = (int)(i / nb), b = (int)(i - (long long)r * nb);
        const int row = rows[r];
        float v[32];
        if (row < 0 || row >= N) {
            if (b == 0 && err) atomicOr(err, kErrBadLaunch);
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = __int_as_float(0x7fc00000);
        } else {
            const uint8_t* blk = w + ((size_t)row * nb + b) * BB;
            const float d = half_bits_to_float((uint32_t)blk[0] | ((uint32_t)blk[1] << 8));
            if constexpr (F == 0) {
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int q = blk[2 + j];
                    v[j] = __fmul_rn(d, (float)((q & 15) - 8));
                    v[16 + j] = __fmul_rn(d, (float)((q >> 4) - 8));
                }
            } else {
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] = __fmul_rn(d, (float)(int8_t)blk[2 + j]);
            }
        }
        float* o = out + (size_t)r * ldo + (size_t)b * 32;
        if ((reinterpret_cast<uintptr_t>(o) & 15) == 0) {
#pragma unroll
            for (int j = 0; j < 32; j += 4) *reinterpret_cast<float4*>(o + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) o[j] = v[j];
        }
    }
}

}  // namespace

cudaError_t launch_dequantize_rows(cudaStream_t s, int fmt, const uint8_t* w, int N, int K, const int32_t* rows,
                                   int nrows, float* out, long long ldo, unsigned* err, int num_sms) {
    const long long total = (long long)nrows * (K / 32);
    if (total == 0) return cudaSuccess;
    const long long grid = std::min<long long>((total + 255) / 256, (long long)num_sms * 8);
    if (fmt == 0)
        dequantize_rows_kernel<0><<<(unsigned)grid, 256, 0, s>>>(w, N, K, rows, nrows, out, ldo, err);
    else
        dequantize_rows_kernel<1><<<(unsigned)grid, 256, 0, s>>>(w, N, K, rows, nrows, out, ldo, err);
    return cudaGetLastError();
}

}  // namespace smk
