// decode.cuh — launchers of the decode-step kernels (decode.cu) shared with the
// C-ABI layer (smk_api.cu).
#pragma once

#include <algorithm>
#include <cuda_runtime.h>

namespace smk {

// Largest row (values) add_rmsnorm takes.
int add_rmsnorm_max_n();
// For each of M rows: x += delta (delta may be null), h = w · (x · fl(1/sqrt(mean(x²) + eps))).
cudaError_t launch_add_rmsnorm(cudaStream_t s, bool pdl, int M, int n, float* x, long long ldx, const float* delta,
                               long long ldd, const float* w, double eps, float* h, long long ldh);
// RoPE of q and k at position pos (or *pos_dev), q to qout, k and v to row pos of the caches.
cudaError_t launch_rope_kv(cudaStream_t s, bool pdl, const float* qkv, const float* inv_freq, const int* pos_dev,
                           int pos, int nh, int nkv, int hd, bool interleaved, float* qout, float* kc, float* vc,
                           int cap, unsigned* err);
// Attention of one token's q over len (or *len_dev) cached positions; max_len bounds
// the length (chunks of the grid); ws [nkv][chunks][nh/nkv][hd + 2] floats and
// tickets [nkv] (zero) when attention_chunks(max_len) > 1.
int attention_chunks(int max_len);
int attention_max_rep();
int attention_max_hd();
cudaError_t launch_attention(cudaStream_t s, bool pdl, const float* q, const float* kc, const float* vc, float* out,
                             const int* len_dev, int len, int max_len, int nh, int nkv, int hd, int cap, float scale,
                             float* ws, unsigned* tickets, unsigned* err);
// The two above in one kernel: RoPE of this token's qkv at position pos (or
// *pos_dev), k and v written to that row of the caches, attention over
// positions 0 .. pos; max_len > pos bounds the chunks (ws and tickets as above).
cudaError_t launch_rope_attention(cudaStream_t s, bool pdl, const float* qkv, const float* inv_freq, const int* pos_dev,
                                  int pos, int max_len, int nh, int nkv, int hd, bool interleaved, float* kc, float* vc,
                                  int cap, float scale, float* out, float* ws, unsigned* tickets, unsigned* err);

}  // namespace smk
