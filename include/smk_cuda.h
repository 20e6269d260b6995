/*
 * smk_cuda.h — C ABI of the B200 (sm_100a) decode-GEMV library,
 * libsmk_cuda.so. Plain pointers and sizes; no CUDA, C++ or framework types
 * in the signatures (a stream is an opaque `void*`, a cudaStream_t).
 *
 * It replaces, for the decode-GEMV path only, the CPU kernel-table entries of
 * Mattral/simd-ml-kernels 0.3.0 (file:line into that tree):
 *   GemvQ4_0Fn / GemvQ8_0Fn = void(int N, int K, const float* x,
 *       const uint8_t* Wq, float* y)                     src/dispatch/kernels.hpp:50-53,70-71
 *   quantize_q4_0_rows / quantize_q8_0_rows             src/kernels/quant/q4_0.hpp:60, q8_0.hpp:58
 *   quantize_x_q8                                       src/kernels/quant/q8_0.hpp:64
 *   SgemmFn / Sgemm16Fn with trans_b, M <= 8 (x·Wᵀ)     src/dispatch/kernels.hpp:38-45,66-68
 *                                                       (dot path: gemm/avx2_gemm_packed.cpp:715-732)
 * with the same semantics: x quantized to Q8 blocks (FP32 scales) once per
 * call; a NaN or ±Inf anywhere in a row of x makes that row's outputs NaN;
 * K == 0 gives zeros; N == 0 (or M == 0) writes nothing; K % 32 != 0 is an
 * argument error. There is no CPU fallback: every entry point runs CUDA
 * kernels (or fails).
 *
 * Two kinds of entry points:
 *   smk_*           device pointers, asynchronous on `stream`, capturable in
 *                   a CUDA graph (no synchronisation; a call that needs
 *                   library scratch for the first time at a size allocates
 *                   it, during a capture too, and keeps replaced buffers
 *                   until smk_ctx_destroy).
 *   smk_*_host      any mix of host and device pointers (told apart with
 *                   cudaPointerGetAttributes); host operands are staged
 *                   through library-owned device buffers; returns when y is
 *                   written. These are the reference's synchronous contract.
 *
 * Errors: every function returns an smk_status; smk_last_error() gives the
 * message of the calling thread's last failure.
 */
#ifndef SMK_CUDA_H
#define SMK_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum smk_status {
    SMK_OK = 0,
    SMK_ERR_ARGUMENT = 1,   /* shape / size / value rejected (reference: ArgumentError) */
    SMK_ERR_DTYPE = 2,      /* element type not supported for this call (reference: DTypeError) */
    SMK_ERR_CUDA = 3,       /* a CUDA runtime call failed */
    SMK_ERR_DEVICE = 4,     /* a kernel reported an error (e.g. a bounded wait ran out) */
    SMK_ERR_REJECTED = 5    /* quantize: NaN/Inf input or a block scale that overflows binary16 */
} smk_status;

/* Weight formats of smk_gemv_q / smk_quantize. */
typedef enum smk_qformat { SMK_Q4_0 = 0, SMK_Q8_0 = 1 } smk_qformat;
/* Element types of the dense path. */
typedef enum smk_dtype { SMK_F32 = 0, SMK_F16 = 1, SMK_BF16 = 2 } smk_dtype;

typedef struct smk_ctx smk_ctx;

/* Library version string, e.g. "0.1.0 (sm_100a)". */
const char* smk_version(void);
/* Message of the calling thread's last failed call ("" if none). */
const char* smk_last_error(void);

/* A context per device: its device number, SM count, scratch buffers, the
 * staging buffers of the _host calls and the error word of the kernels.
 * Replaces the reference's process-wide kernels() table (kernels.hpp:84). */
smk_status smk_ctx_create(int device, smk_ctx** out);
smk_status smk_ctx_destroy(smk_ctx* ctx);
/* Options (smk_ctx_set):
 *   SMK_OPT_PDL     1: launch with programmatic dependent launch, so a GEMV
 *                   starts streaming its weights while the previous GEMV of
 *                   the stream finishes. Requires that no kernel immediately
 *                   before it in the stream writes its weights. Default 0.
 *   SMK_OPT_WARPS   warps per CTA of the quantized fast kernel (1..16).
 *   SMK_OPT_STAGES  shared-memory stages per warp of that kernel, each one
 *                   tile of weights (1..8).
 *   SMK_OPT_CTAS_PER_SM  resident CTAs per SM of that kernel (1..8).
 *                   For these three, 0 (the default) picks per call: 16 warps;
 *                   1 stage and up to 2 CTAs per SM for GEMVs of up to 64
 *                   tiles per SM (latency-bound), else 2 stages and 1 CTA
 *                   per SM.
 *   SMK_OPT_TILE_ORDER  how that kernel's row tiles are spread over its CTAs:
 *                   1 interleaved, 2 or 0 (default) a contiguous range per
 *                   CTA.
 *   SMK_OPT_HOST_GRAPHS  1 (default): a smk_gemv_q_host call with device
 *                   weights that repeats the shape and operand addresses of
 *                   one of the last 64 keys replays a CUDA graph of its copy
 *                   and kernel (captured on its second occurrence); 0: every
 *                   call launches directly. Setting any option drops the
 *                   captured graphs.
 *   SMK_OPT_DENSE_MMA  1 (default): smk_gemv_dense with bfloat16 weights and
 *                   4..8 rows of x, or float16 weights and 6..8 rows of float32
 *                   x, takes the tensor-core kernel (x split exactly into bf16
 *                   parts, fp16 weights into two); 0: the CUDA-core kernel.
 *   SMK_OPT_PREFETCH_DELAY  SM clock cycles (0..100000) that the Q4_0
 *                   one-row kernel of K = 2048-multiple shapes (without a fused
 *                   norm, residual or gather) holds back its first weight
 *                   copies when it starts. Under SMK_OPT_PDL it
 *                   starts while the GEMV before it is about to read its x;
 *                   a short hold measured faster in such chains. Results do
 *                   not depend on it. Default 100. */
enum { SMK_OPT_PDL = 1, SMK_OPT_WARPS = 2, SMK_OPT_STAGES = 3, SMK_OPT_CTAS_PER_SM = 4, SMK_OPT_TILE_ORDER = 5,
       SMK_OPT_HOST_GRAPHS = 6, SMK_OPT_DENSE_MMA = 7, SMK_OPT_PREFETCH_DELAY = 8 };
smk_status smk_ctx_set(smk_ctx* ctx, int option, long long value);
smk_status smk_ctx_get(smk_ctx* ctx, int option, long long* value);
/* The CUDA device that owns `ptr` (device or managed memory), or -1 for host memory. */
smk_status smk_pointer_device(const void* ptr, int* device);
/* Page-locked host memory, mapped into every device's address space (an
 * addition; no reference counterpart). Results written here by a *_host call
 * need no copy back: the kernel stores into them directly. */
smk_status smk_host_alloc(size_t bytes, void** out);
smk_status smk_host_free(void* ptr);
/* Reads and clears the device error word (0: no kernel error since the last read). */
smk_status smk_device_error(smk_ctx* ctx, unsigned* code, void* stream);

/* ---- quantized decode GEMV (replaces KernelTable::gemv_q4_0 / gemv_q8_0) ----
 * y[m][n] = Σ_k x[m][k]·W[n][k] for m < M <= 8 rows of x, W as ggml blocks
 * (N rows of K/32 blocks: Q4_0 18 bytes, Q8_0 34 bytes per block), each row of
 * x quantized to Q8 blocks as the reference's quantize_x_q8. x [M, ldx] fp32,
 * y [M, ldy] fp32. M == 1 with ldx = K, ldy = N is the reference's call. */
smk_status smk_gemv_q(smk_ctx* ctx, smk_qformat fmt, int M, int N, int K, const float* x, int64_t ldx,
                      const uint8_t* Wq, float* y, int64_t ldy, void* stream);
smk_status smk_gemv_q4_0(smk_ctx* ctx, int N, int K, const float* x, const uint8_t* Wq, float* y, void* stream);
smk_status smk_gemv_q8_0(smk_ctx* ctx, int N, int K, const float* x, const uint8_t* Wq, float* y, void* stream);
/* The decode step's down projection with its SwiGLU input formed on the fly:
 * y = (silu(gate) * up) @ W.T, silu(g) = g / (1 + exp(-g)) as the reference
 * (src/kernels/scalar_kernels.cpp:196-198), the product formed once per call
 * while x is quantized to Q8 (into the context's scratch for this stream), then
 * the GEMV on those blocks; replaces w_down(silu(w_gate(h)) * w_up(h)) of the
 * reference's examples/llama/llama.py:434 without a separate SiLU and product
 * pass over fp32 values.
 * Device pointers, asynchronous; gate [M, ldg], up [M, ldu]. An addition. */
smk_status smk_gemv_q_silu_mul(smk_ctx* ctx, smk_qformat fmt, int M, int N, int K, const float* gate, int64_t ldg,
                               const float* up, int64_t ldu, const uint8_t* Wq, float* y, int64_t ldy, void* stream);
/* out[i] = silu(gate[i]) * up[i], i < n, the same arithmetic (device pointers). */
smk_status smk_silu_mul(smk_ctx* ctx, int64_t n, const float* gate, const float* up, float* out, void* stream);
/* Host-or-device pointers, synchronous. The exact contract of GemvQ4_0Fn / GemvQ8_0Fn. */
smk_status smk_gemv_q_host(smk_ctx* ctx, smk_qformat fmt, int M, int N, int K, const float* x, const uint8_t* Wq,
                           float* y);

/* ---- dense decode GEMV (replaces sgemm / sgemm_f16 / sgemm_bf16 with trans_b, M <= 8) ----
 * C[m][n] = alpha·Σ_k X[m][k]·W[n][k] + beta·C[m][n]; beta == 0: C is not read.
 * x_type is w_type (the reference's contract) or SMK_F32 (fp32 activations
 * against 16-bit weights, an addition). X [M, ldx], W [N, ldw], C [M, ldc]. */
smk_status smk_gemv_dense(smk_ctx* ctx, smk_dtype w_type, smk_dtype x_type, int M, int N, int K, float alpha,
                          const void* X, int64_t ldx, const void* W, int64_t ldw, float beta, float* C, int64_t ldc,
                          void* stream);
smk_status smk_gemv_dense_host(smk_ctx* ctx, smk_dtype w_type, smk_dtype x_type, int M, int N, int K, float alpha,
                               const void* X, const void* W, float beta, float* C);

/* ---- rows of a quantized matrix as float32 (replaces dequantize_rows of
 * examples/llama/gguf_reader.py:113-129 for Q4_0 / Q8_0: the embedding lookup
 * of a decode step) ----
 * out[r][k] (row stride ldo) = value k of row rows[r] of Wq (N rows of K/32
 * blocks): fp16(d)·(q − 8) for Q4_0, fp16(d)·q for Q8_0, exact. rows is an
 * int32 array in device memory; an index outside [0, N) gives a row of NaN and
 * a nonzero smk_device_error. Device pointers, asynchronous. */
smk_status smk_dequantize_rows(smk_ctx* ctx, smk_qformat fmt, int N, int K, const uint8_t* Wq, const int32_t* rows,
                               int nrows, float* out, int64_t ldo, void* stream);

/* ---- INT8 decode GEMV (replaces GemmU8S8Fn with trans_b = true, M <= 8:
 * src/dispatch/kernels.hpp:47,69; the M = 1 row path
 * src/kernels/gemm/int8_rows.hpp) ----
 * C[i][j] = a_scale·b_scales[j]·Σ_k (A[i][k] − a_zero_point)·W[j][k];
 * A uint8 [M, lda], W int8 [N, ldw] (the nn.Linear layout), b_scales [N],
 * C float32 [M, ldc] (overwritten). The sums are exact and C is the
 * reference's scalar-table value float(double(a_scale)·b_scales[j]·sum)
 * (src/kernels/scalar_kernels.cpp:148-170). a_zero_point in [0, 255],
 * a_scale finite. Device pointers, asynchronous on `stream`. */
smk_status smk_gemv_u8s8(smk_ctx* ctx, int M, int N, int K, const uint8_t* A, int64_t lda, int a_zero_point,
                         const int8_t* W, int64_t ldw, float a_scale, const float* b_scales, float* C, int64_t ldc,
                         void* stream);
/* Host-or-device pointers, contiguous operands, synchronous. */
smk_status smk_gemv_u8s8_host(smk_ctx* ctx, int M, int N, int K, const uint8_t* A, int a_zero_point, const int8_t* W,
                              float a_scale, const float* b_scales, float* C);

/* ---- weight quantization on the device (replaces quantize_q4_0_rows / quantize_q8_0_rows) ----
 * W [rows, K] fp32 -> rows·K/32 blocks, byte-identical to ggml's
 * quantize_row_q4_0_ref / quantize_row_q8_0_ref. Synchronous (the rejection
 * flag is read back): SMK_ERR_REJECTED for NaN/Inf or a binary16 scale overflow. */
smk_status smk_quantize(smk_ctx* ctx, smk_qformat fmt, int64_t rows, int K, const float* W, uint8_t* out,
                        void* stream);
smk_status smk_quantize_host(smk_ctx* ctx, smk_qformat fmt, int64_t rows, int K, const float* W, uint8_t* out);

/* ---- test hooks (bit-exactness checks; same device code as the GEMV) ----
 * smk_quantize_x: x [M, K] -> qs [M, K] int8 and dx [M, K/32] fp32 (NaN for a
 * block with a non-finite value), the activation quantization of the GEMV.
 * smk_block_sums: the GEMV's exact per-block integer sums, out [M, N, K/32]
 * int32, produced by the production kernel's dump mode. Device pointers. */
smk_status smk_quantize_x(smk_ctx* ctx, int M, int K, const float* x, int64_t ldx, int8_t* qs, float* dx,
                          void* stream);
smk_status smk_block_sums(smk_ctx* ctx, smk_qformat fmt, int M, int N, int K, const float* x, int64_t ldx,
                          const uint8_t* Wq, int32_t* out, void* stream);
/* Test hook, no reference counterpart: the activation quantizer's exact steps
 * (RN(a/127) by an FMA remainder, RN(1/d) by one Newton-Raphson step from the
 * hardware approximation, round half away from zero by a biased truncation)
 * against CUDA's __fdiv_rn, __frcp_rn and roundf over their whole domains
 * (every finite a >= 0, every 2^-126 <= d <= 2^126, every |t| <= 128): out[0..2]
 * receive the mismatch counts, all zero on a correct build. Synchronous. */
smk_status smk_check_x_arith(smk_ctx* ctx, unsigned long long* out /* [3] */);

/* ---- the rest of a Llama decode step, around the GEMVs ----
 * Replace the NumPy code of the reference's decoder (examples/llama/llama.py):
 * rms_norm (:184-188) with the residual add before it (step, :414-439), RoPE
 * (rope_cos_sin / apply_rope :131-178 and Llama._rope) with the KV-cache write,
 * and Llama._attention (:398-412). Device pointers, asynchronous on `stream`,
 * programmatic dependent launch when SMK_OPT_PDL is set. */

/* For each of M rows: x += delta (delta may be NULL; x is updated in place), then
 * h = w * (x * f32(1 / sqrt(f32(sum(x^2) / n) + eps))), n <= 8192. */
smk_status smk_add_rmsnorm(smk_ctx* ctx, int M, int n, float* x, int64_t ldx, const float* delta, int64_t ldd,
                           const float* w, double eps, float* h, int64_t ldh, void* stream);
/* One token's qkv = [q (nh heads) | k (nkv) | v (nkv)] of head_dim hd: q and k
 * rotated by the angles f32(pos) * inv_freq[i] (pairs (i, i + hd/2), or (2i, 2i+1)
 * when interleaved), q to q_out [nh][hd], k and v to row pos of k_cache / v_cache
 * [nkv][capacity][hd]. pos is *pos_dev when pos_dev is not NULL (a graph replayed
 * for each token; outside the cache: nothing written, smk_device_error set). */
smk_status smk_rope_kv(smk_ctx* ctx, const float* qkv, const float* inv_freq, const int32_t* pos_dev, int pos, int nh,
                       int nkv, int hd, int interleaved, float* q_out, float* k_cache, float* v_cache, int capacity,
                       void* stream);
/* Grouped-query attention of one token: query head h uses KV head h / (nh/nkv);
 * out[h] = softmax(scale * q[h] . K[0..len)) . V[0..len), len = *len_dev when
 * len_dev is not NULL, else len; max_len >= every len (it sizes the grid).
 * nh/nkv <= 8, hd a multiple of 32 up to 128. */
smk_status smk_attention_decode(smk_ctx* ctx, const float* q, const float* k_cache, const float* v_cache, float* out,
                                const int32_t* len_dev, int len, int max_len, int nh, int nkv, int hd, int capacity,
                                float scale, void* stream);
/* A quantized GEMV with the decode step's neighbours fused in (device
 * pointers, asynchronous; the fast kernels' conditions: K % 256 == 0, Wq
 * 16-byte aligned):
 *   w_norm != NULL: y = (RMSNorm(x) * w_norm) @ W^T, the reference's rms_norm
 *                   (examples/llama/llama.py:184-188) applied to each row of
 *                   x inside the GEMV's x quantization (x is not modified);
 *   up != NULL:     x replaced by silu(x) * up (as smk_gemv_q_silu_mul);
 *   r != NULL:      y = r + (...) @ W^T, the residual add of Llama.step
 *                   (:414-439) in the GEMV's store; r may be y (in place).
 * w_norm and up exclude each other. */
smk_status smk_gemv_q_fused(smk_ctx* ctx, smk_qformat fmt, int M, int N, int K, const float* x, int64_t ldx,
                            const float* up, int64_t ldu, const float* w_norm, double eps, const uint8_t* Wq,
                            const float* r, int64_t ldr, float* y, int64_t ldy, void* stream);
/* smk_rope_kv and smk_attention_decode as one kernel (the decode step's form):
 * this token's qkv (not rotated) at position pos (*pos_dev when pos_dev is not
 * NULL), k and v written to row pos of the caches, attention over positions
 * 0 .. pos, pos < max_len <= capacity. The same outputs as the two calls. */
smk_status smk_rope_attention(smk_ctx* ctx, const float* qkv, const float* inv_freq, const int32_t* pos_dev, int pos,
                              int max_len, int nh, int nkv, int hd, int interleaved, float* k_cache, float* v_cache,
                              int capacity, float scale, float* out, void* stream);

/* ---- quantized decode GEMV without any allocation -------------------------
 * No counterpart in the reference. For callers that cannot call cudaMalloc:
 * hosts whose memory pools own every device allocation, servers that plan all
 * memory at start-up and allocate nothing per request, plugins inside either.
 * Same result as smk_gemv_q (same kernels), with these differences:
 *   - no smk_ctx: runs on the calling thread's current device; Wq, x and y
 *     are device memory; argument and CUDA errors through smk_last_error(),
 *     errors that kernels report (a bounded wait that ran out) through
 *     smk_noalloc_device_error;
 *   - the quantized activations go to a fixed scratch array of
 *     SMK_NOALLOC_SCRATCH_BYTES inside the library, which every GPU that loads
 *     the library holds until the process exits; a call needing more
 *     (M * ceil(K/8192) > 102) is rejected with SMK_ERR_ARGUMENT;
 *   - the first call on each device looks up the array's device address and
 *     the SM count (set-up, once per device, with that device current); make
 *     that first call before any stream capture;
 *   - every call on a device shares the one array (it keeps the last call's
 *     contents), so calls whose kernels overlap on the GPU — on different
 *     streams, or from different threads — race: serialise them.
 * It calls no cudaMalloc, cudaFree or other allocating routine. */
#define SMK_NOALLOC_SCRATCH_BYTES (1u << 20)
smk_status smk_gemv_q_noalloc(smk_qformat fmt, int M, int N, int K, const float* x, int64_t ldx, const uint8_t* Wq,
                              float* y, int64_t ldy, void* stream);
/* The error word of the current device's smk_gemv_q_noalloc kernels (no
 * reference counterpart): waits for `stream`, stores the word in *code and
 * clears it. The word collects the bits of every call since the last read;
 * 0: none of them reported an error. Allocates nothing. */
smk_status smk_noalloc_device_error(unsigned* code, void* stream);

/* ---- row-sharded GEMV with the all-gather of y fused in (one process per GPU) ----
 * Replaces the row slicing of gemv_slice (src/dispatch/dispatch.cpp:373-379)
 * across GPUs, plus an all-gather of the y slices; an addition with no
 * reference counterpart beyond that slicing. Each rank creates one gather
 * object (a device buffer holding two full-y areas [m_max][world * npad],
 * two receive areas of the same entries as 64-bit words, a staging slice and a
 * control block), passes its 64-byte IPC handle to every peer (any host
 * channel: torch.distributed, MPI, ...), and connects with all ranks'
 * handles in rank order. Every rank then makes the same sequence of
 * smk_gemv_q_gather calls on the same shapes: each computes this rank's
 * npad-row slice (N_local <= npad valid rows; the padding rows read 0) and
 * stores it over NVLink into every peer's receive area, each value with the
 * step's tag in one 64-bit store; on the same stream a wait kernel polls the
 * tags (bounded, about 1 s; smk_device_error reports a timeout) and copies the
 * peers' slices into this rank's full-y area. *y_full receives this step's
 * area: [M][world * npad] floats, rank r's rows at r * npad. Only this rank
 * writes it, on `stream`; it stays valid until this rank's next
 * smk_gemv_q_gather call: queue every kernel that reads it on `stream` (or
 * copy it) before making that call. The two areas alternate between steps. */
typedef struct smk_gather smk_gather;
#define SMK_IPC_HANDLE_BYTES 64
smk_status smk_gather_create(smk_ctx* ctx, int world, int rank, int npad, int m_max, smk_gather** out,
                             void* ipc_handle /* SMK_IPC_HANDLE_BYTES */);
smk_status smk_gather_connect(smk_gather* g, const void* ipc_handles /* world * SMK_IPC_HANDLE_BYTES, by rank */);
smk_status smk_gather_destroy(smk_gather* g);
smk_status smk_gemv_q_gather(smk_ctx* ctx, smk_gather* g, smk_qformat fmt, int M, int N_local, int K, const float* x,
                             int64_t ldx, const uint8_t* Wq, float** y_full, void* stream);
/* A gather step that carries no data (no reference counterpart): signals every
 * peer and waits (bounded) for their signals, on the device; every rank makes
 * the same calls. A cross-GPU barrier in stream order, and with
 * smk_gather_pingpong the measure of the gather's fixed cost. */
smk_status smk_gather_barrier(smk_gather* g, void* stream);
/* Diagnostic (no reference counterpart): ranks 0 and 1 bounce a flag over
 * NVLink `iters` times inside one kernel each; rank 0 gets in *ns the
 * nanoseconds of the last iters - iters/8 round trips (the first ones absorb
 * the launches' skew; other ranks get 0). Both ranks call it together;
 * synchronous. relaxed: plain system-scope stores and loads instead of
 * release / acquire ones. */
smk_status smk_gather_pingpong(smk_gather* g, int iters, int relaxed, unsigned long long* ns, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SMK_CUDA_H */
