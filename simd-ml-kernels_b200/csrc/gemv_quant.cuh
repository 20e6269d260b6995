// gemv_quant.cuh — launch parameters of the Q4_0 / Q8_0 decode-GEMV kernels
// (gemv_quant.cu) shared with the C-ABI layer (smk_api.cu, gemv_noalloc.cu).
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace smk {

enum QFmt : int { kQ4_0 = 0, kQ8_0 = 1 };

constexpr int kQK = 32;           // values per block
constexpr int kSbBlocks = 8;      // blocks per superblock (256 values)
constexpr int kMaxRows = 8;       // rows of x per call (M)

__host__ __device__ constexpr int block_bytes(int fmt) { return fmt == kQ4_0 ? 18 : 34; }
__host__ __device__ constexpr int sb_bytes(int fmt) { return 8 * block_bytes(fmt); }   // 144 / 272

// Work decomposition. A row of K/32 ggml blocks is nsbp = ceil(K/256)
// "superblocks" of 8 blocks. A warp tile is TR rows × G superblocks,
// TR·G = 32 (one superblock per lane: lane = r·G + g); ksteps tiles cover a
// row (superblock sb = ks·G + g).
//
// Quantized activations (shared memory or a global buffer), "lane-major":
//   quants of x row m, k-step ks, block j of the superblock, half h (values
//   16h .. 16h+15), lane g: 16 bytes at (((m·ksteps + ks)·16 + 2j + h)·32 + g)·16
//   (dx, bias) of that block as float2 (bias = −8·Σ quants, as int bits) at
//   xd_base + (((m·ksteps + ks)·8 + j)·32 + g)·8,  xd_base = M·ksteps·8192.
// Lanes of a warp read consecutive 16-byte (8-byte) chunks, one bank set per
// 8 (16) lanes, and within a superblock every offset from the lane's base is
// a compile-time constant. A block whose values are not all finite stores
// dx = NaN, which makes every output of that x row NaN, the reference's rule
// (q8_0_scalar.cpp:142-164).
__host__ __device__ inline size_t xq_total_bytes(int M, int ksteps) { return (size_t)M * ksteps * 10240; }

// The four-row layout (Q4_0, one row of x, K a multiple of 2048; QGemvParams::r4):
// a k-step is 2048 values (8 superblocks) and lane l = 4g + j of a warp takes
// blocks 2j, 2j+1 of superblock g in all four rows of its tile. Its 80 bytes of
// quantized x sit together: slot (ks·32 + l) at byte slot·80 holds the quants of
// block 2j (32 bytes), of block 2j+1 (32 bytes), then (dx, bias) of each as float
// pairs (bias = 0x4B400000 − 8·Σ quants as int bits). 2560 bytes per k-step.
__host__ __device__ inline size_t xq_r4_bytes(int ksteps) { return (size_t)ksteps * 2560; }
__host__ __device__ inline size_t xq_off(int ksteps, int m, int ks, int j, int h, int g) {
    return (((((size_t)m * ksteps + ks) * 16 + 2 * j + h) * 32) + g) * 16;
}
__host__ __device__ inline size_t xd_off(int M, int ksteps, int m, int ks, int j, int g) {
    return (size_t)M * ksteps * 8192 + (((((size_t)m * ksteps + ks) * 8 + j) * 32) + g) * 8;
}

struct QGemvParams {
    const float* x;        // [M, ldx] fp32 activations (device); with `up`, the gate
    long long ldx;
    const float* up;       // nullptr, or [M, ldu]: the activations are silu(x) * up, formed while quantizing
    long long ldu;
    const uint8_t* w;      // N rows of K/32 blocks (device)
    float* y;              // [M, ldy]
    long long ldy;
    int M, N, K;
    int nb;                // K / 32
    int nsbp;              // ceil(nb / 8)
    int G, log2G, TR, ksteps, ntiles;
    int stages;            // shared-memory stages per warp (fast kernel)
    int r4;                // fast kernel: the four-row layout (Q4_0, M = 1, K % 2048 == 0); set by plan_tiles
    int contiguous;        // fast kernel: 1 = each CTA takes a contiguous range of tiles, 0 = tiles interleaved over CTAs
    int cta_q, cta_r;      // contiguous ranges: ntiles = cta_q · grid + cta_r (set by the launcher, see cta_first_tile)
    int issue_delay;       // four-row kernel: SM cycles its warps hold back their first weight copies
    int split;             // tensor-core kernel: K parts per 16-row tile (set by its launcher)
    // Tensor-core kernel with x larger than shared memory: K is cut into
    // kparts parts across CTAs, each CTA holding only its part's slice of x
    // (xnb blocks at most; xnb = nb when kparts == 1). The CTAs' sums go to
    // partial [kparts][M][N], and the last CTA of each tile range (counted on
    // tickets, zeroed by the quantize kernel of the same call) adds the parts
    // in K order into y.
    int kparts;
    int xnb;
    float* partial;
    unsigned* tickets;
    const struct GatherArgs* gather;   // fused all-gather of y over peer GPUs, or nullptr (device copy)
    // Fast kernel, y wanted in page-locked host memory: y goes to device
    // memory as usual, and the CTA that finishes last (counted on *ticket,
    // zero between launches) copies the M rows of N values to yhost (the
    // buffer's device-mapped address, rows ldy apart like y). nullptr: off.
    float* yhost;
    unsigned* ticket;
    const uint8_t* xq;     // quantized x in global memory (nullptr: each CTA quantizes into shared memory)
    int32_t* dump;         // test-only: per-block integer sums [M, N, nb], or nullptr
    unsigned* err;         // device error word
    // The decode step's neighbours fused in (fast kernels): nw != nullptr:
    // each row of x is RMS-normalised and scaled by nw before it is quantized,
    // h = nw · (x · fl(1/sqrt(fl(Σx²/K) + neps))) (the reference's rms_norm);
    // res != nullptr: y = fl(res + x·Wᵀ), rows ldr apart (res may be y: the
    // residual stream updated in place, each value read and written by one lane).
    const float* nw;
    double neps;
    const float* res;
    long long ldr;
};

// All-gather of y fused into the fast kernel's epilogue (row-sharded GEMV,
// one process per GPU). Every rank owns one buffer, mapped into its peers'
// address spaces: two full-y areas [M_max][world·npad] of floats (alternate
// steps; only this rank writes them), two receive areas of the same entries
// as 64-bit words (the peers' slices: value bits low, step tag high) and a
// control block of 32-bit words: [0] epoch (completed gather steps),
// [kGatherTicket] the wait kernel's CTA count, [kGatherSignals + s] rank s's
// latest barrier step.
//
// A step's tag is epoch + 1. A word that shows the tag holds that step's
// value (one 64-bit store is single-copy atomic), so the receiver polls the
// data itself: no fence, no flag, no second NVLink crossing.
constexpr int kMaxRanks = 8;
constexpr int kGatherTicket = 1;
constexpr int kGatherSignals = 8;
constexpr int kGatherPingWord = 32;   // control word of the NVLink ping-pong diagnostic
struct GatherArgs {
    float* y;                               // this rank's full-y areas
    unsigned long long* ll[kMaxRanks];      // rank r's receive areas
    unsigned* ctrl[kMaxRanks];              // rank r's control block
    long long area;                         // entries per area (≥ M_max · world · npad)
    int world, rank, npad;
};

// Fill the tiling of p (p.M, p.N, p.K set): the fast kernel's G = the
// smallest power of two >= nsbp, at most 32; the generic kernel's G = 32.
// fmt given and the four-row conditions met (fast, Q4_0, M == 1, allow_r4 and
// r4_shape): the four-row layout, G = 8, TR = 4, one k-step per 2048 values.
void plan_tiles(QGemvParams& p, bool fast, int fmt = -1, bool allow_r4 = true, int num_sms = 148);
// Shapes that take the four-row layout: K == 2048; or K a multiple of 2048, at
// least 8192, with N <= 16384 (x quantized once into global memory) and at
// least 8 four-row tiles per SM, or K >= 16384.
bool r4_shape(int N, int K, int num_sms);
// Four-row plans with fewer than 8 tiles per SM (K >= 16384): the kernel
// that splits each tile's k-steps over several warps (x in global memory).
bool r4_split(const QGemvParams& p, int num_sms);
// Bytes of quantized x of this plan (either layout).
inline size_t x_bytes(const QGemvParams& p) { return p.r4 ? xq_r4_bytes(p.ksteps) : xq_total_bytes(p.M, p.ksteps); }

// Sets the message smk_last_error() returns on this thread.
void set_last_error(const char* msg);

// CTAs per SM of `fn` at this launch shape; raises the kernel's dynamic
// shared-memory limit as needed. Cached per (device, kernel, threads, smem).
cudaError_t occupancy(const void* fn, int threads, size_t smem, int* per_sm);

// Host-side launchers (gemv_quant.cu). All return cudaGetLastError() of the launch.
struct LaunchCfg {
    cudaStream_t stream;
    bool pdl;              // programmatic dependent launch
    int num_sms;
    int warps;             // warps per CTA of the fast kernel
    int ctas_per_sm = 1;   // cap on resident CTAs per SM of the fast kernel
};

// Quantize p.x (or silu(p.x) * p.up) into the layout of the plan (lane-major,
// or four-row when p.r4) at xq (global memory, x_bytes(p) bytes).
cudaError_t launch_quantize_x(const LaunchCfg& c, const QGemvParams& p, uint8_t* xq);
// n floats from device-mapped page-locked host memory to device memory (a host
// call's x), by a kernel: a GEMV launched after it with programmatic dependent
// launch streams its weights meanwhile.
cudaError_t launch_stage_x(cudaStream_t s, const float* src, float* dst, long long n, int num_sms);
// Test hook: mismatch counts of the x quantizer's exact helpers (bad[3], zeroed
// by the caller) against CUDA's divide, reciprocal and roundf.
cudaError_t launch_check_x_arith(cudaStream_t s, unsigned long long* bad);
// out[i] = silu(gate[i]) * up[i] for i < n, as the fused GEMV forms its
// activations (test hook and unfused path).
cudaError_t launch_silu_mul(cudaStream_t s, long long n, const float* gate, const float* up, float* out);
// y = x · Wᵀ. fast: K % 256 == 0 and w 16-byte aligned (ggml superblocks
// stream as whole 16-byte units); otherwise the generic kernel.
cudaError_t launch_gemv_q(const LaunchCfg& c, int fmt, QGemvParams p, bool fast, size_t* smem_used);
// Size of the fast kernel's dynamic shared memory for this launch.
size_t gemv_q_smem(int fmt, const QGemvParams& p, int warps, int stages, bool x_in_smem);

// After a fused GEMV of M rows on the same stream: wait (bounded,
// kErrPeerTimeout on err) until every peer's slice of the step shows the
// step's tag in this rank's receive area, copy it into the full-y area, and
// advance the epoch once the GEMV has completed. blocks: 1 .. number of SMs
// (kGatherWaitThreads threads each).
constexpr int kGatherWaitThreads = 256;
cudaError_t launch_gather_wait(const LaunchCfg& c, const GatherArgs* g_dev, int M, int blocks, unsigned* err);
// A gather step without data: a cross-GPU barrier in stream order (one warp;
// system-scope release / acquire signals, bounded wait).
cudaError_t launch_gather_barrier(const LaunchCfg& c, const GatherArgs* g_dev, unsigned* err);
// Diagnostic: `iters` round trips of a flag between ranks 0 and 1 over NVLink
// inside one kernel (one warp each; other ranks return at once); rank 0 writes
// the elapsed nanoseconds to *ns. Values base+1 .. base+iters; bounded waits.
cudaError_t launch_gather_pingpong(cudaStream_t s, const GatherArgs* g_dev, unsigned base, int iters, bool relaxed,
                                   unsigned* err, unsigned long long* ns);

// Tensor-core path for kMmaMinRows..8 rows of x (fast-kernel conditions):
// x quantized by launch_quantize_x_mma into xmma_bytes(nb) bytes at p.xq,
// then launch_gemv_q_mma with p.stages stages per warp.
constexpr int kMmaMinRows = 3;
constexpr int kMmaMaxTickets = 1024;   // tile ranges of a K-parted launch (zeroed by the quantize kernel)
size_t xmma_bytes(int nb);
// Shared memory of the kernel holding xnb blocks of x (x_in_smem) or none.
size_t gemv_q_mma_smem(int fmt, int stages, int xnb, bool x_in_smem);
cudaError_t launch_quantize_x_mma(const LaunchCfg& c, const QGemvParams& p, uint8_t* xq);
// x_in_smem: each CTA copies the quantized x into shared memory first.
cudaError_t launch_gemv_q_mma(const LaunchCfg& c, int fmt, const QGemvParams& p, bool x_in_smem);

// Weight quantizers (ggml quantize_row_q4_0_ref / q8_0_ref, bit-exact).
// *reject gets 1 when a value is NaN/Inf or a scale overflows binary16.
cudaError_t launch_quantize_w(cudaStream_t s, int fmt, const float* W, long long rows, int K, uint8_t* out,
                              unsigned* reject);

}  // namespace smk
