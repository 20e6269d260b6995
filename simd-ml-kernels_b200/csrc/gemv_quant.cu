// gemv_quant.cu — sm_100a decode GEMV on ggml Q4_0 / Q8_0 weights, M ≤ 8
// rows of x:  y[m][n] = Σ_b fp16(dw[n][b]) · dx[m][b] · Σ_i qw[n][b][i] · qx[m][b][i]
// (reference: src/kernels/quant/q4_0.hpp:23-30, q8_0.hpp:19-30; x quantized to
// Q8 blocks once per call with FP32 scales, q8_0_scalar.cpp:113-166).
//
// Fast kernel (K % 256 == 0, weights 16-byte aligned): a row of K/32 ggml
// blocks is K/256 "superblocks" of 8 blocks = 144 bytes (Q4_0) or 272 (Q8_0),
// both multiples of 16, so every superblock of every row starts on a 16-byte
// boundary. Each warp owns a private ring of shared-memory stages filled by
// 1-D bulk TMA copies (cp.async.bulk, no multicast) and completed on an
// mbarrier per stage; a stage is a tile of TR rows × G superblocks with one
// superblock per lane (TR·G = 32), read back with 128-bit shared loads (the
// 144/272-byte lane stride puts each 8-lane phase on distinct banks). The
// quants are unpacked in registers: Q4_0 nibbles as q & 0x0F0F0F0F and
// q & 0xF0F0F0F0 against x's two 16-value halves with dp4a.u32.s32, the
// second sum divided by 16 exactly, from the start value −8·Σqx (the
// reference's bias trick, q4_0_rows.hpp:25-31); Q8_0 with signed dp4a. Per
// block the exact int32 sum is scaled by fp16(dw)·dx in FP32 and accumulated
// in FP32 per lane; the G lanes of a row are summed with shuffles.
//
// The weights do not depend on earlier kernels of the stream (the library
// never writes weights from a GEMV-preceding kernel), so each warp issues its
// first stages before griddepcontrol.wait: under programmatic dependent
// launch the next GEMV's weight stream starts while the previous one drains.
// x and y are only touched after the wait.

#include "gemv_quant.cuh"
#include "smk_device.cuh"

#include <algorithm>
#include <cfloat>
#include <map>
#include <mutex>
#include <tuple>

namespace smk {

namespace {

constexpr int kThreadsQuantX = 256;

__device__ __forceinline__ size_t xq_off(int nsbp, int m, int h, int j, int sb) {
    return ((size_t)((m * 2 + h) * 8 + j) * nsbp + sb) * 16;
}
__device__ __forceinline__ size_t xd_off(int M, int nsbp, int m, int j, int sb) {
    return xq_quant_bytes(M, nsbp) + ((size_t)(m * 8 + j) * nsbp + sb) * 8;
}

// Quantize x [M, K] into the swizzled layout at xb (shared or global memory).
// Eight threads per 32-value block, four values each; tid in [0, nthreads),
// nthreads a multiple of 8. Bit-exact with the reference's quantize_x_q8
// (q8_0_scalar.cpp:45-61,113-118): amax/127 and 1/d as IEEE divisions,
// w·id rounded once, then rounded half away from zero. Each thread first
// loads the values of up to kXUnroll blocks, so the prologue of a GEMV waits
// for one round trip to L2 rather than one per block.
constexpr int kXUnroll = 4;

__device__ __forceinline__ float4 load_x4(const float* p) {
    if ((reinterpret_cast<uintptr_t>(p) & 15) == 0) return *reinterpret_cast<const float4*>(p);
    return make_float4(p[0], p[1], p[2], p[3]);
}

__device__ __forceinline__ void quantize_x_block(float4 v, int gq, unsigned gmask, int M, int nsbp, int m, int b,
                                                 uint8_t* xb) {
    unsigned fin = finite_bits(v.x) & finite_bits(v.y) & finite_bits(v.z) & finite_bits(v.w);
    float amax = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) {
        amax = fmaxf(amax, __shfl_xor_sync(gmask, amax, o));
        fin &= __shfl_xor_sync(gmask, fin, o);
    }
    const float d = __fdiv_rn(amax, 127.0f);
    float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    if (!(id <= FLT_MAX)) id = 0.0f;
    const int q0 = fin ? (int)roundf(__fmul_rn(v.x, id)) : 0;
    const int q1 = fin ? (int)roundf(__fmul_rn(v.y, id)) : 0;
    const int q2 = fin ? (int)roundf(__fmul_rn(v.z, id)) : 0;
    const int q3 = fin ? (int)roundf(__fmul_rn(v.w, id)) : 0;
    const uint32_t word = (uint32_t)(q0 & 0xff) | ((uint32_t)(q1 & 0xff) << 8) | ((uint32_t)(q2 & 0xff) << 16) |
                          ((uint32_t)(q3 & 0xff) << 24);
    int s = q0 + q1 + q2 + q3;
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) s += __shfl_xor_sync(gmask, s, o);
    const int sb = b >> 3, j = b & 7;
    *reinterpret_cast<uint32_t*>(xb + xq_off(nsbp, m, gq >> 2, j, sb) + (gq & 3) * 4) = word;
    if (gq == 0) {
        const float dxv = fin ? d : __int_as_float(0x7fc00000);
        *reinterpret_cast<float2*>(xb + xd_off(M, nsbp, m, j, sb)) = make_float2(dxv, __int_as_float(-8 * s));
    }
}

__device__ __forceinline__ void quantize_x_rows(const float* __restrict__ x, long long ldx, int M, int nb,
                                                int nsbp, uint8_t* xb, int tid, int nthreads) {
    const int gq = tid & 7;
    const unsigned gmask = 0xffu << ((tid & 31) & ~7);
    const int total = M * nb, stride = nthreads >> 3;
    for (int base = tid >> 3; base < total; base += kXUnroll * stride) {
        float4 v[kXUnroll];
#pragma unroll
        for (int u = 0; u < kXUnroll; ++u) {
            const int blk = base + u * stride;
            if (blk < total) {
                const int m = blk / nb, b = blk - m * nb;
                v[u] = load_x4(x + (size_t)m * ldx + (size_t)b * kQK + gq * 4);
            }
        }
#pragma unroll
        for (int u = 0; u < kXUnroll; ++u) {
            const int blk = base + u * stride;
            if (blk < total) {
                const int m = blk / nb, b = blk - m * nb;
                quantize_x_block(v[u], gq, gmask, M, nsbp, m, b, xb);
            }
        }
    }
}

__global__ void __launch_bounds__(kThreadsQuantX) quantize_x_kernel(const float* __restrict__ x, long long ldx,
                                                                     int M, int nb, int nsbp, uint8_t* xq) {
    pdl_launch_dependents();
    pdl_wait_primary();   // x comes from the previous kernel; xq may still be read by it
    quantize_x_rows(x, ldx, M, nb, nsbp, xq, blockIdx.x * blockDim.x + threadIdx.x, gridDim.x * blockDim.x);
}

template <bool kShared>
__device__ __forceinline__ uint4 ld_x16(const uint8_t* p) {
    if constexpr (kShared) return *reinterpret_cast<const uint4*>(p);
    else return __ldg(reinterpret_cast<const uint4*>(p));
}
template <bool kShared>
__device__ __forceinline__ float2 ld_x8(const uint8_t* p) {
    if constexpr (kShared) return *reinterpret_cast<const float2*>(p);
    else return __ldg(reinterpret_cast<const float2*>(p));
}

// One block: integer sums against every x row, then acc[m] += isum·(dw·dx).
template <int F, int M, bool kShX, bool kDump>
__device__ __forceinline__ void block_dot(const uint32_t (&q)[8], float dw, const uint8_t* xb, int nsbp, int j,
                                          int sb, float (&acc)[M], int32_t* dump, size_t dump_stride, size_t dump_idx) {
#pragma unroll
    for (int m = 0; m < M; ++m) {
        const uint4 xl = ld_x16<kShX>(xb + xq_off(nsbp, m, 0, j, sb));
        const uint4 xh = ld_x16<kShX>(xb + xq_off(nsbp, m, 1, j, sb));
        const float2 db = ld_x8<kShX>(xb + xd_off(M, nsbp, m, j, sb));
        int isum;
        if constexpr (F == kQ4_0) {
            // q[0..3]: the 16 nibble bytes; low nibbles are values 0-15, high 16-31.
            int a = __float_as_int(db.y);
            a = dp4a_us(q[0] & 0x0F0F0F0Fu, xl.x, a);
            a = dp4a_us(q[1] & 0x0F0F0F0Fu, xl.y, a);
            a = dp4a_us(q[2] & 0x0F0F0F0Fu, xl.z, a);
            a = dp4a_us(q[3] & 0x0F0F0F0Fu, xl.w, a);
            int h = dp4a_us(q[0] & 0xF0F0F0F0u, xh.x, 0);
            h = dp4a_us(q[1] & 0xF0F0F0F0u, xh.y, h);
            h = dp4a_us(q[2] & 0xF0F0F0F0u, xh.z, h);
            h = dp4a_us(q[3] & 0xF0F0F0F0u, xh.w, h);
            isum = a + (h >> 4);   // h is 16·Σ hi·x: exact
        } else {
            int a = dp4a_ss(q[0], xl.x, 0);
            a = dp4a_ss(q[1], xl.y, a);
            a = dp4a_ss(q[2], xl.z, a);
            a = dp4a_ss(q[3], xl.w, a);
            a = dp4a_ss(q[4], xh.x, a);
            a = dp4a_ss(q[5], xh.y, a);
            a = dp4a_ss(q[6], xh.z, a);
            isum = dp4a_ss(q[7], xh.w, a);
        }
        if constexpr (kDump) dump[m * dump_stride + dump_idx] = isum;
        acc[m] = fmaf((float)isum, __fmul_rn(dw, db.x), acc[m]);
    }
}

// One superblock (8 blocks) at sp in shared memory.
template <int F, int M, bool kShX, bool kDump>
__device__ __forceinline__ void superblock(const uint8_t* sp, const uint8_t* xb, int nsbp, int sb, float (&acc)[M],
                                           int32_t* dump, size_t dump_stride, size_t dump_row) {
    if constexpr (F == kQ4_0) {
        uint32_t w[36];
#pragma unroll
        for (int i = 0; i < 9; ++i) {
            const uint4 v = *reinterpret_cast<const uint4*>(sp + 16 * i);
            w[4 * i] = v.x; w[4 * i + 1] = v.y; w[4 * i + 2] = v.z; w[4 * i + 3] = v.w;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            uint32_t q[8], sc;
            if (j % 2 == 0) {   // block starts on a word: scale in the low half, quants 2 bytes in
                const int b = 9 * (j / 2);
                sc = w[b] & 0xffffu;
#pragma unroll
                for (int i = 0; i < 4; ++i) q[i] = funnel(w[b + i], w[b + i + 1], 16);
            } else {            // scale in the high half of a word, quants word-aligned
                const int b = 9 * (j / 2) + 4;
                sc = w[b] >> 16;
#pragma unroll
                for (int i = 0; i < 4; ++i) q[i] = w[b + 1 + i];
            }
            block_dot<F, M, kShX, kDump>(q, half_bits_to_float(sc), xb, nsbp, j, sb, acc, dump, dump_stride,
                                         dump_row + sb * 8 + j);
        }
    } else {
#pragma unroll
        for (int H = 0; H < 2; ++H) {   // blocks 4H..4H+3 lie in words 32H .. 32H+35
            uint32_t w[36];
#pragma unroll
            for (int i = 0; i < 9; ++i) {
                const uint4 v = *reinterpret_cast<const uint4*>(sp + 128 * H + 16 * i);
                w[4 * i] = v.x; w[4 * i + 1] = v.y; w[4 * i + 2] = v.z; w[4 * i + 3] = v.w;
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int j = 4 * H + u;
                uint32_t q[8], sc;
                if (j % 2 == 0) {
                    const int b = 17 * j / 2 - 32 * H;
                    sc = w[b] & 0xffffu;
#pragma unroll
                    for (int i = 0; i < 8; ++i) q[i] = funnel(w[b + i], w[b + i + 1], 16);
                } else {
                    const int b = (34 * j - 2) / 4 - 32 * H;
                    sc = w[b] >> 16;
#pragma unroll
                    for (int i = 0; i < 8; ++i) q[i] = w[b + 1 + i];
                }
                block_dot<F, M, kShX, kDump>(q, half_bits_to_float(sc), xb, nsbp, j, sb, acc, dump, dump_stride,
                                             dump_row + sb * 8 + j);
            }
        }
    }
}

// Issue the bulk copies of work item `it` (tile, k-step) into its stage.
template <int F>
__device__ __forceinline__ void issue_item(const QGemvParams& p, int it, int gw, int GW, uint8_t* stages,
                                           uint64_t* bars, int lane) {
    constexpr int SBB = sb_bytes(F);
    const int tile = gw + (it / p.ksteps) * GW, ks = it - (it / p.ksteps) * p.ksteps;
    const int slot = it % p.stages;
    const int rows = min(p.TR, p.N - tile * p.TR);
    const int sb0 = ks * p.G;
    const int cnt = min(p.G, p.nsbp - sb0);
    const uint32_t bytes = (uint32_t)cnt * SBB;
    if (lane == 0) mbar_arrive_expect_tx(&bars[slot], bytes * rows);
    __syncwarp();
    if (p.ksteps == 1 && p.G == p.nsbp) {
        // Whole rows, back to back in memory and in the stage: one copy.
        if (lane == 0)
            tma_load_1d(stages + (size_t)slot * 32 * SBB, p.w + (size_t)tile * p.TR * ((size_t)p.nsbp * SBB),
                        bytes * rows, &bars[slot]);
    } else if (lane < rows) {
        const size_t row = (size_t)tile * p.TR + lane;
        const uint8_t* src = p.w + row * ((size_t)p.nsbp * SBB) + (size_t)sb0 * SBB;
        tma_load_1d(stages + (size_t)slot * 32 * SBB + (size_t)lane * p.G * SBB, src, bytes, &bars[slot]);
    }
}

template <int F, int M, bool kXGlobal, bool kDump>
__global__ void __launch_bounds__(256) gemv_q_fast(const QGemvParams p) {
    constexpr int SBB = sb_bytes(F);
    extern __shared__ __align__(128) uint8_t smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;

    uint64_t* bars = reinterpret_cast<uint64_t*>(smem) + warp * p.stages;
    size_t off = ((size_t)nwarps * p.stages * 8 + 127) & ~(size_t)127;
    uint8_t* xs = smem + off;
    if constexpr (!kXGlobal) off += (xq_total_bytes(M, p.nsbp) + 127) & ~(size_t)127;
    uint8_t* stages = smem + off + (size_t)warp * p.stages * 32 * SBB;

    pdl_launch_dependents();

    // Tiles of this warp: gw, gw + GW, ... (interleaved over CTAs so every SM
    // gets a near-equal share); each tile is ksteps items.
    const int GW = gridDim.x * nwarps;
    const int gw = warp * gridDim.x + blockIdx.x;
    const int my_tiles = gw < p.ntiles ? (p.ntiles - 1 - gw) / GW + 1 : 0;
    const int nitems = my_tiles * p.ksteps;

    if (lane == 0) {
        for (int s = 0; s < p.stages; ++s) mbar_init(&bars[s], 1);
        fence_mbar_init();
    }
    __syncwarp();
    const int pre = min(p.stages, nitems);
    for (int it = 0; it < pre; ++it) issue_item<F>(p, it, gw, GW, stages, bars, lane);

    pdl_wait_primary();
    if constexpr (!kXGlobal) {
        quantize_x_rows(p.x, p.ldx, M, p.nb, p.nsbp, xs, threadIdx.x, blockDim.x);
        __syncthreads();
    }
    const uint8_t* xb = kXGlobal ? p.xq : xs;

    const int r = lane >> p.log2G, g = lane & (p.G - 1);
    float acc[M];
#pragma unroll
    for (int m = 0; m < M; ++m) acc[m] = 0.0f;

    for (int it = 0; it < nitems; ++it) {
        const int slot = it % p.stages;
        if (!mbar_wait_bounded(&bars[slot], (uint32_t)((it / p.stages) & 1), p.err)) {
            // Give the copies still in flight a bounded chance to land before
            // the CTA's shared memory is released, then stop.
            for (int k = it + 1; k < min(nitems, it + p.stages); ++k)
                mbar_wait_bounded(&bars[k % p.stages], (uint32_t)((k / p.stages) & 1), nullptr);
            return;
        }
        const int tile = gw + (it / p.ksteps) * GW, ks = it - (it / p.ksteps) * p.ksteps;
        const int row = tile * p.TR + r, sb = ks * p.G + g;
        if (row < p.N && sb < p.nsbp)
            superblock<F, M, !kXGlobal, kDump>(stages + (size_t)slot * 32 * SBB + (size_t)lane * SBB, xb, p.nsbp, sb,
                                               acc, p.dump, (size_t)p.N * p.nb, (size_t)row * p.nb);
        if (ks == p.ksteps - 1) {
#pragma unroll
            for (int m = 0; m < M; ++m) {
                float v = acc[m];
                for (int o = p.G >> 1; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                if (g == 0 && row < p.N) p.y[(size_t)m * p.ldy + row] = v;
                acc[m] = 0.0f;
            }
        }
        __syncwarp();
        if (it + p.stages < nitems) {
            fence_proxy_async_smem();
            issue_item<F>(p, it + p.stages, gw, GW, stages, bars, lane);
        }
    }
}

// Generic kernel: any K % 32 == 0 and any weight alignment. One warp per row,
// lanes over blocks, byte loads; x already quantized in global memory.
template <int F, int M, bool kDump>
__global__ void __launch_bounds__(256) gemv_q_generic(const QGemvParams p) {
    constexpr int BB = block_bytes(F);
    pdl_launch_dependents();
    pdl_wait_primary();
    const int lane = threadIdx.x & 31;
    const int nwarps_total = gridDim.x * (blockDim.x >> 5);
    const size_t row_bytes = (size_t)p.nb * BB;
    for (int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < p.N; row += nwarps_total) {
        float acc[M];
#pragma unroll
        for (int m = 0; m < M; ++m) acc[m] = 0.0f;
        for (int b = lane; b < p.nb; b += 32) {
            const uint8_t* blk = p.w + (size_t)row * row_bytes + (size_t)b * BB;
            const uint32_t sc = (uint32_t)__ldg(blk) | ((uint32_t)__ldg(blk + 1) << 8);
            uint32_t q[8];
#pragma unroll
            for (int i = 0; i < (F == kQ4_0 ? 4 : 8); ++i)
                q[i] = (uint32_t)__ldg(blk + 2 + 4 * i) | ((uint32_t)__ldg(blk + 3 + 4 * i) << 8) |
                       ((uint32_t)__ldg(blk + 4 + 4 * i) << 16) | ((uint32_t)__ldg(blk + 5 + 4 * i) << 24);
            block_dot<F, M, false, kDump>(q, half_bits_to_float(sc), p.xq, p.nsbp, b & 7, b >> 3, acc, p.dump,
                                          (size_t)p.N * p.nb, (size_t)row * p.nb + b);
        }
#pragma unroll
        for (int m = 0; m < M; ++m) {
            float v = acc[m];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (lane == 0) p.y[(size_t)m * p.ldy + row] = v;
        }
    }
}

// ---- weight quantizers -------------------------------------------------------

// ggml quantize_row_q4_0_ref / q8_0_ref (reference q4_0_scalar.cpp:33-78,
// q8_0_scalar.cpp:45-111): eight threads per block, four values each.
template <int F>
__global__ void __launch_bounds__(256) quantize_w_kernel(const float* __restrict__ W, long long nblocks,
                                                         uint8_t* __restrict__ out, unsigned* reject) {
    constexpr int BB = block_bytes(F);
    const int gq = threadIdx.x & 7;
    const unsigned gmask = 0xffu << ((threadIdx.x & 31) & ~7);
    const long long groups = (long long)gridDim.x * (blockDim.x >> 3);
    for (long long blk = (long long)blockIdx.x * (blockDim.x >> 3) + (threadIdx.x >> 3); blk < nblocks;
         blk += groups) {
        const float* wp = W + blk * kQK + gq * 4;
        float v[4] = {wp[0], wp[1], wp[2], wp[3]};
        unsigned fin = finite_bits(v[0]) & finite_bits(v[1]) & finite_bits(v[2]) & finite_bits(v[3]);
        uint8_t* o = out + blk * BB;
        if constexpr (F == kQ4_0) {
            // First value of the largest magnitude (lowest index on ties) keeps its sign.
            float amax = 0.0f, mx = 0.0f;
            int idx = 1 << 30;
#pragma unroll
            for (int i = 0; i < 4; ++i)
                if (amax < fabsf(v[i])) { amax = fabsf(v[i]); mx = v[i]; idx = gq * 4 + i; }
#pragma unroll
            for (int s = 4; s > 0; s >>= 1) {
                const float oa = __shfl_xor_sync(gmask, amax, s), om = __shfl_xor_sync(gmask, mx, s);
                const int oi = __shfl_xor_sync(gmask, idx, s);
                if (oa > amax || (oa == amax && oi < idx)) { amax = oa; mx = om; idx = oi; }
                fin &= __shfl_xor_sync(gmask, fin, s);
            }
            const float d = __fdiv_rn(mx, -8.0f);
            float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
            if (!(fabsf(id) <= FLT_MAX)) id = 0.0f;
            int q[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) q[i] = min(15, (int)__fadd_rn(__fmul_rn(v[i], id), 8.5f));
            // Value i pairs with value 16 + i: lanes 0-3 take lanes 4-7's quants as high nibbles.
            int hi[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) hi[i] = __shfl_down_sync(gmask, q[i], 4, 8);
            const uint32_t h = f32_to_f16_bits(d);
            if (gq < 4) {
#pragma unroll
                for (int i = 0; i < 4; ++i) o[2 + gq * 4 + i] = (uint8_t)(q[i] | (hi[i] << 4));
            }
            if (gq == 0) {
                o[0] = (uint8_t)(h & 0xff);
                o[1] = (uint8_t)(h >> 8);
                if (!fin || (h & 0x7fffu) == 0x7c00u) atomicOr(reject, 1u);
            }
        } else {
            float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
            for (int s = 4; s > 0; s >>= 1) {
                amax = fmaxf(amax, __shfl_xor_sync(gmask, amax, s));
                fin &= __shfl_xor_sync(gmask, fin, s);
            }
            const float d = __fdiv_rn(amax, 127.0f);
            float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
            if (!(id <= FLT_MAX)) id = 0.0f;
#pragma unroll
            for (int i = 0; i < 4; ++i) o[2 + gq * 4 + i] = (uint8_t)(int8_t)(int)roundf(__fmul_rn(v[i], id));
            if (gq == 0) {
                const uint32_t h = f32_to_f16_bits(d);
                o[0] = (uint8_t)(h & 0xff);
                o[1] = (uint8_t)(h >> 8);
                if (!fin || (h & 0x7fffu) == 0x7c00u) atomicOr(reject, 1u);
            }
        }
    }
}

// ---- launch helpers ------------------------------------------------------------

// CTAs per SM of a kernel at a launch shape, computed once per (device,
// kernel, threads, shared memory); the kernel's dynamic shared-memory limit is
// raised to the largest size seen. Host calls here are not stream operations,
// and after the first call at a shape none are made, so launches stay cheap
// and legal under stream capture.
struct OccKey {
    int dev;
    const void* fn;
    int threads;
    size_t smem;
    bool operator<(const OccKey& o) const {
        return std::tie(dev, fn, threads, smem) < std::tie(o.dev, o.fn, o.threads, o.smem);
    }
};

cudaError_t occupancy_cached(const void* fn, int threads, size_t smem, int* per_sm) {
    static std::mutex mu;
    static std::map<OccKey, int> cache;
    static std::map<std::pair<int, const void*>, size_t> smem_set;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> g(mu);
    const OccKey key{dev, fn, threads, smem};
    auto it = cache.find(key);
    if (it != cache.end()) {
        *per_sm = it->second;
        return cudaSuccess;
    }
    size_t& lim = smem_set[{dev, fn}];
    if (smem > lim) {
        e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        lim = smem;
    }
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(per_sm, fn, threads, smem);
    if (e != cudaSuccess) return e;
    cache[key] = *per_sm;
    return cudaSuccess;
}

template <typename K>
cudaError_t launch(K kernel, dim3 grid, dim3 block, size_t smem, const LaunchCfg& c, const QGemvParams& p) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = c.stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = c.pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, p);
}

template <int F, int M>
cudaError_t launch_fast_m(const LaunchCfg& c, const QGemvParams& p, size_t smem, bool dump) {
    void (*k)(QGemvParams);
    if (p.xq) k = gemv_q_fast<F, M, true, false>;
    else if (dump) k = gemv_q_fast<F, M, false, true>;
    else k = gemv_q_fast<F, M, false, false>;
    int per_sm = 0;
    cudaError_t e = occupancy_cached((const void*)k, c.warps * 32, smem, &per_sm);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorInvalidConfiguration;
    // Persistent: at most ctas_per_sm CTAs per SM (one by default, which
    // leaves room for the next GEMV's CTA beside it under programmatic
    // dependent launch); small problems still spread over every SM.
    const long long cap = (long long)std::min(per_sm, std::max(c.ctas_per_sm, 1)) * c.num_sms;
    const long long want = std::max<long long>(((long long)p.ntiles + c.warps - 1) / c.warps,
                                               std::min<long long>(p.ntiles, c.num_sms));
    const long long grid = std::min(want, cap);
    return launch(k, dim3((unsigned)std::max<long long>(grid, 1)), dim3(c.warps * 32), smem, c, p);
}

template <int F, int M>
cudaError_t launch_generic_m(const LaunchCfg& c, const QGemvParams& p, bool dump) {
    auto k = dump ? gemv_q_generic<F, M, true> : gemv_q_generic<F, M, false>;
    const int warps = 8;
    const long long want = ((long long)p.N + warps - 1) / warps;
    const long long grid = std::min<long long>(want, (long long)c.num_sms * 8);
    return launch(k, dim3((unsigned)std::max<long long>(grid, 1)), dim3(warps * 32), 0, c, p);
}

template <int F>
cudaError_t dispatch_m(const LaunchCfg& c, const QGemvParams& p, bool fast, size_t smem, bool dump) {
    switch (p.M) {
#define SMK_CASE(MM) \
    case MM: return fast ? launch_fast_m<F, MM>(c, p, smem, dump) : launch_generic_m<F, MM>(c, p, dump);
        SMK_CASE(1) SMK_CASE(2) SMK_CASE(3) SMK_CASE(4) SMK_CASE(5) SMK_CASE(6) SMK_CASE(7) SMK_CASE(8)
#undef SMK_CASE
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace

cudaError_t occupancy(const void* fn, int threads, size_t smem, int* per_sm) {
    return occupancy_cached(fn, threads, smem, per_sm);
}

size_t gemv_q_smem(int fmt, int M, int nsbp, int warps, int stages, bool x_in_smem) {
    size_t off = ((size_t)warps * stages * 8 + 127) & ~(size_t)127;
    if (x_in_smem) off += (xq_total_bytes(M, nsbp) + 127) & ~(size_t)127;
    return off + (size_t)warps * stages * 32 * sb_bytes(fmt);
}

cudaError_t launch_quantize_x(const LaunchCfg& c, const float* x, long long ldx, int M, int K, uint8_t* xq) {
    const int nb = K / kQK, nsbp = (nb + 7) / 8;
    const long long groups = (long long)M * nb;
    const long long grid = std::min<long long>((groups + kThreadsQuantX / 8 - 1) / (kThreadsQuantX / 8),
                                               (long long)c.num_sms * 4);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)std::max<long long>(grid, 1));
    cfg.blockDim = dim3(kThreadsQuantX);
    cfg.stream = c.stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = c.pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, quantize_x_kernel, x, ldx, M, nb, nsbp, xq);
}

cudaError_t launch_gemv_q(const LaunchCfg& c, int fmt, QGemvParams p, bool fast, size_t* smem_used) {
    const bool dump = p.dump != nullptr;
    size_t smem = 0;
    if (fast) smem = gemv_q_smem(fmt, p.M, p.nsbp, c.warps, p.stages, p.xq == nullptr);
    if (smem_used) *smem_used = smem;
    return fmt == kQ4_0 ? dispatch_m<kQ4_0>(c, p, fast, smem, dump) : dispatch_m<kQ8_0>(c, p, fast, smem, dump);
}

cudaError_t launch_quantize_w(cudaStream_t s, int fmt, const float* W, long long rows, int K, uint8_t* out,
                              unsigned* reject) {
    const long long nblocks = rows * (K / kQK);
    if (nblocks == 0) return cudaSuccess;
    const long long grid = std::min<long long>((nblocks + 31) / 32, 148LL * 16);
    if (fmt == kQ4_0)
        quantize_w_kernel<kQ4_0><<<(unsigned)grid, 256, 0, s>>>(W, nblocks, out, reject);
    else
        quantize_w_kernel<kQ8_0><<<(unsigned)grid, 256, 0, s>>>(W, nblocks, out, reject);
    return cudaGetLastError();
}

}  // namespace smk
