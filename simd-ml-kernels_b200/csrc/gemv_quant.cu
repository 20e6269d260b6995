// gemv_quant.cu — sm_100a decode GEMV on ggml Q4_0 / Q8_0 weights, M ≤ 8
// rows of x:  y[m][n] = Σ_b fp16(dw[n][b]) · dx[m][b] · Σ_i qw[n][b][i] · qx[m][b][i]
// (reference: src/kernels/quant/q4_0.hpp:23-30, q8_0.hpp:19-30; x quantized to
// Q8 blocks once per call with FP32 scales, q8_0_scalar.cpp:113-166).
//
// Fast kernel (K % 256 == 0, weights 16-byte aligned): a row of K/32 ggml
// blocks is K/256 superblocks of 8 blocks = 144 bytes (Q4_0) or 272 (Q8_0),
// both multiples of 16, so every superblock of every row starts on a 16-byte
// boundary. Each warp owns a ring of shared-memory stages that it fills with
// 1-D bulk TMA copies (cp.async.bulk, no multicast), completed on one
// mbarrier per stage; a stage is a tile of TR rows × G superblocks, one
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

#include <cudaTypedefs.h>

#include <algorithm>
#include <cfloat>
#include <map>
#include <mutex>
#include <tuple>

namespace smk {

namespace {

constexpr int kThreadsQuantX = 256;

// ---- activation quantization --------------------------------------------------

// Eight threads per 32-value block, four values each. Bit-exact with the
// reference's quantize_x_q8 (q8_0_scalar.cpp:45-61,113-118): amax/127 and 1/d
// as IEEE divisions, w·id rounded once, then rounded half away from zero.
// Each thread first loads the values of up to kXUnroll blocks, so a GEMV's
// prologue waits for one round trip to L2 rather than one per block.
constexpr int kXUnroll = 4;

__device__ __forceinline__ float4 load_x4(const float* p) {
    if ((reinterpret_cast<uintptr_t>(p) & 15) == 0) return *reinterpret_cast<const float4*>(p);
    return make_float4(p[0], p[1], p[2], p[3]);
}

struct XGeom {
    int M, nb, log2G, ksteps;
    int r4;   // the four-row layout (one row of x)
};

// The decode step's SwiGLU input of the down projection, silu(g) * u, with
// silu(g) = g / (1 + exp(−g)) as the reference defines it
// (src/kernels/scalar_kernels.cpp:196-198; silu_avx2.cpp:1-26): IEEE divide
// and product, CUDA's expf (a few ulp), so the value is within the reference's
// own SiLU tolerance of 1e-35 + 1e-6·|SiLU(g)| before the product. For
// g < −88.7, exp(−g) overflows, the denominator is +inf and the result −0;
// silu(−inf) = NaN and silu(+inf) = +inf, as the reference's kernels.
__device__ __forceinline__ float silu_mul1(float g, float u) {
    return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
}
__device__ __forceinline__ float4 silu_mul4(float4 g, float4 u) {
    return make_float4(silu_mul1(g.x, u.x), silu_mul1(g.y, u.y), silu_mul1(g.z, u.z), silu_mul1(g.w, u.w));
}

// One row's 4 activation values at element offset k: x, or silu(x) * up.
__device__ __forceinline__ float4 load_act4(const float* xr, const float* ur, size_t k) {
    return ur ? silu_mul4(load_x4(xr + k), load_x4(ur + k)) : load_x4(xr + k);
}

// ---- RMSNorm fused into the quantization (the reference's rms_norm,
// examples/llama/llama.py:184-188, in add_rmsnorm_kernel's arithmetic) ----

// Σ over the CTA of each thread's partial: a shuffle tree per warp, then the
// warps' sums in warp order, the same order in every CTA of a launch (so
// every CTA derives the same scale). All threads call it; all get the sum.
__device__ __forceinline__ float cta_sum(float v) {
    __shared__ float red[32];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    __syncthreads();   // red may still be read by a previous call's threads
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float s = 0.0f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) s = __fadd_rn(s, red[w]);
    return s;
}
// fl(1 / sqrt(fl(ss / n) + eps)), the root and quotient in double.
__device__ __forceinline__ float rms_inv(float ss, int n, double eps) {
    return (float)(1.0 / sqrt((double)__fdiv_rn(ss, (float)n) + eps));
}
__device__ __forceinline__ float sq_sum4(float4 v) {
    return __fadd_rn(__fadd_rn(__fmul_rn(v.x, v.x), __fmul_rn(v.y, v.y)),
                     __fadd_rn(__fmul_rn(v.z, v.z), __fmul_rn(v.w, v.w)));
}
// h = w · (v · inv), each product rounded.
__device__ __forceinline__ float4 norm4v(float4 v, float4 g, float inv) {
    return make_float4(__fmul_rn(g.x, __fmul_rn(v.x, inv)), __fmul_rn(g.y, __fmul_rn(v.y, inv)),
                       __fmul_rn(g.z, __fmul_rn(v.z, inv)), __fmul_rn(g.w, __fmul_rn(v.w, inv)));
}
// inv of row xr (n values, n % 4 == 0) read by the whole CTA, quads strided over its threads.
__device__ __forceinline__ float cta_row_rms_inv(const float* xr, int n, double eps) {
    float ss = 0.0f;
    for (int i = threadIdx.x * 4; i < n; i += blockDim.x * 4) ss = __fadd_rn(ss, sq_sum4(load_x4(xr + i)));
    return rms_inv(cta_sum(ss), n, eps);
}

// One thread's 4 values of a 32-value block, quantized to Q8: all 32 lanes of
// the warp call this together (full-mask shuffles; the xor offsets stay inside
// each 8-lane group of one block).
struct Q8Quad {
    uint32_t word;   // the 4 int8 quants, value 0 in the low byte
    float dx;        // the block's scale; NaN when a value of the block is not finite
    int s;           // Σ of the block's 32 quants
};

__device__ __forceinline__ Q8Quad quantize_quad(float4 v) {
    constexpr unsigned gmask = 0xffffffffu;
    // max |v| over the block as integer bits: for non-negative floats the bit
    // order is the value order, and +inf / NaN lie above every finite value, so
    // one reduction gives both amax and whether the block is finite.
    unsigned a = max(max(__float_as_uint(v.x) & 0x7fffffffu, __float_as_uint(v.y) & 0x7fffffffu),
                     max(__float_as_uint(v.z) & 0x7fffffffu, __float_as_uint(v.w) & 0x7fffffffu));
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) a = max(a, __shfl_xor_sync(gmask, a, o));
    const bool fin = a < 0x7f800000u;
    const float d = div127_rn(__uint_as_float(a));   // RN(amax / 127)
    // RN(1 / d), 0 when d is 0 or the reciprocal overflows (the reference's id).
    float id = d != 0.0f ? rcp_rn(d) : 0.0f;
    if (!(id <= FLT_MAX)) id = 0.0f;
    // |v·id| <= 127·(1 + 2^-22) < 128 for a finite block.
    const int q0 = fin ? round_half_away(__fmul_rn(v.x, id)) : 0;
    const int q1 = fin ? round_half_away(__fmul_rn(v.y, id)) : 0;
    const int q2 = fin ? round_half_away(__fmul_rn(v.z, id)) : 0;
    const int q3 = fin ? round_half_away(__fmul_rn(v.w, id)) : 0;
    Q8Quad r;
    r.word = (uint32_t)(q0 & 0xff) | ((uint32_t)(q1 & 0xff) << 8) | ((uint32_t)(q2 & 0xff) << 16) |
             ((uint32_t)(q3 & 0xff) << 24);
    int s = q0 + q1 + q2 + q3;
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) s += __shfl_xor_sync(gmask, s, o);
    r.s = s;
    r.dx = fin ? d : __int_as_float(0x7fc00000);
    return r;
}

// int → float without a conversion instruction: for |v| < 2^22 the float with
// bits 0x4B400000 + v is 1.5·2^23 + v exactly (ulp 1 in [2^23, 2^24)), so
// subtracting 1.5·2^23 leaves float(v) exactly. A block's bias −8·Σq rides in the
// same integer add: float(isum) = bits(c + magic − 8Σq) − 1.5·2^23, with
// |isum| ≤ 32·15·127 + 8·32·127 far below 2^22 (Q8_0: ≤ 32·127·127).
constexpr int kIntToFloatMagic = 0x4B400000;
constexpr float kIntToFloatMagicF = 12582912.0f;

// quantize_quad, stored in the lane-major layout; lanes with valid == false
// compute on their (zero) values and store nothing.
__device__ __forceinline__ void quantize_x_block(float4 v, int gq, bool valid, const XGeom& xg, int m, int b,
                                                 uint8_t* xb) {
    const Q8Quad q = quantize_quad(v);
    if (xg.r4) {   // slot (ks·32 + 4g + j) of the four-row layout, b = 64·ks + 8g + 2j + odd
        const unsigned ks = (unsigned)b >> 6, g = ((unsigned)b >> 3) & 7u, jb = (unsigned)b & 7u;
        uint8_t* slot = xb + (ks * 32u + g * 4u + (jb >> 1)) * 80u;
        if (!valid) return;
        *reinterpret_cast<uint32_t*>(slot + (jb & 1u) * 32u + (unsigned)gq * 4u) = q.word;
        // The bias carries the magic number: the block's sum leaves dp4a as the bit
        // pattern of 1.5·2^23 + isum, and one exact subtraction makes it a float.
        if (gq == 0)
            *reinterpret_cast<float2*>(slot + 64u + (jb & 1u) * 8u) =
                make_float2(q.dx, __int_as_float(kIntToFloatMagic - 8 * q.s));
        return;
    }
    // Offsets in 32 bits (the layout stays far below 4 GiB), no division.
    const unsigned sb = (unsigned)b >> 3, j = (unsigned)b & 7u;
    const unsigned ks = sb >> xg.log2G, g = sb & ((1u << xg.log2G) - 1u);
    const unsigned mk = (unsigned)m * (unsigned)xg.ksteps + ks;
    if (!valid) return;
    *reinterpret_cast<uint32_t*>(xb + ((mk * 16u + 2u * j + (unsigned)(gq >> 2)) * 32u + g) * 16u + (gq & 3) * 4) =
        q.word;
    if (gq == 0) {
        *reinterpret_cast<float2*>(xb + (unsigned)xg.M * (unsigned)xg.ksteps * 8192u + ((mk * 8u + j) * 32u + g) * 8u) =
            make_float2(q.dx, __int_as_float(-8 * q.s));
    }
}

// Quantize x [M, K] into the lane-major layout at xb; tid in [0, nthreads),
// nthreads a multiple of 32. Warp w takes blocks 4w .. 4w+3 (one per 8-lane
// group), then the next 4·warps, so every lane of a warp runs every
// iteration. MT: rows of x known at compile time (0: xg.M).
// nw != nullptr: each row RMS-normalised first (the whole CTA computes the
// row's scale: every thread of the CTA must call this).
template <int MT>
__device__ __forceinline__ void quantize_x_rows(const float* __restrict__ x, long long ldx,
                                                const float* __restrict__ up, long long ldu, const XGeom& xg,
                                                uint8_t* xb, int tid, int nthreads, const float* nw = nullptr,
                                                double neps = 0.0) {
    const int gq = tid & 7, grp = (tid & 31) >> 3;
    const int wstride = (nthreads >> 5) * 4, nb = xg.nb;
    const int rows = MT > 0 ? MT : xg.M;
#pragma unroll
    for (int m = 0; m < (MT > 0 ? MT : kMaxRows); ++m) {
        if (m >= rows) break;
        const float* xr = x + (size_t)m * ldx + gq * 4;
        const float* ur = up ? up + (size_t)m * ldu + gq * 4 : nullptr;
        const float inv = nw ? cta_row_rms_inv(x + (size_t)m * ldx, nb * kQK, neps) : 0.0f;
        for (int wbase = (tid >> 5) * 4; wbase < nb; wbase += kXUnroll * wstride) {
            float4 v[kXUnroll];
            if (nw) {
                float4 gw[kXUnroll];
#pragma unroll
                for (int u = 0; u < kXUnroll; ++u) {   // x and the norm's weights, all loads in flight together
                    const int b = wbase + u * wstride + grp;
                    v[u] = b < nb ? load_x4(xr + (size_t)b * kQK) : make_float4(0.f, 0.f, 0.f, 0.f);
                    gw[u] = b < nb ? load_x4(nw + (size_t)b * kQK + gq * 4) : make_float4(0.f, 0.f, 0.f, 0.f);
                }
#pragma unroll
                for (int u = 0; u < kXUnroll; ++u) v[u] = norm4v(v[u], gw[u], inv);
            } else {
#pragma unroll
                for (int u = 0; u < kXUnroll; ++u) {
                    const int b = wbase + u * wstride + grp;
                    v[u] = b < nb ? load_act4(xr, ur, (size_t)b * kQK) : make_float4(0.f, 0.f, 0.f, 0.f);
                }
            }
#pragma unroll
            for (int u = 0; u < kXUnroll; ++u) {
                if (wbase + u * wstride >= nb) break;   // warp-uniform
                const int b = wbase + u * wstride + grp;
                quantize_x_block(v[u], gq, b < nb, xg, m, b, xb);
            }
        }
    }
}

__global__ void __launch_bounds__(kThreadsQuantX) quantize_x_kernel(const float* __restrict__ x, long long ldx,
                                                                     const float* __restrict__ up, long long ldu,
                                                                     XGeom xg, uint8_t* xq, const float* nw,
                                                                     double neps) {
    pdl_launch_dependents();
    pdl_wait_primary();   // x comes from the previous kernel; xq may still be read by it
    quantize_x_rows<0>(x, ldx, up, ldu, xg, xq, blockIdx.x * blockDim.x + threadIdx.x, gridDim.x * blockDim.x, nw,
                       neps);
}

__global__ void __launch_bounds__(256) silu_mul_kernel(long long n, const float* __restrict__ g,
                                                       const float* __restrict__ u, float* __restrict__ out) {
    pdl_launch_dependents();
    pdl_wait_primary();
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        out[i] = silu_mul1(g[i], u[i]);
}

// Test hook: the exact helpers of quantize_quad against CUDA's own operations over
// their whole domains; bad[0] divisions (every finite a >= 0), bad[1] reciprocals
// (every 2^-126 <= d <= 2^126), bad[2] roundings (every |t| <= 128) that differ.
// A host-memory call's activations: n floats from page-locked host memory
// mapped into the device's address space (src) to device memory (dst), 16
// bytes per thread when both are aligned. A kernel rather than a copy-engine
// transfer: the GEMV after it launches at once under programmatic dependent
// launch and streams its weights while these loads cross the bus, and a CUDA
// graph of the call holds kernels only.
__global__ void __launch_bounds__(512) stage_x_kernel(const float* __restrict__ src, float* __restrict__ dst,
                                                      long long n) {
    pdl_launch_dependents();
    pdl_wait_primary();
    const long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x, nt = (long long)gridDim.x * blockDim.x;
    if (((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15) == 0) {
        for (long long i = t; i < n / 4; i += nt)
            reinterpret_cast<float4*>(dst)[i] = reinterpret_cast<const float4*>(src)[i];
        for (long long i = n / 4 * 4 + t; i < n; i += nt) dst[i] = src[i];
    } else {
        for (long long i = t; i < n; i += nt) dst[i] = src[i];
    }
}

__global__ void __launch_bounds__(256) check_x_arith_kernel(unsigned long long* bad) {
    unsigned long long b0 = 0, b1 = 0, b2 = 0;
    const unsigned long long stride = (unsigned long long)gridDim.x * blockDim.x;
    const unsigned long long t0 = (unsigned long long)blockIdx.x * blockDim.x + threadIdx.x;
    for (unsigned long long i = t0; i < 0x7f800000ull; i += stride) {
        const float a = __uint_as_float((unsigned)i);
        b0 += __float_as_uint(div127_rn(a)) != __float_as_uint(__fdiv_rn(a, 127.0f));
    }
    for (unsigned long long i = 0x00800000ull + t0; i <= 0x7e800000ull; i += stride) {
        const float d = __uint_as_float((unsigned)i);
        b1 += __float_as_uint(rcp_rn(d)) != __float_as_uint(__frcp_rn(d));
    }
    for (unsigned long long i = t0; i <= 0x43000000ull; i += stride) {   // 0 .. 128
        const float t = __uint_as_float((unsigned)i);
        b2 += (round_half_away(t) != (int)roundf(t)) + (round_half_away(-t) != (int)roundf(-t));
    }
    atomicAdd(&bad[0], b0);
    atomicAdd(&bad[1], b1);
    atomicAdd(&bad[2], b2);
}

// ---- integer block dots -----------------------------------------------------------

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

// The x data of one lane for one superblock: quants at xq + (2j + h)·512 and
// (dx, bias) at xd + j·256, for each row m at + m·mstride_q / m·mstride_d.
struct XPtr {
    const uint8_t* xq;
    const uint8_t* xd;
    size_t mstride_q, mstride_d;
};

// One block j: integer sums against every x row, then acc[m] += isum·(dw·dx).
template <int F, int M, bool kShX, bool kDump>
__device__ __forceinline__ void block_dot(const uint32_t (&q)[8], float dw, const XPtr& xp, int j, float (&acc)[M],
                                          int32_t* dump, size_t dump_stride, size_t dump_idx) {
#pragma unroll
    for (int m = 0; m < M; ++m) {
        const uint4 xl = ld_x16<kShX>(xp.xq + m * xp.mstride_q + (2 * j) * 512);
        const uint4 xh = ld_x16<kShX>(xp.xq + m * xp.mstride_q + (2 * j + 1) * 512);
        const float2 db = ld_x8<kShX>(xp.xd + m * xp.mstride_d + j * 256);
        int isum;
        if constexpr (F == kQ4_0) {
            // q[0..3]: the 16 nibble bytes; low nibbles are values 0-15, high 16-31.
            // Four chains of two dp4a each (integer sums: any grouping is exact).
            int a = dp4a_us(q[0] & 0x0F0F0F0Fu, xl.x, __float_as_int(db.y));
            int a2 = dp4a_us(q[1] & 0x0F0F0F0Fu, xl.y, 0);
            int h = dp4a_us(q[0] & 0xF0F0F0F0u, xh.x, 0);
            int h2 = dp4a_us(q[1] & 0xF0F0F0F0u, xh.y, 0);
            a = dp4a_us(q[2] & 0x0F0F0F0Fu, xl.z, a);
            a2 = dp4a_us(q[3] & 0x0F0F0F0Fu, xl.w, a2);
            h = dp4a_us(q[2] & 0xF0F0F0F0u, xh.z, h);
            h2 = dp4a_us(q[3] & 0xF0F0F0F0u, xh.w, h2);
            isum = (a + a2) + ((h + h2) >> 4);   // h + h2 is 16·Σ hi·x: exact
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

// One superblock (8 blocks) of weights at sp (shared memory, 16-byte aligned).
template <int F, int M, bool kShX, bool kDump>
__device__ __forceinline__ void superblock(const uint8_t* sp, const XPtr& xp, float (&acc)[M], int32_t* dump,
                                           size_t dump_stride, size_t dump_base) {
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
            block_dot<F, M, kShX, kDump>(q, half_bits_to_float(sc), xp, j, acc, dump, dump_stride, dump_base + j);
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
                block_dot<F, M, kShX, kDump>(q, half_bits_to_float(sc), xp, j, acc, dump, dump_stride, dump_base + j);
            }
        }
    }
}

// ---- the fast kernel -----------------------------------------------------------------

// The CTA that finishes last copies y from device memory into the mapped
// page-locked output. Every SM that writes host memory has its writes flushed
// over the bus before the kernel can complete; measured on a B200, one CTA
// copying 32 KB after the others stored y in device memory ends about 1.6 µs
// sooner than 296 CTAs each storing their rows into host memory. Every thread
// of the CTA calls this once, after its last store of y.
__device__ __forceinline__ void copy_y_to_host(const QGemvParams& p) {
    __shared__ unsigned last;
    __threadfence();   // this thread's rows of y before the CTA's ticket
    __syncthreads();
    if (threadIdx.x == 0) last = atomicAdd(p.ticket, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!last) return;
    __threadfence();   // every other CTA's rows, seen through their tickets
    const size_t n = (size_t)p.N;
    const bool vec = (n & 3) == 0 && (p.ldy & 3) == 0 && ((reinterpret_cast<uintptr_t>(p.y) | reinterpret_cast<uintptr_t>(p.yhost)) & 15) == 0;
    for (int m = 0; m < p.M; ++m) {
        const float* src = p.y + (size_t)m * p.ldy;
        float* dst = p.yhost + (size_t)m * p.ldy;
        if (vec) {
            const float4* s4 = reinterpret_cast<const float4*>(src);
            float4* d4 = reinterpret_cast<float4*>(dst);
            for (size_t i = threadIdx.x; i < (n >> 2); i += blockDim.x) d4[i] = __ldcg(s4 + i);
        } else {
            for (size_t i = threadIdx.x; i < n; i += blockDim.x) dst[i] = __ldcg(src + i);
        }
    }
    if (threadIdx.x == 0) *p.ticket = 0u;   // for the next launch, which the stream orders after this one
}

// Issue the bulk copies of one work item (tile, k-step ks) of this warp into stage `slot`.
template <int F>
__device__ __forceinline__ void issue_item(const QGemvParams& p, int tile, int ks, int slot, uint8_t* stages,
                                           uint64_t* bars, int lane) {
    constexpr int SBB = sb_bytes(F);
    const int rows = min(p.TR, p.N - tile * p.TR);
    const int sb0 = ks * p.G;
    const int cnt = min(p.G, p.nsbp - sb0);
    const uint32_t bytes = (uint32_t)cnt * SBB;
    const size_t row_bytes = (size_t)p.nsbp * SBB;
    uint8_t* dst = stages + (size_t)slot * (32 * SBB);
    if (lane == 0) mbar_arrive_expect_tx(&bars[slot], bytes * rows);
    __syncwarp();
    if (p.ksteps == 1 && p.G == p.nsbp) {
        // Whole rows, back to back in memory and in the stage: one copy.
        if (lane == 0) tma_load_1d(dst, p.w + (size_t)tile * p.TR * row_bytes, bytes * rows, &bars[slot]);
    } else if (lane < rows) {
        const uint8_t* src = p.w + ((size_t)tile * p.TR + lane) * row_bytes + (size_t)sb0 * SBB;
        tma_load_1d(dst + (size_t)lane * p.G * SBB, src, bytes, &bars[slot]);
    }
}

// Position of a warp in its sequence of work items, advanced without division.
struct ItemCursor {
    int tile, ks, slot;
    uint32_t phase;
    __device__ __forceinline__ void next(const QGemvParams& p, int GW) {
        if (++ks == p.ksteps) { ks = 0; tile += GW; }
        if (++slot == p.stages) { slot = 0; phase ^= 1u; }
    }
};

// Fused all-gather, this rank's side of a step: the entry of its output row 0,
// slice row 0 in area (epoch & 1), and the step's tag. Read after
// griddepcontrol.wait: the previous step's wait kernel, which advances the
// epoch, has completed by then.
struct GatherStep {
    long long off;
    unsigned tag;
};
__device__ __forceinline__ GatherStep gather_step(const GatherArgs* ga) {
    const unsigned epoch = *reinterpret_cast<volatile const unsigned*>(ga->ctrl[ga->rank]);
    return {(long long)(epoch & 1u) * ga->area + (long long)ga->rank * ga->npad, epoch + 1u};
}
// The padding rows [n, npad) of this rank's slice, output rows 0 .. M-1: zeros
// in this rank's area and, tagged, in every peer's (the peers wait for every
// entry of the slice), by thread t of nt.
__device__ __forceinline__ void gather_pad(const GatherArgs* ga, int M, int n, int t, int nt) {
    const int pad = ga->npad - n;
    if (pad <= 0) return;
    const GatherStep gs = gather_step(ga);
    const long long cols = (long long)ga->world * ga->npad;
    const unsigned long long w = tagged_word(0.0f, gs.tag);
    for (int i = t; i < M * pad; i += nt) {
        const int m = i / pad, row = n + i % pad;
        const long long o = gs.off + m * cols + row;
        ga->y[o] = 0.0f;
        for (int rk = 0; rk < ga->world; ++rk)
            if (rk != ga->rank) st_relaxed_sys_u64(ga->ll[rk] + o, w);
    }
}

// After a warp's last item. With a fused gather the kernel's y is this rank's
// staging slice (p.y, output rows p.ldy apart): the loop stores exactly as
// without a gather, and nothing of the gather stays live in its registers.
// Here the values of the warp's finished tiles (TR rows each, M output rows)
// go from there into this rank's full-y area and, as tagged words, into every
// peer's receive area, one entry per lane. The tiles are the ones before
// `end` (the warp's cursor after its loop) in steps of `step`, down to the
// CTA's first tile (p.contiguous) or 0; ctaid is read anew so that nothing
// from before the loop has to be kept. The receivers wait for the step's last
// tile in any case, so sending after the loop costs them nothing.
// First tile of CTA bx's contiguous range (the range of bx is [first(bx),
// first(bx + 1))): an even share of the tiles, the first cta_r CTAs one more.
// The launcher splits ntiles = cta_q · grid + cta_r, so the device divides nothing.
__device__ __forceinline__ int cta_first_tile(const QGemvParams& p, int bx) { return bx * p.cta_q + min(bx, p.cta_r); }

__device__ __forceinline__ void gather_send(const QGemvParams& p, int M, int TR, int end, int step, int lane) {
    const GatherArgs* ga = p.gather;
    __syncwarp();   // the lanes' stores to p.y are visible to the whole warp
    unsigned bx;
    asm volatile("mov.u32 %0, %%ctaid.x;" : "=r"(bx));
    const int lo = p.contiguous ? cta_first_tile(p, (int)bx) : 0;
    const GatherStep gs = gather_step(ga);
    const long long cols = (long long)ga->world * ga->npad;
    const int per = M * TR;
    // Entries (tile, output row, tile row) of every finished tile spread over
    // the lanes, so that their loads are in flight together (a tile of one row
    // would otherwise leave 31 lanes idle and the tiles one L2 trip apart).
    const int first = end - step, ntiles = first >= lo ? (first - lo) / step + 1 : 0;
    for (int i = lane; i < ntiles * per; i += 32) {
        const int ti = i / per, e = i - ti * per, tile = first - ti * step;
        const int m = e / TR, row = tile * TR + (e - m * TR);
        if (row < p.N) {
            const float v = p.y[(size_t)m * p.ldy + row];
            const long long o = gs.off + m * cols + row;
            ga->y[o] = v;
            const unsigned long long w = tagged_word(v, gs.tag);
            for (int rk = 0; rk < ga->world; ++rk)
                if (rk != ga->rank) st_relaxed_sys_u64(ga->ll[rk] + o, w);
        }
    }
}

template <int F, int M, bool kXGlobal, bool kDump>
__device__ __forceinline__ void gemv_q_fast_body(const QGemvParams& p) {
    constexpr int SBB = sb_bytes(F);
    extern __shared__ __align__(128) uint8_t smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;

    uint64_t* bars = reinterpret_cast<uint64_t*>(smem) + warp * p.stages;
    size_t off = ((size_t)nwarps * p.stages * 8 + 127) & ~(size_t)127;
    uint8_t* xs = smem + off;
    if constexpr (!kXGlobal) off += (xq_total_bytes(M, p.ksteps) + 127) & ~(size_t)127;
    uint8_t* stages = smem + off + (size_t)warp * p.stages * 32 * SBB;

    // A fused gather's wait kernel reads the epoch when it starts, so it may
    // only launch once the previous one has completed: after griddepcontrol.wait.
    if (!p.gather) pdl_launch_dependents();

    // Tiles of this warp: gw, gw + GW, ...; each tile is ksteps items. With
    // p.contiguous the CTA owns a contiguous, even share of the tiles (each SM
    // streams one region of W) and its warps take them in turn; otherwise the
    // tiles are interleaved over every warp of the grid.
    int GW, gw, tiles_end;
    if (p.contiguous) {
        GW = nwarps;
        gw = cta_first_tile(p, blockIdx.x) + warp;
        tiles_end = cta_first_tile(p, blockIdx.x + 1);
    } else {
        GW = gridDim.x * nwarps;
        gw = warp * gridDim.x + blockIdx.x;
        tiles_end = p.ntiles;
    }
    const int my_tiles = gw < tiles_end ? (tiles_end - 1 - gw) / GW + 1 : 0;
    const int nitems = my_tiles * p.ksteps;

    if (lane == 0) {
        for (int s = 0; s < p.stages; ++s) mbar_init(&bars[s], 1);
        fence_mbar_init();
    }
    __syncwarp();
    // Cursors: `cur` consumes, `iss` issues (p.stages items ahead).
    ItemCursor cur{gw, 0, 0, 0u}, iss{gw, 0, 0, 0u};
    int issued = 0;
    for (; issued < min(p.stages, nitems); ++issued) {
        issue_item<F>(p, iss.tile, iss.ks, iss.slot, stages, bars, lane);
        iss.next(p, GW);
    }

    pdl_wait_primary();
    if (p.gather) pdl_launch_dependents();
    if constexpr (!kXGlobal) {
        const XGeom xg{M, p.nb, p.log2G, p.ksteps, 0};
        quantize_x_rows<M>(p.x, p.ldx, p.up, p.ldu, xg, xs, threadIdx.x, blockDim.x, p.nw, p.neps);
        __syncthreads();
    }
    const uint8_t* xb = kXGlobal ? p.xq : xs;

    const int r = lane >> p.log2G, g = lane & (p.G - 1);
    // Fused all-gather: this step's y goes into this rank's full-y area
    // (epoch & 1) and, tagged, into every peer's receive area, at this rank's slice.
    if (p.gather && blockIdx.x == 0) gather_pad(p.gather, M, p.N, threadIdx.x, blockDim.x);
    XPtr xp;
    xp.mstride_q = (size_t)p.ksteps * 8192;
    xp.mstride_d = (size_t)p.ksteps * 2048;
    const uint8_t* xd0 = xb + (size_t)M * p.ksteps * 8192;
    float acc[M];
#pragma unroll
    for (int m = 0; m < M; ++m) acc[m] = 0.0f;

    for (int it = 0; it < nitems; ++it) {
        if (__any_sync(0xffffffffu, !mbar_wait_bounded(&bars[cur.slot], cur.phase, p.err))) {   // warp-uniform
            // Give the copies still in flight a bounded chance to land before
            // the CTA's shared memory is released, then stop.
            ItemCursor c2 = cur;
            for (int k = it + 1; k < issued; ++k) {
                c2.next(p, GW);
                mbar_wait_bounded(&bars[c2.slot], c2.phase, nullptr);
            }
            break;
        }
        const int row = cur.tile * p.TR + r, sb = cur.ks * p.G + g;
        xp.xq = xb + ((size_t)cur.ks * 16 * 32 + g) * 16;
        xp.xd = xd0 + ((size_t)cur.ks * 8 * 32 + g) * 8;
        const uint8_t* sp = stages + (size_t)cur.slot * (32 * SBB) + (size_t)lane * SBB;
        const size_t dstride = (size_t)p.N * p.nb, dbase = (size_t)row * p.nb + (size_t)sb * 8;
        // A full tile (every lane has a row and a superblock: warp-uniform)
        // runs without a per-lane guard.
        if ((cur.tile + 1) * p.TR <= p.N && (cur.ks + 1) * p.G <= p.nsbp)
            superblock<F, M, !kXGlobal, kDump>(sp, xp, acc, p.dump, dstride, dbase);
        else if (row < p.N && sb < p.nsbp)
            superblock<F, M, !kXGlobal, kDump>(sp, xp, acc, p.dump, dstride, dbase);
        if (cur.ks == p.ksteps - 1) {
#pragma unroll
            for (int m = 0; m < M; ++m) {
                float v = acc[m];
                for (int o = p.G >> 1; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                if (g == 0 && row < p.N)
                    p.y[(size_t)m * p.ldy + row] = p.res ? __fadd_rn(p.res[(size_t)m * p.ldr + row], v) : v;
                acc[m] = 0.0f;
            }
        }
        __syncwarp();
        if (issued < nitems) {
            fence_proxy_async_smem();
            issue_item<F>(p, iss.tile, iss.ks, iss.slot, stages, bars, lane);
            iss.next(p, GW);
            ++issued;
        }
        cur.next(p, GW);
    }
    if (p.gather) gather_send(p, M, p.TR, cur.tile, GW, lane);
    if (p.yhost) copy_y_to_host(p);   // every warp gets here, the ones that gave up too
}

template <int F, int M, bool kXGlobal, bool kDump>
__global__ void __launch_bounds__(512) gemv_q_fast(const QGemvParams p) {
    gemv_q_fast_body<F, M, kXGlobal, kDump>(p);
}

// Q4_0 with one or two rows runs two 512-thread CTAs per SM on small
// matrices (the launch tuning): at most 64 registers a thread.
template <int F, int M, bool kXGlobal, bool kDump>
__global__ void __launch_bounds__(512, 2) gemv_q_fast2(const QGemvParams p) {
    gemv_q_fast_body<F, M, kXGlobal, kDump>(p);
}

// After this rank's fused-gather GEMV of a step: poll this rank's receive area
// until every peer entry of the step (M output rows × (world − 1) slices of
// npad) shows the step's tag, copy the values into the full-y area, then, once
// the GEMV has completed (its own slice is in the area by then), advance the
// epoch: the last CTA to finish, counted on the ticket word. The polling
// starts as soon as the CTAs find room, while the GEMV may still run, and a
// peer's word is usable the moment it lands. Each thread polls eight entries
// at a time with independent loads. A wait longer than kWaitLimitNs sets
// kErrPeerTimeout and leaves the remaining entries of that thread as they
// were; the epoch still advances.
__global__ void __launch_bounds__(kGatherWaitThreads) gather_wait_kernel(const GatherArgs* __restrict__ ga, int M,
                                                                          unsigned* err) {
    pdl_launch_dependents();
    const int W = ga->world, me = ga->rank;
    const unsigned np = (unsigned)ga->npad;
    unsigned* ctrl = ga->ctrl[me];
    const unsigned epoch = *reinterpret_cast<volatile const unsigned*>(ctrl);
    const unsigned tag = epoch + 1u;
    const long long base = (long long)(epoch & 1u) * ga->area, cols = (long long)W * np;
    const unsigned seg = (unsigned)(W - 1) * np, total = (unsigned)M * seg;
    const unsigned nthr = gridDim.x * blockDim.x;
    const unsigned long long* src = ga->ll[me];
    float* dst = ga->y;
    bool ok = true;
    constexpr int kPer = 8;
    for (unsigned e0 = blockIdx.x * blockDim.x + threadIdx.x; ok && e0 < total; e0 += kPer * nthr) {
        long long off[kPer];
        unsigned need = 0;
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
            const unsigned e = e0 + j * nthr;
            off[j] = 0;
            if (e < total) {
                const unsigned m = e / seg, rem = e - m * seg, pi = rem / np, row = rem - pi * np;
                const unsigned rk = pi + (pi >= (unsigned)me ? 1u : 0u);
                off[j] = base + m * cols + (long long)rk * np + row;
                need |= 1u << j;
            }
        }
        const unsigned long long t0 = globaltimer();
        for (uint32_t it = 0; need; ++it) {
            unsigned long long w[kPer];
#pragma unroll
            for (int j = 0; j < kPer; ++j) w[j] = (need >> j & 1u) ? ld_relaxed_sys_u64(src + off[j]) : 0ull;
#pragma unroll
            for (int j = 0; j < kPer; ++j)
                if ((need >> j & 1u) && (unsigned)(w[j] >> 32) == tag) {
                    dst[off[j]] = __uint_as_float((unsigned)w[j]);
                    need &= ~(1u << j);
                }
            if (need && (it & 15u) == 15u && globaltimer() - t0 > kWaitLimitNs) ok = false;
            if (!ok) break;
        }
    }
    pdl_wait_primary();   // this rank's GEMV of the step has completed
    ok = __syncthreads_and(ok);
    if (threadIdx.x == 0) {
        if (!ok && err) atomicOr(err, kErrPeerTimeout);
        bool last = true;
        if (gridDim.x > 1) {
            __threadfence();
            last = atomicAdd(ctrl + kGatherTicket, 1u) == gridDim.x - 1;
        }
        if (last) {
            if (gridDim.x > 1) ctrl[kGatherTicket] = 0u;
            *reinterpret_cast<volatile unsigned*>(ctrl) = epoch + 1u;
        }
    }
}

// A gather step without data, one warp: a cross-GPU barrier in stream order.
// After the previous kernel on the stream has completed, signal every peer
// (this rank's word in its control block: the step's tag, a system-scope
// release that also publishes the earlier kernels' stores), wait (bounded)
// until every peer's word here has reached the tag, then advance the epoch.
// A peer is at most one step ahead, and its words only grow, so ≥ (in
// wrap-around arithmetic) is the test. On a timeout the epoch still advances
// and the error word gets kErrPeerTimeout.
__global__ void __launch_bounds__(32) gather_barrier_kernel(const GatherArgs* __restrict__ ga, unsigned* err) {
    pdl_launch_dependents();
    pdl_wait_primary();
    const int lane = threadIdx.x;
    unsigned* ctrl = ga->ctrl[ga->rank];
    const unsigned epoch = *reinterpret_cast<volatile unsigned*>(ctrl);
    const unsigned want = epoch + 1u;
    bool ok = true;
    if (lane < ga->world && lane != ga->rank) {
        __threadfence_system();
        st_release_sys_u32(ga->ctrl[lane] + kGatherSignals + ga->rank, want);
        const unsigned* sig = ctrl + kGatherSignals + lane;
        const unsigned long long t0 = globaltimer();
        for (uint32_t i = 0; (int)(ld_acquire_sys(sig) - want) < 0; ++i) {
            if ((i & 63u) == 0 && globaltimer() - t0 > kWaitLimitNs) {
                ok = false;
                break;
            }
        }
    }
    ok = __all_sync(0xffffffffu, ok);
    if (lane == 0) {
        if (!ok && err) atomicOr(err, kErrPeerTimeout);
        *reinterpret_cast<volatile unsigned*>(ctrl) = want;
    }
}

// Release / acquire at system scope (what orders data stores before a flag), or
// relaxed (a lone flag, or data that carries its own step tag).
__device__ __forceinline__ void pingpong_store(unsigned* p, unsigned v, int relaxed) {
    if (relaxed) asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
    else asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned pingpong_load(const unsigned* p, int relaxed) {
    unsigned v;
    if (relaxed) asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    else v = ld_acquire_sys(p);
    return v;
}

// The NVLink signalling floor: ranks 0 and 1 bounce a flag `iters` times inside
// one kernel each (one warp), rank 0 timing the last iters − iters/8 round trips
// with %globaltimer.
// The flag goes into the peer's control word kGatherPingWord, as a
// system-scope release store read back with acquire loads (what a barrier
// signal costs) or as relaxed ones (what a tagged data word costs).
__global__ void __launch_bounds__(32) gather_pingpong_kernel(const GatherArgs* __restrict__ ga, unsigned base,
                                                             int iters, int relaxed, unsigned* err,
                                                             unsigned long long* ns) {
    if (threadIdx.x != 0 || ga->world < 2 || ga->rank > 1) return;
    const int me = ga->rank, peer = 1 - me;
    unsigned* mine = ga->ctrl[me] + kGatherPingWord;
    unsigned* theirs = ga->ctrl[peer] + kGatherPingWord;
    // The first eighth of the round trips absorbs the two launches' skew; the
    // time covers the rest (iters − iters/8).
    const int warm = iters / 8;
    unsigned long long t0 = globaltimer();
    for (int i = 1; i <= iters; ++i) {
        if (i == warm + 1) t0 = globaltimer();
        const unsigned v = base + (unsigned)i;
        if (me == 0) pingpong_store(theirs, v, relaxed);
        const unsigned long long tw = globaltimer();
        for (uint32_t k = 0; pingpong_load(mine, relaxed) != v; ++k) {
            if ((k & 63u) == 0 && globaltimer() - tw > kWaitLimitNs) {
                if (err) atomicOr(err, kErrPeerTimeout);
                return;
            }
        }
        if (me == 1) pingpong_store(theirs, v, relaxed);
    }
    if (me == 0 && ns) *ns = globaltimer() - t0;
}

// ---- Q4_0, one row of x, K a multiple of 2048: four weight rows per lane -----------------
//
// In the layout above, the TR lanes that share a superblock column (one per row of
// the tile) each read the same 40 bytes of quantized x per block from shared
// memory, and those reads (four times the bytes the dots need, ~80 shared-memory
// wavefronts per 4-row item) set the pace of the block dots: measured on B200 in a
// config-0 chain, ~1,250 cycles per item against ~530 for its weights. Here a warp
// item is 4 rows × one k-step of 2048 values (the same 4,608-byte stage), and lane
// l = 4g + j takes blocks 2j and 2j+1 of superblock g in all four rows: its 80
// bytes of x (xq_r4_bytes layout) are loaded once and serve four rows from
// registers, and its weights are 9 words per row at byte 1152·row + 144·g + 36·j
// of the stage (32 distinct banks across the warp). Per block the arithmetic is the
// fast kernel's: the exact int32 isum from the −8·Σq start (plus kIntToFloatMagic, so the
// sum converts to float by one exact subtraction instead of an integer-to-float
// conversion), then acc = fma(float(isum), fp16(dw)·dx, acc); each lane adds its two blocks of every
// k-step in order, and a fixed shuffle tree adds the 32 lanes, so the result
// depends on neither the launch shape nor where x was quantized.
//
// With K = 2048 and 16 warps (one quad of x per thread), the first item's weights
// are read from shared memory while the loads of x are in flight: a GEMV chained
// under programmatic dependent launch waits ~1,200 cycles for x behind the next
// GEMV's weight stream, and the 36 words per lane fill that wait.

// Two blocks of one row (lane words w[0..8]: block 2j's scale and quants from byte
// 2, block 2j+1's scale in the high half of w[4] and quants in w[5..8]).
__device__ __forceinline__ float r4_row(const uint32_t (&w)[9], const uint4& x0l, const uint4& x0h, const uint4& x1l,
                                        const uint4& x1h, const uint4& dd, float acc) {
    uint32_t q[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) q[i] = funnel(w[i], w[i + 1], 16);
    int a = dp4a_us(q[0] & 0x0F0F0F0Fu, x0l.x, (int)dd.y), h = dp4a_us(q[0] & 0xF0F0F0F0u, x0h.x, 0);
    a = dp4a_us(q[1] & 0x0F0F0F0Fu, x0l.y, a);
    h = dp4a_us(q[1] & 0xF0F0F0F0u, x0h.y, h);
    a = dp4a_us(q[2] & 0x0F0F0F0Fu, x0l.z, a);
    h = dp4a_us(q[2] & 0xF0F0F0F0u, x0h.z, h);
    a = dp4a_us(q[3] & 0x0F0F0F0Fu, x0l.w, a);
    h = dp4a_us(q[3] & 0xF0F0F0F0u, x0h.w, h);
    acc = fmaf(__fsub_rn(__int_as_float(a + (h >> 4)), kIntToFloatMagicF), __fmul_rn(half_bits_to_float(w[0]), __uint_as_float(dd.x)),
               acc);
    a = dp4a_us(w[5] & 0x0F0F0F0Fu, x1l.x, (int)dd.w);
    h = dp4a_us(w[5] & 0xF0F0F0F0u, x1h.x, 0);
    a = dp4a_us(w[6] & 0x0F0F0F0Fu, x1l.y, a);
    h = dp4a_us(w[6] & 0xF0F0F0F0u, x1h.y, h);
    a = dp4a_us(w[7] & 0x0F0F0F0Fu, x1l.z, a);
    h = dp4a_us(w[7] & 0xF0F0F0F0u, x1h.z, h);
    a = dp4a_us(w[8] & 0x0F0F0F0Fu, x1l.w, a);
    h = dp4a_us(w[8] & 0xF0F0F0F0u, x1h.w, h);
    return fmaf(__fsub_rn(__int_as_float(a + (h >> 4)), kIntToFloatMagicF),
                __fmul_rn(half_bits_to_float(w[4] >> 16), __uint_as_float(dd.z)), acc);
}

// Rows of the first item read into registers while x is in flight (the rest of
// the 64 registers a thread has hold the quantization and the ring's state).
constexpr int kR4PreRows = 1;

// One item: x slot at xslot (shared or global memory), the rows' words from the
// stage, the first kPre rows from pre[] (the item loaded ahead).
template <bool kShX, int kPre>
__device__ __forceinline__ void r4_item(const uint8_t* stage, const uint8_t* xslot, int lane, float (&acc)[4],
                                        const uint32_t (&pre)[kR4PreRows * 9]) {
    const uint4 x0l = ld_x16<kShX>(xslot), x0h = ld_x16<kShX>(xslot + 16), x1l = ld_x16<kShX>(xslot + 32),
                x1h = ld_x16<kShX>(xslot + 48), dd = ld_x16<kShX>(xslot + 64);
    const uint32_t* wp = reinterpret_cast<const uint32_t*>(stage + (lane >> 2) * 144 + (lane & 3) * 36);
#pragma unroll
    for (int rr = 0; rr < 4; ++rr) {
        uint32_t w[9];
#pragma unroll
        for (int i = 0; i < 9; ++i) w[i] = rr < kPre ? pre[(9 * rr + i) % (kR4PreRows * 9)] : wp[rr * 288 + i];
        acc[rr] = r4_row(w, x0l, x0h, x1l, x1h, dd, acc[rr]);
    }
}

// Sums of the four rows over the 32 lanes; lane l ends with row l >> 3.
__device__ __forceinline__ float r4_reduce(const float (&a)[4], int lane) {
    constexpr unsigned kAll = 0xffffffffu;
    const bool up = lane & 16, up2 = lane & 8;
    const float k0 = (up ? a[2] : a[0]) + __shfl_xor_sync(kAll, up ? a[0] : a[2], 16);
    const float k1 = (up ? a[3] : a[1]) + __shfl_xor_sync(kAll, up ? a[1] : a[3], 16);
    float k = (up2 ? k1 : k0) + __shfl_xor_sync(kAll, up2 ? k0 : k1, 8);
    k += __shfl_xor_sync(kAll, k, 4);
    k += __shfl_xor_sync(kAll, k, 2);
    return k + __shfl_xor_sync(kAll, k, 1);
}

// The four-row kernel's optional work, chosen at compile time: config 0 is
// latency-bound enough that even branches never taken cost (measured on B200 in
// a chain: 2.59 against 2.47 us per step with the residual, norm and gather
// checks as runtime branches). kExtGather: the fused all-gather (p.gather);
// kExtNorm: the RMSNorm of x (p.nw); kExtRes: the residual add (p.res).
constexpr int kExtGather = 1, kExtNorm = 2, kExtRes = 4;

template <bool kXGlobal, int kExt>
__device__ __forceinline__ void gemv_q4_r4_body(const QGemvParams& p) {
    constexpr bool kGather = (kExt & kExtGather) != 0, kNorm = (kExt & kExtNorm) != 0, kRes = (kExt & kExtRes) != 0;
    constexpr int SBB = 144;
    extern __shared__ __align__(128) uint8_t smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;

    uint64_t* bars = reinterpret_cast<uint64_t*>(smem) + warp * p.stages;
    size_t off = ((size_t)nwarps * p.stages * 8 + 127) & ~(size_t)127;
    uint8_t* xs = smem + off;
    if constexpr (!kXGlobal) off += (xq_r4_bytes(p.ksteps) + 127) & ~(size_t)127;
    uint8_t* stages = smem + off + (size_t)warp * p.stages * 32 * SBB;

    if constexpr (!kGather) pdl_launch_dependents();   // with a gather: after griddepcontrol.wait (as above)

    int GW, gw, tiles_end;
    if (p.contiguous) {
        GW = nwarps;
        gw = cta_first_tile(p, blockIdx.x) + warp;
        tiles_end = cta_first_tile(p, blockIdx.x + 1);
    } else {
        GW = gridDim.x * nwarps;
        gw = warp * gridDim.x + blockIdx.x;
        tiles_end = p.ntiles;
    }
    const int my_tiles = gw < tiles_end ? (tiles_end - 1 - gw) / GW + 1 : 0;
    const int nitems = my_tiles * p.ksteps;

    if (lane == 0) {
        for (int s = 0; s < p.stages; ++s) mbar_init(&bars[s], 1);
        fence_mbar_init();
    }
    __syncwarp();
    ItemCursor cur{gw, 0, 0, 0u}, iss{gw, 0, 0, 0u};
    int issued = 0;
    // Chained under programmatic dependent launch, this kernel starts while the
    // GEMV before it is about to read its x. Holding the first weight copies
    // back p.issue_delay cycles (a bounded spin) measured faster on B200 for the
    // plain kernel (config 0: 2.39 against 2.57 us per chained step at 100
    // cycles, less gain from 200 cycles on; 64-bit tile-range divisions that
    // once preceded the copies had acted as such a hold) and no faster for the
    // decode step's fused variants, which therefore never hold. The copies
    // still land long before this kernel's own x.
    if (kExt == 0 && p.issue_delay > 0) {
        const long long t0 = clock64();
        for (int spin = 0; spin < 4096 && clock64() - t0 < p.issue_delay; ++spin) {
        }
    }
    for (; issued < min(p.stages, nitems); ++issued) {
        issue_item<kQ4_0>(p, iss.tile, iss.ks, iss.slot, stages, bars, lane);
        iss.next(p, GW);
    }

    pdl_wait_primary();
    if constexpr (kGather) pdl_launch_dependents();
    uint32_t pre[kR4PreRows * 9];
    bool have_pre = false;
    if constexpr (!kXGlobal) {
        const XGeom xg{1, p.nb, 3, p.ksteps, 1};
        if (p.ksteps == 1 && blockDim.x == 512) {
            // 64 blocks × 8 threads: one quad of x per thread, loaded first.
            const int gq = threadIdx.x & 7, b = threadIdx.x >> 3;
            float4 v = load_act4(p.x, p.up, (size_t)b * kQK + gq * 4);
            // The norm's weights load together with x: one L2 round trip for both.
            float4 nwq = make_float4(0.f, 0.f, 0.f, 0.f);
            if constexpr (kNorm) nwq = load_x4(p.nw + (size_t)b * kQK + gq * 4);
            if (nitems > 0) {
                const bool ok = mbar_wait_bounded(&bars[0], 0, p.err);
                have_pre = __all_sync(0xffffffffu, ok);
                if (have_pre) {
                    const uint32_t* wp = reinterpret_cast<const uint32_t*>(stages + (lane >> 2) * 144 + (lane & 3) * 36);
#pragma unroll
                    for (int i = 0; i < kR4PreRows * 9; ++i) pre[i] = wp[(i / 9) * 288 + i % 9];
                }
            }
            // Fused RMSNorm: the row's sum of squares from the quads in the
            // threads' registers (the whole row: 512 threads × 4 values).
            if constexpr (kNorm) v = norm4v(v, nwq, rms_inv(cta_sum(sq_sum4(v)), p.K, p.neps));
            quantize_x_block(v, gq, true, xg, 0, b, xs);
        } else {
            quantize_x_rows<1>(p.x, p.ldx, p.up, p.ldu, xg, xs, threadIdx.x, blockDim.x, kNorm ? p.nw : nullptr,
                               p.neps);
        }
        __syncthreads();
    }
    const uint8_t* xb = kXGlobal ? p.xq : xs;

    const int r = lane >> 3, g = lane & 7;
    if constexpr (kGather) {
        if (blockIdx.x == 0) gather_pad(p.gather, 1, p.N, threadIdx.x, blockDim.x);
    }
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};

    float resv = 0.0f;   // fused residual: the row's value, loaded when its tile starts
    for (int it = 0; it < nitems; ++it) {
        const uint8_t* xslot = xb + ((size_t)cur.ks * 32 + lane) * 80;
        const uint8_t* st = stages + (size_t)cur.slot * (32 * SBB);
        if constexpr (kRes) {
            if (cur.ks == 0 && g == 0 && cur.tile * 4 + r < p.N) resv = p.res[cur.tile * 4 + r];
        }
        if (it == 0 && have_pre) {
            r4_item<!kXGlobal, kR4PreRows>(st, xslot, lane, acc, pre);
        } else {
            if (__any_sync(0xffffffffu, !mbar_wait_bounded(&bars[cur.slot], cur.phase, p.err))) {   // warp-uniform
                ItemCursor c2 = cur;
                for (int k = it + 1; k < issued; ++k) {
                    c2.next(p, GW);
                    mbar_wait_bounded(&bars[c2.slot], c2.phase, nullptr);
                }
                break;
            }
            r4_item<!kXGlobal, 0>(st, xslot, lane, acc, pre);
        }
        if (cur.ks == p.ksteps - 1) {
            const float v = r4_reduce(acc, lane);
            const int row = cur.tile * 4 + r;
            if (g == 0 && row < p.N) p.y[row] = kRes ? __fadd_rn(resv, v) : v;
#pragma unroll
            for (int k = 0; k < 4; ++k) acc[k] = 0.0f;
        }
        __syncwarp();
        if (issued < nitems) {
            fence_proxy_async_smem();
            issue_item<kQ4_0>(p, iss.tile, iss.ks, iss.slot, stages, bars, lane);
            iss.next(p, GW);
            ++issued;
        }
        cur.next(p, GW);
    }
    if constexpr (kGather) gather_send(p, 1, 4, cur.tile, GW, lane);
    if (p.yhost) copy_y_to_host(p);   // every warp gets here, the ones that gave up too
}

template <bool kXGlobal, int kExt>
__global__ void __launch_bounds__(512, 2) gemv_q4_r4(const QGemvParams p) {
    gemv_q4_r4_body<kXGlobal, kExt>(p);
}

// The instantiation for p (the gather never comes with the decode-step fusions).
template <bool kXGlobal>
void (*r4_kernel(const QGemvParams& p))(QGemvParams) {
    if (p.gather) return gemv_q4_r4<kXGlobal, kExtGather>;
    if (p.nw && p.res) return gemv_q4_r4<kXGlobal, kExtNorm | kExtRes>;
    if (p.nw) return gemv_q4_r4<kXGlobal, kExtNorm>;
    if (p.res) return gemv_q4_r4<kXGlobal, kExtRes>;
    return gemv_q4_r4<kXGlobal, 0>;
}

// ---- four-row kernel, K split over warps ----------------------------------------------
//
// Few four-row tiles and long rows (K a multiple of 2048, at least 8192, fewer
// than 8 tiles per SM: the Llama down projection 2048×8192, a 70B layer's
// 8192×28672 sharded over GPUs): one warp per tile would leave most warps idle
// and walk all of K alone. Here the k-steps of a tile are split over S warps
// of a CTA (p.split). CTA c takes the tile groups c, c + grid, ... of T =
// warps / S tiles; warp w works on tile w / S of a group over the k-steps
// [part·ks/S, (part+1)·ks/S), part = w % S, with x quantized once in global
// memory (the four-row slot layout). Each warp's four row sums (r4_reduce) go
// to shared memory and the part-0 warp adds the S parts in part order:
// deterministic, within the reference's bound (rounded differently from one
// warp walking K). Variants: the residual add (kExtRes) and the fused gather
// (kExtGather); an RMSNorm of x happens in the quantize kernel before.
__host__ __device__ inline size_t r4s_smem(int warps, int stages) {
    return (((size_t)warps * stages * 8 + 127) & ~(size_t)127) + (((size_t)warps * 16 + 127) & ~(size_t)127) +
           (size_t)warps * stages * 32 * 144;
}

template <int kExt>
__global__ void __launch_bounds__(512, 2) gemv_q4_r4s(const QGemvParams p) {
    constexpr bool kGather = (kExt & kExtGather) != 0, kRes = (kExt & kExtRes) != 0;
    constexpr int SBB = 144;
    extern __shared__ __align__(128) uint8_t smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const int S = p.split, T = nwarps / S, part = warp % S, tl = warp / S;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem) + warp * p.stages;
    size_t off = ((size_t)nwarps * p.stages * 8 + 127) & ~(size_t)127;
    float* sums = reinterpret_cast<float*>(smem + off);   // [warp][row of the tile]
    off += ((size_t)nwarps * 16 + 127) & ~(size_t)127;
    uint8_t* stages = smem + off + (size_t)warp * p.stages * 32 * SBB;

    if constexpr (!kGather) pdl_launch_dependents();
    const int ks_lo = part * p.ksteps / S, nks = (part + 1) * p.ksteps / S - ks_lo;
    const int ngroups = (p.ntiles + T - 1) / T, bx = (int)blockIdx.x, nbx = (int)gridDim.x;
    const int rounds = bx < ngroups ? (ngroups - 1 - bx) / nbx + 1 : 0;   // CTA-uniform
    auto tile_of = [&](int rd) { return (bx + rd * nbx) * T + tl; };
    int valid = rounds;   // rounds with this warp's tile inside N (only the last group runs past it)
    while (valid > 0 && tile_of(valid - 1) >= p.ntiles) --valid;
    const int nitems = valid * nks;
    if (lane == 0) {
        for (int i = 0; i < p.stages; ++i) mbar_init(&bars[i], 1);
        fence_mbar_init();
    }
    __syncwarp();
    int i_r = 0, i_k = 0, i_slot = 0, issued = 0;
    auto issue_next = [&]() {
        issue_item<kQ4_0>(p, tile_of(i_r), ks_lo + i_k, i_slot, stages, bars, lane);
        if (++i_k == nks) { i_k = 0; ++i_r; }
        if (++i_slot == p.stages) i_slot = 0;
        ++issued;
    };
    while (issued < min(p.stages, nitems)) issue_next();   // weights only: x is the previous kernel's output

    pdl_wait_primary();
    if constexpr (kGather) pdl_launch_dependents();
    GatherStep gs{0, 0u};
    if constexpr (kGather) {
        gs = gather_step(p.gather);
        if (bx == 0) gather_pad(p.gather, 1, p.N, threadIdx.x, blockDim.x);
    }
    const int r = lane >> 3, g = lane & 7;
    const uint32_t no_pre[kR4PreRows * 9] = {};
    int failed = 0, c_slot = 0, consumed = 0;
    uint32_t c_phase = 0;
    for (int rd = 0; rd < rounds; ++rd) {   // CTA-uniform: every warp meets every barrier
        float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        if (rd < valid) {
            for (int k = 0; k < nks && !failed; ++k) {
                if (__any_sync(0xffffffffu, !mbar_wait_bounded(&bars[c_slot], c_phase, p.err))) {   // warp-uniform
                    failed = 1;
                    break;
                }
                const uint8_t* xslot = p.xq + ((size_t)(ks_lo + k) * 32 + lane) * 80;
                r4_item<false, 0>(stages + (size_t)c_slot * (32 * SBB), xslot, lane, acc, no_pre);
                __syncwarp();
                if (issued < nitems) {
                    fence_proxy_async_smem();
                    issue_next();
                }
                ++consumed;
                if (++c_slot == p.stages) { c_slot = 0; c_phase ^= 1u; }
            }
        }
        const float v = r4_reduce(acc, lane);
        if (g == 0) sums[warp * 4 + r] = v;
        const int any_failed = __syncthreads_or(failed);
        if (part == 0 && g == 0 && rd < valid && !any_failed) {
            const int row = tile_of(rd) * 4 + r;
            if (row < p.N) {
                float t = sums[tl * S * 4 + r];
                for (int q = 1; q < S; ++q) t = __fadd_rn(t, sums[(tl * S + q) * 4 + r]);   // the parts in K order
                if constexpr (kRes) t = __fadd_rn(p.res[row], t);
                p.y[row] = t;
                if constexpr (kGather) {
                    const GatherArgs* ga = p.gather;
                    const long long o = gs.off + row;
                    ga->y[o] = t;
                    const unsigned long long w = tagged_word(t, gs.tag);
                    for (int rk = 0; rk < ga->world; ++rk)
                        if (rk != ga->rank) st_relaxed_sys_u64(ga->ll[rk] + o, w);
                }
            }
        }
        __syncthreads();   // the sums are read before the next round writes them
    }
    if (failed) {   // this warp's copies still in flight land (bounded) before the CTA exits
        for (int k = consumed; k < issued; ++k)
            mbar_wait_bounded(&bars[k % p.stages], (uint32_t)((k / p.stages) & 1), nullptr);
    }
    if (p.yhost) copy_y_to_host(p);
}

// ---- tensor-core kernel for 3..8 rows of x -------------------------------------------
//
// With several rows of x, the block dots are an integer matrix product per
// 32-value block: W [16 rows × 32] · Xᵀ [32 × 8 rows of x] on the
// mma.sync m16n8k32 integer shape (u8 × s8 for Q4_0 nibbles, s8 × s8 for Q8_0),
// one MMA per (16 rows, block), exact int32 per-block sums. The A fragment
// of lane (g = lane/4, t = lane%4) is the words t of rows g and g+8, plus
// (k + 16): a Q4_0 block's quant word t holds elements 4t..4t+3 in its low
// nibbles and 16+4t..16+4t+3 in its high nibbles, so a0 = q & 0x0F0F0F0F and
// a2 = (q >> 4) & 0x0F0F0F0F. The B fragment is words t and 4+t of the Q8
// quants of x row g (rows ≥ M are zero). The result lands as rows g, g+8 ×
// x rows 2t, 2t+1 in the lane that keeps them: each lane walks every block of
// its two rows in order and accumulates
//     acc = fl(acc + fl(float(isum) · fl(dw · dx)))
// exactly as the reference's scalar kernel (q4_0_scalar.cpp:82-99,
// q8_0_scalar.cpp:170-192, no contraction), so the outputs equal the scalar
// reference's bit for bit. Weights stream as in the fast kernel: per-warp
// rings of TMA stages (16 rows × 16 (Q4_0) or 8 (Q8_0) blocks each, rows
// padded so the 8 row groups of a fragment load hit distinct banks), issued
// before griddepcontrol.wait.

// Q8 activations for the MMA path, written by quantize_x_mma_kernel: per
// block b the B-fragment words of row m (0..7) for lane t, (word t, word 4+t)
// side by side at ((b·8 + m)·4 + t)·8 bytes; after nb·256 bytes, 64 bytes per
// block: c(m) = kIntToFloatMagic − 8·Σq(m) of rows 0..7 (32 bytes), then dx of
// rows 0..7 (32 bytes), so lane t reads the pairs of x rows (2t, 2t+1) with one
// 8-byte load each; the c pair is the first half of the MMA's accumulator
// input. Rows ≥ M have c = kIntToFloatMagic and dx = 0. float(isum) comes from
// the magic-number add (kIntToFloatMagic).
constexpr int kMmaWarps = 16;
// A warp item is 16 rows × 8 blocks, fetched as one box of a 2-D tensor map
// over the weights (rows of nb·block bytes; Q4_0 as bytes, Q8_0 as 16-bit
// elements so that the 272-byte box row fits the 256-element box limit).
// In shared memory the box rows lie densely at 144 / 272 bytes: 36 / 68
// words, 4 (mod 32), so the 8 row groups of a fragment load fall on
// distinct banks.
template <int F> __host__ __device__ constexpr int mma_kb() { return 8; }
template <int F> __host__ __device__ constexpr int mma_rs() { return 8 * block_bytes(F); }
// Quantized x per block for the MMA path: B fragments 256 bytes, accumulator
// inputs and scales 64 bytes (at nb·256 + b·64).
constexpr int kMmaXFragBytes = 256, kMmaXcdBytes = 64;

__global__ void __launch_bounds__(kThreadsQuantX) quantize_x_mma_kernel(const float* __restrict__ x, long long ldx,
                                                                         const float* __restrict__ up, long long ldu,
                                                                         int M, int nb, uint8_t* xq, unsigned* tickets) {
    pdl_launch_dependents();
    pdl_wait_primary();   // x comes from the previous kernel; xq may still be read by it
    // The K-parted GEMV that follows counts finished CTAs per tile range here.
    if (tickets && blockIdx.x == 0)
        for (int i = threadIdx.x; i < kMmaMaxTickets; i += blockDim.x) tickets[i] = 0u;
    const int gq = threadIdx.x & 7;
    const long long groups = (long long)nb * 8;   // (block, row) pairs, rows padded to 8
    const long long stride = (long long)gridDim.x * (blockDim.x >> 3);
    for (long long base = ((long long)blockIdx.x * blockDim.x + (threadIdx.x & ~31)) >> 3; base < groups;
         base += stride) {   // warp-uniform
        const long long grp = base + ((threadIdx.x & 31) >> 3);
        const bool valid = grp < groups;
        const int b = (int)(grp >> 3), m = (int)(grp & 7);
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (valid && m < M)
            v = load_act4(x + (size_t)m * ldx, up ? up + (size_t)m * ldu : nullptr, (size_t)b * kQK + gq * 4);
        const Q8Quad q = quantize_quad(v);
        if (!valid) continue;
        reinterpret_cast<uint32_t*>(xq)[((size_t)(b * 8 + m) * 4 + (gq & 3)) * 2 + (gq >> 2)] = m < M ? q.word : 0u;
        if (gq == 0) {
            uint8_t* cd = xq + (size_t)nb * kMmaXFragBytes + (size_t)b * kMmaXcdBytes;
            reinterpret_cast<int*>(cd)[m] = m < M ? kIntToFloatMagic - 8 * q.s : kIntToFloatMagic;
            reinterpret_cast<float*>(cd + 32)[m] = m < M ? q.dx : 0.0f;
        }
    }
}

// c = A·B + (m.x, m.y, m.x, m.y): the int32 sums of rows (g, g+8) × x rows
// (2t, 2t+1) start from the magic-number bits of their x row (kIntToFloatMagic,
// with the Q4_0 bias −8·Σq folded in), so c comes out as the bits of a float
// whose value is 2^23 + 2^22 + isum: one exact subtraction converts it. m is
// loaded as one pair, the first half of the accumulator input the instruction
// takes.
template <int F>
__device__ __forceinline__ void mma_q(const uint32_t (&a)[4], uint2 b, int2 m, int (&c)[4]) {
    const int4 cin = make_int4(m.x, m.y, m.x, m.y);
    if constexpr (F == kQ4_0)
        asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                     "{%10,%11,%12,%13};"
                     : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
                     : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b.x), "r"(b.y), "r"(cin.x), "r"(cin.y),
                       "r"(cin.z), "r"(cin.w));
    else
        asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                     "{%10,%11,%12,%13};"
                     : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
                     : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b.x), "r"(b.y), "r"(cin.x), "r"(cin.y),
                       "r"(cin.z), "r"(cin.w));
}

template <int F>
__device__ __forceinline__ void mma_issue(const CUtensorMap* wmap, int tile, int ks, uint8_t* slot, uint64_t* bar,
                                          int lane) {
    constexpr int RS = mma_rs<F>();
    if (lane == 0) {
        mbar_arrive_expect_tx(bar, 16u * RS);   // the whole box, rows past N zero-filled
        tma_load_2d(slot, wmap, ks * (F == kQ4_0 ? RS : RS / 2), tile * 16, bar);
    }
}

// The fragment words of one pair of blocks (2i, 2i+1) of a 16-row item for
// lane (g, t): A of both blocks, and the words holding the rows' fp16 scales
// (the even block's in the low half of sc[0][rr], the odd block's in the high
// half of sc[1][rr]). wr: word 0 of row g of the item, wt = wr + t; the rest of
// each address is a constant (pair and rr unrolled), so the loads need no
// address arithmetic.
template <int F>
__device__ __forceinline__ void mma_frag_pair(const uint32_t* wr, const uint32_t* wt, int pair, uint32_t (&ae)[4],
                                              uint32_t (&ao)[4], uint32_t (&sc)[2][2]) {
    constexpr int PW = 2 * block_bytes(F) / 4, RW = mma_rs<F>() / 4;   // words per block pair, per row
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
        const uint32_t* w = wr + rr * 8 * RW + pair * PW;
        const uint32_t* u = wt + rr * 8 * RW + pair * PW;
        if constexpr (F == kQ4_0) {
            // even block: scale in bytes 0-1, quant word t at byte 2 + 4t; odd block:
            // scale in bytes 18-19 (high half of word 4), quant word t is word 5 + t.
            const uint32_t qe = funnel(u[0], u[1], 16), qo = u[5];
            ae[rr] = qe & 0x0F0F0F0Fu;
            ae[2 + rr] = (qe >> 4) & 0x0F0F0F0Fu;
            ao[rr] = qo & 0x0F0F0F0Fu;
            ao[2 + rr] = (qo >> 4) & 0x0F0F0F0Fu;
            sc[0][rr] = w[0];
            sc[1][rr] = w[4];
        } else {
            // even block: quant word u at byte 2 + 4u; odd block (byte 34 on): scale in
            // the high half of word 8, quant word u is word 9 + u.
            ae[rr] = funnel(u[0], u[1], 16);
            ae[2 + rr] = funnel(u[4], u[5], 16);
            ao[rr] = u[9];
            ao[2 + rr] = u[13];
            sc[0][rr] = w[0];
            sc[1][rr] = w[8];
        }
    }
}

// acc[rr] += isum · (dw · dx) for rows g + 8·rr and x rows (2t, 2t+1), in the
// reference's order and roundings: every product and sum rounded on its own,
// never contracted. c holds the magic-number bits (mma_q), so float(isum) is
// one exact subtraction. The subtraction and dw·dx of a lane's two x rows go
// through the packed FP32 unit (fadd2_rn / fmul2_rn: two IEEE operations each).
// The product that is added to acc is a scalar __fmul_rn: a packed product
// feeding a packed sum is contracted into a fused multiply-add by the code
// generator even with explicit rounding, and so is the product written as a
// packed fma with −0 (measured on B200: 35–44 % of such pairs, and 75 % of
// 8-step sums of the fma form, differ from the scalar roundings), which would
// break the reference's order. kHi: the scales sit in the high halves of sc
// (the odd block of a pair).
template <bool kHi>
__device__ __forceinline__ void mma_accumulate(const int (&c)[4], const uint32_t (&sc)[2], float2 dx,
                                               float2 (&acc)[2]) {
    const float2 unmagic = make_float2(-12582912.0f, -12582912.0f);
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
        const float dw = kHi ? half_hi_to_float(sc[rr]) : half_lo_to_float(sc[rr]);
        const float2 i = fadd2_rn(make_float2(__int_as_float(c[2 * rr]), __int_as_float(c[2 * rr + 1])), unmagic);
        const float2 sc2 = fmul2_rn(make_float2(dw, dw), dx);
        acc[rr].x = __fadd_rn(acc[rr].x, __fmul_rn(i.x, sc2.x));
        acc[rr].y = __fadd_rn(acc[rr].y, __fmul_rn(i.y, sc2.y));
    }
}

// Shared-memory layout of gemv_q_mma: barriers (one per stage per warp, then
// one for x), the MMA-layout x when kXS, the partial sums of split tiles
// (a float4 per lane per warp), then the per-warp rings.
__host__ __device__ inline size_t mma_x_offset(int warps, int stages) {
    return ((size_t)(warps * stages + 1) * 8 + 127) & ~(size_t)127;
}
__host__ __device__ inline size_t mma_part_offset(int warps, int stages, int nb, bool xs) {
    return mma_x_offset(warps, stages) + (xs ? (((size_t)nb * (kMmaXFragBytes + kMmaXcdBytes) + 127) & ~(size_t)127) : 0);
}
__host__ __device__ inline size_t mma_ring_offset(int warps, int stages, int nb, bool xs) {
    return mma_part_offset(warps, stages, nb, xs) + (size_t)warps * 32 * 16;
}

template <bool kXS, typename T>
__device__ __forceinline__ T ld_xfrag(const T* p) {
    if constexpr (kXS) return *p;
    else return __ldg(p);
}

// kXS: the quantized x (xmma_bytes(nb)) is copied into shared memory once per
// CTA by one bulk copy; otherwise its fragments are read from global memory.
//
// Work split: a CTA takes groups of T = warps / S consecutive 16-row tiles;
// warp w works on tile w / S of the group over the K part w % S (p.split = S
// parts of the k-steps). With S = 1 every row's blocks are summed by one lane
// in block order (the reference's order); with S > 1 each part's sum is kept
// in shared memory and part 0 adds the S partial sums in order, so the result
// is deterministic but rounded differently. The launcher splits K only when
// the tiles alone cannot fill the GPU.
//
// kGather: y is this rank's staging slice of a row-sharded GEMV (p.gather), and
// every final output also goes to this rank's full-y area and, as a tagged
// word, to every peer's receive area (the one-row kernels' fused gather).
template <int F, bool kXS, bool kGather>
__global__ void __launch_bounds__(kMmaWarps * 32, 1) gemv_q_mma(const QGemvParams p, const __grid_constant__ CUtensorMap wmap) {
    constexpr int KB = mma_kb<F>(), RS = mma_rs<F>(), ITEM = 16 * RS;
    extern __shared__ __align__(128) uint8_t smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem) + warp * p.stages;
    uint64_t* xbar = reinterpret_cast<uint64_t*>(smem) + nwarps * p.stages;
    const int xnb = p.xnb > 0 ? p.xnb : p.nb;   // blocks of x a CTA holds in shared memory
    uint8_t* xsm = smem + mma_x_offset(nwarps, p.stages);
    float4* parts = reinterpret_cast<float4*>(smem + mma_part_offset(nwarps, p.stages, xnb, kXS));
    uint8_t* ring = smem + mma_ring_offset(nwarps, p.stages, xnb, kXS) + (size_t)warp * p.stages * ITEM;

    if constexpr (!kGather) pdl_launch_dependents();   // with a gather: after griddepcontrol.wait
    const int ntiles = (p.N + 15) / 16, ksteps = p.nb / KB;   // K % 256 == 0: whole items
    // K parts across CTAs (kparts > 1): CTA c works on part c / C of K, over
    // the tile groups of its index c % C within the part.
    const int P = p.kparts > 1 ? p.kparts : 1;
    const int cn = (int)gridDim.x / P, kp = (int)blockIdx.x / cn, cj = (int)blockIdx.x % cn;
    const int kq0 = kp * ksteps / P, kspan = (kp + 1) * ksteps / P - kq0;   // this CTA's items
    const int xb0 = kq0 * KB;                                               // its first block of x
    const int S = p.split, T = nwarps / S, part = warp % S, tl = warp / S;
    const int ks_lo = kq0 + part * kspan / S, nks = kq0 + (part + 1) * kspan / S - ks_lo;
    const bool grouped = S > 1 || P > 1;
    // Rounds of this warp. S == 1: the CTA owns a contiguous range of tiles
    // (an even share, so every SM streams one region of W) and its warps
    // take them in turn (no CTA barrier). S > 1: the CTA's groups of T tiles,
    // CTA-uniform (a barrier per round); only the last group can hold a tile
    // past N.
    const int c_lo = (int)((long long)blockIdx.x * ntiles / gridDim.x);
    const int c_hi = (int)((long long)(blockIdx.x + 1) * ntiles / gridDim.x);
    int my_groups, valid_groups;
    if (!grouped) {
        my_groups = valid_groups = c_lo + warp < c_hi ? (c_hi - 1 - c_lo - warp) / nwarps + 1 : 0;
    } else {
        const int ngroups = (ntiles + T - 1) / T;
        my_groups = cj < ngroups ? (ngroups - 1 - cj) / cn + 1 : 0;
        const int last_tile = my_groups > 0 ? (cj + (my_groups - 1) * cn) * T + tl : 0;
        valid_groups = my_groups > 0 && last_tile >= ntiles ? my_groups - 1 : my_groups;
    }
    auto tile_of = [&](int r) { return !grouped ? c_lo + warp + r * nwarps : (cj + r * cn) * T + tl; };
    const int nitems = valid_groups * nks;
    if (lane == 0) {
        for (int i = 0; i < p.stages; ++i) mbar_init(&bars[i], 1);
        if (kXS && threadIdx.x == 0) mbar_init(xbar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    // Issue cursor over (group round, k-step); items are consumed in the same order.
    int i_r = 0, i_ks = 0, i_slot = 0, issued = 0;
    auto issue_next = [&]() {
        const int tile = tile_of(i_r);
        mma_issue<F>(&wmap, tile, ks_lo + i_ks, ring + (size_t)i_slot * ITEM, &bars[i_slot], lane);
        if (++i_ks == nks) { i_ks = 0; ++i_r; }
        if (++i_slot == p.stages) i_slot = 0;
        ++issued;
    };
    while (issued < min(p.stages, nitems)) issue_next();

    pdl_wait_primary();   // x was quantized by the previous kernel
    // The gather's wait kernel reads the epoch when it starts: launched only once
    // the previous one has finished, which the wait above implies.
    if constexpr (kGather) pdl_launch_dependents();
    GatherStep gs{0, 0u};
    long long gcols = 0;
    if constexpr (kGather) {
        gs = gather_step(p.gather);
        gcols = (long long)p.gather->world * p.gather->npad;
        if (blockIdx.x == 0) gather_pad(p.gather, p.M, p.N, threadIdx.x, blockDim.x);
    }
    // A final output value: y, and with a gather the full-y areas.
    auto emit = [&](int m, int row, float v) {
        p.y[(size_t)m * p.ldy + row] = v;
        if constexpr (kGather) {
            const GatherArgs* ga = p.gather;
            const long long o = gs.off + m * gcols + row;
            ga->y[o] = v;
            const unsigned long long w = tagged_word(v, gs.tag);
            for (int rk = 0; rk < ga->world; ++rk)
                if (rk != ga->rank) st_relaxed_sys_u64(ga->ll[rk] + o, w);
        }
    };
    const uint8_t* xbase = p.xq;
    int failed = 0;
    int xnb_here = p.nb, xoff = 0;   // blocks of x at xbase, and the block index of the first
    if constexpr (kXS) {
        // This CTA's slice of x, blocks [xb0, xb0 + kspan·KB): its quants and
        // its (dx, bias) pairs, two bulk copies (all of x when P == 1).
        xnb_here = kspan * KB;
        xoff = xb0;
        if (threadIdx.x == 0) {
            const uint32_t qbytes = (uint32_t)xnb_here * kMmaXFragBytes, dbytes = (uint32_t)xnb_here * kMmaXcdBytes;
            mbar_arrive_expect_tx(xbar, qbytes + dbytes);
            tma_load_1d(xsm, p.xq + (size_t)xb0 * kMmaXFragBytes, qbytes, xbar);
            tma_load_1d(xsm + qbytes, p.xq + (size_t)p.nb * kMmaXFragBytes + (size_t)xb0 * kMmaXcdBytes, dbytes,
                        xbar);
        }
        failed = !mbar_wait_bounded(xbar, 0u, p.err);
        xbase = xsm;
    }
    failed = __syncthreads_or(failed);
    // This lane's fragments of block 0 of the x held at xbase: B words of row g
    // at (b·8 + g)·4 + t; the accumulator input pair and the dx pair of x rows
    // (2t, 2t+1) in the block's 64 bytes; and its weight row g.
    const uint2* xf_lane = reinterpret_cast<const uint2*>(xbase) + g * 4 + t;
    const uint8_t* xcd = xbase + (size_t)xnb_here * kMmaXFragBytes;
    const int2* xc_lane = reinterpret_cast<const int2*>(xcd) + t;
    const float2* xd_lane = reinterpret_cast<const float2*>(xcd + 32) + t;
    const uint32_t* ring_w = reinterpret_cast<const uint32_t*>(ring) + g * (RS / 4);

    int c_slot = 0, consumed = 0;
    uint32_t c_phase = 0;
    for (int r = 0; r < my_groups; ++r) {   // S > 1: CTA-uniform, every warp meets every barrier
        const int tile = tile_of(r);
        float2 acc[2] = {make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f)};
        if (r < valid_groups) {
            for (int k = 0; k < nks && !failed; ++k) {
                // Warp-uniform verdict: every lane leaves together or none does.
                if (__any_sync(0xffffffffu, !mbar_wait_bounded(&bars[c_slot], c_phase, p.err))) {
                    failed = 1;
                    break;
                }
                const uint32_t* wr = ring_w + c_slot * (ITEM / 4);
                const int bx = (ks_lo + k) * KB - xoff;   // the item's first block within the x held at xbase
                const uint2* xfi = xf_lane + bx * 32;
                const int2* xci = xc_lane + bx * (kMmaXcdBytes / 8);
                const float2* xdi = xd_lane + bx * (kMmaXcdBytes / 8);
                // All MMAs of the item first, then the scaling in block order.
                int c[KB][4];
                uint32_t sc[KB][2];
                float2 dxs[KB];
                const int2 magic2 = make_int2(kIntToFloatMagic, kIntToFloatMagic);
#pragma unroll
                for (int pr = 0; pr < KB / 2; ++pr) {
                    const uint2 xe = ld_xfrag<kXS>(xfi + pr * 64);
                    const uint2 xo = ld_xfrag<kXS>(xfi + pr * 64 + 32);
                    uint32_t ae[4], ao[4], s2[2][2];
                    mma_frag_pair<F>(wr, wr + t, pr, ae, ao, s2);
                    mma_q<F>(ae, xe, F == kQ4_0 ? ld_xfrag<kXS>(xci + (2 * pr) * (kMmaXcdBytes / 8)) : magic2,
                             c[2 * pr]);
                    mma_q<F>(ao, xo, F == kQ4_0 ? ld_xfrag<kXS>(xci + (2 * pr + 1) * (kMmaXcdBytes / 8)) : magic2,
                             c[2 * pr + 1]);
                    dxs[2 * pr] = ld_xfrag<kXS>(xdi + (2 * pr) * (kMmaXcdBytes / 8));
                    dxs[2 * pr + 1] = ld_xfrag<kXS>(xdi + (2 * pr + 1) * (kMmaXcdBytes / 8));
                    sc[2 * pr][0] = s2[0][0];
                    sc[2 * pr][1] = s2[0][1];
                    sc[2 * pr + 1][0] = s2[1][0];
                    sc[2 * pr + 1][1] = s2[1][1];
                }
#pragma unroll
                for (int j = 0; j < KB; ++j) {
                    if (j & 1) mma_accumulate<true>(c[j], sc[j], dxs[j], acc);
                    else mma_accumulate<false>(c[j], sc[j], dxs[j], acc);
                }
                __syncwarp();
                if (issued < nitems) {
                    fence_proxy_async_smem();
                    issue_next();
                }
                ++consumed;
                if (++c_slot == p.stages) { c_slot = 0; c_phase ^= 1u; }
            }
        }
        if (!grouped) {
            if (r < valid_groups && !failed) {
#pragma unroll
                for (int rr = 0; rr < 2; ++rr) {
                    const int row = tile * 16 + g + 8 * rr;
                    if (row < p.N && 2 * t < p.M) emit(2 * t, row, acc[rr].x);
                    if (row < p.N && 2 * t + 1 < p.M) emit(2 * t + 1, row, acc[rr].y);
                }
            }
        } else {
            parts[warp * 32 + lane] = make_float4(acc[0].x, acc[0].y, acc[1].x, acc[1].y);
            __syncthreads();
            if (part == 0 && r < valid_groups && !failed) {
                float4 sum = parts[warp * 32 + lane];
                for (int q = 1; q < S; ++q) {   // the parts of the tile in K order
                    const float4 v = parts[(warp + q) * 32 + lane];
                    sum.x = __fadd_rn(sum.x, v.x);
                    sum.y = __fadd_rn(sum.y, v.y);
                    sum.z = __fadd_rn(sum.z, v.z);
                    sum.w = __fadd_rn(sum.w, v.w);
                }
                const float vals[4] = {sum.x, sum.y, sum.z, sum.w};
                // One K part of several: the sums go to this part's partial rows.
                float* out = P > 1 ? p.partial + (size_t)kp * p.M * p.N : p.y;
                const long long ldo = P > 1 ? p.N : p.ldy;
#pragma unroll
                for (int rr = 0; rr < 2; ++rr) {
                    const int row = tile * 16 + g + 8 * rr;
#pragma unroll
                    for (int j = 0; j < 2; ++j)
                        if (row < p.N && 2 * t + j < p.M) {
                            if (P > 1) out[(size_t)(2 * t + j) * ldo + row] = vals[2 * rr + j];
                            else emit(2 * t + j, row, vals[2 * rr + j]);
                        }
                }
            }
            __syncthreads();
        }
    }
    if (P > 1) {
        // The last of the P CTAs with this index (same tile groups, other K
        // parts) adds the parts in K order: deterministic whatever the order
        // in which the CTAs finish.
        __shared__ unsigned last_cta;
        __threadfence();   // this thread's partial rows before the ticket
        __syncthreads();
        if (threadIdx.x == 0) last_cta = atomicAdd(&p.tickets[cj], 1u) == (unsigned)(P - 1);
        __syncthreads();
        if (last_cta && !failed) {
            __threadfence();   // the other CTAs' rows, seen through their tickets
            for (int r = 0; r < my_groups; ++r) {
                const int row0 = (cj + r * cn) * T * 16;
                const int nrows = min(T * 16, p.N - row0);
                for (int i = threadIdx.x; i < p.M * nrows; i += blockDim.x) {
                    const int m = i / nrows, row = row0 + i % nrows;
                    float sum = __ldcg(p.partial + (size_t)m * p.N + row);
                    for (int q = 1; q < P; ++q)
                        sum = __fadd_rn(sum, __ldcg(p.partial + ((size_t)q * p.M + m) * p.N + row));
                    emit(m, row, sum);
                }
            }
        }
    }
    if (failed) {
        // Let this warp's copies still in flight land (bounded) before the CTA exits.
        for (int k = consumed; k < issued; ++k) {
            const int s2 = k % p.stages;
            mbar_wait_bounded(&bars[s2], (uint32_t)((k / p.stages) & 1), nullptr);
        }
    }
}

// ---- the generic kernel --------------------------------------------------------------

// Any K % 32 == 0 and any weight alignment. One warp per row, lanes over
// blocks, byte loads; x already quantized in global memory (layout G = 32).
template <int F, int M, bool kDump>
__global__ void __launch_bounds__(256) gemv_q_generic(const QGemvParams p) {
    constexpr int BB = block_bytes(F);
    pdl_launch_dependents();
    pdl_wait_primary();
    const int lane = threadIdx.x & 31;
    const int nwarps_total = gridDim.x * (blockDim.x >> 5);
    const size_t row_bytes = (size_t)p.nb * BB;
    XPtr xp;
    xp.mstride_q = (size_t)p.ksteps * 8192;
    xp.mstride_d = (size_t)p.ksteps * 2048;
    const uint8_t* xd0 = p.xq + (size_t)M * p.ksteps * 8192;
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
            const int sb = b >> 3, ks = sb >> 5, g = sb & 31;
            xp.xq = p.xq + ((size_t)ks * 16 * 32 + g) * 16;
            xp.xd = xd0 + ((size_t)ks * 8 * 32 + g) * 8;
            block_dot<F, M, false, kDump>(q, half_bits_to_float(sc), xp, b & 7, acc, p.dump, (size_t)p.N * p.nb,
                                          (size_t)row * p.nb + b);
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

template <typename Kern, typename... Args>
cudaError_t launch(Kern kernel, dim3 grid, dim3 block, size_t smem, const LaunchCfg& c, Args... args) {
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
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// The split four-row kernel for p (x quantized in global memory, few tiles):
// S parts per tile, the largest power of two up to 16 and the k-steps whose
// parts still fit the GPU's warps in one round; stages: two when a part has
// more than one k-step.
cudaError_t launch_r4_split(const LaunchCfg& c, const QGemvParams& p) {
    const int warps = 16;
    QGemvParams q = p;
    q.split = 1;
    while (q.split < warps && 2 * q.split <= p.ksteps &&
           (long long)p.ntiles * 2 * q.split <= (long long)c.num_sms * warps)
        q.split *= 2;
    q.stages = (p.ksteps + q.split - 1) / q.split > 1 ? 2 : 1;
    void (*k)(QGemvParams);
    if (p.gather) k = gemv_q4_r4s<kExtGather>;
    else if (p.res) k = gemv_q4_r4s<kExtRes>;
    else k = gemv_q4_r4s<0>;
    const size_t smem = r4s_smem(warps, q.stages);
    int per_sm = 0;
    cudaError_t e = occupancy_cached((const void*)k, warps * 32, smem, &per_sm);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorInvalidConfiguration;
    const int T = warps / q.split;
    const long long groups = (p.ntiles + T - 1) / T;
    const long long grid = std::max<long long>(1, std::min<long long>(groups, (long long)per_sm * c.num_sms));
    return launch(k, dim3((unsigned)grid), dim3(warps * 32), smem, c, q);
}

template <int F, int M>
cudaError_t launch_fast_m(const LaunchCfg& c, const QGemvParams& p, size_t smem, bool dump) {
    void (*k)(QGemvParams);
    if constexpr (F == 0 && M == 1) {
        if (p.r4 && r4_split(p, c.num_sms)) {
            if (!p.xq) return cudaErrorInvalidValue;   // x quantized (and normalised) in global memory first
            return launch_r4_split(c, p);
        }
        if (p.r4) k = p.xq ? r4_kernel<true>(p) : r4_kernel<false>(p);
        else if (p.xq) k = gemv_q_fast2<F, M, true, false>;
        else if (dump) k = gemv_q_fast<F, M, false, true>;
        else k = gemv_q_fast2<F, M, false, false>;
    } else if constexpr (F == 0 && M <= 2) {
        if (p.xq) k = gemv_q_fast2<F, M, true, false>;
        else if (dump) k = gemv_q_fast<F, M, false, true>;
        else k = gemv_q_fast2<F, M, false, false>;
    } else {
        if (p.xq) k = gemv_q_fast<F, M, true, false>;
        else if (dump) k = gemv_q_fast<F, M, false, true>;
        else k = gemv_q_fast<F, M, false, false>;
    }
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
    const int grid = (int)std::max<long long>(std::min(want, cap), 1);
    QGemvParams q = p;
    q.cta_q = p.ntiles / grid;
    q.cta_r = p.ntiles % grid;
    return launch(k, dim3((unsigned)grid), dim3(c.warps * 32), smem, c, q);
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

bool r4_shape(int N, int K, int num_sms) {
    if (K == 2048) return true;
    // Longer rows, where x is quantized once into global memory (K >= 8192,
    // N <= 16384), with tiles for every warp (8 per SM) or K >= 16384 (then
    // fewer tiles take the split-K kernel, r4_split). Measured on B200,
    // graph-chained: 8192x28672 23.6 us against 28.8; 28672x8192 (x in shared
    // memory) and, at K = 8192, the Llama down projection 2048x8192 were slower
    // this way, split or not (6.88 us in the superblock kernel, 7.50 split).
    return K % 2048 == 0 && K >= 8192 && N <= 16384 && ((long long)N >= 32LL * num_sms || K >= 16384);
}

bool r4_split(const QGemvParams& p, int num_sms) {
    return p.r4 && p.ksteps >= 8 && (long long)p.ntiles < 8LL * num_sms;
}

void plan_tiles(QGemvParams& p, bool fast, int fmt, bool allow_r4, int num_sms) {
    p.nb = p.K / kQK;
    p.nsbp = (p.nb + 7) / 8;
    p.r4 = fast && allow_r4 && fmt == kQ4_0 && p.M == 1 && p.K > 0 && r4_shape(p.N, p.K, num_sms);
    if (p.r4) {
        p.G = 8;
        p.log2G = 3;
        p.TR = 4;
        p.ksteps = p.K / 2048;
        p.ntiles = (p.N + 3) / 4;
        return;
    }
    int G = 1, lg = 0;
    if (fast) {
        while (G < p.nsbp && G < 32) { G <<= 1; ++lg; }
    } else {
        G = 32;
        lg = 5;
    }
    p.G = G;
    p.log2G = lg;
    p.TR = 32 / G;
    p.ksteps = std::max(1, (p.nsbp + G - 1) / G);
    p.ntiles = (p.N + p.TR - 1) / p.TR;
}

size_t gemv_q_smem(int fmt, const QGemvParams& p, int warps, int stages, bool x_in_smem) {
    size_t off = ((size_t)warps * stages * 8 + 127) & ~(size_t)127;
    if (x_in_smem) off += (x_bytes(p) + 127) & ~(size_t)127;
    return off + (size_t)warps * stages * 32 * sb_bytes(fmt);
}

cudaError_t launch_quantize_x(const LaunchCfg& c, const QGemvParams& p, uint8_t* xq) {
    const long long groups = (long long)p.M * p.nb;
    const long long grid = std::min<long long>((groups + kThreadsQuantX / 8 - 1) / (kThreadsQuantX / 8),
                                               (long long)c.num_sms * 4);
    const XGeom xg{p.M, p.nb, p.log2G, p.ksteps, p.r4};
    return launch(quantize_x_kernel, dim3((unsigned)std::max<long long>(grid, 1)), dim3(kThreadsQuantX), 0, c, p.x,
                  p.ldx, p.up, p.ldu, xg, xq, p.nw, p.neps);
}

cudaError_t launch_stage_x(cudaStream_t s, const float* src, float* dst, long long n, int num_sms) {
    if (n <= 0) return cudaSuccess;
    const long long grid = std::min<long long>((n / 4 + 511) / 512 + 1, (long long)num_sms);
    stage_x_kernel<<<(unsigned)grid, 512, 0, s>>>(src, dst, n);
    return cudaGetLastError();
}

cudaError_t launch_check_x_arith(cudaStream_t s, unsigned long long* bad) {
    check_x_arith_kernel<<<148 * 8, 256, 0, s>>>(bad);
    return cudaGetLastError();
}

cudaError_t launch_silu_mul(cudaStream_t s, long long n, const float* gate, const float* up, float* out) {
    if (n <= 0) return cudaSuccess;
    const long long grid = std::min<long long>((n + 255) / 256, 148LL * 8);
    silu_mul_kernel<<<(unsigned)grid, 256, 0, s>>>(n, gate, up, out);
    return cudaGetLastError();
}

cudaError_t launch_gemv_q(const LaunchCfg& c, int fmt, QGemvParams p, bool fast, size_t* smem_used) {
    const bool dump = p.dump != nullptr;
    size_t smem = 0;
    if (fast) smem = gemv_q_smem(fmt, p, c.warps, p.stages, p.xq == nullptr);
    if (smem_used) *smem_used = smem;
    return fmt == kQ4_0 ? dispatch_m<kQ4_0>(c, p, fast, smem, dump) : dispatch_m<kQ8_0>(c, p, fast, smem, dump);
}

cudaError_t launch_gather_wait(const LaunchCfg& c, const GatherArgs* g_dev, int M, int blocks, unsigned* err) {
    return launch(gather_wait_kernel, dim3(blocks), dim3(kGatherWaitThreads), 0, c, g_dev, M, err);
}

cudaError_t launch_gather_barrier(const LaunchCfg& c, const GatherArgs* g_dev, unsigned* err) {
    return launch(gather_barrier_kernel, dim3(1), dim3(32), 0, c, g_dev, err);
}

cudaError_t launch_gather_pingpong(cudaStream_t s, const GatherArgs* g_dev, unsigned base, int iters, bool relaxed,
                                   unsigned* err, unsigned long long* ns) {
    gather_pingpong_kernel<<<1, 32, 0, s>>>(g_dev, base, iters, relaxed ? 1 : 0, err, ns);
    return cudaGetLastError();
}

size_t xmma_bytes(int nb) { return (size_t)nb * (kMmaXFragBytes + kMmaXcdBytes); }

cudaError_t launch_quantize_x_mma(const LaunchCfg& c, const QGemvParams& p, uint8_t* xq) {
    const long long groups = (long long)p.nb * 8;
    const long long grid = std::min<long long>((groups + kThreadsQuantX / 8 - 1) / (kThreadsQuantX / 8),
                                               (long long)c.num_sms * 4);
    return launch(quantize_x_mma_kernel, dim3((unsigned)std::max<long long>(grid, 1)), dim3(kThreadsQuantX), 0, c,
                  p.x, p.ldx, p.up, p.ldu, p.M, p.nb, xq, p.kparts > 1 ? p.tickets : nullptr);
}

size_t gemv_q_mma_smem(int fmt, int stages, int xnb, bool x_in_smem) {
    const int rs = fmt == kQ4_0 ? mma_rs<kQ4_0>() : mma_rs<kQ8_0>();
    return mma_ring_offset(kMmaWarps, stages, xnb, x_in_smem) + (size_t)kMmaWarps * stages * 16 * rs;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// against the driver library); null when the driver does not offer it.
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return (PFN_cuTensorMapEncodeTiled_v12000) nullptr;
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    }();
    return fn;
}

// The weights as a 2-D tensor: N rows of nb·block bytes (16-byte multiple,
// since nb % 8 == 0), boxes of 16 rows × 8 blocks.
cudaError_t encode_weight_map(int fmt, const QGemvParams& p, CUtensorMap* map) {
    PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
    if (!enc) return cudaErrorNotSupported;
    const bool q4 = fmt == kQ4_0;
    const cuuint64_t row_bytes = (cuuint64_t)p.nb * block_bytes(fmt);
    const cuuint64_t dims[2] = {q4 ? row_bytes : row_bytes / 2, (cuuint64_t)p.N};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {q4 ? (cuuint32_t)mma_rs<kQ4_0>() : (cuuint32_t)mma_rs<kQ8_0>() / 2, 16u};
    const cuuint32_t estr[2] = {1u, 1u};
    const CUresult r = enc(map, q4 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_UINT16, 2,
                           const_cast<uint8_t*>(p.w), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t launch_gemv_q_mma(const LaunchCfg& c, int fmt, const QGemvParams& p, bool x_in_smem) {
    CUtensorMap wmap;
    cudaError_t me = encode_weight_map(fmt, p, &wmap);
    if (me != cudaSuccess) return me;
    void (*k)(QGemvParams, CUtensorMap);
    if (p.gather) {
        if (fmt == kQ4_0) k = x_in_smem ? gemv_q_mma<kQ4_0, true, true> : gemv_q_mma<kQ4_0, false, true>;
        else k = x_in_smem ? gemv_q_mma<kQ8_0, true, true> : gemv_q_mma<kQ8_0, false, true>;
    } else {
        if (fmt == kQ4_0) k = x_in_smem ? gemv_q_mma<kQ4_0, true, false> : gemv_q_mma<kQ4_0, false, false>;
        else k = x_in_smem ? gemv_q_mma<kQ8_0, true, false> : gemv_q_mma<kQ8_0, false, false>;
    }
    const int P = p.kparts > 1 ? p.kparts : 1;
    if (P > 1 && (!x_in_smem || !p.partial || !p.tickets)) return cudaErrorInvalidValue;
    const size_t smem = gemv_q_mma_smem(fmt, p.stages, p.xnb > 0 ? p.xnb : p.nb, x_in_smem);
    int per_sm = 0;
    cudaError_t e = occupancy_cached((const void*)k, kMmaWarps * 32, smem, &per_sm);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorInvalidConfiguration;
    // Split K (S parts per tile, a power of two up to the warps of a CTA and the
    // k-steps) until the tiles' parts fill about 3/4 of the GPU's warps.
    const long long ntiles = ((long long)p.N + 15) / 16, ksteps = p.nb / 8;
    const long long cap = (long long)std::min(per_sm, std::max(c.ctas_per_sm, 1)) * c.num_sms;
    QGemvParams q = p;
    q.split = 1;
    long long grid;
    if (P > 1) {
        // K parts across CTAs: C CTAs per part, the same tile groups in every
        // part; within a CTA the part may be split again (S) while the groups
        // do not fill the CTA slots of a part.
        const long long kspan = ksteps / P, cap_part = std::max(1LL, cap / P);
        while (q.split < kMmaWarps && 2LL * q.split <= kspan && ntiles * P * q.split * 4 < cap * kMmaWarps * 3)
            q.split *= 2;
        while (q.split < kMmaWarps && 2LL * q.split <= kspan &&
               (ntiles * q.split + kMmaWarps - 1) / kMmaWarps < cap_part)
            q.split *= 2;
        const long long T = kMmaWarps / q.split;
        const long long C = std::min((ntiles + T - 1) / T, cap_part);
        if (C > kMmaMaxTickets) return cudaErrorInvalidConfiguration;
        return launch(k, dim3((unsigned)(C * P)), dim3(kMmaWarps * 32), smem, c, q, wmap);
    }
    while (q.split < kMmaWarps && 2LL * q.split <= ksteps && ntiles * q.split * 4 < cap * kMmaWarps * 3) q.split *= 2;
    if (q.split == 1) {   // tiles interleaved over every warp of the grid
        grid = std::min(std::max((ntiles + kMmaWarps - 1) / kMmaWarps, std::min<long long>(ntiles, c.num_sms)), cap);
    } else {              // groups of kMmaWarps / S tiles per CTA: enough groups for every CTA slot
        while (q.split < kMmaWarps && 2LL * q.split <= ksteps && (ntiles * q.split + kMmaWarps - 1) / kMmaWarps < cap)
            q.split *= 2;
        const long long T = kMmaWarps / q.split;
        grid = std::min((ntiles + T - 1) / T, cap);
    }
    return launch(k, dim3((unsigned)std::max<long long>(grid, 1)), dim3(kMmaWarps * 32), smem, c, q, wmap);
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
