// gemv_dense_mma.cu — sm_100a tensor-core decode GEMV for bfloat16 weights and
// 4..8 rows of x: the reference's sgemm_bf16 / sgemm with trans_b on its
// dot_rows path (src/kernels/gemm/avx2_gemm_packed.cpp:358-448; scalar order
// src/kernels/scalar_kernels.cpp:69-84), C = alpha · X · Wᵀ + beta · C.
//
// Why: the CUDA-core kernel (gemv_dense.cu) re-reads x from shared memory for
// every weight row and keeps an accumulator per (row, x row) in registers, so
// at M = 8 it runs three warps per scheduler and stays latency-bound (0.43 of
// HBM). Here every 16 × 16 tile of W meets all 8 rows of x in one
// mma.sync.m16n8k16 with fp32 accumulation.
//
// Exactness: bf16 × bf16 products are exact in fp32. x (fp32, 24-bit
// significand) is split exactly into three bf16 parts, x = hi + mid + lo: hi
// is x truncated to bf16, mid the remainder truncated, lo what is left, which
// has at most 8 significant bits. Each part meets W in its own MMA, so every
// product is exact and only the fp32 sums round (the dense bound of the
// reference's tests, 2(K+2)·2^-24·Σ|x||w|). Each part has its own
// accumulator (three independent MMA chains); mid + lo, then hi + that, at
// the end. bf16 x is its own single part.
//
// Layout: a split kernel writes the parts once per call in B-fragment order
// (dm_xfrag_bytes: per 16-value block kb, per part, 32 lanes × (two bf16x2
// words)), 192 KB at K = 4096. A warp item is 16 rows × 128 values of W: two
// tensor-map boxes of 16 × 64 bf16 with the 128-byte swizzle (A fragments by
// ldmatrix), plus that k-range's x fragments by one bulk copy (an L2 hit),
// in one ring stage with one mbarrier. Weight boxes of the first stages are
// issued before griddepcontrol.wait; their x fragments after it, since the
// split kernel before writes them.
//
// Work: each CTA takes a contiguous range of 16-row tiles, in rounds of T
// tiles; within a round warp w takes tile w / S and K part w % S (S parts of
// the K items, S a power of two chosen so that the warps have work), and part
// 0 adds the S parts' sums in order through shared memory. Deterministic.
//
// Special values: an infinite weight that meets a zero part of x makes a NaN
// in the mid + lo accumulator where the reference's single product gives ±inf;
// an output whose mid + lo sum is NaN while its hi sum is not is recomputed by
// its lane in plain fp32 (rare: W holds an infinity). NaN or infinite x keeps
// the reference's results (hi carries the value, the other parts are zero).

#include "gemv_dense.cuh"
#include "gemv_quant.cuh"
#include "smk_device.cuh"

#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdint>

namespace smk {

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();   // gemv_quant.cu

namespace {

constexpr int kDMWarps = 8;
constexpr int kDMStages = 2;
constexpr int kDMItemK = 128;                  // K values of W per warp item
constexpr int kDMBox = 64;                     // bf16 values per box row (128 bytes, the swizzle span)
constexpr int kDMWBytes = 16 * kDMItemK * 2;   // weight bytes of an item (two boxes)

__host__ __device__ constexpr int dm_xbytes(int np) { return 8 * np * 256; }   // x fragments of an item
__host__ __device__ constexpr int dm_stage(int np) { return kDMWBytes + dm_xbytes(np); }   // multiple of 1024

// Shared memory: barriers, the S parts' sums (8 floats per lane per warp), then
// the rings on a 1024-byte boundary (the swizzle's period).
__host__ __device__ inline size_t dm_parts_offset() { return ((size_t)kDMWarps * kDMStages * 8 + 127) & ~(size_t)127; }
__host__ __device__ inline size_t dm_ring_offset() { return dm_parts_offset() + (size_t)kDMWarps * 32 * 8 * 4; }
__host__ __device__ inline size_t dm_smem(int np) {
    return dm_ring_offset() + 1024 + (size_t)kDMWarps * kDMStages * dm_stage(np);
}

// x = hi + mid + lo exactly, each a bf16 (bits in the low 16 of the result).
// Non-finite x: hi carries it (NaN as the canonical quiet NaN), mid = lo = 0.
__device__ __forceinline__ void split3(float x, uint32_t (&part)[3]) {
    const uint32_t b = __float_as_uint(x);
    if ((b & 0x7f800000u) == 0x7f800000u) {
        part[0] = (b & 0x007fffffu) ? 0x7fc0u : (b >> 16);
        part[1] = part[2] = 0u;
        return;
    }
    const uint32_t hb = b & 0xffff0000u;
    const float r = __fsub_rn(x, __uint_as_float(hb));   // exact: x and hi agree in sign and leading bits
    const uint32_t mb = __float_as_uint(r) & 0xffff0000u;
    const float l = __fsub_rn(r, __uint_as_float(mb));   // exact, at most 8 significant bits
    part[0] = hb >> 16;
    part[1] = mb >> 16;
    part[2] = __float_as_uint(l) >> 16;
}

template <int XK>
__device__ __forceinline__ float x_at(const void* x, long long i) {
    if constexpr (XK == kF32) return static_cast<const float*>(x)[i];
    else return __uint_as_float((uint32_t)static_cast<const uint16_t*>(x)[i] << 16);
}

// x [M, K] into the fragment layout at xf: thread (kb, lane) writes lane's
// words of block kb for every part. NP = 3 (fp32 x) or 1 (bf16 x, exact).
template <int XK, int NP>
__global__ void __launch_bounds__(256) dense_split_x_kernel(const void* __restrict__ x, long long ldx, int M, int K,
                                                            uint2* __restrict__ xf) {
    pdl_launch_dependents();
    pdl_wait_primary();   // x may come from the previous kernel, which may still read xf
    const long long total = (long long)(K / 16) * 32;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int kb = (int)(i >> 5), lane = (int)(i & 31), g = lane >> 2, t = lane & 3;
        float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};   // k = 16kb + 2t, +1, +8, +9 of x row g
        if (g < M) {
            const long long k0 = (long long)g * ldx + 16 * kb + 2 * t;
            v[0] = x_at<XK>(x, k0);
            v[1] = x_at<XK>(x, k0 + 1);
            v[2] = x_at<XK>(x, k0 + 8);
            v[3] = x_at<XK>(x, k0 + 9);
        }
        uint32_t p[4][3];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            if constexpr (NP == 3) split3(v[e], p[e]);
            else p[e][0] = __float_as_uint(v[e]) >> 16;   // bf16 x: the value itself
        }
#pragma unroll
        for (int q = 0; q < NP; ++q)
            xf[((size_t)kb * NP + q) * 32 + lane] = make_uint2(p[0][q] | (p[1][q] << 16), p[2][q] | (p[3][q] << 16));
    }
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

// d += A·B: A 16 × 16 bf16 (rows of W), B 16 × 8 bf16 (rows of x as columns), fp32.
// A function of its register operands only (not volatile), so the compiler
// schedules it by its dependencies; the shared-memory loads feeding it stay
// ordered after the stage's barrier wait.
__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint2 b) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b.x), "r"(b.y));
}

struct DMGeom {
    int ntiles;   // ceil(N / 16)
    int nk;       // K / kDMItemK
    int S;        // K parts per tile (power of two, <= kDMWarps)
};

// One output recomputed in plain fp32 (x in its own type, W bf16 or fp16), k in order.
template <int WK, int XK>
__device__ float dense_dot_fp32(const DenseParams& p, int row, int m) {
    const uint16_t* w = static_cast<const uint16_t*>(p.w) + (size_t)row * p.ldw;
    float s = 0.0f;
    for (int k = 0; k < p.K; ++k) {
        const float wv = WK == kF16 ? __half2float(__ushort_as_half(w[k])) : __uint_as_float((uint32_t)w[k] << 16);
        s = __fmaf_rn(x_at<XK>(p.x, (long long)m * p.ldx + k), wv, s);
    }
    return s;
}

// An A-fragment register of two fp16 weights as two registers of bf16 pairs,
// w = hi + lo exactly: hi is w (exact in fp32) truncated to bf16, lo the
// remainder, at most 3 significant bits (fp16 has 11, bf16 8), exact in bf16
// for every finite fp16 including subnormals. An infinity leaves lo = NaN:
// its outputs are recomputed in plain fp32 (the NaN check below).
__device__ __forceinline__ void split_f16x2(uint32_t h, uint32_t& hi, uint32_t& lo) {
    const float f0 = half_lo_to_float(h), f1 = half_hi_to_float(h);
    const uint32_t b0 = __float_as_uint(f0), b1 = __float_as_uint(f1);
    hi = __byte_perm(b0, b1, 0x7632);
    const float r0 = __fsub_rn(f0, __uint_as_float(b0 & 0xffff0000u)), r1 = __fsub_rn(f1, __uint_as_float(b1 & 0xffff0000u));
    lo = __byte_perm(__float_as_uint(r0), __float_as_uint(r1), 0x7632);
}

// WK: kBF16 (W used as it is) or kF16 (each weight split into two bf16 parts,
// so every part of x meets both: six MMAs per 16 × 16 tile, all products exact).
template <int WK, int XK, int NP>
__global__ void __launch_bounds__(kDMWarps * 32, 1) gemv_dense_mma(const DenseParams p, const DMGeom g,
                                                                   const __grid_constant__ CUtensorMap wmap) {
    constexpr int XB = dm_xbytes(NP), STAGE = dm_stage(NP);
    extern __shared__ __align__(128) uint8_t smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int gq = lane >> 2, t = lane & 3;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem) + warp * kDMStages;
    float* parts = reinterpret_cast<float*>(smem + dm_parts_offset());
    const uint32_t raw = smem_addr(smem);
    const uint32_t ring_addr = (raw + (uint32_t)dm_ring_offset() + 1023u) & ~1023u;
    uint8_t* ring = smem + (ring_addr - raw) + (size_t)warp * kDMStages * STAGE;
    const uint32_t ring_w = ring_addr + (uint32_t)(warp * kDMStages * STAGE);
    const uint8_t* xf = static_cast<const uint8_t*>(p.xfrag);

    pdl_launch_dependents();
    const int S = g.S, T = kDMWarps / S, part = warp % S, tl = warp / S;
    const int k_lo = part * g.nk / S, nks = (part + 1) * g.nk / S - k_lo;
    const int c_lo = (int)((long long)blockIdx.x * g.ntiles / gridDim.x);
    const int c_hi = (int)((long long)(blockIdx.x + 1) * g.ntiles / gridDim.x);
    const int rounds = (c_hi - c_lo + T - 1) / T;   // CTA-uniform
    auto tile_of = [&](int r) { return c_lo + r * T + tl; };
    int my_rounds = 0;   // rounds in which this warp has a tile (a prefix of the rounds)
    while (my_rounds < rounds && tile_of(my_rounds) < c_hi) ++my_rounds;
    const int nitems = my_rounds * nks;
    if (lane == 0) {
        for (int i = 0; i < kDMStages; ++i) mbar_init(&bars[i], 1);
        fence_mbar_init();
    }
    __syncwarp();
    int i_r = 0, i_k = 0, i_slot = 0, issued = 0;
    auto issue_w = [&](int slot, int tile, int kk) {
        if (lane == 0) {
            uint64_t* bar = &bars[slot];
            uint8_t* dst = ring + (size_t)slot * STAGE;
            mbar_arrive_expect_tx(bar, (uint32_t)STAGE);   // whole boxes (zero past N) and the x fragments
            tma_load_2d(dst, &wmap, kk * kDMItemK, tile * 16, bar);
            tma_load_2d(dst + 16 * kDMBox * 2, &wmap, kk * kDMItemK + kDMBox, tile * 16, bar);
        }
    };
    auto issue_x = [&](int slot, int kk) {
        if (lane == 0)
            tma_load_1d(ring + (size_t)slot * STAGE + kDMWBytes, xf + (size_t)kk * XB, (uint32_t)XB, &bars[slot]);
    };
    int pre_k[kDMStages];
    const int npre = min(kDMStages, nitems);
    for (; issued < npre; ++issued) {   // weights only: the x fragments are the previous kernel's output
        pre_k[issued] = k_lo + i_k;
        issue_w(i_slot, tile_of(i_r), k_lo + i_k);
        if (++i_k == nks) { i_k = 0; ++i_r; }
        if (++i_slot == kDMStages) i_slot = 0;
    }
    pdl_wait_primary();
    for (int i = 0; i < npre; ++i) issue_x(i, pre_k[i]);

    const int li = lane >> 3, wrow = (lane & 7) + 8 * (li & 1);
    int failed = 0, c_slot = 0, consumed = 0;
    uint32_t c_phase = 0;
    for (int r = 0; r < rounds; ++r) {   // CTA-uniform: every warp meets every barrier
        // One accumulator per part: three independent MMA chains (hi, mid, lo);
        // fp16 weights: one per product of their parts (six chains), so no chain
        // takes more than one MMA per block, folded into mid and lo at the end.
        float hi[4] = {0.f, 0.f, 0.f, 0.f}, mid[4] = {0.f, 0.f, 0.f, 0.f}, lo[4] = {0.f, 0.f, 0.f, 0.f};
        float mid2[4] = {0.f, 0.f, 0.f, 0.f}, lo2[4] = {0.f, 0.f, 0.f, 0.f}, lo3[4] = {0.f, 0.f, 0.f, 0.f};
        if (r < my_rounds) {
            for (int k = 0; k < nks && !failed; ++k) {
                if (__any_sync(0xffffffffu, !mbar_wait_bounded(&bars[c_slot], c_phase, p.err))) {
                    failed = 1;
                    break;
                }
                const uint32_t st = ring_w + (uint32_t)(c_slot * STAGE);
                const uint2* xs = reinterpret_cast<const uint2*>(ring + (size_t)c_slot * STAGE + kDMWBytes);
                // Four 16-value blocks at a time: their A fragments and x fragments
                // loaded first, then their MMAs.
#pragma unroll
                for (int k4 = 0; k4 < 8; k4 += 4) {
                    uint32_t a[4][4];
                    uint2 bx[4][NP];
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const int kb = k4 + u, box = kb >> 2, chunk = 2 * (kb & 3) + (li >> 1);
                        ldsm_x4(a[u], st + (uint32_t)(box * 16 * kDMBox * 2 + wrow * kDMBox * 2 +
                                                      ((chunk ^ (wrow & 7)) << 4)));
#pragma unroll
                        for (int q = 0; q < NP; ++q) bx[u][q] = xs[(kb * NP + q) * 32 + lane];
                    }
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        if constexpr (WK == kF16) {   // fp32 x only (NP == 3)
                            uint32_t ah[4], al[4];
#pragma unroll
                            for (int i = 0; i < 4; ++i) split_f16x2(a[u][i], ah[i], al[i]);
                            mma_bf16(hi, ah, bx[u][0]);
                            mma_bf16(mid, ah, bx[u][1]);
                            mma_bf16(mid2, al, bx[u][0]);
                            mma_bf16(lo, ah, bx[u][2]);
                            mma_bf16(lo2, al, bx[u][1]);
                            mma_bf16(lo3, al, bx[u][2]);
                        } else {
                            mma_bf16(hi, a[u], bx[u][0]);
                            if constexpr (NP == 3) {
                                mma_bf16(mid, a[u], bx[u][1]);
                                mma_bf16(lo, a[u], bx[u][2]);
                            }
                        }
                    }
                }
                __syncwarp();
                if (issued < nitems) {
                    fence_proxy_async_smem();
                    issue_w(i_slot, tile_of(i_r), k_lo + i_k);
                    issue_x(i_slot, k_lo + i_k);
                    if (++i_k == nks) { i_k = 0; ++i_r; }
                    if (++i_slot == kDMStages) i_slot = 0;
                    ++issued;
                }
                ++consumed;
                if (++c_slot == kDMStages) { c_slot = 0; c_phase ^= 1u; }
            }
        }
        if constexpr (WK == kF16) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                mid[i] = __fadd_rn(mid[i], mid2[i]);
                lo[i] = __fadd_rn(__fadd_rn(lo[i], lo2[i]), lo3[i]);
            }
        }
        if (S > 1) {   // part 0 adds the parts' sums, in part order
#pragma unroll
            for (int i = 0; i < 4; ++i) lo[i] = __fadd_rn(mid[i], lo[i]);   // the low parts' sum, then the parts
            float* mine = parts + (warp * 32 + lane) * 8;
#pragma unroll
            for (int i = 0; i < 4; ++i) { mine[i] = hi[i]; mine[4 + i] = lo[i]; }
            __syncthreads();
            if (part == 0) {
                for (int q = 1; q < S; ++q) {
                    const float* o = parts + ((warp + q) * 32 + lane) * 8;
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        hi[i] = __fadd_rn(hi[i], o[i]);
                        lo[i] = __fadd_rn(lo[i], o[4 + i]);
                    }
                }
            }
            __syncthreads();
        }
        if (S == 1) {
#pragma unroll
            for (int i = 0; i < 4; ++i) lo[i] = __fadd_rn(mid[i], lo[i]);
        }
        if (part == 0 && r < my_rounds && !failed) {
            const int tile = tile_of(r);
#pragma unroll
            for (int rr = 0; rr < 2; ++rr) {
                const int row = tile * 16 + gq + 8 * rr;
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    const int m = 2 * t + j;
                    if (row < p.N && m < p.M) {
                        const float h = hi[2 * rr + j], l = lo[2 * rr + j];
                        const float v = (isnan(l) && !isnan(h)) ? dense_dot_fp32<WK, XK>(p, row, m) : __fadd_rn(h, l);
                        float* c = p.y + (size_t)m * p.ldy + row;
                        const float cb = p.beta == 0.0f ? 0.0f : (p.beta == 1.0f ? *c : __fmul_rn(p.beta, *c));
                        *c = __fadd_rn(cb, __fmul_rn(p.alpha, v));
                    }
                }
            }
        }
    }
    if (failed) {   // let this warp's copies still in flight land (bounded) before the CTA exits
        for (int k = consumed; k < issued; ++k) mbar_wait_bounded(&bars[k % kDMStages], (uint32_t)((k / kDMStages) & 1), nullptr);
    }
}

}  // namespace

namespace {

template <typename Kern, typename... Args>
cudaError_t launch_dm(Kern kernel, long long grid, int threads, size_t smem, cudaStream_t s, bool pdl, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

int dm_parts_of(int x_kind) { return x_kind == kF32 ? 3 : 1; }

}  // namespace

size_t dense_mma_scratch(int w_kind, int x_kind, int M, int K, long long ldw, const void* w) {
    if (!(w_kind == kBF16 && (x_kind == kF32 || x_kind == kBF16)) && !(w_kind == kF16 && x_kind == kF32)) return 0;
    if (M < kDenseMmaMinRows || M > 8 || K < kDMItemK || K % kDMItemK != 0) return 0;
    // fp16 weights: six MMAs and the split of every weight per tile; measured on
    // B200 at 14336x4096, 36.2 us here against 44.8 (M = 8) and 32.3 (M = 4) on
    // the CUDA-core kernel, so from 6 rows.
    if (w_kind == kF16 && M < kDenseMmaMinRowsF16) return 0;
    if ((ldw * 2) % 16 != 0 || (reinterpret_cast<uintptr_t>(w) & 15) != 0) return 0;
    int dev = 0, optin = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess)
        return 0;
    if (dm_smem(dm_parts_of(x_kind)) > (size_t)optin) return 0;
    return (size_t)(K / 16) * dm_parts_of(x_kind) * 256;
}

cudaError_t launch_gemv_dense_mma(cudaStream_t s, bool pdl, int num_sms, int w_kind, int x_kind, const DenseParams& p) {
    if (!p.xfrag) return cudaErrorInvalidValue;
    PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
    if (!enc) return cudaErrorNotSupported;
    // W as a 2-D tensor of bf16: N rows of K (row stride ldw), boxes of 16 rows
    // × 64 values with the 128-byte swizzle, zero fill past N.
    CUtensorMap wmap;
    const cuuint64_t dims[2] = {(cuuint64_t)p.K, (cuuint64_t)p.N};
    const cuuint64_t strides[1] = {(cuuint64_t)p.ldw * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kDMBox, 16u};
    const cuuint32_t estr[2] = {1u, 1u};
    if (enc(&wmap, w_kind == kF16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
            const_cast<void*>(p.w), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return cudaErrorNotSupported;
    const int np = dm_parts_of(x_kind);
    // The split: (K/16) blocks × 32 lanes.
    const long long pairs = (long long)(p.K / 16) * 32;
    const long long sgrid = std::max<long long>(1, std::min<long long>((pairs + 255) / 256, (long long)num_sms * 4));
    cudaError_t e;
    if (x_kind == kF32)
        e = launch_dm(dense_split_x_kernel<kF32, 3>, sgrid, 256, 0, s, pdl, p.x, p.ldx, p.M, p.K,
                      static_cast<uint2*>(p.xfrag));
    else
        e = launch_dm(dense_split_x_kernel<kBF16, 1>, sgrid, 256, 0, s, pdl, p.x, p.ldx, p.M, p.K,
                      static_cast<uint2*>(p.xfrag));
    if (e != cudaSuccess) return e;
    DMGeom g;
    g.ntiles = (p.N + 15) / 16;
    g.nk = p.K / kDMItemK;
    const long long grid = std::max<long long>(1, std::min<long long>(g.ntiles, num_sms));
    // K parts per tile: the largest power of two (at most the warps of a CTA and
    // the K items) whose tile parts still fit the grid's warps once.
    g.S = 1;
    while (g.S < kDMWarps && 2 * g.S <= g.nk && (long long)g.ntiles * g.S * 2 <= grid * kDMWarps) g.S *= 2;
    const size_t smem = dm_smem(np);
    auto k = w_kind == kF16 ? gemv_dense_mma<kF16, kF32, 3>
                            : (x_kind == kF32 ? gemv_dense_mma<kBF16, kF32, 3> : gemv_dense_mma<kBF16, kBF16, 1>);
    int per_sm = 0;
    e = occupancy((const void*)k, kDMWarps * 32, smem, &per_sm);   // also raises the kernel's shared-memory limit
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorNotSupported;
    // The split kernel wrote xfrag: the GEMV waits for it before its x copies
    // (griddepcontrol.wait), and streams its weights meanwhile.
    return launch_dm(k, grid, kDMWarps * 32, smem, s, true, p, g, wmap);
}

}  // namespace smk
