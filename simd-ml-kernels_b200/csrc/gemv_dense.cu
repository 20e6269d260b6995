// gemv_dense.cu — sm_100a dense decode GEMV, M ≤ 8 rows of x against W [N, K]
// in float32 / binary16 / bfloat16, FP32 accumulation (see gemv_dense.cuh).
//
// Bound by reading W once: each warp walks TR = 4 rows of W along K with
// 128-bit streaming loads (L1 no-allocate), converts 16-bit weights to FP32 in
// registers (exact), and uses each converted weight for all M rows of x, which
// the CTA stages in shared memory as FP32 (exact for the 16-bit types). No
// tensor cores: with M ≤ 8 the arithmetic is far below the HBM roof
// (≤ 16 FLOP per weight element), and FP32 x has no exact tensor-core type.
// Per lane FP32 FMA chains, then a shuffle reduction; the epilogue applies
// the reference's order: C = fl(beta·C) (0 when beta == 0: C is never read),
// then C + fl(alpha·sum).

#include "gemv_dense.cuh"
#include "gemv_quant.cuh"
#include "smk_device.cuh"

#include <algorithm>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace smk {

namespace {

constexpr int kTR = 4;            // rows of W per warp
constexpr int kWarps = 8;
constexpr size_t kXSmemMax = 96 * 1024;

template <int KIND>
__device__ __forceinline__ float to_f32(const void* base, long long i) {
    if constexpr (KIND == kF32) return reinterpret_cast<const float*>(base)[i];
    const unsigned short h = reinterpret_cast<const unsigned short*>(base)[i];
    if constexpr (KIND == kF16) return __half2float(__ushort_as_half(h));
    return __uint_as_float((uint32_t)h << 16);
}

// 16 bytes of W as FP32 values: 4 (float32) or 8 (16-bit).
template <int WK>
struct Vec {
    static constexpr int kElems = WK == kF32 ? 4 : 8;
    float v[kElems];
    __device__ __forceinline__ void load(const void* p) {
        const uint4 u = ld_stream_v4(p);
        if constexpr (WK == kF32) {
            v[0] = __uint_as_float(u.x); v[1] = __uint_as_float(u.y);
            v[2] = __uint_as_float(u.z); v[3] = __uint_as_float(u.w);
        } else {
            const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                if constexpr (WK == kF16) {
                    v[2 * i] = __half2float(__ushort_as_half((unsigned short)(w[i] & 0xffffu)));
                    v[2 * i + 1] = __half2float(__ushort_as_half((unsigned short)(w[i] >> 16)));
                } else {
                    v[2 * i] = __uint_as_float(w[i] << 16);
                    v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
                }
            }
        }
    }
};

template <int WK, int XK, int M, bool kVec, bool kXSmem>
__global__ void __launch_bounds__(kWarps * 32) gemv_dense_kernel(const DenseParams p) {
    extern __shared__ __align__(16) float xs[];
    constexpr int ES = WK == kF32 ? 4 : 2;
    constexpr int VE = 16 / ES;
    const int lane = threadIdx.x & 31;
    const int Kp = (p.K + 3) & ~3;   // shared row stride: 16-byte aligned rows
    pdl_launch_dependents();
    pdl_wait_primary();
    if constexpr (kXSmem) {
        for (long long i = threadIdx.x; i < (long long)M * p.K; i += blockDim.x) {
            const int m = (int)(i / p.K);
            const long long k = i - (long long)m * p.K;
            xs[(long long)m * Kp + k] = to_f32<XK>(p.x, m * p.ldx + k);
        }
        __syncthreads();
    }
    auto xval = [&](int m, int k) -> float {
        if constexpr (kXSmem) return xs[(long long)m * Kp + k];
        else return to_f32<XK>(p.x, m * p.ldx + k);
    };

    const int groups = (p.N + kTR - 1) / kTR;
    const int gwarps = gridDim.x * kWarps;
    for (int grp = blockIdx.x * kWarps + (threadIdx.x >> 5); grp < groups; grp += gwarps) {
        const int r0 = grp * kTR;
        const int nr = min(kTR, p.N - r0);
        float acc[kTR][M];
#pragma unroll
        for (int r = 0; r < kTR; ++r)
#pragma unroll
            for (int m = 0; m < M; ++m) acc[r][m] = 0.0f;

        int kdone = 0;
        if constexpr (kVec) {
            const int nvec = p.K / VE;
            const char* wrow = reinterpret_cast<const char*>(p.w) + (size_t)r0 * p.ldw * ES;
            const size_t rstride = (size_t)p.ldw * ES;
            for (int v = lane; v < nvec; v += 32) {
                Vec<WK> wv[kTR];
#pragma unroll
                for (int r = 0; r < kTR; ++r)
                    if (r < nr) wv[r].load(wrow + r * rstride + (size_t)v * 16);
                const int k0 = v * VE;
#pragma unroll
                for (int m = 0; m < M; ++m) {
                    float xv[VE];
                    if constexpr (kXSmem) {
                        const float4* xp = reinterpret_cast<const float4*>(xs + (size_t)m * Kp + k0);
#pragma unroll
                        for (int q = 0; q < VE / 4; ++q) {
                            const float4 t = xp[q];
                            xv[4 * q] = t.x; xv[4 * q + 1] = t.y; xv[4 * q + 2] = t.z; xv[4 * q + 3] = t.w;
                        }
                    } else {
#pragma unroll
                        for (int e = 0; e < VE; ++e) xv[e] = xval(m, k0 + e);
                    }
#pragma unroll
                    for (int r = 0; r < kTR; ++r)
#pragma unroll
                        for (int e = 0; e < VE; ++e) acc[r][m] = fmaf(wv[r].v[e], xv[e], acc[r][m]);
                }
            }
            kdone = nvec * VE;
        }
        for (int k = kdone + lane; k < p.K; k += 32) {
#pragma unroll
            for (int r = 0; r < kTR; ++r) {
                if (r >= nr) continue;
                const float wv = to_f32<WK>(p.w, (long long)(r0 + r) * p.ldw + k);
#pragma unroll
                for (int m = 0; m < M; ++m) acc[r][m] = fmaf(wv, xval(m, k), acc[r][m]);
            }
        }
#pragma unroll
        for (int r = 0; r < kTR; ++r)
#pragma unroll
            for (int m = 0; m < M; ++m) {
                float s = acc[r][m];
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
                if (lane == 0 && r < nr) {
                    float* c = p.y + (size_t)m * p.ldy + r0 + r;
                    const float cb = p.beta == 0.0f ? 0.0f : (p.beta == 1.0f ? *c : __fmul_rn(p.beta, *c));
                    *c = p.K == 0 ? cb : __fadd_rn(cb, __fmul_rn(p.alpha, s));
                }
            }
    }
}

// ---- the streaming kernel ---------------------------------------------------------
//
// W rows reach shared memory by 1-D bulk TMA copies (never multicast) into a
// ring of stages per warp, as in the quantized kernel: a warp item is kDTR
// rows × kDRowBytes of K, each stage one item, one mbarrier per stage, the
// first stages issued before griddepcontrol.wait so the weight stream starts
// while the previous kernel finishes. Lane l reads 16 bytes at l·16 and
// 512 + l·16 of each row chunk (consecutive lanes, consecutive banks),
// converts them to FP32 in registers and accumulates pairs of adjacent k
// with packed FP32 FMA (__ffma2_rn: two IEEE fmas), against x staged as FP32
// in shared memory. Each (row, m) sum is the two pair halves added, a
// shuffle tree over the 32 lanes, then the reference's epilogue.

constexpr int kDTR = 4;              // rows per warp item
constexpr int kDRowBytes = 1024;     // bytes of one row per item
constexpr int kDWarps = 8;

template <int WK>
__device__ __forceinline__ void widen(const uint4 u, float2 (&f)[16 / (WK == kF32 ? 4 : 2) / 2]) {
    if constexpr (WK == kF32) {
        f[0] = make_float2(__uint_as_float(u.x), __uint_as_float(u.y));
        f[1] = make_float2(__uint_as_float(u.z), __uint_as_float(u.w));
    } else {
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            if constexpr (WK == kF16)
                f[i] = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
            else
                f[i] = make_float2(__uint_as_float(w[i] << 16), __uint_as_float(w[i] & 0xffff0000u));
        }
    }
}

struct DenseGeom {
    int ksteps;    // items per tile (ceil(K·es / kDRowBytes))
    int ntiles;    // ceil(N / kDTR)
    int stages;    // ring slots per warp
    int kp;        // shared x row stride in floats
    int xvec;      // x rows 16-byte aligned with K a multiple of the vector: vector staging
};

// x [M, K] into shared memory as FP32 (row stride kp), every thread keeping
// kXInFlight 16-byte loads in flight per round, so staging costs a few L2 round
// trips rather than one per element.
constexpr int kXInFlight = 8;

// With 16-bit weights lane l reads 16-byte chunks 2l and 2l + 1 of a half
// row of x, once per row of x and weight vector. Stored in order, lanes l and
// l + 4 of each 8-lane shared-memory wavefront would hit the same banks. So
// the rows are kept with chunk c at position c ^ ((c >> 3) & 1), which puts
// the 8 lanes on 8 distinct bank groups for both of their chunks (row stride
// a multiple of 8 floats, so the swap stays inside the row).
__device__ __forceinline__ int xswz(int c) { return c ^ ((c >> 3) & 1); }

template <int XK, int M, bool kSwz>
__device__ __forceinline__ void stage_x(const DenseParams& p, const DenseGeom& g, float* xs) {
    const int nt = blockDim.x, t = threadIdx.x;
    if (g.xvec) {
        constexpr int EV = XK == kF32 ? 4 : 8;   // elements per 16-byte vector
        const int per_row = p.K / EV;
#pragma unroll 1
        for (int m = 0; m < M; ++m) {
            const uint4* src = reinterpret_cast<const uint4*>(
                reinterpret_cast<const uint8_t*>(p.x) + (size_t)m * p.ldx * (XK == kF32 ? 4 : 2));
            float* dst = xs + (size_t)m * g.kp;
            for (int v0 = t; v0 < per_row; v0 += kXInFlight * nt) {
                uint4 u[kXInFlight];
#pragma unroll
                for (int i = 0; i < kXInFlight; ++i)
                    if (v0 + i * nt < per_row) u[i] = src[v0 + i * nt];
#pragma unroll
                for (int i = 0; i < kXInFlight; ++i) {
                    const int v = v0 + i * nt;
                    if (v >= per_row) break;
                    if constexpr (XK == kF32) {
                        *reinterpret_cast<uint4*>(dst + 4 * (kSwz ? xswz(v) : v)) = u[i];
                    } else {
                        float2 f[4];
                        widen<XK>(u[i], f);
                        const int c0 = kSwz ? xswz(2 * v) : 2 * v, c1 = kSwz ? xswz(2 * v + 1) : 2 * v + 1;
                        *reinterpret_cast<float4*>(dst + 4 * c0) = make_float4(f[0].x, f[0].y, f[1].x, f[1].y);
                        *reinterpret_cast<float4*>(dst + 4 * c1) = make_float4(f[2].x, f[2].y, f[3].x, f[3].y);
                    }
                }
            }
        }
    } else {
#pragma unroll 1
        for (int m = 0; m < M; ++m)
            for (int k = t; k < p.K; k += nt)
                xs[(size_t)m * g.kp + (kSwz ? 4 * xswz(k >> 2) + (k & 3) : k)] = to_f32<XK>(p.x, m * p.ldx + k);
    }
}

template <int WK>
__device__ __forceinline__ void dense_issue(const DenseParams& p, const DenseGeom& g, int tile, int ks, uint8_t* slot,
                                            uint64_t* bar, int lane) {
    constexpr int ES = WK == kF32 ? 4 : 2;
    const int rows = min(kDTR, p.N - tile * kDTR);
    const long long kb = (long long)ks * kDRowBytes;
    const long long left = (long long)p.K * ES - kb;
    const uint32_t bytes = (uint32_t)(left < kDRowBytes ? left : kDRowBytes);
    if (lane == 0) mbar_arrive_expect_tx(bar, bytes * rows);
    __syncwarp();
    if (lane < rows) {
        const uint8_t* src = reinterpret_cast<const uint8_t*>(p.w) +
                             ((long long)tile * kDTR + lane) * p.ldw * ES + kb;
        tma_load_1d(slot + lane * kDRowBytes, src, bytes, bar);
    }
}

template <int WK, int XK, int M, int WARPS>
__global__ void __launch_bounds__(WARPS * 32, 1) gemv_dense_tma(const DenseParams p, const DenseGeom g) {
    constexpr int ES = WK == kF32 ? 4 : 2;
    constexpr int EPV = 16 / ES;                 // elements per 16-byte vector
    constexpr int HALF = kDRowBytes / 2 / ES;    // elements per half row chunk
    constexpr int ITEM = kDTR * kDRowBytes;
    extern __shared__ __align__(128) uint8_t smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem) + warp * g.stages;
    uint64_t* xbar = reinterpret_cast<uint64_t*>(smem) + nwarps * g.stages;   // x copies (FP32 x)
    size_t off = ((size_t)(nwarps * g.stages + 1) * 8 + 127) & ~(size_t)127;
    float* xs = reinterpret_cast<float*>(smem + off);
    off += ((size_t)M * g.kp * 4 + 127) & ~(size_t)127;
    uint8_t* ring = smem + off + (size_t)warp * g.stages * ITEM;

    pdl_launch_dependents();
    const int GW = gridDim.x * nwarps;
    const int gw = warp * gridDim.x + blockIdx.x;
    const int my_tiles = gw < g.ntiles ? (g.ntiles - 1 - gw) / GW + 1 : 0;
    const int nitems = my_tiles * g.ksteps;
    constexpr bool kSwz = WK != kF32;               // x chunk order (xswz) for 16-bit weights
    constexpr bool kXBulk = XK == kF32 && !kSwz;    // FP32 x rows in order go by bulk copies
    if (lane == 0) {
        for (int i = 0; i < g.stages; ++i) mbar_init(&bars[i], 1);
        if (kXBulk && threadIdx.x == 0) mbar_init(xbar, 1);
        fence_mbar_init();
    }
    if (kXBulk) __syncthreads();   // xbar initialised before any thread waits on it
    else __syncwarp();
    int c_tile = gw, c_ks = 0, c_slot = 0, i_tile = gw, i_ks = 0, i_slot = 0;
    uint32_t c_phase = 0;
    int issued = 0;
    for (; issued < min(g.stages, nitems); ++issued) {
        dense_issue<WK>(p, g, i_tile, i_ks, ring + (size_t)i_slot * ITEM, &bars[i_slot], lane);
        if (++i_ks == g.ksteps) { i_ks = 0; i_tile += GW; }
        if (++i_slot == g.stages) i_slot = 0;
    }

    pdl_wait_primary();   // x and C may come from the previous kernel
    if (kXBulk && g.xvec) {
        // One bulk copy per row of x (K·4 bytes, 16-byte aligned on both sides).
        if (threadIdx.x == 0) {
            mbar_arrive_expect_tx(xbar, (uint32_t)M * (uint32_t)p.K * 4u);
            for (int m = 0; m < M; ++m)
                tma_load_1d(xs + (size_t)m * g.kp, reinterpret_cast<const float*>(p.x) + (size_t)m * p.ldx,
                            (uint32_t)p.K * 4u, xbar);
        }
        if (!mbar_wait_bounded(xbar, 0u, p.err)) {
            // x never arrived: drain this warp's weight copies (bounded) and stop.
            for (int k = 0; k < issued; ++k) mbar_wait_bounded(&bars[k], 0u, nullptr);
            return;
        }
    } else {
        stage_x<XK, M, kSwz>(p, g, xs);
        __syncthreads();
    }

    float2 acc[kDTR][M];
#pragma unroll
    for (int r = 0; r < kDTR; ++r)
#pragma unroll
        for (int m = 0; m < M; ++m) acc[r][m] = make_float2(0.0f, 0.0f);

    for (int it = 0; it < nitems; ++it) {
        if (__any_sync(0xffffffffu, !mbar_wait_bounded(&bars[c_slot], c_phase, p.err))) {   // warp-uniform
            for (int k = it + 1; k < issued; ++k) {   // let the copies in flight land, then stop
                const int s2 = (c_slot + (k - it)) % g.stages;
                const uint32_t ph = c_phase ^ (uint32_t)(((c_slot + (k - it)) / g.stages) & 1);
                mbar_wait_bounded(&bars[s2], ph, nullptr);
            }
            return;
        }
        const uint8_t* st = ring + (size_t)c_slot * ITEM;
        const int kb = c_ks * (kDRowBytes / ES);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int e0 = h * HALF + lane * EPV;
            if (kb + e0 < p.K) {   // K·es is a multiple of 16: the whole vector is in range
                float2 wv[kDTR][EPV / 2];
#pragma unroll
                for (int r = 0; r < kDTR; ++r)
                    widen<WK>(*reinterpret_cast<const uint4*>(st + r * kDRowBytes + h * (kDRowBytes / 2) + lane * 16),
                              wv[r]);
#pragma unroll
                for (int m = 0; m < M; ++m) {
                    const float* xr = xs + m * g.kp;
                    const int c0 = (kb + e0) >> 2;   // chunk of the row: kb + e0 is a multiple of 4
                    float2 xv[EPV / 2];
#pragma unroll
                    for (int q = 0; q < EPV / 4; ++q) {
                        const float4 t = *reinterpret_cast<const float4*>(xr + 4 * (kSwz ? xswz(c0 + q) : c0 + q));
                        xv[2 * q] = make_float2(t.x, t.y);
                        xv[2 * q + 1] = make_float2(t.z, t.w);
                    }
                    // j outer, rows inner: consecutive FFMA2s feed different
                    // accumulators (each still adds its terms in j order).
#pragma unroll
                    for (int j = 0; j < EPV / 2; ++j)
#pragma unroll
                        for (int r = 0; r < kDTR; ++r) acc[r][m] = __ffma2_rn(wv[r][j], xv[j], acc[r][m]);
                }
            }
        }
        if (c_ks == g.ksteps - 1) {
            const int r0 = c_tile * kDTR;
#pragma unroll
            for (int r = 0; r < kDTR; ++r)
#pragma unroll
                for (int m = 0; m < M; ++m) {
                    float v = acc[r][m].x + acc[r][m].y;
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                    if (lane == 0 && r0 + r < p.N) {
                        float* c = p.y + (size_t)m * p.ldy + r0 + r;
                        const float cb = p.beta == 0.0f ? 0.0f : (p.beta == 1.0f ? *c : __fmul_rn(p.beta, *c));
                        *c = __fadd_rn(cb, __fmul_rn(p.alpha, v));
                    }
                    acc[r][m] = make_float2(0.0f, 0.0f);
                }
        }
        __syncwarp();
        if (issued < nitems) {
            fence_proxy_async_smem();
            dense_issue<WK>(p, g, i_tile, i_ks, ring + (size_t)i_slot * ITEM, &bars[i_slot], lane);
            if (++i_ks == g.ksteps) { i_ks = 0; i_tile += GW; }
            if (++i_slot == g.stages) i_slot = 0;
            ++issued;
        }
        if (++c_ks == g.ksteps) { c_ks = 0; c_tile += GW; }
        if (++c_slot == g.stages) { c_slot = 0; c_phase ^= 1u; }
    }
}

int smem_optin_of_current_device() {
    static int cached[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
    if (!cached[dev]) {
        int v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess) return 0;
        cached[dev] = v;
    }
    return cached[dev];
}

// The streaming kernel when W's rows and x fit its rules: 16-byte aligned W
// and row stride, K·es a multiple of 16, x as FP32 in shared memory beside a
// ring of at least two stages per warp. Returns cudaErrorNotSupported when
// they do not (the caller then takes the plain kernel).
template <int WK, int XK, int M>
cudaError_t launch_tma(cudaStream_t s, bool pdl, int num_sms, const DenseParams& p) {
    constexpr int ES = WK == kF32 ? 4 : 2;
    if (p.K <= 0 || ((long long)p.K * ES) % 16 != 0 || ((long long)p.ldw * ES) % 16 != 0 ||
        (reinterpret_cast<uintptr_t>(p.w) & 15) != 0)
        return cudaErrorNotSupported;
    DenseGeom g;
    g.ksteps = (int)(((long long)p.K * ES + kDRowBytes - 1) / kDRowBytes);
    g.ntiles = (p.N + kDTR - 1) / kDTR;
    g.kp = (p.K + 7) & ~7;   // an even number of 16-byte chunks per row (xswz stays in the row)
    {
        const int xes = XK == kF32 ? 4 : 2;
        g.xvec = (reinterpret_cast<uintptr_t>(p.x) & 15) == 0 && ((long long)p.ldx * xes) % 16 == 0 &&
                 ((long long)p.K * xes) % 16 == 0;
    }
    const int optin = smem_optin_of_current_device();
    const size_t xbytes = ((size_t)M * g.kp * 4 + 127) & ~(size_t)127;
    // More warps hide the shared-memory and FMA latency of the larger M;
    // 12 warps of the M = 8 kernel still fit the register file.
    constexpr int WARPS = M <= 2 ? kDWarps : 12;
    const size_t per_stage = (size_t)WARPS * kDTR * kDRowBytes;
    const size_t fixed = xbytes + 256 + 1024;   // x, barriers (rounded), slack
    if (optin <= 0 || (size_t)optin < fixed + 2 * per_stage) return cudaErrorNotSupported;
    g.stages = (int)std::min<size_t>(6, ((size_t)optin - fixed) / per_stage);
    const size_t smem = (((size_t)(WARPS * g.stages + 1) * 8 + 127) & ~(size_t)127) + xbytes + g.stages * per_stage;
    auto k = gemv_dense_tma<WK, XK, M, WARPS>;
    int per_sm = 0;
    cudaError_t e = occupancy((const void*)k, WARPS * 32, smem, &per_sm);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorNotSupported;
    const long long want = std::max<long long>(((long long)g.ntiles + WARPS - 1) / WARPS,
                                               std::min<long long>(g.ntiles, num_sms));
    const long long grid = std::max<long long>(1, std::min<long long>(want, num_sms));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(WARPS * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k, p, g);
}

template <int WK, int XK, int M>
cudaError_t launch_m(cudaStream_t s, bool pdl, int num_sms, const DenseParams& p) {
    const cudaError_t t = launch_tma<WK, XK, M>(s, pdl, num_sms, p);
    if (t != cudaErrorNotSupported) return t;
    constexpr int ES = WK == kF32 ? 4 : 2;
    const bool vec = ((reinterpret_cast<uintptr_t>(p.w) & 15) == 0) && (((size_t)p.ldw * ES) % 16 == 0);
    const size_t xbytes = (size_t)M * ((p.K + 3) & ~3) * 4;
    const bool xsm = xbytes <= kXSmemMax;
    void (*k)(DenseParams);
    if (vec) k = xsm ? gemv_dense_kernel<WK, XK, M, true, true> : gemv_dense_kernel<WK, XK, M, true, false>;
    else k = xsm ? gemv_dense_kernel<WK, XK, M, false, true> : gemv_dense_kernel<WK, XK, M, false, false>;
    const size_t smem = xsm ? xbytes : 0;
    int per_sm = 0;
    cudaError_t e = occupancy((const void*)k, kWarps * 32, smem, &per_sm);
    if (e != cudaSuccess) return e;
    const long long groups = ((long long)p.N + kTR - 1) / kTR;
    const long long want = (groups + kWarps - 1) / kWarps;
    const long long grid = std::max<long long>(1, std::min<long long>(want, (long long)std::max(per_sm, 1) * num_sms));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(kWarps * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k, p);
}

template <int WK, int XK>
cudaError_t launch_kinds(cudaStream_t s, bool pdl, int num_sms, const DenseParams& p) {
    switch (p.M) {
#define SMK_CASE(MM) case MM: return launch_m<WK, XK, MM>(s, pdl, num_sms, p);
        SMK_CASE(1) SMK_CASE(2) SMK_CASE(3) SMK_CASE(4) SMK_CASE(5) SMK_CASE(6) SMK_CASE(7) SMK_CASE(8)
#undef SMK_CASE
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace

cudaError_t launch_gemv_dense(cudaStream_t s, bool pdl, int num_sms, int w_kind, int x_kind, const DenseParams& p) {
    if (w_kind == kF32 && x_kind == kF32) return launch_kinds<kF32, kF32>(s, pdl, num_sms, p);
    if (w_kind == kF16 && x_kind == kF16) return launch_kinds<kF16, kF16>(s, pdl, num_sms, p);
    if (w_kind == kF16 && x_kind == kF32) return launch_kinds<kF16, kF32>(s, pdl, num_sms, p);
    if (w_kind == kBF16 && x_kind == kBF16) return launch_kinds<kBF16, kBF16>(s, pdl, num_sms, p);
    if (w_kind == kBF16 && x_kind == kF32) return launch_kinds<kBF16, kF32>(s, pdl, num_sms, p);
    return cudaErrorInvalidValue;
}

}  // namespace smk
