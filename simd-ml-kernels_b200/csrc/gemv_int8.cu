// gemv_int8.cu — sm_100a INT8 decode GEMV: the reference's sgemm_u8s8 with
// trans_b for M ≤ 8 rows of A (see gemv_int8.cuh).
//
// Bound by reading W once, like the dense and quantized GEMVs. W rows stream
// into per-warp shared-memory rings by 1-D bulk TMA copies (never multicast):
// a warp item is kITR = 4 rows × 1 KB of K, one mbarrier per stage, the first
// stages issued before griddepcontrol.wait so the stream starts while the
// previous kernel finishes. A is staged in shared memory (one bulk copy per
// row when its rows are 16-byte aligned) or, when it is too large, read
// through L1.
//
// Arithmetic: Σ_k (A − zp)·W = Σ_k A·W − zp·Σ_k W, both sums exact integers.
// Lane l takes 16 bytes at l·16 and 512 + l·16 of each 1 KB row chunk;
// dp4a.u32.s32 (unsigned A bytes × signed W bytes) gives Σ A·W and
// dp4a.s32.s32 against 0x01010101 gives Σ W, in int32 per lane (exact: a
// lane adds at most 32·255·128 per item and a tile spans at most
// kIMaxSteps = 1024 items). The warp then combines them in int64 and reduces
// over its lanes. The epilogue is the scalar table's
// (src/kernels/scalar_kernels.cpp:166-167): C = float(double(a_scale) ·
// b_scales[j] · double(sum)), where the first product is exact in double, so
// every output is bitwise the reference's scalar result.

#include "gemv_int8.cuh"
#include "gemv_quant.cuh"
#include "smk_device.cuh"

#include <algorithm>

namespace smk {

namespace {

constexpr int kITR = 4;            // rows of W per warp item
constexpr int kIRowBytes = 1024;   // values of one row per item
constexpr int kIMaxSteps = 1024;   // items per tile that keep the int32 lane sums exact

struct U8S8Geom {
    int ksteps;    // items per tile, ceil(K / kIRowBytes)
    int ntiles;    // ceil(N / kITR)
    int stages;    // ring slots per warp
    int kp;        // shared row stride of A in bytes (K rounded up to 16)
};

// The scalar table's epilogue: (a_scale · b_scale) is exact in double (two
// 24-bit significands), times the exact sum with one double rounding, then
// one rounding to float.
__device__ __forceinline__ float u8s8_out(float a_scale, float b_scale, long long sum) {
    return __double2float_rn(__dmul_rn(__dmul_rn((double)a_scale, (double)b_scale), (double)sum));
}

__device__ __forceinline__ long long warp_sum_ll(long long v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ uint4 ld_nc_v4(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}

__device__ __forceinline__ void u8s8_issue(const U8S8Params& p, int tile, int ks, uint8_t* slot, uint64_t* bar,
                                           int lane) {
    const int rows = min(kITR, p.N - tile * kITR);
    const long long kb = (long long)ks * kIRowBytes;
    const long long left = (long long)p.K - kb;
    const uint32_t bytes = (uint32_t)(left < kIRowBytes ? left : kIRowBytes);
    if (lane == 0) mbar_arrive_expect_tx(bar, bytes * rows);
    __syncwarp();
    if (lane < rows)
        tma_load_1d(slot + lane * kIRowBytes, p.w + ((long long)tile * kITR + lane) * p.ldw + kb, bytes, bar);
}

template <int M, int WARPS, bool kASmem>
__global__ void __launch_bounds__(WARPS * 32, 1) gemv_u8s8_tma(const U8S8Params p, const U8S8Geom g) {
    constexpr int ITEM = kITR * kIRowBytes;
    extern __shared__ __align__(128) uint8_t smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem) + warp * g.stages;
    uint64_t* abar = reinterpret_cast<uint64_t*>(smem) + nwarps * g.stages;   // A copies
    size_t off = ((size_t)(nwarps * g.stages + 1) * 8 + 127) & ~(size_t)127;
    uint8_t* as = smem + off;
    if constexpr (kASmem) off += ((size_t)M * g.kp + 127) & ~(size_t)127;
    uint8_t* ring = smem + off + (size_t)warp * g.stages * ITEM;

    pdl_launch_dependents();
    const int GW = gridDim.x * nwarps;
    const int gw = warp * gridDim.x + blockIdx.x;
    const int my_tiles = gw < g.ntiles ? (g.ntiles - 1 - gw) / GW + 1 : 0;
    const int nitems = my_tiles * g.ksteps;
    const bool abulk = kASmem && ((reinterpret_cast<uintptr_t>(p.a) | (uintptr_t)p.lda) & 15) == 0;
    if (lane == 0) {
        for (int i = 0; i < g.stages; ++i) mbar_init(&bars[i], 1);
        if (abulk && threadIdx.x == 0) mbar_init(abar, 1);
        fence_mbar_init();
    }
    if (abulk) __syncthreads();   // abar initialised before any thread waits on it
    else __syncwarp();
    int c_tile = gw, c_ks = 0, c_slot = 0, i_tile = gw, i_ks = 0, i_slot = 0;
    uint32_t c_phase = 0;
    int issued = 0;
    for (; issued < min(g.stages, nitems); ++issued) {
        u8s8_issue(p, i_tile, i_ks, ring + (size_t)i_slot * ITEM, &bars[i_slot], lane);
        if (++i_ks == g.ksteps) { i_ks = 0; i_tile += GW; }
        if (++i_slot == g.stages) i_slot = 0;
    }

    pdl_wait_primary();   // A may come from the previous kernel
    if constexpr (kASmem) {
        if (abulk) {
            // One bulk copy per row of A (K bytes, K a multiple of 16).
            if (threadIdx.x == 0) {
                mbar_arrive_expect_tx(abar, (uint32_t)M * (uint32_t)p.K);
                for (int m = 0; m < M; ++m)
                    tma_load_1d(as + (size_t)m * g.kp, p.a + (size_t)m * p.lda, (uint32_t)p.K, abar);
            }
            if (!mbar_wait_bounded(abar, 0u, p.err)) {
                // A never arrived: drain this warp's weight copies (bounded) and stop.
                for (int k = 0; k < issued; ++k) mbar_wait_bounded(&bars[k], 0u, nullptr);
                return;
            }
        } else {
            for (long long i = threadIdx.x; i < (long long)M * p.K; i += blockDim.x) {
                const int m = (int)(i / p.K);
                const long long k = i - (long long)m * p.K;
                as[(size_t)m * g.kp + k] = p.a[m * p.lda + k];
            }
            __syncthreads();
        }
    }

    int sab[kITR][M], sb[kITR];
#pragma unroll
    for (int r = 0; r < kITR; ++r) {
        sb[r] = 0;
#pragma unroll
        for (int m = 0; m < M; ++m) sab[r][m] = 0;
    }
    const bool zp = p.zp != 0;   // Σ W is needed only for a nonzero zero point

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
        const int kb = c_ks * kIRowBytes;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int e0 = h * (kIRowBytes / 2) + lane * 16;
            if (kb + e0 < p.K) {   // K is a multiple of 16: the whole vector is in range
                uint4 wv[kITR];
#pragma unroll
                for (int r = 0; r < kITR; ++r) wv[r] = *reinterpret_cast<const uint4*>(st + r * kIRowBytes + e0);
                if (zp) {
                    // Word outer, rows inner: consecutive dp4a feed different sums.
#pragma unroll
                    for (int r = 0; r < kITR; ++r) sb[r] = dp4a_ss(wv[r].x, 0x01010101u, sb[r]);
#pragma unroll
                    for (int r = 0; r < kITR; ++r) sb[r] = dp4a_ss(wv[r].y, 0x01010101u, sb[r]);
#pragma unroll
                    for (int r = 0; r < kITR; ++r) sb[r] = dp4a_ss(wv[r].z, 0x01010101u, sb[r]);
#pragma unroll
                    for (int r = 0; r < kITR; ++r) sb[r] = dp4a_ss(wv[r].w, 0x01010101u, sb[r]);
                }
#pragma unroll
                for (int m = 0; m < M; ++m) {
                    uint4 av;
                    if constexpr (kASmem) av = *reinterpret_cast<const uint4*>(as + (size_t)m * g.kp + kb + e0);
                    else av = ld_nc_v4(p.a + (size_t)m * p.lda + kb + e0);
#pragma unroll
                    for (int r = 0; r < kITR; ++r) sab[r][m] = dp4a_us(av.x, wv[r].x, sab[r][m]);
#pragma unroll
                    for (int r = 0; r < kITR; ++r) sab[r][m] = dp4a_us(av.y, wv[r].y, sab[r][m]);
#pragma unroll
                    for (int r = 0; r < kITR; ++r) sab[r][m] = dp4a_us(av.z, wv[r].z, sab[r][m]);
#pragma unroll
                    for (int r = 0; r < kITR; ++r) sab[r][m] = dp4a_us(av.w, wv[r].w, sab[r][m]);
                }
            }
        }
        if (c_ks == g.ksteps - 1) {
            const int r0 = c_tile * kITR;
#pragma unroll
            for (int r = 0; r < kITR; ++r) {
                const float bscale = lane == 0 && r0 + r < p.N ? p.scales[r0 + r] : 0.0f;
#pragma unroll
                for (int m = 0; m < M; ++m) {
                    const long long v = warp_sum_ll((long long)sab[r][m] - (long long)p.zp * sb[r]);
                    if (lane == 0 && r0 + r < p.N) p.y[(size_t)m * p.ldy + r0 + r] = u8s8_out(p.a_scale, bscale, v);
                    sab[r][m] = 0;
                }
                sb[r] = 0;
            }
        }
        __syncwarp();
        if (issued < nitems) {
            fence_proxy_async_smem();
            u8s8_issue(p, i_tile, i_ks, ring + (size_t)i_slot * ITEM, &bars[i_slot], lane);
            if (++i_ks == g.ksteps) { i_ks = 0; i_tile += GW; }
            if (++i_slot == g.stages) i_slot = 0;
            ++issued;
        }
        if (++c_ks == g.ksteps) { c_ks = 0; c_tile += GW; }
        if (++c_slot == g.stages) { c_slot = 0; c_phase ^= 1u; }
    }
}

// Any K (including 0 and K % 16 != 0), any alignment, any K size: one warp
// per row of W, lanes over K with byte loads, int64 sums. The parity path for
// shapes the streaming kernel does not take.
constexpr int kPlainWarps = 8;

template <int M>
__global__ void __launch_bounds__(kPlainWarps * 32) gemv_u8s8_plain(const U8S8Params p) {
    pdl_launch_dependents();
    pdl_wait_primary();
    const int lane = threadIdx.x & 31;
    const int gwarps = gridDim.x * kPlainWarps;
    for (int row = blockIdx.x * kPlainWarps + (threadIdx.x >> 5); row < p.N; row += gwarps) {
        long long acc[M];
#pragma unroll
        for (int m = 0; m < M; ++m) acc[m] = 0;
        const int8_t* wr = p.w + (size_t)row * p.ldw;
        for (int k = lane; k < p.K; k += 32) {
            const int b = wr[k];
#pragma unroll
            for (int m = 0; m < M; ++m) acc[m] += (long long)(((int)p.a[(size_t)m * p.lda + k] - p.zp) * b);
        }
        const float bscale = p.scales[row];
#pragma unroll
        for (int m = 0; m < M; ++m) {
            const long long v = warp_sum_ll(acc[m]);
            if (lane == 0) p.y[(size_t)m * p.ldy + row] = u8s8_out(p.a_scale, bscale, v);
        }
    }
}

int smem_optin() {
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

template <typename Kern, typename... Args>
cudaError_t launch_ex(Kern k, long long grid, int threads, size_t smem, cudaStream_t s, bool pdl, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)std::max<long long>(grid, 1));
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k, args...);
}

// The streaming kernel when W's rows fit its rules (16-byte aligned base and
// row stride, K a multiple of 16, at most kIMaxSteps items per row) and a ring
// of at least two stages per warp fits beside A (or A is read through L1,
// which needs 16-byte aligned rows of A). cudaErrorNotSupported otherwise.
template <int M, int WARPS>
cudaError_t launch_tma(cudaStream_t s, bool pdl, int num_sms, const U8S8Params& p) {
    if (p.K <= 0 || p.K % 16 != 0 || p.ldw % 16 != 0 || (reinterpret_cast<uintptr_t>(p.w) & 15) != 0)
        return cudaErrorNotSupported;
    U8S8Geom g;
    g.ksteps = (p.K + kIRowBytes - 1) / kIRowBytes;
    if (g.ksteps > kIMaxSteps) return cudaErrorNotSupported;
    g.ntiles = (p.N + kITR - 1) / kITR;
    g.kp = (p.K + 15) & ~15;
    const int optin = smem_optin();
    const size_t per_stage = (size_t)WARPS * kITR * kIRowBytes;
    const size_t bars = ((size_t)(WARPS * 8 + 1) * 8 + 127) & ~(size_t)127;
    const size_t abytes = ((size_t)M * g.kp + 127) & ~(size_t)127;
    const bool a_aligned = ((reinterpret_cast<uintptr_t>(p.a) | (uintptr_t)p.lda) & 15) == 0;
    bool asmem = optin > 0 && (size_t)optin >= bars + abytes + 2 * per_stage;
    if (!asmem && !a_aligned) return cudaErrorNotSupported;
    const size_t fixed = bars + (asmem ? abytes : 0);
    if (optin <= 0 || (size_t)optin < fixed + 2 * per_stage) return cudaErrorNotSupported;
    g.stages = (int)std::min<size_t>(6, ((size_t)optin - fixed) / per_stage);
    const size_t smem = (((size_t)(WARPS * g.stages + 1) * 8 + 127) & ~(size_t)127) + (asmem ? abytes : 0) +
                        g.stages * per_stage;
    auto k = asmem ? gemv_u8s8_tma<M, WARPS, true> : gemv_u8s8_tma<M, WARPS, false>;
    int per_sm = 0;
    cudaError_t e = occupancy((const void*)k, WARPS * 32, smem, &per_sm);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorNotSupported;
    const long long want = std::max<long long>(((long long)g.ntiles + WARPS - 1) / WARPS,
                                               std::min<long long>(g.ntiles, num_sms));
    const long long grid = std::max<long long>(1, std::min<long long>(want, num_sms));
    return launch_ex(k, grid, WARPS * 32, smem, s, pdl, p, g);
}

template <int M>
cudaError_t launch_m(cudaStream_t s, bool pdl, int num_sms, const U8S8Params& p) {
    // 16 warps per CTA: measured on B200 at M = 1, 4, 8 and N = 4096, 14336
    // (K = 4096), it beat 8 and 12 warps at every point (M = 1, N = 14336:
    // 10.4 us against 11.8 and 13.2 us).
    const cudaError_t t = launch_tma<M, 16>(s, pdl, num_sms, p);
    if (t != cudaErrorNotSupported) return t;
    auto k = gemv_u8s8_plain<M>;
    int per_sm = 0;
    cudaError_t e = occupancy((const void*)k, kPlainWarps * 32, 0, &per_sm);
    if (e != cudaSuccess) return e;
    const long long want = ((long long)p.N + kPlainWarps - 1) / kPlainWarps;
    const long long grid = std::min<long long>(want, (long long)std::max(per_sm, 1) * num_sms);
    return launch_ex(k, grid, kPlainWarps * 32, 0, s, pdl, p);
}

}  // namespace

cudaError_t launch_gemv_u8s8(cudaStream_t s, bool pdl, int num_sms, const U8S8Params& p) {
    switch (p.M) {
#define SMK_CASE(MM) case MM: return launch_m<MM>(s, pdl, num_sms, p);
        SMK_CASE(1) SMK_CASE(2) SMK_CASE(3) SMK_CASE(4) SMK_CASE(5) SMK_CASE(6) SMK_CASE(7) SMK_CASE(8)
#undef SMK_CASE
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace smk
