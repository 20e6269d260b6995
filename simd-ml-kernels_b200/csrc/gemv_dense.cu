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

template <int WK, int XK, int M>
cudaError_t launch_m(cudaStream_t s, bool pdl, int num_sms, const DenseParams& p) {
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
