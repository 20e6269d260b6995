// decode.cu — the rest of a Llama decode step on sm_100a, around the GEMVs:
// residual add fused with RMSNorm, RoPE fused with the KV-cache write, and
// grouped-query attention of one token over the cache. The reference runs
// these on the host in NumPy (examples/llama/llama.py: rms_norm :184-188,
// RoPE :131-178 and _rope, _attention :398-412, step :414-439).
//
// All three are small, latency-bound kernels of a chain of ~7 launches per
// layer. Each takes part in programmatic dependent launch like the GEMVs: it
// lets the next kernel launch at entry and reads its inputs only after
// griddepcontrol.wait, so a chain of them costs one grid boundary per kernel
// and no host round trip.

#include "decode.cuh"
#include "smk_device.cuh"

#include <cmath>
#include <cfloat>

namespace smk {

namespace {

template <int kThreads>
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) red[warp] = v;
    __syncthreads();
    v = lane < kThreads / 32 ? red[lane] : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;   // every thread of the CTA
}

// ---- residual add + RMSNorm --------------------------------------------------------
//
// Row r: x += delta (when delta is given; x is the residual stream, updated in
// place), then h = w * (x * inv) with var = fl(Σx² / n) and
// inv = fl(1 / sqrt(var + eps)) formed in double, the reference's rms_norm
// (weight * (x * float32(1 / math.sqrt(float(var) + eps)))); its float32 mean
// is a pairwise NumPy sum, here a shuffle tree, so var agrees to rounding.
// One CTA per row; each thread keeps its values in registers between the passes.
constexpr int kNormThreads = 512;
constexpr int kNormPerThread = 16;   // rows up to 8192 values

__global__ void __launch_bounds__(kNormThreads) add_rmsnorm_kernel(float* __restrict__ x, long long ldx,
                                                                   const float* __restrict__ delta, long long ldd,
                                                                   const float* __restrict__ w, double eps, int n,
                                                                   float* __restrict__ h, long long ldh) {
    __shared__ float red[kNormThreads / 32];
    pdl_launch_dependents();
    pdl_wait_primary();
    float* xr = x + (size_t)blockIdx.x * ldx;
    const float* dr = delta ? delta + (size_t)blockIdx.x * ldd : nullptr;
    float v[kNormPerThread];
    float ss = 0.0f;
#pragma unroll
    for (int u = 0; u < kNormPerThread; ++u) {
        const int i = threadIdx.x + u * kNormThreads;
        v[u] = 0.0f;
        if (i < n) {
            float t = xr[i];
            if (dr) {
                t = __fadd_rn(t, dr[i]);
                xr[i] = t;
            }
            v[u] = t;
            ss = __fadd_rn(ss, __fmul_rn(t, t));
        }
    }
    ss = block_sum<kNormThreads>(ss, red);
    const float var = __fdiv_rn(ss, (float)n);
    const float inv = (float)(1.0 / sqrt((double)var + eps));
    float* hr = h + (size_t)blockIdx.x * ldh;
#pragma unroll
    for (int u = 0; u < kNormPerThread; ++u) {
        const int i = threadIdx.x + u * kNormThreads;
        if (i < n) hr[i] = __fmul_rn(w[i], __fmul_rn(v[u], inv));
    }
}

// ---- RoPE + KV-cache write ---------------------------------------------------------
//
// qkv holds one token's q (nh heads), k and v (nkv heads each) of head_dim hd.
// q and k are rotated by the angles pos·inv_freq[i] (float32 product, as the
// reference's rope_cos_sin): pairs (i, i + hd/2) with cos/sin of angle i (the
// Hugging Face layout, apply_rope: x·cos + rotate_half(x)·sin), or, when
// interleaved, pairs (2i, 2i+1) (the layout of GGUF files, Llama._rope). Each
// output is fl(fl(a·c) ± fl(b·s)) in the reference's order; cos and sin come
// from CUDA's cosf / sinf. q goes to qout [nh][hd]; k and v go to row pos of
// the layer's caches [nkv][cap][hd]. pos comes from *pos_dev when given (a
// graph replayed for every token), else from pos; pos outside [0, cap) writes
// nothing and sets kErrBadLaunch.
// Pair i of one head of hd values at position pos: (a, b) = (src[ia], src[ib])
// rotated by the angle fl(pos·inv_freq[i]) into dst[ia], dst[ib].
__device__ __forceinline__ void rope_pair(const float* src, float* dst, const float* inv_freq, int pos, int i, int hd,
                                          int interleaved) {
    const float ang = __fmul_rn((float)pos, inv_freq[i]);
    const float c = cosf(ang), s = sinf(ang);
    const int ia = interleaved ? 2 * i : i, ib = interleaved ? 2 * i + 1 : i + hd / 2;
    const float a = src[ia], b = src[ib];
    dst[ia] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));   // a·cos − b·sin
    dst[ib] = __fadd_rn(__fmul_rn(b, c), __fmul_rn(a, s));   // b·cos + a·sin
}

__global__ void __launch_bounds__(512) rope_kv_kernel(const float* __restrict__ qkv, const float* __restrict__ inv_freq,
                                                      const int* __restrict__ pos_dev, int pos_imm, int nh, int nkv,
                                                      int hd, int interleaved, float* __restrict__ qout,
                                                      float* __restrict__ kc, float* __restrict__ vc, int cap,
                                                      unsigned* err) {
    pdl_launch_dependents();
    pdl_wait_primary();
    const int pos = pos_dev ? *pos_dev : pos_imm;
    if (pos < 0 || pos >= cap) {
        if (threadIdx.x == 0 && blockIdx.x == 0 && err) atomicOr(err, kErrBadLaunch);
        return;
    }
    const int half = hd / 2;
    const int pairs = (nh + nkv) * half;
    for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < pairs; t += gridDim.x * blockDim.x) {
        const int head = t / half, i = t - head * half;
        float* dst = head < nh ? qout + (size_t)head * hd
                               : kc + ((size_t)(head - nh) * cap + pos) * hd;
        rope_pair(qkv + (size_t)head * hd, dst, inv_freq, pos, i, hd, interleaved);   // q heads, then k heads
    }
    const float* vsrc = qkv + (size_t)(nh + nkv) * hd;
    for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < nkv * hd; t += gridDim.x * blockDim.x) {
        const int head = t / hd, d = t - head * hd;
        vc[((size_t)head * cap + pos) * hd + d] = vsrc[t];
    }
}

// ---- grouped-query attention of one token --------------------------------------------
//
// For KV head g, query heads g·rep .. g·rep+rep−1 (rep = nh / nkv) attend to
// positions 0 .. L−1 of the layer's caches: scores fl(scale·(q·k)) (the
// reference's sgemm with alpha = float32(1/sqrt(hd))), softmax over the
// positions (max subtracted, exp, normalised: the reference's softmax_row), and
// out = P·V, everything in float32 but the order of the sums. A CTA takes one
// KV head and one chunk of kAttnChunk positions: lane p of a warp owns
// position p (a full row of K from L1/L2, q broadcast from shared memory); for
// the product with V, lanes own output dimensions and warps split the
// positions. With more than one chunk per head, each CTA writes its running
// max m, sum l and unnormalised output o to the workspace, and the CTA that
// finishes last for the head (an atomic ticket, reset for the next call)
// combines them: out = Σ_c o_c e^(m_c − M) / Σ_c l_c e^(m_c − M).
constexpr int kAttnThreads = 256;
constexpr int kAttnChunk = 256;
constexpr int kAttnMaxRep = 8;
constexpr int kAttnMaxHd = 128;

struct AttnArgs {
    const float* q;        // [nh][hd] (rotated)
    float* kc;             // [nkv][cap][hd] (this layer)
    float* vc;
    float* out;            // [nh][hd]
    const int* len_dev;    // positions attended: *len_dev (device), else len
    int len, nh, nkv, hd, cap;
    float scale;
    float* ws;             // [nkv][chunks][rep][hd + 2] partials (chunks > 1)
    unsigned* tickets;     // [nkv], zero between calls
    unsigned* err;
    // RoPE fused in (attention_kernel<true>): q is this token's qkv
    // [q (nh) | k (nkv) | v (nkv)] before rotation, the position is *pos_dev
    // (or pos), and the length pos + 1.
    const float* inv_freq;
    const int* pos_dev;
    int pos, interleaved;
};

// kRope: RoPE and the KV-cache write fused in. Every CTA rotates the q heads of
// its KV head into shared memory itself; the CTA whose chunk holds the token's
// position rotates the token's k and writes k and v to that row of the caches
// before it reads them (no other CTA reads that row in this call). The
// rotations are rope_kv_kernel's, so the outputs equal rope_kv followed by
// attention bit for bit.
template <bool kRope>
__global__ void __launch_bounds__(kAttnThreads) attention_kernel(const AttnArgs a) {
    __shared__ __align__(16) float qs[kAttnMaxRep * kAttnMaxHd];
    __shared__ float ps[kAttnMaxRep * kAttnChunk];                      // scores, then exp
    __shared__ float red[kAttnThreads / 32 * kAttnMaxRep];
    __shared__ float accs[kAttnThreads / 32 * kAttnMaxRep * kAttnMaxHd];   // per-warp partial outputs
    __shared__ unsigned last;
    pdl_launch_dependents();
    pdl_wait_primary();
    const int g = blockIdx.x, chunk = blockIdx.y, nchunks = gridDim.y;
    const int rep = a.nh / a.nkv, hd = a.hd;
    int L;
    if constexpr (kRope) {
        const int pos = a.pos_dev ? *a.pos_dev : a.pos;
        if (pos < 0 || pos >= a.cap) {   // only a device-side position can get here
            if (threadIdx.x == 0 && chunk == 0 && a.err) atomicOr(a.err, kErrBadLaunch);
            return;   // every CTA of the launch returns alike: no ticket is taken
        }
        L = pos + 1;
        const int half = hd / 2;
        for (int t = threadIdx.x; t < rep * half; t += kAttnThreads) {
            const int h = t / half, i = t - h * half;
            rope_pair(a.q + (size_t)(g * rep + h) * hd, qs + h * hd, a.inv_freq, pos, i, hd, a.interleaved);
        }
        if (pos / kAttnChunk == chunk) {
            const float* ksrc = a.q + (size_t)(a.nh + g) * hd;
            float* krow = a.kc + ((size_t)g * a.cap + pos) * hd;
            for (int i = threadIdx.x; i < half; i += kAttnThreads)
                rope_pair(ksrc, krow, a.inv_freq, pos, i, hd, a.interleaved);
            const float* vsrc = a.q + (size_t)(a.nh + a.nkv + g) * hd;
            float* vrow = a.vc + ((size_t)g * a.cap + pos) * hd;
            for (int d = threadIdx.x; d < hd; d += kAttnThreads) vrow[d] = vsrc[d];
        }
    } else {
        L = a.len_dev ? *a.len_dev : a.len;
        if (L > a.cap) {   // only a device-side length can get here (the host checks its own)
            if (threadIdx.x == 0 && a.err) atomicOr(a.err, kErrBadLaunch);
            L = a.cap;
        }
        for (int t = threadIdx.x; t < rep * hd; t += kAttnThreads) qs[t] = a.q[(size_t)g * rep * hd + t];
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = kAttnThreads / 32;
    const int p0 = chunk * kAttnChunk, p1 = min(L, p0 + kAttnChunk), np = max(0, p1 - p0);
    __syncthreads();   // q in shared memory; the token's k and v rows written (kRope)
    const float* K = a.kc + (size_t)g * a.cap * hd;
    const float* V = a.vc + (size_t)g * a.cap * hd;
    // Scores: position p0 + j at thread j (kAttnChunk <= threads · passes). The
    // K row is read 8 float4 at a time, all 8 loads in flight before the FMAs.
    for (int j = threadIdx.x; j < np; j += kAttnThreads) {
        const float4* kr = reinterpret_cast<const float4*>(K + (size_t)(p0 + j) * hd);
        float acc[kAttnMaxRep];
#pragma unroll
        for (int h = 0; h < kAttnMaxRep; ++h) acc[h] = 0.0f;
        for (int d0 = 0; d0 < hd / 4; d0 += 8) {   // hd a multiple of 32: whole groups of 8
            float4 kv[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) kv[u] = kr[d0 + u];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
#pragma unroll
                for (int h = 0; h < kAttnMaxRep; ++h) {
                    if (h < rep) {
                        const float4 qv = reinterpret_cast<const float4*>(qs + h * hd)[d0 + u];
                        acc[h] = fmaf(qv.x, kv[u].x, acc[h]);
                        acc[h] = fmaf(qv.y, kv[u].y, acc[h]);
                        acc[h] = fmaf(qv.z, kv[u].z, acc[h]);
                        acc[h] = fmaf(qv.w, kv[u].w, acc[h]);
                    }
                }
            }
        }
#pragma unroll
        for (int h = 0; h < kAttnMaxRep; ++h)
            if (h < rep) ps[h * kAttnChunk + j] = __fmul_rn(a.scale, acc[h]);
    }
    __syncthreads();
    // Per head: max and sum of exp over this chunk.
    float mh[kAttnMaxRep], lh[kAttnMaxRep];
#pragma unroll
    for (int h = 0; h < kAttnMaxRep; ++h) {
        if (h >= rep) break;
        float m = -INFINITY;
        for (int j = threadIdx.x; j < np; j += kAttnThreads) m = fmaxf(m, ps[h * kAttnChunk + j]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (lane == 0) red[warp * kAttnMaxRep + h] = m;
    }
    __syncthreads();
#pragma unroll
    for (int h = 0; h < kAttnMaxRep; ++h) {
        if (h >= rep) break;
        float m = -INFINITY;
        for (int w = 0; w < nwarps; ++w) m = fmaxf(m, red[w * kAttnMaxRep + h]);
        mh[h] = m;
    }
    __syncthreads();
#pragma unroll
    for (int h = 0; h < kAttnMaxRep; ++h) {
        if (h >= rep) break;
        float l = 0.0f;
        for (int j = threadIdx.x; j < np; j += kAttnThreads) {
            const float e = expf(__fsub_rn(ps[h * kAttnChunk + j], mh[h]));
            ps[h * kAttnChunk + j] = e;
            l = __fadd_rn(l, e);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
        if (lane == 0) red[warp * kAttnMaxRep + h] = l;
    }
    __syncthreads();
#pragma unroll
    for (int h = 0; h < kAttnMaxRep; ++h) {
        if (h >= rep) break;
        float l = 0.0f;
        for (int w = 0; w < nwarps; ++w) l += red[w * kAttnMaxRep + h];
        lh[h] = l;
    }
    // o[h][d] = Σ_j e[h][j]·V[p0+j][d]: lanes own dimensions d = lane + 32u,
    // warps take positions j = warp, warp + nwarps, ...; then a sum over warps.
    const int du = hd / 32;   // dimensions per lane (hd a multiple of 32)
    float o[kAttnMaxRep][kAttnMaxHd / 32];
#pragma unroll
    for (int h = 0; h < kAttnMaxRep; ++h)
#pragma unroll
        for (int u = 0; u < kAttnMaxHd / 32; ++u) o[h][u] = 0.0f;
    // Four positions per pass, their V rows loaded together; the FMAs then go
    // in position order, as one position per pass would.
    constexpr int kVPass = 4;
    for (int j0 = warp; j0 < np; j0 += kVPass * nwarps) {
        float vv[kVPass][kAttnMaxHd / 32];
#pragma unroll
        for (int i = 0; i < kVPass; ++i) {
            const int j = j0 + i * nwarps;
            const float* vr = V + (size_t)(p0 + min(j, np - 1)) * hd;
#pragma unroll
            for (int u = 0; u < kAttnMaxHd / 32; ++u) vv[i][u] = u < du ? vr[lane + 32 * u] : 0.0f;
        }
#pragma unroll
        for (int i = 0; i < kVPass; ++i) {
            const int j = j0 + i * nwarps;
            if (j >= np) break;   // warp-uniform
#pragma unroll
            for (int h = 0; h < kAttnMaxRep; ++h) {
                if (h >= rep) break;
                const float e = ps[h * kAttnChunk + j];
#pragma unroll
                for (int u = 0; u < kAttnMaxHd / 32; ++u) o[h][u] = fmaf(e, vv[i][u], o[h][u]);
            }
        }
    }
    // Sum over warps through shared memory.
    float* acc = accs;   // [nwarps][rep][hd]
#pragma unroll
    for (int h = 0; h < kAttnMaxRep; ++h) {
        if (h >= rep) break;
#pragma unroll
        for (int u = 0; u < kAttnMaxHd / 32; ++u)
            if (u < du) acc[((size_t)warp * rep + h) * hd + lane + 32 * u] = o[h][u];
    }
    __syncthreads();
    const size_t gout = (size_t)g * rep * hd;
    for (int t = threadIdx.x; t < rep * hd; t += kAttnThreads) {
        float s = 0.0f;
        for (int w = 0; w < nwarps; ++w) s += acc[(size_t)w * rep * hd + t];
        const int h = t / hd;
        if (nchunks == 1) {
            a.out[gout + t] = np > 0 ? __fdiv_rn(s, lh[h]) : __int_as_float(0x7fc00000);
        } else {
            float* wsr = a.ws + (((size_t)g * nchunks + chunk) * rep + h) * (hd + 2);
            wsr[t - h * hd] = s;
            if (t - h * hd == 0) {
                wsr[hd] = mh[h];
                wsr[hd + 1] = lh[h];
            }
        }
    }
    if (nchunks == 1) return;
    // The last CTA of this KV head combines the chunks.
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last = atomicAdd(&a.tickets[g], 1u) == (unsigned)nchunks - 1;
    __syncthreads();
    if (!last) return;
    __threadfence();
    for (int t = threadIdx.x; t < rep * hd; t += kAttnThreads) {
        const int h = t / hd, d = t - h * hd;
        float M = -INFINITY;
        for (int c = 0; c < nchunks; ++c) {
            const float* wsr = a.ws + (((size_t)g * nchunks + c) * rep + h) * (hd + 2);
            if (__ldcg(wsr + hd + 1) > 0.0f) M = fmaxf(M, __ldcg(wsr + hd));
        }
        float num = 0.0f, den = 0.0f;
        for (int c = 0; c < nchunks; ++c) {
            const float* wsr = a.ws + (((size_t)g * nchunks + c) * rep + h) * (hd + 2);
            const float l = __ldcg(wsr + hd + 1);
            if (!(l > 0.0f)) continue;
            const float f = expf(__fsub_rn(__ldcg(wsr + hd), M));
            num = fmaf(__ldcg(wsr + d), f, num);
            den = fmaf(l, f, den);
        }
        a.out[gout + t] = __fdiv_rn(num, den);
    }
    if (threadIdx.x == 0) a.tickets[g] = 0u;   // for the next call, which the stream orders after this one
}

template <typename Kern, typename... Args>
cudaError_t launch_pdl(Kern kernel, dim3 grid, dim3 block, cudaStream_t s, bool pdl, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

}  // namespace

int add_rmsnorm_max_n() { return kNormThreads * kNormPerThread; }

cudaError_t launch_add_rmsnorm(cudaStream_t s, bool pdl, int M, int n, float* x, long long ldx, const float* delta,
                               long long ldd, const float* w, double eps, float* h, long long ldh) {
    if (M <= 0 || n <= 0) return cudaSuccess;
    return launch_pdl(add_rmsnorm_kernel, dim3(M), dim3(kNormThreads), s, pdl, x, ldx, delta, ldd, w, eps, n, h, ldh);
}

cudaError_t launch_rope_kv(cudaStream_t s, bool pdl, const float* qkv, const float* inv_freq, const int* pos_dev,
                           int pos, int nh, int nkv, int hd, bool interleaved, float* qout, float* kc, float* vc,
                           int cap, unsigned* err) {
    const int pairs = (nh + nkv) * (hd / 2);
    const int grid = std::max(1, std::min(16, (pairs + 511) / 512));
    return launch_pdl(rope_kv_kernel, dim3(grid), dim3(512), s, pdl, qkv, inv_freq, pos_dev, pos, nh, nkv, hd,
                      interleaved ? 1 : 0, qout, kc, vc, cap, err);
}

int attention_chunks(int max_len) { return std::max(1, (max_len + kAttnChunk - 1) / kAttnChunk); }
int attention_max_rep() { return kAttnMaxRep; }
int attention_max_hd() { return kAttnMaxHd; }

cudaError_t launch_attention(cudaStream_t s, bool pdl, const float* q, const float* kc, const float* vc, float* out,
                             const int* len_dev, int len, int max_len, int nh, int nkv, int hd, int cap, float scale,
                             float* ws, unsigned* tickets, unsigned* err) {
    AttnArgs a = {};
    a.q = q; a.kc = const_cast<float*>(kc); a.vc = const_cast<float*>(vc); a.out = out; a.len_dev = len_dev;
    a.len = len; a.nh = nh; a.nkv = nkv; a.hd = hd; a.cap = cap; a.scale = scale;
    a.ws = ws; a.tickets = tickets; a.err = err;
    const int chunks = attention_chunks(max_len);
    return launch_pdl(attention_kernel<false>, dim3(nkv, chunks), dim3(kAttnThreads), s, pdl, a);
}

cudaError_t launch_rope_attention(cudaStream_t s, bool pdl, const float* qkv, const float* inv_freq, const int* pos_dev,
                                  int pos, int max_len, int nh, int nkv, int hd, bool interleaved, float* kc, float* vc,
                                  int cap, float scale, float* out, float* ws, unsigned* tickets, unsigned* err) {
    AttnArgs a = {};
    a.q = qkv; a.kc = kc; a.vc = vc; a.out = out; a.len_dev = nullptr; a.len = 0;
    a.nh = nh; a.nkv = nkv; a.hd = hd; a.cap = cap; a.scale = scale;
    a.ws = ws; a.tickets = tickets; a.err = err;
    a.inv_freq = inv_freq; a.pos_dev = pos_dev; a.pos = pos; a.interleaved = interleaved ? 1 : 0;
    const int chunks = attention_chunks(max_len);
    return launch_pdl(attention_kernel<true>, dim3(nkv, chunks), dim3(kAttnThreads), s, pdl, a);
}

}  // namespace smk
