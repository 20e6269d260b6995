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

#include <cudaTypedefs.h>

#include <algorithm>

namespace smk {

// cuTensorMapEncodeTiled through the runtime (gemv_quant.cu).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();

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

// ---- the tensor-core kernel (several rows of A) -----------------------------------------
//
// With several rows of A the dp4a kernel spends about 40 instructions per
// lane on every 16 bytes of weights (8 rows of Σ A·W plus Σ W), and the
// integer pipe, not HBM, sets the pace. Here one integer MMA
// (mma.sync m16n8k32 .s8.u8, exact int32 sums) takes 16 weight rows × 32
// values against all 8 rows of A at once:
//   * weights: a warp item is 16 rows × 256 bytes of K, two boxes of a 2-D
//     tensor map (16 rows × 128 bytes, 128-byte swizzle: chunk c of row r at
//     chunk c ^ (r & 7)), read with ldmatrix.x4 (conflict-free through the
//     swizzle) straight into the A fragments;
//   * activations: the 8 rows of A (zero past M) in shared memory with rows
//     kpa = round_up(K, 256) + 16 bytes apart (16 bytes of skew per row: the
//     ldmatrix reads of the B fragments are conflict-free);
//   * Σ W for a nonzero zero point: with M < 8 row M of the staged A is all
//     ones, so column M of the MMA result is Σ W; with M = 8 one more MMA
//     against a constant ones fragment;
//   * split K: S parts of a row tile run on the CTA's warps (groups of
//     16 / S tiles) and part 0 adds the integer sums, so the result does not
//     depend on S. The epilogue is the dp4a kernel's (the scalar table's).
// Sums stay exact in int32 while K <= 65536 (|Σ| <= K·255·128 < 2^31).

constexpr int kUMWarps = 16;
constexpr int kUMBox = 128;              // bytes of K per TMA box: the 128-byte swizzle span
constexpr int kUMItemK = 2 * kUMBox;     // bytes of K per warp item
constexpr int kUMItem = 16 * kUMItemK;   // 4 KB per item
constexpr int kUMMaxK = 65536;

struct U8S8MmaGeom {
    int ntiles;    // ceil(N / 16)
    int kitems;    // ceil(K / 256)
    int split;     // S
    int stages;    // ring slots per warp
    int kpa;       // shared row stride of A (bytes)
    int ones;      // Σ W: 0 not needed (zp == 0), 1 row M of A is ones, 2 an extra MMA
};

__host__ __device__ inline size_t um_a_offset(int stages) { return ((size_t)(kUMWarps * stages + 1) * 8 + 127) & ~(size_t)127; }
__host__ __device__ inline size_t um_parts_offset(int stages, int kpa) {
    return um_a_offset(stages) + (((size_t)8 * kpa + 127) & ~(size_t)127);
}
__host__ __device__ inline size_t um_ring_offset(int stages, int kpa) {
    return (um_parts_offset(stages, kpa) + (size_t)kUMWarps * 32 * 24 + 1023) & ~(size_t)1023;
}
__host__ __device__ inline size_t um_smem(int stages, int kpa) {
    return um_ring_offset(stages, kpa) + (size_t)kUMWarps * stages * kUMItem + 1024;   // + alignment slack
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

__device__ __forceinline__ void mma_s8u8(int (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <int M>
__global__ void __launch_bounds__(kUMWarps * 32, 1) gemv_u8s8_mma(const U8S8Params p, const U8S8MmaGeom g,
                                                                const __grid_constant__ CUtensorMap wmap) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int gq = lane >> 2, t = lane & 3;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem) + warp * g.stages;
    uint8_t* as = smem + um_a_offset(g.stages);
    int* parts = reinterpret_cast<int*>(smem + um_parts_offset(g.stages, g.kpa));
    // The ring starts on a 1024-byte boundary (the 128-byte swizzle's period).
    const uint32_t raw_addr = smem_addr(smem);
    const uint32_t ring_addr = (raw_addr + (uint32_t)um_ring_offset(g.stages, g.kpa) + 1023u) & ~1023u;
    uint8_t* ring = smem + (ring_addr - raw_addr) + (size_t)warp * g.stages * kUMItem;
    const uint32_t ring_w = ring_addr + (uint32_t)(warp * g.stages * kUMItem);

    pdl_launch_dependents();
    const int S = g.split, T = kUMWarps / S, part = warp % S, tl = warp / S;
    const int ks_lo = part * g.kitems / S, nks = (part + 1) * g.kitems / S - ks_lo;
    const int ngroups = (g.ntiles + T - 1) / T;
    const int my_groups = (int)blockIdx.x < ngroups ? (ngroups - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    auto tile_of = [&](int r) { return ((int)blockIdx.x + r * (int)gridDim.x) * T + tl; };
    const int valid_groups = my_groups > 0 && tile_of(my_groups - 1) >= g.ntiles ? my_groups - 1 : my_groups;
    const int nitems = valid_groups * nks;
    if (lane == 0) {
        for (int i = 0; i < g.stages; ++i) mbar_init(&bars[i], 1);
        fence_mbar_init();
    }
    __syncthreads();
    int i_r = 0, i_ks = 0, i_slot = 0, issued = 0;
    auto issue_next = [&]() {
        if (lane == 0) {
            uint64_t* bar = &bars[i_slot];
            uint8_t* dst = ring + (size_t)i_slot * kUMItem;
            const int x = (ks_lo + i_ks) * kUMItemK, y = tile_of(i_r) * 16;
            mbar_arrive_expect_tx(bar, (uint32_t)kUMItem);   // whole boxes, zero-filled past K and N
            tma_load_2d(dst, &wmap, x, y, bar);
            tma_load_2d(dst + 16 * kUMBox, &wmap, x + kUMBox, y, bar);
        }
        if (++i_ks == nks) { i_ks = 0; ++i_r; }
        if (++i_slot == g.stages) i_slot = 0;
        ++issued;
    };
    while (issued < min(g.stages, nitems)) issue_next();

    pdl_wait_primary();   // A may come from the previous kernel
    {
        // The 8 rows of A in shared memory: rows < M from A (zero past K),
        // row M all ones when Σ W comes from the MMA (g.ones == 1), others zero.
        const int chunks = g.kpa / 16;
        const bool avec = ((reinterpret_cast<uintptr_t>(p.a) | (uintptr_t)p.lda) & 15) == 0;
        for (int i = threadIdx.x; i < 8 * chunks; i += blockDim.x) {
            const int row = i / chunks, k0 = (i - row * chunks) * 16;
            uint4 v = make_uint4(0u, 0u, 0u, 0u);
            if (row < M) {
                const uint8_t* src = p.a + (size_t)row * p.lda;
                if (avec && k0 + 16 <= p.K) {
                    v = *reinterpret_cast<const uint4*>(src + k0);
                } else {
                    uint32_t w[4] = {0u, 0u, 0u, 0u};
                    for (int b = 0; b < 16 && k0 + b < p.K; ++b) w[b >> 2] |= (uint32_t)src[k0 + b] << (8 * (b & 3));
                    v = make_uint4(w[0], w[1], w[2], w[3]);
                }
            } else if (row == M && g.ones == 1) {
                v = make_uint4(0x01010101u, 0x01010101u, 0x01010101u, 0x01010101u);
            }
            *reinterpret_cast<uint4*>(as + (size_t)row * g.kpa + k0) = v;
        }
        __syncthreads();
    }
    const uint32_t as_addr = smem_addr(as);
    // ldmatrix row addresses of this lane: A fragments (weights) and B (activations).
    const int li = lane >> 3;                          // which 8x8 matrix this lane addresses
    const int wrow = (lane & 7) + 8 * (li & 1);        // weight row of the tile
    const uint32_t b_lane = as_addr + (uint32_t)((lane & 7) * g.kpa + 16 * li);

    int failed = 0;
    int c_slot = 0, consumed = 0;
    uint32_t c_phase = 0;
    for (int r = 0; r < my_groups; ++r) {   // CTA-uniform: every warp meets every barrier
        const int tile = tile_of(r);
        int c[4] = {0, 0, 0, 0}, cs[4] = {0, 0, 0, 0};
        if (r < valid_groups) {
            for (int k = 0; k < nks && !failed; ++k) {
                if (__any_sync(0xffffffffu, !mbar_wait_bounded(&bars[c_slot], c_phase, p.err))) {
                    failed = 1;
                    break;
                }
                const uint32_t st = ring_w + (uint32_t)(c_slot * kUMItem);
                const uint32_t kk = (uint32_t)((ks_lo + k) * kUMItemK);
#pragma unroll
                for (int s2 = 0; s2 < 4; ++s2) {   // two 32-value slices per B load
                    uint32_t b[4];
                    ldmatrix_x4(b, b_lane + kk + 64u * s2);
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int s = 2 * s2 + h, box = s >> 2, sb = s & 3;
                        const int chunk = 2 * sb + (li >> 1);
                        uint32_t a[4];
                        ldmatrix_x4(a, st + (uint32_t)(box * 16 * kUMBox + wrow * kUMBox + ((chunk ^ (wrow & 7)) << 4)));
                        mma_s8u8(c, a, b[2 * h], b[2 * h + 1]);
                        if (g.ones == 2) mma_s8u8(cs, a, 0x01010101u, 0x01010101u);
                    }
                }
                __syncwarp();
                if (issued < nitems) {
                    fence_proxy_async_smem();
                    issue_next();
                }
                ++consumed;
                if (++c_slot == g.stages) { c_slot = 0; c_phase ^= 1u; }
            }
        }
        // Parts of a tile: part 0 adds the others' integer sums.
        int* mine = parts + (warp * 32 + lane) * 6;
        mine[0] = c[0]; mine[1] = c[1]; mine[2] = c[2]; mine[3] = c[3]; mine[4] = cs[0]; mine[5] = cs[2];
        __syncthreads();
        if (part == 0 && r < valid_groups && !failed) {
            for (int q = 1; q < S; ++q) {
                const int* o = parts + ((warp + q) * 32 + lane) * 6;
                c[0] += o[0]; c[1] += o[1]; c[2] += o[2]; c[3] += o[3]; cs[0] += o[4]; cs[2] += o[5];
            }
            long long sb0 = 0, sb1 = 0;   // Σ W of rows gq and gq + 8
            if (g.ones == 1) {
                const int src = gq * 4 + (M >> 1);
                sb0 = __shfl_sync(0xffffffffu, (M & 1) ? c[1] : c[0], src);
                sb1 = __shfl_sync(0xffffffffu, (M & 1) ? c[3] : c[2], src);
            } else if (g.ones == 2) {
                sb0 = cs[0];
                sb1 = cs[2];
            }
#pragma unroll
            for (int rr = 0; rr < 2; ++rr) {
                const int row = tile * 16 + gq + 8 * rr;
                if (row < p.N) {
                    const float bscale = p.scales[row];
                    const long long sbv = rr ? sb1 : sb0;
#pragma unroll
                    for (int j = 0; j < 2; ++j) {
                        const int n = 2 * t + j;
                        if (n < M)
                            p.y[(size_t)n * p.ldy + row] =
                                u8s8_out(p.a_scale, bscale, (long long)c[2 * rr + j] - (long long)p.zp * sbv);
                    }
                }
            }
        }
        __syncthreads();
    }
    if (failed) {
        for (int k = consumed; k < issued; ++k)
            mbar_wait_bounded(&bars[k % g.stages], (uint32_t)((k / g.stages) & 1), nullptr);
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

// The weights as a 2-D tensor of bytes: N rows of K (row stride ldw), boxes
// of 16 rows x 128 bytes with the 128-byte swizzle, zero fill past K and N.
cudaError_t encode_u8s8_map(const U8S8Params& p, CUtensorMap* map) {
    PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
    if (!enc) return cudaErrorNotSupported;
    const cuuint64_t dims[2] = {(cuuint64_t)p.K, (cuuint64_t)p.N};
    const cuuint64_t strides[1] = {(cuuint64_t)p.ldw};
    const cuuint32_t box[2] = {(cuuint32_t)kUMBox, 16u};
    const cuuint32_t estr[2] = {1u, 1u};
    const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t*>(p.w), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorNotSupported;
}

// The tensor-core kernel for kU8S8MmaMinRows..8 rows when W's rows suit a
// tensor map (16-byte aligned base and stride, K a multiple of 16, at most
// kUMMaxK) and A fits in shared memory beside two stages per warp;
// cudaErrorNotSupported otherwise.
template <int M>
cudaError_t launch_mma(cudaStream_t s, bool pdl, int num_sms, const U8S8Params& p) {
    if (p.K <= 0 || p.K % 16 != 0 || p.K > kUMMaxK || p.ldw % 16 != 0 || (reinterpret_cast<uintptr_t>(p.w) & 15) != 0)
        return cudaErrorNotSupported;
    U8S8MmaGeom g;
    g.ntiles = (p.N + 15) / 16;
    g.kitems = (p.K + kUMItemK - 1) / kUMItemK;
    g.kpa = g.kitems * kUMItemK + 16;
    g.ones = p.zp == 0 ? 0 : (M < 8 ? 1 : 2);
    const int optin = smem_optin();
    g.stages = 0;
    for (int st = 4; st >= 2 && !g.stages; --st)
        if (optin > 0 && um_smem(st, g.kpa) <= (size_t)optin) g.stages = st;
    if (!g.stages) return cudaErrorNotSupported;
    CUtensorMap wmap;
    cudaError_t e = encode_u8s8_map(p, &wmap);
    if (e != cudaSuccess) return e;
    const size_t smem = um_smem(g.stages, g.kpa);
    auto k = gemv_u8s8_mma<M>;
    int per_sm = 0;
    e = occupancy((const void*)k, kUMWarps * 32, smem, &per_sm);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorNotSupported;
    // Split K while the tiles' parts fill under 3/4 of the warps, then until
    // the groups of 16 / S tiles cover every CTA slot.
    const long long cap = (long long)num_sms * per_sm, ntiles = g.ntiles;
    g.split = 1;
    while (g.split < kUMWarps && 2 * g.split <= g.kitems && ntiles * g.split * 4 < cap * kUMWarps * 3) g.split *= 2;
    while (g.split < kUMWarps && 2 * g.split <= g.kitems && (ntiles * g.split + kUMWarps - 1) / kUMWarps < cap)
        g.split *= 2;
    const long long T = kUMWarps / g.split;
    const long long grid = std::max<long long>(1, std::min((ntiles + T - 1) / T, cap));
    return launch_ex(k, grid, kUMWarps * 32, smem, s, pdl, p, g, wmap);
}

template <int M>
cudaError_t launch_m(cudaStream_t s, bool pdl, int num_sms, const U8S8Params& p) {
    if constexpr (M >= kU8S8MmaMinRows) {
        const cudaError_t t = launch_mma<M>(s, pdl, num_sms, p);
        if (t != cudaErrorNotSupported) return t;
    }
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
