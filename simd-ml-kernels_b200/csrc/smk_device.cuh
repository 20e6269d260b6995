// smk_device.cuh — device-side building blocks shared by the sm_100a kernels:
// mbarriers, 1-D bulk TMA copies (cp.async.bulk, no multicast), programmatic
// dependent launch (griddepcontrol), bounded waits that report through an
// error word instead of hanging, and the integer dot products of the block
// formats.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_fp16.h>

namespace smk {

// Device error codes, OR-ed into the error word the launch gets (read and
// cleared by smk_device_error()).
enum : unsigned {
    kErrWaitTimeout = 1u,   // an mbarrier wait ran past its deadline
    kErrBadLaunch = 2u,     // a kernel saw parameters its launch code should have rejected
    kErrPeerTimeout = 4u,   // a peer GPU's gather signal did not arrive in time
};

// A wait on an mbarrier gives up after this long (ns of %globaltimer): far
// above any legitimate wait (a few µs), short enough to keep a broken launch
// from holding the GPU.
constexpr unsigned long long kWaitLimitNs = 1000ull * 1000ull * 1000ull;

__device__ __forceinline__ unsigned long long globaltimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t)::"memory");
    return t;
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

// Make the barrier initialisations visible to the async proxy (the TMA unit).
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Order this thread's earlier generic-proxy shared-memory accesses before
// later async-proxy (TMA) writes to the same bytes.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Wait for phase `parity` of *bar to complete, for at most kWaitLimitNs.
// Returns false (and sets kErrWaitTimeout in *err) when the deadline passed.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, unsigned* err) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = globaltimer();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255u) == 0 && globaltimer() - t0 > kWaitLimitNs) {
            if (err) atomicOr(err, kErrWaitTimeout);
            return false;
        }
    }
}

// 1-D bulk copy global -> this CTA's shared memory, completion counted on
// *bar in bytes. dst, src 16-byte aligned; bytes a multiple of 16. Never
// multicast.
__device__ __forceinline__ void tma_load_1d(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// 2-D tiled bulk copy of one box of the tensor described by *map (a kernel
// parameter) at element coordinates (x, y) into this CTA's shared memory,
// completion counted on *bar in bytes (the whole box, out-of-range rows
// zero-filled). dst 128-byte aligned; x·element size a multiple of 16.
// Never multicast.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

// System-scope release increment of a (possibly peer GPU's) counter, and the
// matching acquire load: the writer's earlier stores are visible to a reader
// that observes the new value.
__device__ __forceinline__ void red_release_sys_add(unsigned* p, unsigned v) {
    asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// A float and a 32-bit tag as one 64-bit word (value bits low), and the
// system-scope relaxed accesses that move such words between GPUs: each
// 64-bit element is single-copy atomic, so a reader that sees the tag sees
// the value stored with it.
__device__ __forceinline__ unsigned long long tagged_word(float v, unsigned tag) {
    return (unsigned long long)__float_as_uint(v) | ((unsigned long long)tag << 32);
}
__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long a) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(a) : "memory");
}
__device__ __forceinline__ void st_relaxed_sys_v2_u64(unsigned long long* p, unsigned long long a,
                                                      unsigned long long b) {
    asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys_u32(unsigned* p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Two IEEE float32 products / sums in one packed instruction (sm_100), each
// rounded to nearest on its own. A packed product that feeds a packed sum is
// fused into one multiply-add by the code generator, explicit .rn or not, and
// so is a product written as fma(a, b, −0) (both checked on B200), so use them
// only where no sum consumes a product whose rounding matters.
__device__ __forceinline__ unsigned long long pack_f2(float2 v) {
    return (unsigned long long)__float_as_uint(v.x) | ((unsigned long long)__float_as_uint(v.y) << 32);
}
__device__ __forceinline__ float2 unpack_f2(unsigned long long v) {
    return make_float2(__uint_as_float((unsigned)v), __uint_as_float((unsigned)(v >> 32)));
}
__device__ __forceinline__ float2 fmul2_rn(float2 a, float2 b) {
    unsigned long long d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(pack_f2(a)), "l"(pack_f2(b)));
    return unpack_f2(d);
}
__device__ __forceinline__ float2 fadd2_rn(float2 a, float2 b) {
    unsigned long long d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(pack_f2(a)), "l"(pack_f2(b)));
    return unpack_f2(d);
}

// The binary16 in the low / high half of a word, as float (exact).
__device__ __forceinline__ float half_lo_to_float(uint32_t w) {
    float f;
    asm("{ .reg .f16 l, h; mov.b32 {l, h}, %1; cvt.f32.f16 %0, l; }" : "=f"(f) : "r"(w));
    return f;
}
__device__ __forceinline__ float half_hi_to_float(uint32_t w) {
    float f;
    asm("{ .reg .f16 l, h; mov.b32 {l, h}, %1; cvt.f32.f16 %0, h; }" : "=f"(f) : "r"(w));
    return f;
}

// Programmatic dependent launch. Both are no-ops when the kernel was not
// launched with the programmatic-serialization attribute.
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait_primary() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Σ_i a_i·b_i + c over the four bytes of a and b: a unsigned, b signed.
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
// Both signed.
__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

__device__ __forceinline__ float half_bits_to_float(uint32_t h16) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(h16 & 0xffffu)));
}

// binary32 -> binary16 bit pattern, round to nearest even, by integer
// arithmetic: the float is m·2^(e−150) (e its biased exponent, 1 for
// subnormals), the half with exponent Eh >= −14 has ulp 2^(Eh−10), so the
// value is m·2^−s half ulps with s = 140 + Eh − e; ((Eh + 15) << 10) + q − 1024
// is then the pattern for every rounded q (a carry to 2048 moves into the
// exponent, Eh = −14 gives the subnormals), and patterns at or past 0x7c00
// overflow to infinity. NaN -> 0x7e00 with the sign.
__device__ __forceinline__ uint32_t f32_to_f16_bits(float f) {
    const uint32_t u = __float_as_uint(f);
    const uint32_t sign = (u >> 16) & 0x8000u;
    const uint32_t a = u & 0x7fffffffu;
    if (a > 0x7f800000u) return sign | 0x7e00u;
    if (a == 0x7f800000u) return sign | 0x7c00u;
    int e = (int)(a >> 23);
    uint32_t m = a & 0x7fffffu;
    if (e == 0) e = 1; else m |= 0x800000u;
    const int Eh = max(e - 127, -14);
    const int s = 140 + Eh - e;
    uint32_t q = 0;
    if (s <= 31) {
        q = m >> s;
        const uint32_t rem = m & ((1u << s) - 1u), half = 1u << (s - 1);
        if (rem > half || (rem == half && (q & 1u))) ++q;
    }
    const int bits = ((Eh + 15) << 10) + (int)q - 1024;
    return sign | (bits >= 0x7c00 ? 0x7c00u : (uint32_t)bits);
}

// ---- exact arithmetic of the activation quantizer (quantize_x_q8: d = amax/127,
// id = 1/d, q = round-half-away(v·id), each rounded to nearest as IEEE divides,
// reciprocals and roundf do), in fewer dependent steps. Each is checked bit for bit
// against CUDA's __fdiv_rn / __frcp_rn / roundf over its whole domain by
// smk_check_x_arith (a GPU test).

// RN(a / 127) for finite a >= 0: q = RN(a·c), c = RN(1/127); the remainder
// a − 127·q is exact in one FMA, and RN(q + r·c) is the correctly rounded quotient
// (Brisebarre, Muller and Raina, "Accelerating correctly rounded floating-point
// division when the divisor is known in advance", IEEE Trans. Computers 53(8),
// 2004; for this divisor it holds for every finite a >= 0).
__device__ __forceinline__ float div127_rn(float a) {
    constexpr float c = 0x1.020408p-7f;   // RN(1/127)
    const float q = __fmul_rn(a, c);
    return __fmaf_rn(__fmaf_rn(-127.0f, q, a), c, q);
}

// RN(1 / d): the hardware approximation refined by one Newton-Raphson step with
// the residual e = 1 − d·y formed exactly by an FMA, y' = RN(y + e·y) (Markstein,
// "Computation of elementary functions on the IBM RISC System/6000 processor",
// IBM J. Res. Dev. 34(1), 1990). Correctly rounded for 2^-126 <= |d| <= 2^126
// (every such d checked on B200); outside that range (zero, subnormal, huge,
// non-finite) it defers to __frcp_rn.
__device__ __forceinline__ float rcp_rn(float d) {
    const float a = fabsf(d);
    if (!(a >= 0x1p-126f && a <= 0x1p126f)) return __frcp_rn(d);
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(d));
    return __fmaf_rn(__fmaf_rn(-d, y, 1.0f), y, y);
}

// round-half-away-from-zero(t) as an integer for |t| <= 128: t + copysign(c, t)
// with c = 1/2 − 2^-25, truncated. Adding exactly 1/2 would round 1/2 − 2^-25 + 1/2
// up to 1; with c the sum of a value below a half-integer never reaches the next
// integer, and a half-integer or more always does (checked for every |t| <= 128).
__device__ __forceinline__ int round_half_away(float t) {
    return __float2int_rz(__fadd_rn(t, copysignf(0x1.fffffep-2f, t)));
}

// Bits [s, s+32) of the 64-bit value hi:lo.
__device__ __forceinline__ uint32_t funnel(uint32_t lo, uint32_t hi, uint32_t s) {
    return __funnelshift_r(lo, hi, s);
}

__device__ __forceinline__ bool finite_bits(float v) {
    return (__float_as_uint(v) & 0x7f800000u) != 0x7f800000u;
}

// Loads that bypass L1 allocation for streamed weights.
__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

}  // namespace smk
