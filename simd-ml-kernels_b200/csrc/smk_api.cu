// smk_api.cu — the C ABI (include/smk_cuda.h) over the sm_100a kernels:
// argument checks with the reference's rules, kernel selection and launch
// shapes, library-owned scratch and staging buffers, host staging for the
// synchronous *_host entry points, and error reporting.

#include "../../include/smk_cuda.h"
#include "dequant.cuh"
#include "gemv_dense.cuh"
#include "gemv_int8.cuh"
#include "decode.cuh"
#include "gemv_quant.cuh"

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <limits>
#include <map>
#include <unordered_map>
#include <mutex>
#include <string>
#include <vector>

#include <cuda_runtime.h>
#include <functional>

#define SMK_VERSION "0.1.0 (sm_100a)"

namespace {

thread_local std::string g_last_error;

smk_status fail(smk_status st, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return st;
}

smk_status cuda_fail(cudaError_t e, const char* what) {
    return fail(SMK_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

#define SMK_CUDA(call, what)                            \
    do {                                                \
        cudaError_t e_ = (call);                        \
        if (e_ != cudaSuccess) return cuda_fail(e_, what); \
    } while (0)

// Switch to the context's device for the duration of a call.
struct DeviceGuard {
    int prev = -1;
    bool ok = true;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) ok = cudaSetDevice(dev) == cudaSuccess;
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

// A growable device buffer; old allocations are kept until the context dies,
// so kernels still in flight on them stay valid.
struct DevBuf {
    void* ptr = nullptr;
    size_t bytes = 0;
    std::vector<void*> retired;
    cudaError_t reserve(size_t want) {
        if (want <= bytes) return cudaSuccess;
        size_t n = std::max(want, bytes + bytes / 2);
        n = (n + 4095) & ~(size_t)4095;
        void* p = nullptr;
        // Under a stream capture this thread's capture mode is relaxed for the
        // allocation: cudaMalloc is not stream-ordered, and the buffer it
        // replaces stays allocated (retired), so kernels captured earlier keep
        // valid pointers.
        cudaStreamCaptureMode mode = cudaStreamCaptureModeRelaxed;
        cudaThreadExchangeStreamCaptureMode(&mode);
        cudaError_t e = cudaMalloc(&p, n);
        cudaThreadExchangeStreamCaptureMode(&mode);
        if (e != cudaSuccess) return e;
        if (ptr) retired.push_back(ptr);
        ptr = p;
        bytes = n;
        return cudaSuccess;
    }
    void release() {
        for (void* p : retired) cudaFree(p);
        retired.clear();
        if (ptr) cudaFree(ptr);
        ptr = nullptr;
        bytes = 0;
    }
};

bool is_device_ptr(const void* p) {
    if (!p) return false;
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

size_t align256(size_t n) { return (n + 255) & ~(size_t)255; }

// Where a pointer lives: device (or managed) memory, page-locked host memory
// mapped into the device's address space (the device address is returned),
// or ordinary pageable host memory.
enum class Mem { kDevice, kPinned, kPageable };
Mem mem_kind(const void* p, void** dev_addr) {
    *dev_addr = nullptr;
    cudaPointerAttributes a;
    if (!p || cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return Mem::kPageable;
    }
    if (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged) return Mem::kDevice;
    if (a.type == cudaMemoryTypeHost && a.devicePointer) {
        *dev_addr = a.devicePointer;
        return Mem::kPinned;
    }
    return Mem::kPageable;
}

// Page-locked, device-mapped host buffer, grown on demand.
struct PinnedBuf {
    void* ptr = nullptr;
    size_t bytes = 0;
    cudaError_t reserve(size_t want) {
        if (want <= bytes) return cudaSuccess;
        size_t n = std::max(want, bytes * 2);
        n = (n + 4095) & ~(size_t)4095;
        void* p = nullptr;
        cudaError_t e = cudaHostAlloc(&p, n, cudaHostAllocMapped | cudaHostAllocPortable);
        if (e != cudaSuccess) return e;
        if (ptr) cudaFreeHost(ptr);
        ptr = p;
        bytes = n;
        return cudaSuccess;
    }
    void release() {
        if (ptr) cudaFreeHost(ptr);
        ptr = nullptr;
        bytes = 0;
    }
};

// A synchronous host call captured as a CUDA graph: its operands' addresses
// (the effective ones: a page-locked host source or destination, or the
// context's staging buffer for pageable memory), its shape, and how often it
// has been seen.
struct HostKey {
    int fmt, M, N, K;
    const void* xsrc;
    const void* w;
    const void* yout;
    bool operator==(const HostKey& o) const {
        return fmt == o.fmt && M == o.M && N == o.N && K == o.K && xsrc == o.xsrc && w == o.w && yout == o.yout;
    }
};
struct HostKeyHash {
    size_t operator()(const HostKey& k) const {
        size_t h = std::hash<const void*>()(k.xsrc);
        for (size_t v : {std::hash<const void*>()(k.w), std::hash<const void*>()(k.yout), (size_t)k.fmt,
                         (size_t)k.M, (size_t)k.N, (size_t)k.K})
            h = h * 0x9E3779B97F4A7C15ull + v;
        return h;
    }
};
struct HostGraph {
    cudaGraphExec_t exec = nullptr;
    unsigned long long used = 0;   // the context's call count at the last use (LRU)
    int seen = 0;                  // calls with this key; < 0: capture failed, never retried
};

}  // namespace

void smk::set_last_error(const char* msg) { g_last_error = msg; }

struct smk_ctx {
    int device = 0;
    int num_sms = 148;
    size_t smem_optin = 227 * 1024;
    bool pdl = false;
    // Launch shape of the quantized fast kernel; 0 = chosen per call (see plan_q).
    int warps = 0;
    int stages = 0;
    int ctas_per_sm = 0;
    int tile_order = 0;             // 0 automatic, 1 interleaved, 2 contiguous
    unsigned* d_err = nullptr;      // device error word
    unsigned* d_reject = nullptr;   // quantizer rejection flag
    unsigned* d_ticket = nullptr;   // finished-CTA count of a GEMV that copies y to host memory (zero between launches)
    std::mutex mu_scratch;                    // guards scratch and test_buf
    std::map<cudaStream_t, DevBuf> scratch;   // per-stream quantized-x scratch
    DevBuf test_buf;                          // test hooks
    std::map<cudaStream_t, DevBuf> attn_ws;   // per-stream attention partials and tickets
    std::mutex mu_stage;                      // held for a whole *_host call
    DevBuf staging;                           // *_host operands copied to the device (weights)
    PinnedBuf pinned;                         // *_host activations and outputs in pageable memory
    // Synchronous quantized GEMVs repeated with the same operands replay a
    // CUDA graph of their copy and kernel (guarded by mu_stage).
    bool host_graphs = true;
    bool dense_mma = true;   // SMK_OPT_DENSE_MMA: bf16 weights at 4..8 rows on the tensor-core kernel
    int prefetch_delay = 100;   // SMK_OPT_PREFETCH_DELAY: cycles the four-row kernel holds back its weight copies
    cudaStream_t capture_stream = nullptr;   // non-blocking: captures never touch the legacy stream
    std::unordered_map<HostKey, HostGraph, HostKeyHash> graphs;
    unsigned long long host_calls = 0;
    void clear_graphs() {
        for (auto& kv : graphs)
            if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
        graphs.clear();
    }
};

namespace {

smk::LaunchCfg cfg_for(smk_ctx* c, cudaStream_t s) {
    smk::LaunchCfg l;
    l.stream = s;
    l.pdl = c->pdl;
    l.num_sms = c->num_sms;
    l.warps = c->warps > 0 ? c->warps : 16;
    l.ctas_per_sm = c->ctas_per_sm > 0 ? c->ctas_per_sm : 1;
    return l;
}

// The automatic launch shape (measured on B200 in CUDA-graph chains, config-0
// to LM-head sizes): 16 warps per CTA and contiguous per-CTA tile ranges
// throughout; GEMVs of up to ~64 tiles per SM (latency-bound) take one stage
// per warp with up to 2 CTAs per SM, larger ones two stages and one CTA per
// SM (8192x28672: 29.7 µs against 34.1 for 8 warps x 2 stages x 2 CTAs with
// interleaved tiles; 16384x2048: 5.24 against 5.58 µs for one CTA per SM).
void auto_shape(smk_ctx* c, smk::QGemvParams& p, smk::LaunchCfg* l, int* stages) {
    // Work items: tiles, or (four-row layout) tiles times their 2048-value k-steps.
    const long long items = (long long)p.ntiles * (p.r4 ? p.ksteps : 1);
    const bool large = items >= 64LL * c->num_sms;
    if (c->warps <= 0) l->warps = 16;
    if (c->ctas_per_sm <= 0) l->ctas_per_sm = large ? 1 : 2;
    *stages = c->stages > 0 ? c->stages : (large ? 2 : 1);
    p.contiguous = c->tile_order == 1 ? 0 : 1;
    p.issue_delay = c->prefetch_delay;
}

smk_status check_q_args(smk_qformat fmt, int M, int N, int K) {
    if (fmt != SMK_Q4_0 && fmt != SMK_Q8_0) return fail(SMK_ERR_DTYPE, "unknown block format %d", (int)fmt);
    if (M < 0 || N < 0 || K < 0) return fail(SMK_ERR_ARGUMENT, "N and K must be >= 0");
    if (M > smk::kMaxRows) return fail(SMK_ERR_ARGUMENT, "at most %d rows of x per call (got %d)", smk::kMaxRows, M);
    if (K % 32 != 0) return fail(SMK_ERR_ARGUMENT, "K must be a multiple of 32 (got %d)", K);
    return SMK_OK;
}

// The launch shape of the quantized fast kernel for this call.
struct QPlan {
    bool fast;
    bool x_in_smem;
    size_t x_bytes;
    smk::QGemvParams p;
};

QPlan plan_q(smk_ctx* c, smk::LaunchCfg* l, smk_qformat fmt, int M, int N, int K, const float* x, int64_t ldx,
             const uint8_t* Wq, float* y, int64_t ldy, bool want_dump) {
    QPlan q = {};
    smk::QGemvParams& p = q.p;
    p.x = x; p.ldx = ldx; p.w = Wq; p.y = y; p.ldy = ldy;
    p.M = M; p.N = N; p.K = K;
    p.err = c->d_err;
    q.fast = (K % 256 == 0) && ((reinterpret_cast<uintptr_t>(Wq) & 15) == 0);
    smk::plan_tiles(p, q.fast, fmt, !want_dump, c->num_sms);
    q.x_bytes = smk::x_bytes(p);
    if (q.fast) {
        auto_shape(c, p, l, &p.stages);
        // Quantized x in shared memory while it is small; otherwise one
        // quantize kernel writes it to scratch and every CTA reads it there.
        const size_t budget = 64 * 1024;
        q.x_in_smem = q.x_bytes <= budget || want_dump;
        size_t smem = smk::gemv_q_smem(fmt, p, l->warps, p.stages, q.x_in_smem);
        while (smem > c->smem_optin && p.stages > 1) {
            --p.stages;
            smem = smk::gemv_q_smem(fmt, p, l->warps, p.stages, q.x_in_smem);
        }
        if (smem > c->smem_optin) {   // e.g. a dump of a huge M·K: the generic kernel
            q.fast = false;
            smk::plan_tiles(p, false);
            q.x_bytes = smk::x_bytes(p);
        }
    }
    if (!q.fast) q.x_in_smem = false;
    return q;
}

smk_status run_q(smk_ctx* c, smk_qformat fmt, int M, int N, int K, const float* x, int64_t ldx, const uint8_t* Wq,
                 float* y, int64_t ldy, cudaStream_t s, int32_t* dump,
                 const smk::GatherArgs* gather = nullptr, const float* up = nullptr, int64_t ldu = 0,
                 float* yhost = nullptr, bool force_pdl = false, const float* nw = nullptr, double neps = 0.0,
                 const float* res = nullptr, int64_t ldr = 0) {
    // yhost: the device-mapped address of a page-locked output. The fast
    // kernel then writes y (device memory, same ldy) and copies it there at
    // its end; the other kernels write yhost directly.
    if (M == 0 || N == 0) return SMK_OK;
    if (yhost && (gather || dump)) return fail(SMK_ERR_ARGUMENT, "internal: host output with a gather or dump");
    if (K == 0) {
        if (yhost) y = yhost;
        for (int m = 0; m < M; ++m) SMK_CUDA(cudaMemsetAsync(y + (size_t)m * ldy, 0, (size_t)N * 4, s), "cudaMemsetAsync");
        return SMK_OK;
    }
    smk::LaunchCfg l = cfg_for(c, s);
    if (force_pdl) l.pdl = true;   // the previous kernel writes x only (a host call's stage_x_kernel)
    const bool fused = nw || res;   // RMSNorm before / residual add after: the fast kernels only
    if (!fused && M >= smk::kMmaMinRows && !dump && K % 256 == 0 && (reinterpret_cast<uintptr_t>(Wq) & 15) == 0) {
        // Several rows of x: integer tensor-core kernel (bitwise the reference's
        // scalar order), x quantized once into scratch by its own kernel; with
        // a gather, the outputs also go out to the peers from its stores.
        smk::QGemvParams p = {};
        p.gather = gather;
        p.x = x; p.ldx = ldx; p.w = Wq; p.y = yhost ? yhost : y; p.ldy = ldy;
        p.up = up; p.ldu = ldu;
        p.M = M; p.N = N; p.K = K; p.nb = K / 32;
        p.err = c->d_err;
        // x in shared memory when it fits beside at least 2 stages (K up to ~9K).
        bool xs = false;
        for (int st = c->stages > 0 ? c->stages : 4; st >= 2 && !xs; --st)
            if (smk::gemv_q_mma_smem((int)fmt, st, p.nb, true) <= c->smem_optin) {
                xs = true;
                p.stages = st;
            }
        // Otherwise K in P parts across CTAs, each CTA holding its part's slice
        // of x, when a slice fits (B200, 8 rows, 8192x28672: 39.2 us with P = 2 against
        // 73.7 us reading x through L1).
        for (int P = 2; !xs && P <= 16 && P <= p.nb / 8; P *= 2) {
            const int xnb = (p.nb / 8 + P - 1) / P * 8;
            for (int st = c->stages > 0 ? c->stages : 4; st >= 2 && !xs; --st)
                if (smk::gemv_q_mma_smem((int)fmt, st, xnb, true) <= c->smem_optin) {
                    xs = true;
                    p.stages = st;
                    p.kparts = P;
                    p.xnb = xnb;
                }
        }
        if (!xs) {
            p.stages = c->stages > 0 ? c->stages : 4;
            while (p.stages > 1 && smk::gemv_q_mma_smem((int)fmt, p.stages, p.nb, false) > c->smem_optin) --p.stages;
        }
        l.warps = 16;
        l.ctas_per_sm = c->ctas_per_sm > 0 ? c->ctas_per_sm : 1;
        // Scratch: the quantized x, then (K parts) the parts' sums [P][M][N]
        // and the tile ranges' tickets.
        const size_t xqb = align256(smk::xmma_bytes(p.nb));
        const size_t partb = p.kparts > 1 ? align256((size_t)p.kparts * M * N * 4) : 0;
        const size_t tickb = p.kparts > 1 ? (size_t)smk::kMmaMaxTickets * 4 : 0;
        uint8_t* xq;
        {
            std::lock_guard<std::mutex> g(c->mu_scratch);
            DevBuf& b = c->scratch[s];
            SMK_CUDA(b.reserve(xqb + partb + tickb), "cudaMalloc (scratch)");
            xq = static_cast<uint8_t*>(b.ptr);
        }
        if (p.kparts > 1) {
            p.partial = reinterpret_cast<float*>(xq + xqb);
            p.tickets = reinterpret_cast<unsigned*>(xq + xqb + partb);
        }
        SMK_CUDA(smk::launch_quantize_x_mma(l, p, xq), "quantize_x launch");
        p.xq = xq;
        SMK_CUDA(smk::launch_gemv_q_mma(l, (int)fmt, p, xs), "gemv launch");
        return SMK_OK;
    }
    QPlan q = plan_q(c, &l, fmt, M, N, K, x, ldx, Wq, y, ldy, dump != nullptr);
    q.p.dump = dump;
    q.p.gather = gather;
    q.p.up = up;
    q.p.ldu = ldu;
    q.p.nw = nw;
    q.p.neps = neps;
    q.p.res = res;
    q.p.ldr = ldr;
    if (fused && !q.fast) return fail(SMK_ERR_ARGUMENT, "the fused norm / residual needs K %% 256 == 0 and 16-byte aligned Wq");
    if (yhost) {
        if (q.fast) {
            q.p.yhost = yhost;
            q.p.ticket = c->d_ticket;
        } else {
            q.p.y = yhost;
        }
    }
    if (gather && !q.fast) return fail(SMK_ERR_ARGUMENT, "the fused gather needs K %% 256 == 0 and 16-byte aligned Wq");
    // The SwiGLU product costs an exp and a divide per element: formed once by
    // the quantize kernel into global memory rather than by every CTA of the
    // GEMV (measured on the Llama-1B decode stack: 3,100-3,127 against
    // 2,836-2,855 tok/s).
    if (up && q.fast && q.x_in_smem && !dump) q.x_in_smem = false;
    // Long rows of x and few weight rows per SM: one quantize kernel writes x
    // to scratch once, instead of every CTA quantizing all of K (B200,
    // graph-chained: 8192x28672 28.9 against 33.9 us; the Llama-1B stack
    // 3,177 against 3,132 tok/s). 28672x8192 measured 3 % slower that way and
    // K = 2048 (config 0) far slower, so those keep x in shared memory.
    if (!up && !gather && !dump && q.fast && q.x_in_smem && K >= 8192 && N <= 16384) q.x_in_smem = false;
    // The four-row kernel that splits K over warps reads x from global memory.
    if (q.fast && q.x_in_smem && !dump && smk::r4_split(q.p, c->num_sms)) q.x_in_smem = false;
    if (!q.x_in_smem) {
        uint8_t* xq;
        {
            std::lock_guard<std::mutex> g(c->mu_scratch);
            DevBuf& b = c->scratch[s];
            SMK_CUDA(b.reserve(q.x_bytes), "cudaMalloc (scratch)");
            xq = static_cast<uint8_t*>(b.ptr);
        }
        SMK_CUDA(smk::launch_quantize_x(l, q.p, xq), "quantize_x launch");
        q.p.xq = xq;
    }
    SMK_CUDA(smk::launch_gemv_q(l, fmt, q.p, q.fast, nullptr), "gemv launch");
    return SMK_OK;
}

}  // namespace

extern "C" {

const char* smk_version(void) { return SMK_VERSION; }
const char* smk_last_error(void) { return g_last_error.c_str(); }

smk_status smk_ctx_create(int device, smk_ctx** out) {
    if (!out) return fail(SMK_ERR_ARGUMENT, "out must not be NULL");
    *out = nullptr;
    int n = 0;
    SMK_CUDA(cudaGetDeviceCount(&n), "cudaGetDeviceCount");
    if (device < 0 || device >= n) return fail(SMK_ERR_ARGUMENT, "device %d out of range (%d devices)", device, n);
    DeviceGuard g(device);
    if (!g.ok) return fail(SMK_ERR_CUDA, "cudaSetDevice(%d) failed", device);
    cudaDeviceProp prop;
    SMK_CUDA(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
    if (prop.major < 10)
        return fail(SMK_ERR_CUDA, "device %d (%s, sm_%d%d) is not a Blackwell sm_100 GPU", device, prop.name,
                    prop.major, prop.minor);
    smk_ctx* c = new smk_ctx();
    c->device = device;
    c->num_sms = prop.multiProcessorCount;
    c->smem_optin = prop.sharedMemPerBlockOptin;
    cudaError_t e = cudaMalloc(&c->d_err, 4 * sizeof(unsigned));
    if (e != cudaSuccess) {
        delete c;
        return cuda_fail(e, "cudaMalloc (error word)");
    }
    c->d_reject = c->d_err + 1;
    c->d_ticket = c->d_err + 2;
    e = cudaMemset(c->d_err, 0, 4 * sizeof(unsigned));
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&c->capture_stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
        cudaFree(c->d_err);
        delete c;
        return cuda_fail(e, "context set-up");
    }
    *out = c;
    return SMK_OK;
}

smk_status smk_ctx_destroy(smk_ctx* c) {
    if (!c) return SMK_OK;
    DeviceGuard g(c->device);
    cudaDeviceSynchronize();
    c->clear_graphs();
    if (c->capture_stream) cudaStreamDestroy(c->capture_stream);
    for (auto& kv : c->scratch) kv.second.release();
    for (auto& kv : c->attn_ws) kv.second.release();
    c->staging.release();
    c->pinned.release();
    c->test_buf.release();
    cudaFree(c->d_err);
    delete c;
    return SMK_OK;
}

smk_status smk_ctx_set(smk_ctx* c, int option, long long v) {
    if (!c) return fail(SMK_ERR_ARGUMENT, "ctx must not be NULL");
    {
        // Captured host calls hold the launch settings of their capture.
        std::lock_guard<std::mutex> lock(c->mu_stage);
        c->clear_graphs();
    }
    switch (option) {
        case SMK_OPT_HOST_GRAPHS: c->host_graphs = v != 0; return SMK_OK;
        case SMK_OPT_DENSE_MMA: c->dense_mma = v != 0; return SMK_OK;
        case SMK_OPT_PREFETCH_DELAY:
            if (v < 0 || v > 100000) return fail(SMK_ERR_ARGUMENT, "prefetch delay must be in 0..100000 cycles");
            c->prefetch_delay = (int)v;
            return SMK_OK;
        case SMK_OPT_PDL: c->pdl = v != 0; return SMK_OK;
        case SMK_OPT_WARPS:
            if (v < 0 || v > 16) return fail(SMK_ERR_ARGUMENT, "warps must be in 0..16 (0: automatic)");
            c->warps = (int)v;
            return SMK_OK;
        case SMK_OPT_STAGES:
            if (v < 0 || v > 8) return fail(SMK_ERR_ARGUMENT, "stages must be in 0..8 (0: automatic)");
            c->stages = (int)v;
            return SMK_OK;
        case SMK_OPT_CTAS_PER_SM:
            if (v < 0 || v > 8) return fail(SMK_ERR_ARGUMENT, "CTAs per SM must be in 0..8 (0: automatic)");
            c->ctas_per_sm = (int)v;
            return SMK_OK;
        case SMK_OPT_TILE_ORDER:
            if (v < 0 || v > 2) return fail(SMK_ERR_ARGUMENT, "tile order must be 0, 1 or 2");
            c->tile_order = (int)v;
            return SMK_OK;
        default: return fail(SMK_ERR_ARGUMENT, "unknown option %d", option);
    }
}

smk_status smk_ctx_get(smk_ctx* c, int option, long long* v) {
    if (!c || !v) return fail(SMK_ERR_ARGUMENT, "ctx and value must not be NULL");
    switch (option) {
        case SMK_OPT_PDL: *v = c->pdl; return SMK_OK;
        case SMK_OPT_WARPS: *v = c->warps; return SMK_OK;
        case SMK_OPT_STAGES: *v = c->stages; return SMK_OK;
        case SMK_OPT_CTAS_PER_SM: *v = c->ctas_per_sm; return SMK_OK;
        case SMK_OPT_TILE_ORDER: *v = c->tile_order; return SMK_OK;
        case SMK_OPT_HOST_GRAPHS: *v = c->host_graphs; return SMK_OK;
        case SMK_OPT_DENSE_MMA: *v = c->dense_mma; return SMK_OK;
        case SMK_OPT_PREFETCH_DELAY: *v = c->prefetch_delay; return SMK_OK;
        default: return fail(SMK_ERR_ARGUMENT, "unknown option %d", option);
    }
}

smk_status smk_host_alloc(size_t bytes, void** out) {
    if (!out) return fail(SMK_ERR_ARGUMENT, "out must not be NULL");
    *out = nullptr;
    if (bytes == 0) return SMK_OK;
    SMK_CUDA(cudaHostAlloc(out, bytes, cudaHostAllocMapped | cudaHostAllocPortable), "cudaHostAlloc");
    return SMK_OK;
}

smk_status smk_host_free(void* ptr) {
    if (ptr) SMK_CUDA(cudaFreeHost(ptr), "cudaFreeHost");
    return SMK_OK;
}

smk_status smk_pointer_device(const void* ptr, int* device) {
    if (!device) return fail(SMK_ERR_ARGUMENT, "device must not be NULL");
    *device = -1;
    if (!ptr) return SMK_OK;
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, ptr) != cudaSuccess) {
        cudaGetLastError();
        return SMK_OK;
    }
    if (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged) *device = a.device;
    return SMK_OK;
}

smk_status smk_device_error(smk_ctx* c, unsigned* code, void* stream) {
    if (!c || !code) return fail(SMK_ERR_ARGUMENT, "ctx and code must not be NULL");
    DeviceGuard g(c->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    unsigned h = 0;
    SMK_CUDA(cudaMemcpyAsync(&h, c->d_err, sizeof h, cudaMemcpyDeviceToHost, s), "cudaMemcpyAsync");
    SMK_CUDA(cudaMemsetAsync(c->d_err, 0, sizeof h, s), "cudaMemsetAsync");
    SMK_CUDA(cudaStreamSynchronize(s), "cudaStreamSynchronize");
    *code = h;
    return SMK_OK;
}

smk_status smk_gemv_q(smk_ctx* c, smk_qformat fmt, int M, int N, int K, const float* x, int64_t ldx,
                      const uint8_t* Wq, float* y, int64_t ldy, void* stream) {
    if (!c) return fail(SMK_ERR_ARGUMENT, "ctx must not be NULL");
    smk_status st = check_q_args(fmt, M, N, K);
    if (st != SMK_OK) return st;
    if (M == 0 || N == 0) return SMK_OK;
    if (!y || (K > 0 && (!x || !Wq))) return fail(SMK_ERR_ARGUMENT, "x, Wq and y must not be NULL");
    if (ldy < N || (K > 0 && ldx < K)) return fail(SMK_ERR_ARGUMENT, "ldx >= K and ldy >= N required");
    DeviceGuard g(c->device);
    if (!g.ok) return fail(SMK_ERR_CUDA, "cudaSetDevice(%d) failed", c->device);
    return run_q(c, fmt, M, N, K, x, ldx, Wq, y, ldy, static_cast<cudaStream_t>(stream), nullptr);
}

}  // extern "C"

struct smk_gather {
    smk_ctx* c = nullptr;
    int world = 0, rank = 0, npad = 0, m_max = 0;
    void* base = nullptr;                      // this rank's buffer: full-y areas, receive areas, staging, control
    size_t area_bytes = 0;                     // one full-y area (floats); a receive area is twice that
    size_t staging_bytes = 0;                  // the GEMV's own output [m_max][npad], before it is sent
    void* peer[smk::kMaxRanks] = {};           // mapped peer buffers (peer[rank] = base)
    smk::GatherArgs host = {};
    smk::GatherArgs* dev = nullptr;            // the same, in device memory (kernel argument)
    unsigned long long steps = 0;              // calls so far: which area the next one writes
    unsigned pings = 0;                        // ping-pong values used so far
    bool connected = false;
};

namespace {
constexpr size_t kGatherCtrlBytes = 256;
}

extern "C" {

smk_status smk_gather_create(smk_ctx* c, int world, int rank, int npad, int m_max, smk_gather** out,
                             void* ipc_handle) {
    if (!c || !out || !ipc_handle) return fail(SMK_ERR_ARGUMENT, "ctx, out and ipc_handle must not be NULL");
    *out = nullptr;
    if (world < 1 || world > smk::kMaxRanks || rank < 0 || rank >= world)
        return fail(SMK_ERR_ARGUMENT, "need 1 <= world <= %d and 0 <= rank < world", smk::kMaxRanks);
    if (npad < 1 || m_max < 1 || m_max > smk::kMaxRows) return fail(SMK_ERR_ARGUMENT, "need npad >= 1, 1 <= m_max <= 8");
    static_assert(sizeof(cudaIpcMemHandle_t) == SMK_IPC_HANDLE_BYTES, "IPC handle size");
    DeviceGuard dg(c->device);
    if (!dg.ok) return fail(SMK_ERR_CUDA, "cudaSetDevice(%d) failed", c->device);
    auto* g = new smk_gather();
    g->c = c;
    g->world = world;
    g->rank = rank;
    g->npad = npad;
    g->m_max = m_max;
    if ((size_t)m_max * world * npad > (size_t)INT32_MAX / 2)
        return fail(SMK_ERR_ARGUMENT, "m_max * world * npad too large");
    g->area_bytes = align256((size_t)m_max * world * npad * sizeof(float));
    g->staging_bytes = align256((size_t)m_max * npad * sizeof(float));
    const size_t bytes = 6 * g->area_bytes + g->staging_bytes + kGatherCtrlBytes;
    cudaError_t e = cudaMalloc(&g->base, bytes);
    if (e == cudaSuccess) e = cudaMemset(g->base, 0, bytes);
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(ipc_handle), g->base);
    if (e != cudaSuccess) {
        if (g->base) cudaFree(g->base);
        delete g;
        return cuda_fail(e, "gather buffer");
    }
    *out = g;
    return SMK_OK;
}

smk_status smk_gather_connect(smk_gather* g, const void* ipc_handles) {
    if (!g || !ipc_handles) return fail(SMK_ERR_ARGUMENT, "gather and ipc_handles must not be NULL");
    if (g->connected) return fail(SMK_ERR_ARGUMENT, "gather already connected");
    DeviceGuard dg(g->c->device);
    if (!dg.ok) return fail(SMK_ERR_CUDA, "cudaSetDevice(%d) failed", g->c->device);
    const auto* hs = static_cast<const cudaIpcMemHandle_t*>(ipc_handles);
    for (int r = 0; r < g->world; ++r) {
        if (r == g->rank) {
            g->peer[r] = g->base;
            continue;
        }
        void* p = nullptr;
        const cudaError_t e = cudaIpcOpenMemHandle(&p, hs[r], cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            for (int q = 0; q < r; ++q)
                if (q != g->rank && g->peer[q]) cudaIpcCloseMemHandle(g->peer[q]);
            return cuda_fail(e, "cudaIpcOpenMemHandle (peer gather buffer)");
        }
        g->peer[r] = p;
    }
    smk::GatherArgs& a = g->host;
    a.y = static_cast<float*>(g->base);
    for (int r = 0; r < g->world; ++r) {
        char* b = static_cast<char*>(g->peer[r]);
        a.ll[r] = reinterpret_cast<unsigned long long*>(b + 2 * g->area_bytes);
        a.ctrl[r] = reinterpret_cast<unsigned*>(b + 6 * g->area_bytes + g->staging_bytes);
    }
    a.area = (long long)(g->area_bytes / sizeof(float));
    a.world = g->world;
    a.rank = g->rank;
    a.npad = g->npad;
    SMK_CUDA(cudaMalloc(&g->dev, sizeof(smk::GatherArgs)), "cudaMalloc (gather args)");
    SMK_CUDA(cudaMemcpy(g->dev, &a, sizeof a, cudaMemcpyHostToDevice), "cudaMemcpy (gather args)");
    g->connected = true;
    return SMK_OK;
}

smk_status smk_gather_destroy(smk_gather* g) {
    if (!g) return SMK_OK;
    DeviceGuard dg(g->c->device);
    cudaDeviceSynchronize();
    for (int r = 0; r < g->world; ++r)
        if (r != g->rank && g->peer[r]) cudaIpcCloseMemHandle(g->peer[r]);
    if (g->dev) cudaFree(g->dev);
    if (g->base) cudaFree(g->base);
    delete g;
    return SMK_OK;
}

smk_status smk_gemv_q_gather(smk_ctx* c, smk_gather* g, smk_qformat fmt, int M, int N_local, int K, const float* x,
                             int64_t ldx, const uint8_t* Wq, float** y_full, void* stream) {
    if (!c || !g || !y_full) return fail(SMK_ERR_ARGUMENT, "ctx, gather and y_full must not be NULL");
    if (!g->connected) return fail(SMK_ERR_ARGUMENT, "gather not connected");
    smk_status st = check_q_args(fmt, M, N_local, K);
    if (st != SMK_OK) return st;
    if (M < 1 || M > g->m_max || N_local < 1 || N_local > g->npad || K < 256)
        return fail(SMK_ERR_ARGUMENT, "need 1 <= M <= m_max, 1 <= N_local <= npad and K >= 256");
    if (!x || !Wq || ldx < K) return fail(SMK_ERR_ARGUMENT, "x and Wq must not be NULL; ldx >= K");
    DeviceGuard dg(c->device);
    if (!dg.ok) return fail(SMK_ERR_CUDA, "cudaSetDevice(%d) failed", c->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    float* staging = reinterpret_cast<float*>(static_cast<char*>(g->base) + 6 * g->area_bytes);
    st = run_q(c, fmt, M, N_local, K, x, ldx, Wq, staging, g->npad, s, nullptr, g->dev);
    if (st != SMK_OK) return st;
    smk::LaunchCfg l = cfg_for(c, s);
    // Enough CTAs that each thread polls about eight peer entries, at most one per SM.
    const long long entries = (long long)M * (g->world - 1) * g->npad;
    const int blocks = (int)std::max(1LL, std::min<long long>(c->num_sms, (entries + 8 * smk::kGatherWaitThreads - 1) /
                                                                            (8 * smk::kGatherWaitThreads)));
    SMK_CUDA(smk::launch_gather_wait(l, g->dev, M, blocks, c->d_err), "gather wait launch");
    *y_full = reinterpret_cast<float*>(static_cast<char*>(g->base) + (g->steps & 1) * g->area_bytes);
    ++g->steps;
    return SMK_OK;
}

smk_status smk_gather_barrier(smk_gather* g, void* stream) {
    if (!g) return fail(SMK_ERR_ARGUMENT, "gather must not be NULL");
    if (!g->connected) return fail(SMK_ERR_ARGUMENT, "gather not connected");
    DeviceGuard dg(g->c->device);
    if (!dg.ok) return fail(SMK_ERR_CUDA, "cudaSetDevice(%d) failed", g->c->device);
    SMK_CUDA(smk::launch_gather_barrier(cfg_for(g->c, static_cast<cudaStream_t>(stream)), g->dev, g->c->d_err),
             "gather barrier launch");
    ++g->steps;
    return SMK_OK;
}

smk_status smk_gather_pingpong(smk_gather* g, int iters, int relaxed, unsigned long long* ns, void* stream) {
    if (!g || !ns) return fail(SMK_ERR_ARGUMENT, "gather and ns must not be NULL");
    if (!g->connected) return fail(SMK_ERR_ARGUMENT, "gather not connected");
    if (iters < 1 || iters > (1 << 20)) return fail(SMK_ERR_ARGUMENT, "iters must be in 1..2^20");
    DeviceGuard dg(g->c->device);
    if (!dg.ok) return fail(SMK_ERR_CUDA, "cudaSetDevice(%d) failed", g->c->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    unsigned long long* d_ns = nullptr;
    {
        std::lock_guard<std::mutex> lock(g->c->mu_scratch);
        SMK_CUDA(g->c->test_buf.reserve(sizeof(unsigned long long)), "cudaMalloc (test)");
        d_ns = static_cast<unsigned long long*>(g->c->test_buf.ptr);
        SMK_CUDA(cudaMemsetAsync(d_ns, 0, sizeof *d_ns, s), "cudaMemsetAsync");
        SMK_CUDA(smk::launch_gather_pingpong(s, g->dev, g->pings, iters, relaxed != 0, g->c->d_err, d_ns), "ping-pong launch");
        SMK_CUDA(cudaMemcpyAsync(ns, d_ns, sizeof *ns, cudaMemcpyDeviceToHost, s), "cudaMemcpyAsync");
        SMK_CUDA(cudaStreamSynchronize(s), "cudaStreamSynchronize");
    }
    g->pings += (unsigned)iters;
    return SMK_OK;
}

smk_status smk_gemv_q_silu_mul(smk_ctx* c, smk_qformat fmt, int M, int N, int K, const float* gate, int64_t ldg,
                               const float* up, int64_t ldu, const uint8_t* Wq, float* y, int64_t ldy, void* stream) {
    if (!c) return fail(SMK_ERR_ARGUMENT, "ctx must not be NULL");
    smk_status st = check_q_args(fmt, M, N, K);
    if (st != SMK_OK) return st;
    if (M == 0 || N == 0) return SMK_OK;
    if (!y || (K > 0 && (!gate || !up || !Wq))) return fail(SMK_ERR_ARGUMENT, "gate, up, Wq and y must not be NULL");
    if (ldy < N || (K > 0 && (ldg < K || ldu < K))) return fail(SMK_ERR_ARGUMENT, "ldg, ldu >= K and ldy >= N required");
    DeviceGuard g(c->device);
    if (!g.ok) return fail(SMK_ERR_CUDA, "cudaSetDevice(%d) failed", c->device);
    return run_q(c, fmt, M, N, K, gate, ldg, Wq, y, ldy, static_cast<cudaStream_t>(stream), nullptr, nullptr, up, ldu);
}

smk_status smk_gemv_q_fused(smk_ctx* c, smk_qformat fmt, int M, int N, int K, const float* x, int64_t ldx,
                            const float* up, int64_t ldu, const float* w_norm, double eps, const uint8_t* Wq,
                            const float* r, int64_t ldr, float* y, int64_t ldy, void* stream) {
    if (!c) return fail(SMK_ERR_ARGUMENT, "ctx must not be NULL");
    smk_status st = check_q_args(fmt, M, N, K);
    if (st != SMK_OK) return st;
    if (M == 0 || N == 0) return SMK_OK;
    if (up && w_norm) return fail(SMK_ERR_ARGUMENT, "the SwiGLU input and the RMSNorm cannot be fused together");
    if (K == 0) return fail(SMK_ERR_ARGUMENT, "the fused forms need K > 0");
    if (!y || !x || !Wq) return fail(SMK_ERR_ARGUMENT, "x, Wq and y must not be NULL");
    if (ldy < N || ldx < K || (up && ldu < K) || (r && ldr < N))
        return fail(SMK_ERR_ARGUMENT, "ldx, ldu >= K and ldy, ldr >= N required");
    if (w_norm && !(eps >= 0.0)) return fail(SMK_ERR_ARGUMENT, "eps must be >= 0");
    if (r && r != y) {
        // In place (r == y) each value is read and written by one lane; other
        // overlaps would race.
        const char *rb = reinterpret_cast<const char*>(r), *re = rb + ((size_t)(M - 1) * ldr + N) * 4;
        const char *yb = reinterpret_cast<const char*>(y), *ye = yb + ((size_t)(M - 1) * ldy + N) * 4;
        if (rb < ye && yb < re) return fail(SMK_ERR_ARGUMENT, "r must be y itself or not overlap it");
    }
    DeviceGuard g(c->device);
    if (!g.ok) return fail(SMK_ERR_CUDA, "cudaSetDevice(%d) failed", c->device);
    return run_q(c, fmt, M, N, K, x, ldx, Wq, y, ldy, static_cast<cudaStream_t>(stream), nullptr, nullptr, up, ldu,
                 nullptr, false, w_norm, eps, r, ldr);
}

smk_status smk_silu_mul(smk_ctx* c, int64_t n, const float* gate, const float* up, float* out, void* stream) {
    if (!c) return fail(SMK_ERR_ARGUMENT, "ctx must not be NULL");
    if (n < 0) return fail(SMK_ERR_ARGUMENT, "n must be >= 0");
    if (n == 0) return SMK_OK;
    if (!gate || !up || !out) return fail(SMK_ERR_ARGUMENT, "gate, up and out must not be NULL");
    DeviceGuard g(c->device);
    if (!g.ok) return fail(SMK_ERR_CUDA, "cudaSetDevice(%d) failed", c->device);
    SMK_CUDA(smk::launch_silu_mul(static_cast<cudaStream_t>(stream), n, gate, up, out), "silu_mul launch");
    return SMK_OK;
}

smk_status smk_add_rmsnorm(smk_ctx* c, int M, int n, float* x, int64_t ldx, const float* delta, int64_t ldd,
                           const float* w, double eps, float* h, int64_t ldh, void* stream) {
    if (!c) return fail(SMK_ERR_ARGUMENT, "ctx must not be NULL");
    if (M < 0 || n < 0) return fail(SMK_ERR_ARGUMENT, "M and n must be >= 0");
    if (n > smk::add_rmsnorm_max_n())
        return fail(SMK_ERR_ARGUMENT, "rows of at most %d values (got %d)", smk::add_rmsnorm_max_n(), n);
    if (M == 0 || n == 0) return SMK_OK;
    if (!x || !w || !h) return fail(SMK_ERR_ARGUMENT, "x, w and h must not be NULL");
    if (ldx < n || ldh < n || (delta && ldd < n)) return fail(SMK_ERR_ARGUMENT, "row strides must be >= n");
    if (!(eps >= 0.0)) return fail(SMK_ERR_ARGUMENT, "eps must be >= 0");
    DeviceGuard g(c->device);
    if (!g.ok) return fail(SMK_ERR_CUDA, "cudaSetDevice(%d) failed", c->device);
    SMK_CUDA(smk::launch_add_rmsnorm(static_cast<cudaStream_t>(stream), c->pdl, M, n, x, ldx, delta, ldd, w, eps, h,
                                     ldh),
             "add_rmsnorm launch");
    return SMK_OK;
}

smk_status smk_rope_kv(smk_ctx* c, const float* qkv, const float* inv_freq, const int32_t* pos_dev, int pos, int nh,
                       int nkv, int hd, int interleaved, float* q_out, float* k_cache, float* v_cache, int capacity,
                       void* stream) {
    if (!c) return fail(SMK_ERR_ARGUMENT, "ctx must not be NULL");
    if (nh <= 0 || nkv <= 0 || nh % nkv != 0) return fail(SMK_ERR_ARGUMENT, "heads must be positive, nh a multiple of nkv");
    if (hd <= 0 || hd % 2 != 0) return fail(SMK_ERR_ARGUMENT, "head_dim must be positive and even");
    if (capacity <= 0) return fail(SMK_ERR_ARGUMENT, "capacity must be positive");
    if (!pos_dev && (pos < 0 || pos >= capacity))
        return fail(SMK_ERR_ARGUMENT, "position %d outside the cache (capacity %d)", pos, capacity);
    if (!qkv || !inv_freq || !q_out || !k_cache || !v_cache) return fail(SMK_ERR_ARGUMENT, "pointers must not be NULL");
    DeviceGuard g(c->device);
    if (!g.ok) return fail(SMK_ERR_CUDA, "cudaSetDevice(%d) failed", c->device);
    SMK_CUDA(smk::launch_rope_kv(static_cast<cudaStream_t>(stream), c->pdl, qkv, inv_freq, pos_dev, pos, nh, nkv, hd,
                                 interleaved != 0, q_out, k_cache, v_cache, capacity, c->d_err),
             "rope_kv launch");
    return SMK_OK;
}

namespace {
// The attention workspace of `stream` when max_len takes more than one chunk:
// tickets (one per KV head) at a fixed place at the start of the buffer, zeroed
// when the buffer is allocated and reset by every call that used them; the
// partials after them, sized by the call. One chunk: no workspace (nullptr).
smk_status attention_workspace(smk_ctx* c, cudaStream_t s, int max_len, int nh, int nkv, int hd, float** ws,
                               unsigned** tickets) {
    *ws = nullptr;
    *tickets = nullptr;
    const int chunks = smk::attention_chunks(max_len);
    if (chunks <= 1) return SMK_OK;
    constexpr int kMaxTicketHeads = 256;
    if (nkv > kMaxTicketHeads) return fail(SMK_ERR_ARGUMENT, "at most %d KV heads", kMaxTicketHeads);
    const size_t tb = kMaxTicketHeads * sizeof(unsigned);
    const size_t need = tb + (size_t)nkv * chunks * (nh / nkv) * (hd + 2) * sizeof(float);
    std::lock_guard<std::mutex> lock(c->mu_scratch);
    DevBuf& b = c->attn_ws[s];
    const bool grow = need > b.bytes;
    SMK_CUDA(b.reserve(need), "cudaMalloc (attention workspace)");
    *tickets = static_cast<unsigned*>(b.ptr);
    *ws = reinterpret_cast<float*>(static_cast<uint8_t*>(b.ptr) + tb);
    if (grow) SMK_CUDA(cudaMemsetAsync(b.ptr, 0, tb, s), "cudaMemsetAsync");
    return SMK_OK;
}
}  // namespace

smk_status smk_attention_decode(smk_ctx* c, const float* q, const float* k_cache, const float* v_cache, float* out,
                                const int32_t* len_dev, int len, int max_len, int nh, int nkv, int hd, int capacity,
                                float scale, void* stream) {
    if (!c) return fail(SMK_ERR_ARGUMENT, "ctx must not be NULL");
    if (nh <= 0 || nkv <= 0 || nh % nkv != 0) return fail(SMK_ERR_ARGUMENT, "heads must be positive, nh a multiple of nkv");
    if (nh / nkv > smk::attention_max_rep())
        return fail(SMK_ERR_ARGUMENT, "at most %d query heads per KV head (got %d)", smk::attention_max_rep(), nh / nkv);
    if (hd <= 0 || hd % 32 != 0 || hd > smk::attention_max_hd())
        return fail(SMK_ERR_ARGUMENT, "head_dim must be a multiple of 32 up to %d (got %d)", smk::attention_max_hd(), hd);
    if (capacity <= 0 || max_len <= 0 || max_len > capacity)
        return fail(SMK_ERR_ARGUMENT, "need 0 < max_len <= capacity");
    if (!len_dev && (len < 1 || len > max_len)) return fail(SMK_ERR_ARGUMENT, "len must be in 1..max_len (got %d)", len);
    if (!q || !k_cache || !v_cache || !out) return fail(SMK_ERR_ARGUMENT, "pointers must not be NULL");
    DeviceGuard g(c->device);
    if (!g.ok) return fail(SMK_ERR_CUDA, "cudaSetDevice(%d) failed", c->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    float* ws = nullptr;
    unsigned* tickets = nullptr;
    smk_status st = attention_workspace(c, s, max_len, nh, nkv, hd, &ws, &tickets);
    if (st != SMK_OK) return st;
    SMK_CUDA(smk::launch_attention(s, c->pdl, q, k_cache, v_cache, out, len_dev, len, max_len, nh, nkv, hd, capacity,
                                   scale, ws, tickets, c->d_err),
             "attention launch");
    return SMK_OK;
}

smk_status smk_rope_attention(smk_ctx* c, const float* qkv, const float* inv_freq, const int32_t* pos_dev, int pos,
                              int max_len, int nh, int nkv, int hd, int interleaved, float* k_cache, float* v_cache,
                              int capacity, float scale, float* out, void* stream) {
    if (!c) return fail(SMK_ERR_ARGUMENT, "ctx must not be NULL");
    if (nh <= 0 || nkv <= 0 || nh % nkv != 0) return fail(SMK_ERR_ARGUMENT, "heads must be positive, nh a multiple of nkv");
    if (nh / nkv > smk::attention_max_rep())
        return fail(SMK_ERR_ARGUMENT, "at most %d query heads per KV head (got %d)", smk::attention_max_rep(), nh / nkv);
    if (hd <= 0 || hd % 32 != 0 || hd > smk::attention_max_hd())
        return fail(SMK_ERR_ARGUMENT, "head_dim must be a multiple of 32 up to %d (got %d)", smk::attention_max_hd(), hd);
    if (capacity <= 0 || max_len <= 0 || max_len > capacity)
        return fail(SMK_ERR_ARGUMENT, "need 0 < max_len <= capacity");
    if (!pos_dev && (pos < 0 || pos >= max_len))
        return fail(SMK_ERR_ARGUMENT, "position %d outside 0..max_len-1 (max_len %d)", pos, max_len);
    if (!qkv || !inv_freq || !k_cache || !v_cache || !out) return fail(SMK_ERR_ARGUMENT, "pointers must not be NULL");
    DeviceGuard g(c->device);
    if (!g.ok) return fail(SMK_ERR_CUDA, "cudaSetDevice(%d) failed", c->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    float* ws = nullptr;
    unsigned* tickets = nullptr;
    smk_status st = attention_workspace(c, s, max_len, nh, nkv, hd, &ws, &tickets);
    if (st != SMK_OK) return st;
    SMK_CUDA(smk::launch_rope_attention(s, c->pdl, qkv, inv_freq, pos_dev, pos, max_len, nh, nkv, hd, interleaved != 0,
                                        k_cache, v_cache, capacity, scale, out, ws, tickets, c->d_err),
             "rope + attention launch");
    return SMK_OK;
}

smk_status smk_gemv_q4_0(smk_ctx* c, int N, int K, const float* x, const uint8_t* Wq, float* y, void* stream) {
    return smk_gemv_q(c, SMK_Q4_0, 1, N, K, x, K, Wq, y, N, stream);
}

smk_status smk_gemv_q8_0(smk_ctx* c, int N, int K, const float* x, const uint8_t* Wq, float* y, void* stream) {
    return smk_gemv_q(c, SMK_Q8_0, 1, N, K, x, K, Wq, y, N, stream);
}

smk_status smk_gemv_q_host(smk_ctx* c, smk_qformat fmt, int M, int N, int K, const float* x, const uint8_t* Wq,
                           float* y) {
    if (!c) return fail(SMK_ERR_ARGUMENT, "ctx must not be NULL");
    smk_status st = check_q_args(fmt, M, N, K);
    if (st != SMK_OK) return st;
    if (M == 0 || N == 0) return SMK_OK;
    if (!y || (K > 0 && (!x || !Wq))) return fail(SMK_ERR_ARGUMENT, "x, Wq and y must not be NULL");
    DeviceGuard g(c->device);
    if (!g.ok) return fail(SMK_ERR_CUDA, "cudaSetDevice(%d) failed", c->device);
    const size_t xb = (size_t)M * K * 4, wb = (size_t)N * (K / 32) * smk::block_bytes(fmt), yb = (size_t)M * N * 4;
    // Host activations reach the device through stage_x_kernel, which reads
    // them from page-locked memory (the caller's, or this context's
    // page-locked buffer for a pageable array) over the bus while the GEMV
    // after it already streams its weights (programmatic dependent launch).
    // Host outputs are written by the GEMV into page-locked memory (mapped
    // into the device's address space under unified addressing), which costs
    // less than a copy back; the fast kernel does it from one CTA at its end.
    // Weights in host memory are copied to the device (device-resident
    // weights are the fast path).
    void *xmap = nullptr, *wmap = nullptr, *ymap = nullptr;
    const Mem xk = K > 0 ? mem_kind(x, &xmap) : Mem::kDevice;
    const Mem wk = K > 0 ? mem_kind(Wq, &wmap) : Mem::kDevice;
    const Mem yk = mem_kind(y, &ymap);
    cudaStream_t s = nullptr;   // the legacy default stream: ordered after other blocking streams' work
    std::lock_guard<std::mutex> lock(c->mu_stage);
    const size_t px = xk == Mem::kPageable ? align256(xb) : 0, py = yk == Mem::kPageable ? align256(yb) : 0;
    if (px + py) SMK_CUDA(c->pinned.reserve(px + py), "cudaHostAlloc (staging)");
    char* pin = static_cast<char*>(c->pinned.ptr);
    const size_t dxo = 0, dwo = xk != Mem::kDevice ? align256(xb) : 0;
    const size_t dyo = dwo + (wk != Mem::kDevice ? align256(wb) : 0);   // device copy of y (see run_q)
    const size_t dev_bytes = dyo + align256(yb);
    SMK_CUDA(c->staging.reserve(dev_bytes), "cudaMalloc (staging)");
    char* dst = static_cast<char*>(c->staging.ptr);
    const void* xsrc = x;   // where the copy of x reads (host memory)
    const float* xdev = static_cast<const float*>(xmap);   // the same, device-mapped
    if (xk == Mem::kPageable) {
        std::memcpy(pin, x, xb);
        xsrc = pin;
        void* dm = nullptr;
        SMK_CUDA(cudaHostGetDevicePointer(&dm, pin, 0), "cudaHostGetDevicePointer");
        xdev = static_cast<const float*>(dm);
    }
    const float* dx = xk != Mem::kDevice ? reinterpret_cast<const float*>(dst + dxo) : x;
    const uint8_t* dw = wk != Mem::kDevice ? reinterpret_cast<const uint8_t*>(dst + dwo) : Wq;
    float* dy = y;
    float* yhost = nullptr;
    if (yk == Mem::kPinned) yhost = static_cast<float*>(ymap);
    if (yk == Mem::kPageable) {
        void* dm = nullptr;
        SMK_CUDA(cudaHostGetDevicePointer(&dm, pin + px, 0), "cudaHostGetDevicePointer");
        yhost = static_cast<float*>(dm);
    }
    if (yhost) dy = reinterpret_cast<float*>(dst + dyo);
    // The call's device work: the copies of host operands, then the GEMV.
    auto enqueue = [&](cudaStream_t q) -> smk_status {
        if (wk != Mem::kDevice)
            SMK_CUDA(cudaMemcpyAsync(dst + dwo, Wq, wb, cudaMemcpyHostToDevice, q), "cudaMemcpyAsync (Wq)");
        if (xk != Mem::kDevice)
            SMK_CUDA(smk::launch_stage_x(q, xdev, reinterpret_cast<float*>(dst + dxo), (long long)M * K, c->num_sms),
                     "stage_x launch");
        return run_q(c, fmt, M, N, K, dx, K, dw, dy, N, q, nullptr, nullptr, nullptr, 0, yhost, xk != Mem::kDevice);
    };
    // A call whose operands (effective addresses) and shape repeat a recent
    // one replays a CUDA graph of that work: one launch instead of a copy and
    // a kernel launch, and no host-side planning (the weights stay on the
    // device, where the graph reads them at replay). The graph is captured on
    // the second call with a key, on a private non-blocking stream, and
    // launched into the legacy default stream like the direct path.
    HostGraph* hg = nullptr;
    if (c->host_graphs && wk == Mem::kDevice && K > 0) {
        const HostKey key{(int)fmt, M, N, K, xsrc, Wq, yhost ? static_cast<const void*>(yhost) : y};
        auto it = c->graphs.find(key);
        if (it == c->graphs.end()) {
            constexpr size_t kMaxHostGraphs = 64;
            if (c->graphs.size() >= kMaxHostGraphs) {   // drop the least recently used
                auto lru = c->graphs.begin();
                for (auto j = c->graphs.begin(); j != c->graphs.end(); ++j)
                    if (j->second.used < lru->second.used) lru = j;
                if (lru->second.exec) cudaGraphExecDestroy(lru->second.exec);
                c->graphs.erase(lru);
            }
            it = c->graphs.emplace(key, HostGraph{}).first;
        }
        hg = &it->second;
        hg->used = ++c->host_calls;
        if (!hg->exec && hg->seen >= 0 && ++hg->seen >= 2) {
            cudaStream_t q = c->capture_stream;
            cudaGraph_t graph = nullptr;
            SMK_CUDA(cudaStreamBeginCapture(q, cudaStreamCaptureModeThreadLocal), "cudaStreamBeginCapture");
            st = enqueue(q);
            const cudaError_t e = cudaStreamEndCapture(q, &graph);
            if (st != SMK_OK) {
                if (graph) cudaGraphDestroy(graph);
                return st;
            }
            if (e == cudaSuccess && cudaGraphInstantiate(&hg->exec, graph, 0) != cudaSuccess) hg->exec = nullptr;
            if (graph) cudaGraphDestroy(graph);
            if (!hg->exec) {   // not capturable here: this key takes the direct path from now on
                cudaGetLastError();
                hg->seen = -1;
            }
        }
    }
    if (hg && hg->exec) {
        SMK_CUDA(cudaGraphLaunch(hg->exec, s), "cudaGraphLaunch");
    } else {
        st = enqueue(s);
        if (st != SMK_OK) return st;
    }
    SMK_CUDA(cudaStreamSynchronize(s), "cudaStreamSynchronize");
    if (yk == Mem::kPageable) std::memcpy(y, pin + px, yb);
    return SMK_OK;
}

smk_status smk_gemv_dense(smk_ctx* c, smk_dtype wt, smk_dtype xt, int M, int N, int K, float alpha, const void* X,
                          int64_t ldx, const void* W, int64_t ldw, float beta, float* C, int64_t ldc, void* stream) {
    if (!c) return fail(SMK_ERR_ARGUMENT, "ctx must not be NULL");
    if (wt != SMK_F32 && wt != SMK_F16 && wt != SMK_BF16) return fail(SMK_ERR_DTYPE, "unknown weight type %d", (int)wt);
    if (!(xt == wt || xt == SMK_F32)) return fail(SMK_ERR_DTYPE, "x must have the weights' type or float32");
    if (M < 0 || N < 0 || K < 0) return fail(SMK_ERR_ARGUMENT, "M, N and K must be >= 0");
    if (M > smk::kMaxRows) return fail(SMK_ERR_ARGUMENT, "the decode path takes at most %d rows of x (got %d)",
                                       smk::kMaxRows, M);
    if (M == 0 || N == 0) return SMK_OK;
    if (!C || (K > 0 && (!X || !W))) return fail(SMK_ERR_ARGUMENT, "X, W and C must not be NULL");
    if (ldc < N || (K > 0 && (ldx < K || ldw < K))) return fail(SMK_ERR_ARGUMENT, "leading dimensions too small");
    DeviceGuard g(c->device);
    if (!g.ok) return fail(SMK_ERR_CUDA, "cudaSetDevice(%d) failed", c->device);
    smk::DenseParams p = {};
    p.x = X; p.ldx = ldx; p.w = W; p.ldw = ldw; p.y = C; p.ldy = ldc;
    p.M = M; p.N = N; p.K = K; p.alpha = alpha; p.beta = beta;
    p.err = c->d_err;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const size_t need = c->dense_mma ? smk::dense_mma_scratch((int)wt, (int)xt, M, K, ldw, W) : 0;
    if (need) {   // bf16 weights, several rows of x: the tensor-core kernel and its x split in scratch
        {
            std::lock_guard<std::mutex> lock(c->mu_scratch);
            DevBuf& b = c->scratch[s];
            SMK_CUDA(b.reserve(need), "cudaMalloc (scratch)");
            p.xfrag = b.ptr;
        }
        SMK_CUDA(smk::launch_gemv_dense_mma(s, c->pdl, c->num_sms, (int)wt, (int)xt, p), "dense tensor-core gemv launch");
        return SMK_OK;
    }
    SMK_CUDA(smk::launch_gemv_dense(s, c->pdl, c->num_sms, (int)wt, (int)xt, p), "dense gemv launch");
    return SMK_OK;
}

smk_status smk_gemv_dense_host(smk_ctx* c, smk_dtype wt, smk_dtype xt, int M, int N, int K, float alpha,
                               const void* X, const void* W, float beta, float* C) {
    if (!c) return fail(SMK_ERR_ARGUMENT, "ctx must not be NULL");
    if (M <= 0 || N <= 0) return smk_gemv_dense(c, wt, xt, M, N, K, alpha, X, K, W, K, beta, C, N, nullptr);
    DeviceGuard g(c->device);
    if (!g.ok) return fail(SMK_ERR_CUDA, "cudaSetDevice(%d) failed", c->device);
    const size_t xes = xt == SMK_F32 ? 4 : 2, wes = wt == SMK_F32 ? 4 : 2;
    const size_t xb = (size_t)M * K * xes, wb = (size_t)N * K * wes, cb = (size_t)M * N * 4;
    const bool xh = K > 0 && !is_device_ptr(X), wh = K > 0 && !is_device_ptr(W), ch = !is_device_ptr(C);
    cudaStream_t s = nullptr;
    std::lock_guard<std::mutex> lock(c->mu_stage);
    const size_t ox = 0, ow = ox + (xh ? align256(xb) : 0), oc = ow + (wh ? align256(wb) : 0),
                 total = oc + (ch ? align256(cb) : 0);
    if (total) SMK_CUDA(c->staging.reserve(total), "cudaMalloc (staging)");
    char* base = static_cast<char*>(c->staging.ptr);
    const void* dX = xh ? base + ox : X;
    const void* dW = wh ? base + ow : W;
    float* dC = ch ? reinterpret_cast<float*>(base + oc) : C;
    if (xh) SMK_CUDA(cudaMemcpyAsync(base + ox, X, xb, cudaMemcpyHostToDevice, s), "cudaMemcpyAsync (X)");
    if (wh) SMK_CUDA(cudaMemcpyAsync(base + ow, W, wb, cudaMemcpyHostToDevice, s), "cudaMemcpyAsync (W)");
    if (ch && beta != 0.0f) SMK_CUDA(cudaMemcpyAsync(dC, C, cb, cudaMemcpyHostToDevice, s), "cudaMemcpyAsync (C)");
    smk_status st = smk_gemv_dense(c, wt, xt, M, N, K, alpha, dX, K, dW, K, beta, dC, N, s);
    if (st != SMK_OK) return st;
    if (K == 0 && beta == 0.0f) SMK_CUDA(cudaMemsetAsync(dC, 0, cb, s), "cudaMemsetAsync");
    if (ch) SMK_CUDA(cudaMemcpyAsync(C, dC, cb, cudaMemcpyDeviceToHost, s), "cudaMemcpyAsync (C)");
    SMK_CUDA(cudaStreamSynchronize(s), "cudaStreamSynchronize");
    return SMK_OK;
}

// Argument checks of sgemm_u8s8 (src/bindings/pybind_entry.cpp:866-868) and
// of this decode path.
static smk_status check_u8s8_args(int M, int N, int K, int a_zero_point, float a_scale) {
    if (M < 0 || N < 0 || K < 0) return fail(SMK_ERR_ARGUMENT, "M, N and K must be >= 0");
    if (M > smk::kMaxRows)
        return fail(SMK_ERR_ARGUMENT, "the decode path takes at most %d rows of A (got %d)", smk::kMaxRows, M);
    if (a_zero_point < 0 || a_zero_point > 255)
        return fail(SMK_ERR_ARGUMENT, "a_zero_point must be in [0, 255] (got %d)", a_zero_point);
    if (!std::isfinite(a_scale)) return fail(SMK_ERR_ARGUMENT, "a_scale must be finite");
    return SMK_OK;
}

smk_status smk_gemv_u8s8(smk_ctx* c, int M, int N, int K, const uint8_t* A, int64_t lda, int a_zero_point,
                         const int8_t* W, int64_t ldw, float a_scale, const float* b_scales, float* C, int64_t ldc,
                         void* stream) {
    if (!c) return fail(SMK_ERR_ARGUMENT, "ctx must not be NULL");
    smk_status st = check_u8s8_args(M, N, K, a_zero_point, a_scale);
    if (st != SMK_OK) return st;
    if (M == 0 || N == 0) return SMK_OK;
    if (!C || !b_scales || (K > 0 && (!A || !W))) return fail(SMK_ERR_ARGUMENT, "A, W, b_scales and C must not be NULL");
    if (ldc < N || (K > 0 && (lda < K || ldw < K))) return fail(SMK_ERR_ARGUMENT, "leading dimensions too small");
    DeviceGuard g(c->device);
    if (!g.ok) return fail(SMK_ERR_CUDA, "cudaSetDevice(%d) failed", c->device);
    smk::U8S8Params p;
    p.a = A; p.lda = lda; p.w = W; p.ldw = ldw; p.scales = b_scales; p.y = C; p.ldy = ldc;
    p.M = M; p.N = N; p.K = K; p.zp = a_zero_point; p.a_scale = a_scale;
    p.err = c->d_err;
    SMK_CUDA(smk::launch_gemv_u8s8(static_cast<cudaStream_t>(stream), c->pdl, c->num_sms, p), "u8s8 gemv launch");
    return SMK_OK;
}

smk_status smk_gemv_u8s8_host(smk_ctx* c, int M, int N, int K, const uint8_t* A, int a_zero_point, const int8_t* W,
                              float a_scale, const float* b_scales, float* C) {
    if (!c) return fail(SMK_ERR_ARGUMENT, "ctx must not be NULL");
    smk_status st = check_u8s8_args(M, N, K, a_zero_point, a_scale);
    if (st != SMK_OK) return st;
    if (M == 0 || N == 0) return SMK_OK;
    if (!C || !b_scales || (K > 0 && (!A || !W))) return fail(SMK_ERR_ARGUMENT, "A, W, b_scales and C must not be NULL");
    DeviceGuard g(c->device);
    if (!g.ok) return fail(SMK_ERR_CUDA, "cudaSetDevice(%d) failed", c->device);
    const size_t ab = (size_t)M * K, wb = (size_t)N * K, sb = (size_t)N * 4, cb = (size_t)M * N * 4;
    const bool ah = K > 0 && !is_device_ptr(A), wh = K > 0 && !is_device_ptr(W), sh = !is_device_ptr(b_scales),
               ch = !is_device_ptr(C);
    cudaStream_t s = nullptr;
    std::lock_guard<std::mutex> lock(c->mu_stage);
    const size_t oa = 0, ow = oa + (ah ? align256(ab) : 0), os = ow + (wh ? align256(wb) : 0),
                 oc = os + (sh ? align256(sb) : 0), total = oc + (ch ? align256(cb) : 0);
    if (total) SMK_CUDA(c->staging.reserve(total), "cudaMalloc (staging)");
    char* base = static_cast<char*>(c->staging.ptr);
    const uint8_t* dA = ah ? reinterpret_cast<const uint8_t*>(base + oa) : A;
    const int8_t* dW = wh ? reinterpret_cast<const int8_t*>(base + ow) : W;
    const float* dS = sh ? reinterpret_cast<const float*>(base + os) : b_scales;
    float* dC = ch ? reinterpret_cast<float*>(base + oc) : C;
    if (ah) SMK_CUDA(cudaMemcpyAsync(base + oa, A, ab, cudaMemcpyHostToDevice, s), "cudaMemcpyAsync (A)");
    if (wh) SMK_CUDA(cudaMemcpyAsync(base + ow, W, wb, cudaMemcpyHostToDevice, s), "cudaMemcpyAsync (W)");
    if (sh) SMK_CUDA(cudaMemcpyAsync(base + os, b_scales, sb, cudaMemcpyHostToDevice, s), "cudaMemcpyAsync (b_scales)");
    st = smk_gemv_u8s8(c, M, N, K, dA, K, a_zero_point, dW, K, a_scale, dS, dC, N, s);
    if (st != SMK_OK) return st;
    if (ch) SMK_CUDA(cudaMemcpyAsync(C, dC, cb, cudaMemcpyDeviceToHost, s), "cudaMemcpyAsync (C)");
    SMK_CUDA(cudaStreamSynchronize(s), "cudaStreamSynchronize");
    return SMK_OK;
}

smk_status smk_dequantize_rows(smk_ctx* c, smk_qformat fmt, int N, int K, const uint8_t* Wq, const int32_t* rows,
                               int nrows, float* out, int64_t ldo, void* stream) {
    if (!c) return fail(SMK_ERR_ARGUMENT, "ctx must not be NULL");
    if (fmt != SMK_Q4_0 && fmt != SMK_Q8_0) return fail(SMK_ERR_DTYPE, "unknown block format %d", (int)fmt);
    if (N < 0 || K < 0 || nrows < 0) return fail(SMK_ERR_ARGUMENT, "N, K and nrows must be >= 0");
    if (K % 32 != 0) return fail(SMK_ERR_ARGUMENT, "K must be a multiple of 32 (got %d)", K);
    if (nrows == 0 || K == 0) return SMK_OK;
    if (!Wq || !rows || !out) return fail(SMK_ERR_ARGUMENT, "Wq, rows and out must not be NULL");
    if (ldo < K) return fail(SMK_ERR_ARGUMENT, "ldo must be >= K");
    DeviceGuard g(c->device);
    if (!g.ok) return fail(SMK_ERR_CUDA, "cudaSetDevice(%d) failed", c->device);
    SMK_CUDA(smk::launch_dequantize_rows(static_cast<cudaStream_t>(stream), (int)fmt, Wq, N, K, rows, nrows, out, ldo,
                                         c->d_err, c->num_sms),
             "dequantize launch");
    return SMK_OK;
}

smk_status smk_quantize(smk_ctx* c, smk_qformat fmt, int64_t rows, int K, const float* W, uint8_t* out, void* stream) {
    if (!c) return fail(SMK_ERR_ARGUMENT, "ctx must not be NULL");
    if (fmt != SMK_Q4_0 && fmt != SMK_Q8_0) return fail(SMK_ERR_DTYPE, "unknown block format %d", (int)fmt);
    if (rows < 0 || K < 0 || K % 32 != 0)
        return fail(SMK_ERR_ARGUMENT, "K (the last dimension of W) must be a multiple of 32 (got %d)", K);
    if (rows == 0 || K == 0) return SMK_OK;
    DeviceGuard g(c->device);
    if (!g.ok) return fail(SMK_ERR_CUDA, "cudaSetDevice(%d) failed", c->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    SMK_CUDA(cudaMemsetAsync(c->d_reject, 0, sizeof(unsigned), s), "cudaMemsetAsync");
    SMK_CUDA(smk::launch_quantize_w(s, (int)fmt, W, rows, K, out, c->d_reject), "quantize launch");
    unsigned rej = 0;
    SMK_CUDA(cudaMemcpyAsync(&rej, c->d_reject, sizeof rej, cudaMemcpyDeviceToHost, s), "cudaMemcpyAsync");
    SMK_CUDA(cudaStreamSynchronize(s), "cudaStreamSynchronize");
    if (rej)
        return fail(SMK_ERR_REJECTED, "W must be finite, with every block scale representable in float16");
    return SMK_OK;
}

smk_status smk_quantize_host(smk_ctx* c, smk_qformat fmt, int64_t rows, int K, const float* W, uint8_t* out) {
    if (!c) return fail(SMK_ERR_ARGUMENT, "ctx must not be NULL");
    if (fmt != SMK_Q4_0 && fmt != SMK_Q8_0) return fail(SMK_ERR_DTYPE, "unknown block format %d", (int)fmt);
    if (rows < 0 || K < 0 || K % 32 != 0)
        return fail(SMK_ERR_ARGUMENT, "K (the last dimension of W) must be a multiple of 32 (got %d)", K);
    if (rows == 0 || K == 0) return SMK_OK;
    DeviceGuard g(c->device);
    if (!g.ok) return fail(SMK_ERR_CUDA, "cudaSetDevice(%d) failed", c->device);
    const size_t wb = (size_t)rows * K * 4, ob = (size_t)rows * (K / 32) * smk::block_bytes(fmt);
    const bool wh = !is_device_ptr(W), oh = !is_device_ptr(out);
    cudaStream_t s = nullptr;
    std::lock_guard<std::mutex> lock(c->mu_stage);
    const size_t total = (wh ? align256(wb) : 0) + (oh ? align256(ob) : 0);
    if (total) SMK_CUDA(c->staging.reserve(total), "cudaMalloc (staging)");
    char* base = static_cast<char*>(c->staging.ptr);
    const float* dW = wh ? reinterpret_cast<const float*>(base) : W;
    uint8_t* dO = oh ? reinterpret_cast<uint8_t*>(base + (wh ? align256(wb) : 0)) : out;
    if (wh) SMK_CUDA(cudaMemcpyAsync(base, W, wb, cudaMemcpyHostToDevice, s), "cudaMemcpyAsync (W)");
    smk_status st = smk_quantize(c, fmt, rows, K, dW, dO, s);
    if (st != SMK_OK) return st;
    if (oh) {
        SMK_CUDA(cudaMemcpyAsync(out, dO, ob, cudaMemcpyDeviceToHost, s), "cudaMemcpyAsync (out)");
        SMK_CUDA(cudaStreamSynchronize(s), "cudaStreamSynchronize");
    }
    return SMK_OK;
}

}  // extern "C"

// ---- test hooks --------------------------------------------------------------

namespace {

// Un-swizzle the quantized-x layout (gemv_quant.cuh) into plain int8 [M, K]
// and fp32 [M, K/32].
__global__ void unswizzle_x(const uint8_t* xq, smk::QGemvParams p, int8_t* qs, float* dx) {
    const int K = p.nb * 32;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < (long long)p.M * K;
         i += (long long)gridDim.x * blockDim.x) {
        const int m = (int)(i / K), k = (int)(i % K), b = k / 32, v = k % 32;
        const int sb = b >> 3, j = b & 7, h = v >> 4, ks = sb >> p.log2G, g = sb & (p.G - 1);
        qs[i] = (int8_t)xq[smk::xq_off(p.ksteps, m, ks, j, h, g) + (v & 15)];
        if (v == 0)
            dx[(size_t)m * p.nb + b] = reinterpret_cast<const float2*>(xq + smk::xd_off(p.M, p.ksteps, m, ks, j, g))->x;
    }
}

}  // namespace

extern "C" {

smk_status smk_quantize_x(smk_ctx* c, int M, int K, const float* x, int64_t ldx, int8_t* qs, float* dx, void* stream) {
    if (!c) return fail(SMK_ERR_ARGUMENT, "ctx must not be NULL");
    smk_status st = check_q_args(SMK_Q8_0, M, 1, K);
    if (st != SMK_OK) return st;
    if (M == 0 || K == 0) return SMK_OK;
    DeviceGuard g(c->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    smk::QGemvParams p = {};
    p.x = x; p.ldx = ldx; p.M = M; p.N = 1; p.K = K;
    smk::plan_tiles(p, false);
    uint8_t* xq;
    {
        std::lock_guard<std::mutex> lock(c->mu_scratch);
        SMK_CUDA(c->test_buf.reserve(smk::xq_total_bytes(M, p.ksteps)), "cudaMalloc (test)");
        xq = static_cast<uint8_t*>(c->test_buf.ptr);
    }
    SMK_CUDA(smk::launch_quantize_x(cfg_for(c, s), p, xq), "quantize_x launch");
    unswizzle_x<<<std::min<long long>(((long long)M * K + 255) / 256, 4096), 256, 0, s>>>(xq, p, qs, dx);
    SMK_CUDA(cudaGetLastError(), "unswizzle launch");
    return SMK_OK;
}

smk_status smk_block_sums(smk_ctx* c, smk_qformat fmt, int M, int N, int K, const float* x, int64_t ldx,
                          const uint8_t* Wq, int32_t* out, void* stream) {
    if (!c) return fail(SMK_ERR_ARGUMENT, "ctx must not be NULL");
    smk_status st = check_q_args(fmt, M, N, K);
    if (st != SMK_OK) return st;
    if (M == 0 || N == 0 || K == 0) return SMK_OK;
    DeviceGuard g(c->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    float* y;
    {
        std::lock_guard<std::mutex> lock(c->mu_scratch);
        SMK_CUDA(c->test_buf.reserve((size_t)M * N * 4), "cudaMalloc (test)");
        y = static_cast<float*>(c->test_buf.ptr);
    }
    return run_q(c, fmt, M, N, K, x, ldx, Wq, y, N, s, out);
}

smk_status smk_check_x_arith(smk_ctx* c, unsigned long long* out) {
    if (!c || !out) return fail(SMK_ERR_ARGUMENT, "ctx and out must not be NULL");
    DeviceGuard g(c->device);
    unsigned long long* bad;
    {
        std::lock_guard<std::mutex> lock(c->mu_scratch);
        SMK_CUDA(c->test_buf.reserve(3 * sizeof(unsigned long long)), "cudaMalloc (test)");
        bad = static_cast<unsigned long long*>(c->test_buf.ptr);
        SMK_CUDA(cudaMemset(bad, 0, 3 * sizeof(unsigned long long)), "cudaMemset");
        SMK_CUDA(smk::launch_check_x_arith(nullptr, bad), "check launch");
        SMK_CUDA(cudaMemcpy(out, bad, 3 * sizeof(unsigned long long), cudaMemcpyDeviceToHost), "cudaMemcpy");
    }
    return SMK_OK;
}

}  // extern "C"
