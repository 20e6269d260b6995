// gemv_noalloc.cu — smk_gemv_q_noalloc: the quantized decode GEMV for callers
// that must not allocate GPU memory.
//
// Who needs it: code that runs where cudaMalloc is unavailable or unwelcome —
// inside a host framework that owns every device allocation through its own
// pool (and forbids foreign cudaMalloc calls, which would also implicitly
// synchronise the device), real-time or inference servers that pre-plan all
// memory at start-up and must not allocate on the request path, and plugins
// loaded into such hosts. The regular entry points (smk_gemv_q and friends)
// need an smk_ctx, whose creation allocates an error word and whose calls
// may grow scratch buffers with cudaMalloc; this entry point needs neither.
//
// How: the only scratch the GEMV needs — the activation rows quantized to Q8
// blocks — lives in a file-scope __device__ array of fixed size, which every
// GPU that loads this library reserves for as long as the library stays
// loaded. The caller passes x, the weights and y, all device memory. Each call
// quantizes x into the array and runs the GEMV kernel that reads x from
// global memory (the same kernels as smk_gemv_q's global-scratch path).

#include "../../include/smk_cuda.h"
#include "gemv_quant.cuh"

#include <algorithm>
#include <cstdio>
#include <mutex>
#include <string>

#include <cuda_runtime.h>

namespace {

// Maximum scratch: 1 MiB of quantized activations, 10 KiB per row of x and
// per 8192 values of K: M · ceil(K/8192) up to 102 (K up to 835,584 for one
// row of x; K up to 98,304 for eight).
constexpr size_t kNoAllocScratchBytes = SMK_NOALLOC_SCRATCH_BYTES;

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];
// Error bits of the kernels launched by smk_gemv_q_noalloc on this device (a
// bounded wait that ran out, ...). Zero when the library loads; the kernels
// OR bits in; smk_noalloc_device_error reads and clears it.
static __device__ unsigned g_noalloc_error;

struct DeviceState {
    bool ready = false;
    uint8_t* scratch = nullptr;
    unsigned* error = nullptr;
    int num_sms = 0;
};

constexpr int kMaxDevices = 64;
std::mutex g_mu;
DeviceState g_state[kMaxDevices];

smk_status noalloc_fail(smk_status st, const std::string& msg) {
    smk::set_last_error(msg.c_str());   // read back with smk_last_error()
    return st;
}

// Per-device set-up, done by the first call on each device with that device
// current: the device addresses of the scratch array and the error word
// (host code cannot use the symbols' names as addresses).
smk_status setup(int dev, DeviceState** out) {
    std::lock_guard<std::mutex> g(g_mu);
    DeviceState& s = g_state[dev];
    if (!s.ready) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess)
            return noalloc_fail(SMK_ERR_CUDA, std::string("cudaGetSymbolAddress(scratch): ") + cudaGetErrorString(e));
        s.scratch = static_cast<uint8_t*>(p);
        e = cudaGetSymbolAddress(&p, g_noalloc_error);
        if (e != cudaSuccess)
            return noalloc_fail(SMK_ERR_CUDA, std::string("cudaGetSymbolAddress(error): ") + cudaGetErrorString(e));
        s.error = static_cast<unsigned*>(p);
        e = cudaDeviceGetAttribute(&s.num_sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess)
            return noalloc_fail(SMK_ERR_CUDA, std::string("cudaDeviceGetAttribute: ") + cudaGetErrorString(e));
        s.ready = true;
    }
    *out = &s;
    return SMK_OK;
}

}  // namespace

extern "C" smk_status smk_gemv_q_noalloc(smk_qformat fmt, int M, int N, int K, const float* x, int64_t ldx,
                                         const uint8_t* Wq, float* y, int64_t ldy, void* stream) {
    if (fmt != SMK_Q4_0 && fmt != SMK_Q8_0) return noalloc_fail(SMK_ERR_DTYPE, "unknown block format");
    if (M < 0 || N < 0 || K < 0) return noalloc_fail(SMK_ERR_ARGUMENT, "M, N and K must be >= 0");
    if (M > smk::kMaxRows) return noalloc_fail(SMK_ERR_ARGUMENT, "at most 8 rows of x per call");
    if (K % 32 != 0) return noalloc_fail(SMK_ERR_ARGUMENT, "K must be a multiple of 32");
    const bool fast = (K % 256 == 0) && ((reinterpret_cast<uintptr_t>(Wq) & 15) == 0);
    smk::QGemvParams p = {};
    p.x = x; p.ldx = ldx; p.w = Wq; p.y = y; p.ldy = ldy;
    p.M = M; p.N = N; p.K = K;
    // The plan (and so the accumulation order) of smk_gemv_q on a 148-SM B200.
    smk::plan_tiles(p, fast, (int)fmt, true, 148);
    const size_t need = smk::x_bytes(p);
    if (need > kNoAllocScratchBytes) {
        char buf[256];
        snprintf(buf, sizeof buf,
                 "smk_gemv_q_noalloc: M=%d rows of K=%d need %zu bytes of scratch, more than its fixed %zu "
                 "(M * ceil(K/8192) must be <= %zu); use smk_gemv_q",
                 M, K, need, kNoAllocScratchBytes, kNoAllocScratchBytes / 10240);
        return noalloc_fail(SMK_ERR_ARGUMENT, buf);
    }
    if (M == 0 || N == 0) return SMK_OK;
    if (!y || (K > 0 && (!x || !Wq))) return noalloc_fail(SMK_ERR_ARGUMENT, "x, Wq and y must not be NULL");
    if (ldy < N || (K > 0 && ldx < K)) return noalloc_fail(SMK_ERR_ARGUMENT, "ldx >= K and ldy >= N required");
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return noalloc_fail(SMK_ERR_CUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices) return noalloc_fail(SMK_ERR_ARGUMENT, "device number out of range");
    DeviceState* s = nullptr;
    smk_status st = setup(dev, &s);
    if (st != SMK_OK) return st;
    cudaStream_t strm = static_cast<cudaStream_t>(stream);
    if (K == 0) {
        for (int m = 0; m < M; ++m) {
            e = cudaMemsetAsync(y + (size_t)m * ldy, 0, (size_t)N * 4, strm);
            if (e != cudaSuccess) return noalloc_fail(SMK_ERR_CUDA, cudaGetErrorString(e));
        }
        return SMK_OK;
    }
    // The scratch needs no clearing: the quantize kernel writes every byte the
    // GEMV kernel reads. The error word is not cleared here: it keeps the bits
    // of every call until smk_noalloc_device_error reads it.

    smk::LaunchCfg l;
    l.stream = strm;
    l.pdl = false;
    l.num_sms = s->num_sms;
    l.warps = 8;
    p.xq = s->scratch;
    p.dump = nullptr;
    p.err = s->error;
    p.stages = 2;
    e = smk::launch_quantize_x(l, p, s->scratch);
    if (e != cudaSuccess) return noalloc_fail(SMK_ERR_CUDA, std::string("quantize_x launch: ") + cudaGetErrorString(e));
    e = smk::launch_gemv_q(l, (int)fmt, p, fast, nullptr);
    if (e != cudaSuccess) return noalloc_fail(SMK_ERR_CUDA, std::string("gemv launch: ") + cudaGetErrorString(e));
    return SMK_OK;
}

// The device error word of this device's smk_gemv_q_noalloc calls: waits for
// `stream` (and everything queued on it before), copies the word to *code and
// clears it. 0 means that no kernel of those calls reported an error since the
// last read. Allocates nothing: one device-to-host copy, one memset and a
// stream synchronisation.
extern "C" smk_status smk_noalloc_device_error(unsigned* code, void* stream) {
    if (!code) return noalloc_fail(SMK_ERR_ARGUMENT, "code must not be NULL");
    *code = 0;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return noalloc_fail(SMK_ERR_CUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices) return noalloc_fail(SMK_ERR_ARGUMENT, "device number out of range");
    DeviceState* s = nullptr;
    smk_status st = setup(dev, &s);
    if (st != SMK_OK) return st;
    cudaStream_t strm = static_cast<cudaStream_t>(stream);
    unsigned word = 0;
    e = cudaMemcpyAsync(&word, s->error, sizeof(unsigned), cudaMemcpyDeviceToHost, strm);
    if (e == cudaSuccess) e = cudaMemsetAsync(s->error, 0, sizeof(unsigned), strm);
    if (e == cudaSuccess) e = cudaStreamSynchronize(strm);
    if (e != cudaSuccess) return noalloc_fail(SMK_ERR_CUDA, std::string("reading the error word: ") + cudaGetErrorString(e));
    *code = word;
    return SMK_OK;
}
