// core_pybind.cpp — simd_ml_kernels._core for the B200 build: the decode-GEMV
// entry points of the reference's Python module (src/bindings/pybind_entry.cpp
// of Mattral/simd-ml-kernels 0.3.0), same names, argument order, defaults,
// validation order, error classes and messages, over the C ABI of
// libsmk_cuda.so (include/smk_cuda.h). No kernel runs on the CPU.
//
// Operands are NumPy arrays (host memory: staged to the device, the call
// returns when the result is back, as the reference's calls do) or objects
// exposing __cuda_array_interface__ (device memory: torch CUDA tensors,
// DeviceArray). With every operand on the device and `stream` given, a call
// is asynchronous on that stream, like any CUDA library call.

#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <cstdint>
#include <cstring>
#include <cmath>
#include <limits>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/smk_cuda.h"

namespace py = pybind11;

namespace {

// Registered as simd_ml_kernels.DTypeError (TypeError, RuntimeError) and
// simd_ml_kernels.ArgumentError (ValueError, RuntimeError), as in the reference.
struct DTypeError : std::runtime_error { using std::runtime_error::runtime_error; };
struct ArgumentError : std::runtime_error { using std::runtime_error::runtime_error; };

// ---- one context per device, created on first use ---------------------------

std::mutex g_ctx_mu;
std::vector<smk_ctx*> g_ctx;

int current_device_hint = 0;

smk_ctx* ctx_for(int device) {
    std::lock_guard<std::mutex> g(g_ctx_mu);
    if ((int)g_ctx.size() <= device) g_ctx.resize(device + 1, nullptr);
    if (!g_ctx[device]) {
        smk_ctx* c = nullptr;
        if (smk_ctx_create(device, &c) != SMK_OK)
            throw std::runtime_error(std::string("simd_ml_kernels: no usable B200 device: ") + smk_last_error());
        g_ctx[device] = c;
    }
    return g_ctx[device];
}

// ---- page-locked result arrays -------------------------------------------------
//
// GEMV results returned as new NumPy arrays live in page-locked memory, so the
// kernel stores y straight into the array the caller receives (no staging
// buffer, no copy after the synchronise). Blocks are recycled by byte size when
// their arrays die; a result larger than kMaxBlock, or any result while
// page-locked memory cannot be had, is an ordinary NumPy array.

struct PinnedPool {
    static constexpr size_t kMaxBlock = size_t(4) << 20;   // per result array
    static constexpr size_t kMaxFree = size_t(64) << 20;   // kept for reuse
    std::mutex mu;
    std::vector<std::pair<size_t, void*>> free_list;
    size_t free_bytes = 0;

    void* get(size_t bytes) {
        {
            std::lock_guard<std::mutex> g(mu);
            for (size_t i = 0; i < free_list.size(); ++i) {
                if (free_list[i].first == bytes) {
                    void* p = free_list[i].second;
                    free_list[i] = free_list.back();
                    free_list.pop_back();
                    free_bytes -= bytes;
                    return p;
                }
            }
        }
        void* p = nullptr;
        return smk_host_alloc(bytes, &p) == SMK_OK ? p : nullptr;
    }
    void put(void* p, size_t bytes) {
        {
            std::lock_guard<std::mutex> g(mu);
            if (free_bytes + bytes <= kMaxFree) {
                free_list.emplace_back(bytes, p);
                free_bytes += bytes;
                return;
            }
        }
        smk_host_free(p);
    }
};

PinnedPool* g_pool = new PinnedPool();   // never destroyed: result arrays may outlive the module

struct PinnedBlock {
    void* ptr;
    size_t bytes;
};

py::array_t<float> result_array(const std::vector<py::ssize_t>& shape) {
    size_t n = 1;
    for (py::ssize_t d : shape) n *= (size_t)d;
    const size_t bytes = n * sizeof(float);
    if (bytes == 0 || bytes > PinnedPool::kMaxBlock) return py::array_t<float>(shape);
    void* p = g_pool->get(bytes);
    if (!p) return py::array_t<float>(shape);
    auto* blk = new PinnedBlock{p, bytes};
    py::capsule base(blk, [](void* v) {
        auto* b = static_cast<PinnedBlock*>(v);
        g_pool->put(b->ptr, b->bytes);
        delete b;
    });
    return py::array_t<float>(shape, static_cast<float*>(p), base);
}

void check(smk_status st) {
    if (st == SMK_OK) return;
    const std::string msg = smk_last_error();
    if (st == SMK_ERR_ARGUMENT || st == SMK_ERR_REJECTED) throw ArgumentError(msg);
    if (st == SMK_ERR_DTYPE) throw DTypeError(msg);
    throw std::runtime_error(msg);
}

// ---- an operand: a NumPy array or a __cuda_array_interface__ object --------

struct Arr {
    py::object obj;
    void* ptr = nullptr;
    std::vector<int64_t> shape;
    char kind = 0;          // 'f', 'u', 'i', 'V', ...
    int itemsize = 0;
    std::string name;       // dtype name ("bfloat16" for ml_dtypes)
    bool device = false;
    bool contiguous = true;
    bool writeable = true;
    int device_id = 0;
    int ndim() const { return (int)shape.size(); }
    int64_t size() const {
        int64_t n = 1;
        for (int64_t s : shape) n *= s;
        return n;
    }
};

Arr as_arr(const py::handle& h) {
    Arr a;
    a.obj = py::reinterpret_borrow<py::object>(h);
    if (py::isinstance<py::array>(h)) {
        auto arr = py::reinterpret_borrow<py::array>(h);
        a.ptr = const_cast<void*>(arr.data());
        for (int i = 0; i < arr.ndim(); ++i) a.shape.push_back(arr.shape(i));
        const py::dtype dt = arr.dtype();
        a.kind = dt.kind();
        a.itemsize = (int)dt.itemsize();
        // The dtype's name is only read to tell ml_dtypes.bfloat16 apart and
        // for error messages: fetched for 2-byte types that are not plain
        // numbers, not on every call.
        if (a.itemsize == 2 && a.kind != 'f' && a.kind != 'i' && a.kind != 'u')
            a.name = py::str(dt.attr("name"));
        else
            a.name = std::string(1, a.kind) + std::to_string(a.itemsize);
        a.contiguous = (arr.flags() & py::array::c_style) != 0;
        a.writeable = arr.writeable();
        return a;
    }
    if (py::hasattr(h, "__cuda_array_interface__")) {
        py::dict cai = h.attr("__cuda_array_interface__");
        a.device = true;
        py::tuple data = cai["data"];
        a.ptr = reinterpret_cast<void*>(data[0].cast<uintptr_t>());
        a.writeable = !data[1].cast<bool>();
        for (auto s : cai["shape"].cast<py::tuple>()) a.shape.push_back(s.cast<int64_t>());
        const std::string ts = cai["typestr"].cast<std::string>();
        a.kind = ts.size() > 1 ? ts[1] : 0;
        a.itemsize = ts.size() > 2 ? std::stoi(ts.substr(2)) : 0;
        a.name = std::string(1, a.kind) + std::to_string(a.itemsize);
        if (cai.contains("strides") && !cai["strides"].is_none()) {
            py::tuple st = cai["strides"];
            int64_t expect = a.itemsize;
            for (int i = (int)a.shape.size() - 1; i >= 0; --i) {
                if (a.shape[i] != 1 && st[i].cast<int64_t>() != expect) a.contiguous = false;
                expect *= a.shape[i];
            }
        }
        // The Python layer sets the device of its CUDA operands before a call;
        // no pointer query here, so calls stay legal inside stream capture.
        a.device_id = current_device_hint;
        return a;
    }
    throw DTypeError("expected a numpy.ndarray or a CUDA array (__cuda_array_interface__)");
}

// The reference's validation helpers (pybind_entry.cpp:80-128), same messages.
void check_float32(const Arr& a, const char* name) {
    if (a.kind != 'f' || a.itemsize != 4)
        throw DTypeError(std::string(name) + " must be float32 (dtype=np.float32). "
                         "Call arr.astype(np.float32) before passing.");
}
void check_contiguous(const Arr& a, const char* name) {
    if (!a.contiguous)
        throw ArgumentError(std::string(name) + " must be C-contiguous. "
                            "Call numpy.ascontiguousarray(arr) before passing.");
}
void validate_array(const Arr& a, const char* name) {
    check_float32(a, name);
    check_contiguous(a, name);
}
void check_writeable(const Arr& a, const char* name) {
    if (!a.writeable)
        throw ArgumentError(std::string(name) + " must be writeable. "
                            "The array may be read-only; make a copy first.");
}

// ---- GEMV on ggml blocks (pybind_entry.cpp:944-995) -------------------------

py::object gemv_blocks(const py::handle& xh, const Arr& w, py::ssize_t N, py::ssize_t K, int block_bytes,
                       const char* fmt_name, smk_qformat fmt, const py::object& out, const py::object& stream,
                       bool batched) {
    const Arr x = as_arr(xh);
    validate_array(x, "x");
    if (w.kind != 'u' || w.itemsize != 1)
        throw DTypeError(std::string("Wq must be uint8 (blocks from quantize_") + fmt_name + "; dtype=np.uint8)");
    check_contiguous(w, "Wq");
    if (N < 0 || K < 0) throw ArgumentError("N and K must be >= 0");
    if (K % 32 != 0) throw ArgumentError("K must be a multiple of 32 (got " + std::to_string(K) + ")");
    if (N > std::numeric_limits<int>::max() || K > std::numeric_limits<int>::max())
        throw ArgumentError("N or K is too large");
    int M = 1;
    if (!batched) {
        if (x.ndim() != 1 || x.shape[0] != K)
            throw ArgumentError("x must be 1-D with K = " + std::to_string(K) + " elements");
    } else {
        if (x.ndim() != 2 || x.shape[1] != K)
            throw ArgumentError("x must be 2-D [M, K] with K = " + std::to_string(K));
        if (x.shape[0] > 8) throw ArgumentError("at most 8 rows of x per call (got " + std::to_string(x.shape[0]) + ")");
        M = (int)x.shape[0];
    }
    const py::ssize_t row = K / 32 * block_bytes;
    if (w.size() != N * row)
        throw ArgumentError("Wq must hold N*K/32*" + std::to_string(block_bytes) + " = " + std::to_string(N * row) +
                            " bytes (got " + std::to_string(w.size()) + ")");
    const int dev = x.device ? x.device_id : (w.device ? w.device_id : current_device_hint);
    smk_ctx* c = ctx_for(dev);

    py::object result;
    float* yp = nullptr;
    bool y_device = false;
    if (out.is_none()) {
        if (x.device) throw ArgumentError("out= is required when x is a CUDA array");
        std::vector<py::ssize_t> shp = batched ? std::vector<py::ssize_t>{M, (py::ssize_t)N}
                                               : std::vector<py::ssize_t>{(py::ssize_t)N};
        py::array_t<float> y = result_array(shp);
        yp = y.mutable_data();
        result = y;
    } else {
        const Arr o = as_arr(out);
        validate_array(o, "out");
        check_writeable(o, "out");
        if (o.size() != (int64_t)M * N) throw ArgumentError("out must hold M*N float32 values");
        yp = static_cast<float*>(o.ptr);
        y_device = o.device;
        result = out;
    }
    const bool all_device = x.device && w.device && y_device;
    const bool async = all_device && !stream.is_none();
    void* strm = async ? reinterpret_cast<void*>(stream.cast<uintptr_t>()) : nullptr;   // read with the GIL held
    smk_status st;
    {
        py::gil_scoped_release release;
        if (async) {
            st = smk_gemv_q(c, fmt, M, (int)N, (int)K, static_cast<const float*>(x.ptr), K,
                            static_cast<const uint8_t*>(w.ptr), yp, N, strm);
        } else {
            st = smk_gemv_q_host(c, fmt, M, (int)N, (int)K, static_cast<const float*>(x.ptr),
                                 static_cast<const uint8_t*>(w.ptr), yp);
        }
    }
    check(st);
    return result;
}

// ---- quantize (pybind_entry.cpp:914-938,981-995) ------------------------------

py::object quantize_blocks(const py::handle& wh, int block_bytes, smk_qformat fmt, const char* too_large,
                           const py::object& out, const py::object& stream) {
    const Arr W = as_arr(wh);
    validate_array(W, "W");
    if (W.ndim() < 1) throw ArgumentError("W must have at least 1 dimension (rows of K values)");
    const int64_t K = W.shape.back();
    if (K % 32 != 0)
        throw ArgumentError("K (the last dimension of W) must be a multiple of 32 (got " + std::to_string(K) + ")");
    if (K > std::numeric_limits<int>::max()) throw ArgumentError("K is too large");
    const int64_t rows = K == 0 ? 0 : W.size() / K;
    std::vector<py::ssize_t> shape(W.shape.begin(), W.shape.end());
    shape.back() = K / 32 * block_bytes;
    smk_ctx* c = ctx_for(W.device ? W.device_id : current_device_hint);
    py::object result;
    uint8_t* op;
    if (out.is_none()) {
        if (W.device) throw ArgumentError("out= is required when W is a CUDA array");
        py::array_t<uint8_t> o(shape);
        op = o.mutable_data();
        result = o;
    } else {
        const Arr o = as_arr(out);
        if (o.kind != 'u' || o.itemsize != 1) throw DTypeError("out must be uint8");
        check_contiguous(o, "out");
        if (o.size() != rows * (K / 32) * block_bytes) throw ArgumentError("out has the wrong size");
        op = static_cast<uint8_t*>(o.ptr);
        result = out;
    }
    smk_status st;
    {
        py::gil_scoped_release release;
        st = smk_quantize_host(c, fmt, rows, (int)K, static_cast<const float*>(W.ptr), op);
    }
    (void)stream;
    if (st == SMK_ERR_REJECTED) throw ArgumentError(too_large);
    check(st);
    return result;
}

// ---- dense decode GEMV: sgemm / sgemm_f16 / sgemm_bf16 with trans_b ----------

const char* kDecodeOnly =
    "this build implements the decode GEMV on the B200: C = alpha * A @ B.T + beta * C "
    "with trans_b=True, trans_a=False and at most 8 rows of A";

void output_matrix(const py::object& C, int64_t M, int64_t N, Arr* info) {
    if (!py::isinstance<py::array>(C) && !py::hasattr(C, "__cuda_array_interface__"))
        throw DTypeError("C must be a numpy.ndarray of dtype float32 (or None)");
    Arr a = as_arr(C);
    validate_array(a, "C");
    check_writeable(a, "C");
    if (a.ndim() != 2 || a.shape[0] != M || a.shape[1] != N)
        throw ArgumentError("C must have shape [" + std::to_string(M) + "×" + std::to_string(N) + "]");
    *info = a;
}

py::object dense_call(smk_dtype wt, smk_dtype xt, const Arr& A, const Arr& B, int M, int N, int K, float alpha,
                      float beta, const py::object& C, const py::object& stream) {
    smk_ctx* c = ctx_for(A.device ? A.device_id : (B.device ? B.device_id : current_device_hint));
    py::object result;
    float* cp;
    bool c_device = false;
    if (C.is_none()) {
        if (A.device) throw ArgumentError("C is required when A is a CUDA array");
        py::array_t<float> out = result_array({(py::ssize_t)M, (py::ssize_t)N});
        cp = out.mutable_data();
        if (M * (int64_t)N) std::memset(cp, 0, sizeof(float) * (size_t)M * N);
        result = out;
    } else {
        Arr ci;
        output_matrix(C, M, N, &ci);
        cp = static_cast<float*>(ci.ptr);
        c_device = ci.device;
        result = C;
    }
    const bool async = A.device && B.device && c_device && !stream.is_none();
    void* strm = async ? reinterpret_cast<void*>(stream.cast<uintptr_t>()) : nullptr;   // read with the GIL held
    smk_status st;
    {
        py::gil_scoped_release release;
        if (async)
            st = smk_gemv_dense(c, wt, xt, M, N, K, alpha, A.ptr, K, B.ptr, K, beta, cp, N, strm);
        else
            st = smk_gemv_dense_host(c, wt, xt, M, N, K, alpha, A.ptr, B.ptr, beta, cp);
    }
    check(st);
    return result;
}

// The decode shape of trans_b GEMMs; anything else is outside this build.
void decode_shape(const Arr& A, const Arr& B, bool trans_a, bool trans_b, int* M, int* N, int* K) {
    const int64_t m = A.shape[trans_a ? 1 : 0], k = A.shape[trans_a ? 0 : 1];
    const int64_t n = B.shape[trans_b ? 0 : 1], kb = B.shape[trans_b ? 1 : 0];
    if (kb != k) {
        auto dims = [](const Arr& x) {
            return "[" + std::to_string(x.shape[0]) + "×" + std::to_string(x.shape[1]) + "]";
        };
        throw ArgumentError("Shape mismatch: " + std::string(trans_a ? "A.T" : "A") + " is [" + std::to_string(m) +
                            "×" + std::to_string(k) + "] (A is " + dims(A) + ") but " + (trans_b ? "B.T" : "B") +
                            " is [" + std::to_string(kb) + "×" + std::to_string(n) + "] (B is " + dims(B) + ")");
    }
    if (trans_a || !trans_b || m > 8) throw ArgumentError(kDecodeOnly);
    *M = (int)m;
    *N = (int)n;
    *K = (int)k;
}

// ---- INT8 decode GEMV: sgemm_u8s8 with trans_b (pybind_entry.cpp:837-893) ----

const char* kDecodeOnlyU8S8 =
    "this build implements the INT8 decode GEMV on the B200: sgemm_u8s8 with trans_b=True (B as [N, K]) "
    "and at most 8 rows of A";

py::object py_sgemm_u8s8(const py::handle& Ah, const py::handle& Bh, float a_scale, int a_zero_point,
                         const py::handle& Sh, const py::object& C, bool trans_b, const py::object& stream) {
    // The reference's checks, in its order and with its messages (pybind_entry.cpp:849-876).
    const Arr A = as_arr(Ah), B = as_arr(Bh), S = as_arr(Sh);
    if (A.kind != 'u' || A.itemsize != 1) throw DTypeError("A must be uint8 (quantized activations; dtype=np.uint8)");
    if (B.kind != 'i' || B.itemsize != 1) throw DTypeError("B must be int8 (quantized weights; dtype=np.int8)");
    check_float32(S, "b_scales");
    if (A.ndim() != 2) throw ArgumentError("A must be 2-D");
    if (B.ndim() != 2) throw ArgumentError("B must be 2-D");
    if (S.ndim() != 1) throw ArgumentError("b_scales must be 1-D (one scale per output column)");
    check_contiguous(A, "A");
    check_contiguous(B, "B");
    check_contiguous(S, "b_scales");
    if (a_zero_point < 0 || a_zero_point > 255)
        throw ArgumentError("a_zero_point must be in [0, 255] (got " + std::to_string(a_zero_point) + ")");
    if (!std::isfinite(a_scale)) throw ArgumentError("a_scale must be finite");
    const int64_t M = A.shape[0], K = A.shape[1];
    const int64_t N = B.shape[trans_b ? 0 : 1], Kb = B.shape[trans_b ? 1 : 0];
    if (Kb != K)
        throw ArgumentError("Shape mismatch: A is [" + std::to_string(M) + "×" + std::to_string(K) + "] but " +
                            (trans_b ? "B.T" : "B") + " is [" + std::to_string(Kb) + "×" + std::to_string(N) + "]");
    if (S.shape[0] != N)
        throw ArgumentError("b_scales must have N = " + std::to_string(N) + " elements (got " +
                            std::to_string(S.shape[0]) + ")");
    // With no elements the layout of B does not matter; otherwise the decode contract.
    if (M * N * K != 0 && (!trans_b || M > 8)) throw ArgumentError(kDecodeOnlyU8S8);
    if (N > std::numeric_limits<int>::max() || K > std::numeric_limits<int>::max())
        throw ArgumentError("N or K is too large");
    py::object result;
    float* cp;
    bool c_device = false;
    if (C.is_none()) {
        if (A.device) throw ArgumentError("C is required when A is a CUDA array");
        py::array_t<float> out = result_array({(py::ssize_t)M, (py::ssize_t)N});
        cp = out.mutable_data();
        result = out;
    } else {
        Arr ci;
        output_matrix(C, M, N, &ci);
        cp = static_cast<float*>(ci.ptr);
        c_device = ci.device;
        result = C;
    }
    if (M * N == 0) return result;
    smk_ctx* c = ctx_for(A.device ? A.device_id : (B.device ? B.device_id : current_device_hint));
    const bool async = A.device && B.device && S.device && c_device && !stream.is_none();
    void* strm = async ? reinterpret_cast<void*>(stream.cast<uintptr_t>()) : nullptr;   // read with the GIL held
    smk_status st;
    {
        py::gil_scoped_release release;
        if (async)
            st = smk_gemv_u8s8(c, (int)M, (int)N, (int)K, static_cast<const uint8_t*>(A.ptr), K, a_zero_point,
                               static_cast<const int8_t*>(B.ptr), K, a_scale, static_cast<const float*>(S.ptr), cp, N,
                               strm);
        else
            st = smk_gemv_u8s8_host(c, (int)M, (int)N, (int)K, static_cast<const uint8_t*>(A.ptr), a_zero_point,
                                    static_cast<const int8_t*>(B.ptr), a_scale, static_cast<const float*>(S.ptr), cp);
    }
    check(st);
    return result;
}

py::object py_sgemm(const py::handle& Ah, const py::handle& Bh, const py::object& C, float alpha, float beta,
                    const std::string& isa, bool trans_a, bool trans_b, const py::object& stream) {
    if (!isa.empty()) {
        if (isa == "scalar" || isa == "avx2" || isa == "avx512")
            throw std::runtime_error("isa='" + isa +
                                     "' was requested but this build does not include it. Use isa='' (the kernels "
                                     "chosen for this CPU) or check simd_ml_kernels.build_info()['isa_usable'].");
        throw ArgumentError("isa must be one of: '', 'scalar', 'avx2', 'avx512' (got '" + isa + "')");
    }
    const Arr A = as_arr(Ah), B = as_arr(Bh);
    validate_array(A, "A");
    validate_array(B, "B");
    if (A.ndim() != 2) throw ArgumentError("A must be 2-D");
    if (B.ndim() != 2) throw ArgumentError("B must be 2-D");
    int M, N, K;
    decode_shape(A, B, trans_a, trans_b, &M, &N, &K);
    return dense_call(SMK_F32, SMK_F32, A, B, M, N, K, alpha, beta, C, stream);
}

py::object py_sgemm_f16(const py::handle& Ah, const py::handle& Bh, float alpha, float beta, const py::object& C,
                        bool trans_b, const py::object& stream) {
    const Arr A = as_arr(Ah), B = as_arr(Bh);
    auto check_f16 = [](const Arr& a, const char* name) {
        if (a.kind != 'f' || a.itemsize != 2)
            throw DTypeError(std::string(name) + " must be float16 (dtype=np.float16). "
                             "Call arr.astype(np.float16) before passing.");
        if (!a.contiguous)
            throw ArgumentError(std::string(name) + " must be C-contiguous. "
                                "Call numpy.ascontiguousarray(arr) before passing.");
    };
    check_f16(A, "A");
    check_f16(B, "B");
    if (A.ndim() != 2) throw ArgumentError("A must be 2-D");
    if (B.ndim() != 2) throw ArgumentError("B must be 2-D");
    int M, N, K;
    {
        const int64_t m = A.shape[0], k = A.shape[1];
        const int64_t n = B.shape[trans_b ? 0 : 1], kb = B.shape[trans_b ? 1 : 0];
        if (kb != k)
            throw ArgumentError("Shape mismatch: A is [" + std::to_string(m) + "×" + std::to_string(k) + "] but " +
                                (trans_b ? "B.T" : "B") + " is [" + std::to_string(kb) + "×" + std::to_string(n) +
                                "] (B is [" + std::to_string(B.shape[0]) + "×" + std::to_string(B.shape[1]) + "])");
        if (!trans_b || m > 8) throw ArgumentError(kDecodeOnly);
        M = (int)m; N = (int)n; K = (int)k;
    }
    return dense_call(SMK_F16, SMK_F16, A, B, M, N, K, alpha, beta, C, stream);
}

py::object py_sgemm_bf16(const py::handle& Ah, const py::handle& Bh, float alpha, float beta, const py::object& C,
                         bool trans_b, const py::object& stream) {
    const Arr A = as_arr(Ah), B = as_arr(Bh);
    // uint16 BF16 bit patterns or ml_dtypes.bfloat16 (pybind_entry.cpp:772-806).
    auto check_bf16 = [](const Arr& a, const char* name) {
        if (a.kind == 'u' && a.itemsize == 2) return;
        if (a.itemsize == 2 && a.name == "bfloat16") return;
        std::string msg = std::string(name) +
                          " must hold BF16 values: a uint16 array of BF16 bit patterns or an "
                          "ml_dtypes.bfloat16 array (got " + a.name + ").";
        if (a.kind == 'f' && a.itemsize == 2)
            msg += " float16 is IEEE half precision, not BF16: use sgemm_f16 for float16 inputs.";
        throw DTypeError(msg);
    };
    check_bf16(A, "A");
    check_bf16(B, "B");
    if (A.ndim() != 2) throw ArgumentError("A must be 2-D");
    if (B.ndim() != 2) throw ArgumentError("B must be 2-D");
    check_contiguous(A, "A");
    check_contiguous(B, "B");
    int M, N, K;
    {
        const int64_t m = A.shape[0], k = A.shape[1];
        const int64_t n = B.shape[trans_b ? 0 : 1], kb = B.shape[trans_b ? 1 : 0];
        if (kb != k)
            throw ArgumentError("Shape mismatch: A is [" + std::to_string(m) + "×" + std::to_string(k) + "] but " +
                                (trans_b ? "B.T" : "B") + " is [" + std::to_string(kb) + "×" + std::to_string(n) +
                                "] (B is [" + std::to_string(B.shape[0]) + "×" + std::to_string(B.shape[1]) + "])");
        if (!trans_b || m > 8) throw ArgumentError(kDecodeOnly);
        M = (int)m; N = (int)n; K = (int)k;
    }
    return dense_call(SMK_BF16, SMK_BF16, A, B, M, N, K, alpha, beta, C, stream);
}

// gemv_dense(x, W, out=None): x float32 [M, K] (M <= 8) against W [N, K] in
// float32 / float16 / bfloat16 bits — FP32 activations with 16-bit weights.
py::object py_gemv_dense(const py::handle& xh, const py::handle& wh, const std::string& wtype, const py::object& out,
                         const py::object& stream) {
    const Arr x = as_arr(xh), W = as_arr(wh);
    validate_array(x, "x");
    check_contiguous(W, "W");
    smk_dtype wt;
    if (wtype == "float32") {
        check_float32(W, "W");
        wt = SMK_F32;
    } else if (wtype == "float16") {
        if (W.itemsize != 2) throw DTypeError("W must hold 2-byte float16 values");
        wt = SMK_F16;
    } else if (wtype == "bfloat16") {
        if (W.itemsize != 2) throw DTypeError("W must hold 2-byte bfloat16 values");
        wt = SMK_BF16;
    } else {
        throw ArgumentError("wtype must be 'float32', 'float16' or 'bfloat16'");
    }
    if (x.ndim() != 2 || W.ndim() != 2) throw ArgumentError("x must be [M, K] and W [N, K]");
    if (x.shape[1] != W.shape[1]) throw ArgumentError("x and W must have the same K");
    if (x.shape[0] > 8) throw ArgumentError(kDecodeOnly);
    return dense_call(wt, SMK_F32, x, W, (int)x.shape[0], (int)W.shape[0], (int)x.shape[1], 1.0f, 0.0f, out, stream);
}

// ---- test hooks ----------------------------------------------------------------

void py_quantize_x(uintptr_t x, int M, int K, uintptr_t qs, uintptr_t dx, uintptr_t stream) {
    smk_ctx* c = ctx_for(current_device_hint);
    check(smk_quantize_x(c, M, K, reinterpret_cast<const float*>(x), K, reinterpret_cast<int8_t*>(qs),
                         reinterpret_cast<float*>(dx), reinterpret_cast<void*>(stream)));
}

void py_block_sums(int fmt, uintptr_t x, int M, int N, int K, uintptr_t w, uintptr_t out, uintptr_t stream) {
    smk_ctx* c = ctx_for(current_device_hint);
    check(smk_block_sums(c, (smk_qformat)fmt, M, N, K, reinterpret_cast<const float*>(x), K,
                         reinterpret_cast<const uint8_t*>(w), reinterpret_cast<int32_t*>(out),
                         reinterpret_cast<void*>(stream)));
}

}  // namespace

PYBIND11_MODULE(_core, m) {
    m.doc() = "simd_ml_kernels._core (B200 build): the decode-GEMV path of simd-ml-kernels on sm_100a CUDA kernels.";

    py::register_exception<DTypeError>(m, "DTypeError",
                                       py::make_tuple(py::handle(PyExc_TypeError), py::handle(PyExc_RuntimeError)))
        .attr("__doc__") = "An array argument has the wrong dtype (TypeError and RuntimeError).";
    py::register_exception<ArgumentError>(
        m, "ArgumentError", py::make_tuple(py::handle(PyExc_ValueError), py::handle(PyExc_RuntimeError)))
        .attr("__doc__") = "An argument has the wrong shape, layout or value (ValueError and RuntimeError).";

    m.def("gemv_q4_0",
          [](py::handle x, py::handle Wq, py::ssize_t N, py::ssize_t K, py::object out, py::object stream) {
              return gemv_blocks(x, as_arr(Wq), N, K, 18, "q4_0", SMK_Q4_0, out, stream, false);
          },
          py::arg("x"), py::arg("Wq"), py::arg("N"), py::arg("K"), py::kw_only(), py::arg("out") = py::none(),
          py::arg("stream") = py::none(),
          "gemv_q4_0(x, Wq, N, K) -> float32 [N]: y = x @ W.T, W as quantize_q4_0 blocks; x quantized to Q8 inside.");
    m.def("gemv_q8_0",
          [](py::handle x, py::handle Wq, py::ssize_t N, py::ssize_t K, py::object out, py::object stream) {
              return gemv_blocks(x, as_arr(Wq), N, K, 34, "q8_0", SMK_Q8_0, out, stream, false);
          },
          py::arg("x"), py::arg("Wq"), py::arg("N"), py::arg("K"), py::kw_only(), py::arg("out") = py::none(),
          py::arg("stream") = py::none(),
          "gemv_q8_0(x, Wq, N, K) -> float32 [N]: y = x @ W.T, W as quantize_q8_0 blocks.");
    m.def("gemv_q4_0_batch",
          [](py::handle x, py::handle Wq, py::ssize_t N, py::ssize_t K, py::object out, py::object stream) {
              return gemv_blocks(x, as_arr(Wq), N, K, 18, "q4_0", SMK_Q4_0, out, stream, true);
          },
          py::arg("x"), py::arg("Wq"), py::arg("N"), py::arg("K"), py::kw_only(), py::arg("out") = py::none(),
          py::arg("stream") = py::none(),
          "gemv_q4_0_batch(x [M, K], Wq, N, K) -> float32 [M, N], M <= 8: W read once for all rows; each row "
          "as one gemv_q4_0 call.");
    m.def("gemv_q8_0_batch",
          [](py::handle x, py::handle Wq, py::ssize_t N, py::ssize_t K, py::object out, py::object stream) {
              return gemv_blocks(x, as_arr(Wq), N, K, 34, "q8_0", SMK_Q8_0, out, stream, true);
          },
          py::arg("x"), py::arg("Wq"), py::arg("N"), py::arg("K"), py::kw_only(), py::arg("out") = py::none(),
          py::arg("stream") = py::none());
    m.def("quantize_q4_0",
          [](py::handle W, py::object out, py::object stream) {
              return quantize_blocks(W, 18, SMK_Q4_0,
                                     "W must be finite, with |W| below 8 * 65520 = 524160 (a block scale "
                                     "max|w|/8 must fit float16)",
                                     out, stream);
          },
          py::arg("W"), py::kw_only(), py::arg("out") = py::none(), py::arg("stream") = py::none(),
          "quantize_q4_0(W) -> uint8 [..., K/32*18]: ggml Q4_0 blocks, byte-identical to quantize_row_q4_0_ref.");
    m.def("quantize_q8_0",
          [](py::handle W, py::object out, py::object stream) {
              return quantize_blocks(W, 34, SMK_Q8_0,
                                     "W must be finite, with |W| below 127 * 65520 = 8321040 (a block scale "
                                     "max|w|/127 must fit float16)",
                                     out, stream);
          },
          py::arg("W"), py::kw_only(), py::arg("out") = py::none(), py::arg("stream") = py::none(),
          "quantize_q8_0(W) -> uint8 [..., K/32*34]: ggml Q8_0 blocks, byte-identical to quantize_row_q8_0_ref.");
    m.def("sgemm", &py_sgemm, py::arg("A"), py::arg("B"), py::arg("C") = py::none(), py::arg("alpha") = 1.0f,
          py::arg("beta") = 0.0f, py::arg("isa") = "", py::kw_only(), py::arg("trans_a") = false,
          py::arg("trans_b") = false, py::arg("stream") = py::none(),
          "sgemm(A, B, C=None, alpha=1, beta=0, isa='', *, trans_a=False, trans_b=False): the decode GEMV "
          "x @ W.T (trans_b=True, M <= 8) in float32.");
    m.def("sgemm_f16", &py_sgemm_f16, py::arg("A"), py::arg("B"), py::arg("alpha") = 1.0f, py::arg("beta") = 0.0f,
          py::arg("C") = py::none(), py::kw_only(), py::arg("trans_b") = false, py::arg("stream") = py::none());
    m.def("sgemm_bf16", &py_sgemm_bf16, py::arg("A"), py::arg("B"), py::arg("alpha") = 1.0f,
          py::arg("beta") = 0.0f, py::arg("C") = py::none(), py::kw_only(), py::arg("trans_b") = false,
          py::arg("stream") = py::none());
    m.def("sgemm_u8s8", &py_sgemm_u8s8, py::arg("A"), py::arg("B"), py::arg("a_scale"), py::arg("a_zero_point"),
          py::arg("b_scales"), py::arg("C") = py::none(), py::kw_only(), py::arg("trans_b") = false,
          py::arg("stream") = py::none(),
          "sgemm_u8s8(A, B, a_scale, a_zero_point, b_scales, C=None, *, trans_b=False) -> float32 [M, N]: "
          "C = a_scale * b_scales[j] * sum_k (A - a_zero_point) * B.T, A uint8 [M, K] (M <= 8), B int8 [N, K] "
          "with trans_b=True; exact integer sums, the reference's scalar-table rounding.");
    m.def("gemv_dense", &py_gemv_dense, py::arg("x"), py::arg("W"), py::arg("wtype") = "float32",
          py::arg("out") = py::none(), py::arg("stream") = py::none());
    // The device path of the Python package for torch CUDA tensors: the
    // package validated dtypes, shapes and contiguity (the reference's
    // checks and messages); this only launches.
    m.def("_gemv_q_dev",
          [](int fmt, int M, int N, int K, uintptr_t x, long long ldx, uintptr_t w, uintptr_t y, long long ldy,
             uintptr_t stream, int device) {
              smk_ctx* c = ctx_for(device);
              smk_status st;
              {
                  py::gil_scoped_release release;
                  st = smk_gemv_q(c, (smk_qformat)fmt, M, N, K, reinterpret_cast<const float*>(x), ldx,
                                  reinterpret_cast<const uint8_t*>(w), reinterpret_cast<float*>(y), ldy,
                                  reinterpret_cast<void*>(stream));
              }
              check(st);
          });
    // Host activations against weights already resident on a device (a
    // torch CUDA tensor the package checked: uint8, contiguous): the
    // reference's synchronous NumPy contract without describing W through
    // __cuda_array_interface__ on every call.
    m.def("_gemv_q_host_dw",
          [](int fmt, py::handle x, uintptr_t w, long long wbytes, py::ssize_t N, py::ssize_t K, bool batched,
             int device) {
              Arr wa;
              wa.ptr = reinterpret_cast<void*>(w);
              wa.shape = {wbytes};
              wa.kind = 'u';
              wa.itemsize = 1;
              wa.device = true;
              wa.device_id = device;
              const bool q4 = fmt == 0;
              return gemv_blocks(x, wa, N, K, q4 ? 18 : 34, q4 ? "q4_0" : "q8_0", q4 ? SMK_Q4_0 : SMK_Q8_0,
                                 py::none(), py::none(), batched);
          });
    // Row-sharded GEMV with the all-gather of y fused in (simd_ml_kernels.shard).
    m.def("_gather_create", [](int world, int rank, int npad, int m_max, int device) {
        smk_ctx* c = ctx_for(device);
        smk_gather* g = nullptr;
        char h[SMK_IPC_HANDLE_BYTES];
        check(smk_gather_create(c, world, rank, npad, m_max, &g, h));
        return py::make_tuple(reinterpret_cast<uintptr_t>(g), py::bytes(h, SMK_IPC_HANDLE_BYTES));
    });
    m.def("_gather_connect", [](uintptr_t g, py::bytes handles) {
        const std::string hs = handles;
        check(smk_gather_connect(reinterpret_cast<smk_gather*>(g), hs.data()));
    });
    m.def("_gather_destroy", [](uintptr_t g) { check(smk_gather_destroy(reinterpret_cast<smk_gather*>(g))); });
    m.def("_gather_barrier", [](uintptr_t g, uintptr_t stream) {
        check(smk_gather_barrier(reinterpret_cast<smk_gather*>(g), reinterpret_cast<void*>(stream)));
    });
    m.def("_gather_pingpong", [](uintptr_t g, int iters, int relaxed, uintptr_t stream) {
        unsigned long long ns = 0;
        {
            py::gil_scoped_release nogil;
            check(smk_gather_pingpong(reinterpret_cast<smk_gather*>(g), iters, relaxed, &ns, reinterpret_cast<void*>(stream)));
        }
        return ns;
    });
    m.def("_gemv_q_gather", [](uintptr_t g, int fmt, int M, int N, int K, uintptr_t x, long long ldx, uintptr_t w,
                               uintptr_t stream, int device) {
        smk_ctx* c = ctx_for(device);
        float* y = nullptr;
        smk_status st;
        {
            py::gil_scoped_release release;
            st = smk_gemv_q_gather(c, reinterpret_cast<smk_gather*>(g), (smk_qformat)fmt, M, N, K,
                                   reinterpret_cast<const float*>(x), ldx, reinterpret_cast<const uint8_t*>(w), &y,
                                   reinterpret_cast<void*>(stream));
        }
        check(st);
        return reinterpret_cast<uintptr_t>(y);
    });
    m.def("_gemv_q_silu_mul_dev", [](int fmt, int M, int N, int K, uintptr_t g, long long ldg, uintptr_t u,
                                     long long ldu, uintptr_t w, uintptr_t y, long long ldy, uintptr_t stream,
                                     int device) {
        smk_ctx* c = ctx_for(device);
        smk_status st;
        {
            py::gil_scoped_release release;
            st = smk_gemv_q_silu_mul(c, (smk_qformat)fmt, M, N, K, reinterpret_cast<const float*>(g), ldg,
                                     reinterpret_cast<const float*>(u), ldu, reinterpret_cast<const uint8_t*>(w),
                                     reinterpret_cast<float*>(y), ldy, reinterpret_cast<void*>(stream));
        }
        check(st);
    });
    m.def("_silu_mul", [](long long n, uintptr_t g, uintptr_t u, uintptr_t out, uintptr_t stream, int device) {
        check(smk_silu_mul(ctx_for(device), n, reinterpret_cast<const float*>(g), reinterpret_cast<const float*>(u),
                           reinterpret_cast<float*>(out), reinterpret_cast<void*>(stream)));
    });
    m.def("_dequantize_rows", [](int fmt, int N, int K, uintptr_t w, uintptr_t rows, int nrows, uintptr_t out,
                                 long long ldo, uintptr_t stream, int device) {
        check(smk_dequantize_rows(ctx_for(device), (smk_qformat)fmt, N, K, reinterpret_cast<const uint8_t*>(w),
                                  reinterpret_cast<const int32_t*>(rows), nrows, reinterpret_cast<float*>(out), ldo,
                                  reinterpret_cast<void*>(stream)));
    });
    m.def("_add_rmsnorm", [](int M, int n, uintptr_t x, long long ldx, uintptr_t delta, long long ldd, uintptr_t w,
                             double eps, uintptr_t h, long long ldh, uintptr_t stream, int device) {
        check(smk_add_rmsnorm(ctx_for(device), M, n, reinterpret_cast<float*>(x), ldx,
                              reinterpret_cast<const float*>(delta), ldd, reinterpret_cast<const float*>(w), eps,
                              reinterpret_cast<float*>(h), ldh, reinterpret_cast<void*>(stream)));
    });
    m.def("_rope_kv", [](uintptr_t qkv, uintptr_t inv_freq, uintptr_t pos_dev, int pos, int nh, int nkv, int hd,
                         int interleaved, uintptr_t q_out, uintptr_t kc, uintptr_t vc, int cap, uintptr_t stream,
                         int device) {
        check(smk_rope_kv(ctx_for(device), reinterpret_cast<const float*>(qkv), reinterpret_cast<const float*>(inv_freq),
                          reinterpret_cast<const int32_t*>(pos_dev), pos, nh, nkv, hd, interleaved,
                          reinterpret_cast<float*>(q_out), reinterpret_cast<float*>(kc), reinterpret_cast<float*>(vc),
                          cap, reinterpret_cast<void*>(stream)));
    });
    m.def("_attention_decode", [](uintptr_t q, uintptr_t kc, uintptr_t vc, uintptr_t out, uintptr_t len_dev, int len,
                                  int max_len, int nh, int nkv, int hd, int cap, float scale, uintptr_t stream,
                                  int device) {
        check(smk_attention_decode(ctx_for(device), reinterpret_cast<const float*>(q),
                                   reinterpret_cast<const float*>(kc), reinterpret_cast<const float*>(vc),
                                   reinterpret_cast<float*>(out), reinterpret_cast<const int32_t*>(len_dev), len,
                                   max_len, nh, nkv, hd, cap, scale, reinterpret_cast<void*>(stream)));
    });
    m.def("_gemv_q_fused", [](int fmt, int M, int N, int K, uintptr_t x, long long ldx, uintptr_t up, long long ldu,
                              uintptr_t w_norm, double eps, uintptr_t w, uintptr_t r, long long ldr, uintptr_t y,
                              long long ldy, uintptr_t stream, int device) {
        smk_ctx* c = ctx_for(device);
        smk_status st;
        {
            py::gil_scoped_release release;
            st = smk_gemv_q_fused(c, (smk_qformat)fmt, M, N, K, reinterpret_cast<const float*>(x), ldx,
                                  reinterpret_cast<const float*>(up), ldu, reinterpret_cast<const float*>(w_norm), eps,
                                  reinterpret_cast<const uint8_t*>(w), reinterpret_cast<const float*>(r), ldr,
                                  reinterpret_cast<float*>(y), ldy, reinterpret_cast<void*>(stream));
        }
        check(st);
    });
    m.def("_rope_attention", [](uintptr_t qkv, uintptr_t inv_freq, uintptr_t pos_dev, int pos, int max_len, int nh,
                                int nkv, int hd, int interleaved, uintptr_t kc, uintptr_t vc, int cap, float scale,
                                uintptr_t out, uintptr_t stream, int device) {
        check(smk_rope_attention(ctx_for(device), reinterpret_cast<const float*>(qkv),
                                 reinterpret_cast<const float*>(inv_freq), reinterpret_cast<const int32_t*>(pos_dev),
                                 pos, max_len, nh, nkv, hd, interleaved, reinterpret_cast<float*>(kc),
                                 reinterpret_cast<float*>(vc), cap, scale, reinterpret_cast<float*>(out),
                                 reinterpret_cast<void*>(stream)));
    });
    m.def("version", []() { return std::string(smk_version()); });
    m.def("_set_device", [](int d) { current_device_hint = d; });
    m.def("_ctx_set", [](int option, long long value) { check(smk_ctx_set(ctx_for(current_device_hint), option, value)); });
    m.def("_device_error", [](uintptr_t stream) {
        unsigned code = 0;
        check(smk_device_error(ctx_for(current_device_hint), &code, reinterpret_cast<void*>(stream)));
        return code;
    });
    m.def("_quantize_x", &py_quantize_x);
    m.def("_block_sums", &py_block_sums);
    m.def("_check_x_arith", []() {
        unsigned long long bad[3] = {0, 0, 0};
        {
            py::gil_scoped_release nogil;
            check(smk_check_x_arith(ctx_for(current_device_hint), bad));
        }
        return py::make_tuple(bad[0], bad[1], bad[2]);
    });
}
