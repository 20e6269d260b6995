"""simd_ml_kernels — the B200 (sm_100a) build of simd-ml-kernels' decode-GEMV path.

Drop-in for the reference package's GEMV entry points (same names,
arguments, return types, error classes and messages):

    gemv_q4_0(x, Wq, N, K)        quantize_q4_0(W)
    gemv_q8_0(x, Wq, N, K)        quantize_q8_0(W)
    sgemm(x, W, trans_b=True)     sgemm_f16(x, W, trans_b=True)     sgemm_bf16(x, W, trans_b=True)
    sgemm_u8s8(A, W, a_scale, a_zero_point, b_scales, trans_b=True)

Every call runs CUDA kernels on a Blackwell GPU (there is no CPU path).
NumPy operands are copied to the device and the call returns NumPy results,
as the reference's calls do. torch CUDA tensors stay on the device: the call
is queued on torch's current stream and returns a CUDA tensor.

Additions for this build: gemv_q4_0_batch / gemv_q8_0_batch (up to 8 rows of
x against one read of W), gemv_dense (float32 x against float32 / float16 /
bfloat16 W), gemv_q4_0_silu_mul / gemv_q8_0_silu_mul (the decoder's down
projection on silu(gate) * up), set_pdl (programmatic dependent launch
between GEMVs), and the gguf submodule (llama.cpp model files onto the
device, embedding rows).
"""

from __future__ import annotations

import os as _os
import sys as _sys

from numpy import ndarray as _np_ndarray

from . import _core
from ._core import ArgumentError, DTypeError

__version__ = "0.1.0"

__all__ = [
    "ArgumentError",
    "DTypeError",
    "build_info",
    "detected_isa",
    "gemv_dense",
    "gemv_q4_0",
    "gemv_q4_0_batch",
    "gemv_q8_0",
    "gemv_q8_0_batch",
    "gemv_q4_0_silu_mul",
    "gemv_q8_0_silu_mul",
    "get_num_threads",
    "library_path",
    "quantize_q4_0",
    "quantize_q8_0",
    "set_num_threads",
    "set_pdl",
    "sgemm",
    "sgemm_bf16",
    "sgemm_f16",
    "sgemm_u8s8",
    "silu_mul",
]


def library_path() -> str:
    """Path of libsmk_cuda.so, the C ABI this package calls."""
    return _os.path.join(_os.path.dirname(_os.path.abspath(__file__)), "libsmk_cuda.so")


# ---- torch CUDA tensors --------------------------------------------------------

def _torch():
    return _sys.modules.get("torch")


def _is_cuda_tensor(a) -> bool:
    t = _torch()
    return t is not None and isinstance(a, t.Tensor) and a.is_cuda


class _Cai:
    """A __cuda_array_interface__ view of a torch CUDA tensor with a chosen
    typestr (bfloat16 has none of its own: it travels as 2-byte unsigned bits)."""

    __slots__ = ("__cuda_array_interface__", "tensor")

    def __init__(self, t, typestr: str | None = None):
        self.tensor = t
        item = t.element_size()
        if typestr is None:
            typestr = _TYPESTR[t.dtype]
        self.__cuda_array_interface__ = {
            "data": (t.data_ptr(), False),
            "shape": tuple(t.shape),
            "strides": tuple(s * item for s in t.stride()),
            "typestr": typestr,
            "version": 2,
        }


_TYPESTR = {}


def _typestr_table():
    t = _torch()
    if not _TYPESTR and t is not None:
        _TYPESTR.update({t.float32: "<f4", t.float16: "<f2", t.bfloat16: "<u2", t.uint8: "|u1", t.int8: "|i1",
                         t.int16: "<i2", t.int32: "<i4", t.float64: "<f8"})
    return _TYPESTR


def _wrap(a):
    if _is_cuda_tensor(a):
        _typestr_table()
        return _Cai(a)
    return a


def _stream_of(a):
    t = _torch()
    return t.cuda.current_stream(a.device).cuda_stream


def _device_call(fn, tensors, out_shape, out_dtype, *args, **kw):
    """Run fn on CUDA tensors: allocate the output on the tensors' device and
    queue the call on torch's current stream there."""
    t = _torch()
    dev = next(x.device for x in tensors if _is_cuda_tensor(x))
    out = kw.pop("out", None)
    if out is None:
        out = t.empty(out_shape, dtype=out_dtype, device=dev)
    with t.cuda.device(dev):
        _core._set_device(dev.index if dev.index is not None else t.cuda.current_device())
        fn(*args, out=_wrap(out), stream=_stream_of(out), **kw)
    return out


# ---- the reference's entry points -------------------------------------------------

def _set_device_of(*arrays) -> None:
    for a in arrays:
        if _is_cuda_tensor(a):
            _core._set_device(a.device.index)
            return


_raw_stream = None


def _current_stream(index):
    """The raw cudaStream_t of torch's current stream on a device."""
    global _raw_stream
    t = _torch()
    if _raw_stream is None:
        _raw_stream = getattr(t._C, "_cuda_getCurrentRawStream", False)
    if _raw_stream:
        return _raw_stream(index)
    return t.cuda.current_stream(index).cuda_stream


def _check_dev_gemv(fmt, x, Wq, N, K, out, batched):
    """The reference's argument checks (pybind_entry.cpp:944-971), for CUDA tensors."""
    t = _torch()
    if x.dtype != t.float32:
        raise DTypeError("x must be float32 (dtype=np.float32). Call arr.astype(np.float32) before passing.")
    if not x.is_contiguous():
        raise ArgumentError("x must be C-contiguous. Call numpy.ascontiguousarray(arr) before passing.")
    if Wq.dtype != t.uint8:
        raise DTypeError(f"Wq must be uint8 (blocks from quantize_{fmt}; dtype=np.uint8)")
    if not Wq.is_contiguous():
        raise ArgumentError("Wq must be C-contiguous. Call numpy.ascontiguousarray(arr) before passing.")
    if N < 0 or K < 0:
        raise ArgumentError("N and K must be >= 0")
    if K % 32:
        raise ArgumentError(f"K must be a multiple of 32 (got {K})")
    if not batched:
        if x.dim() != 1 or x.shape[0] != K:
            raise ArgumentError(f"x must be 1-D with K = {K} elements")
        M = 1
    else:
        if x.dim() != 2 or x.shape[1] != K:
            raise ArgumentError(f"x must be 2-D [M, K] with K = {K}")
        M = x.shape[0]
        if M > 8:
            raise ArgumentError(f"at most 8 rows of x per call (got {M})")
    bpb = 18 if fmt == "q4_0" else 34
    if Wq.numel() != N * (K // 32) * bpb:
        raise ArgumentError(f"Wq must hold N*K/32*{bpb} = {N * (K // 32) * bpb} bytes (got {Wq.numel()})")
    if Wq.device != x.device:
        raise ArgumentError("x and Wq must be on the same device")
    if out is not None and (out.dtype != t.float32 or not out.is_contiguous() or out.numel() != M * N
                            or out.device != x.device):
        raise ArgumentError("out must be a contiguous float32 CUDA tensor of M*N values on x's device")
    return M


def _gemv(fmt, core_fn, x, Wq, N, K, out, batched):
    """x a CUDA tensor: validated here, then queued on torch's current stream;
    returns a CUDA tensor. x in host memory: the reference's synchronous
    contract (weights may be device-resident); returns NumPy."""
    if type(x) is not _np_ndarray and _is_cuda_tensor(x):
        t = _torch()
        M = _check_dev_gemv(fmt, x, Wq, N, K, out, batched)
        if out is None:
            out = t.empty((M, N) if batched else (N,), dtype=t.float32, device=x.device)
        index = x.device.index if x.device.index is not None else t.cuda.current_device()
        _core._gemv_q_dev(0 if fmt == "q4_0" else 1, M, N, K, x.data_ptr(), K, Wq.data_ptr(), out.data_ptr(), N,
                          _current_stream(index), index)
        return out
    if out is None and _is_cuda_tensor(Wq):
        # Host x, device-resident weights: checked here, passed as a pointer.
        t = _torch()
        if Wq.dtype != t.uint8:
            raise DTypeError(f"Wq must be uint8 (blocks from quantize_{fmt}; dtype=np.uint8)")
        if not Wq.is_contiguous():
            raise ArgumentError("Wq must be C-contiguous. Call numpy.ascontiguousarray(arr) before passing.")
        return _core._gemv_q_host_dw(0 if fmt == "q4_0" else 1, x, Wq.data_ptr(), Wq.numel(), N, K, batched,
                                     Wq.get_device())
    _set_device_of(Wq, out)
    return core_fn(x, _wrap(Wq), N, K, out=_wrap(out) if out is not None else None)


def gemv_q4_0(x, Wq, N, K, *, out=None):
    """y = x @ W.T [N] float32 for one row x [K], W given as quantize_q4_0 blocks
    (N rows of K/32 blocks of 18 bytes); x is quantized to Q8 blocks inside."""
    return _gemv("q4_0", _core.gemv_q4_0, x, Wq, N, K, out, False)


def gemv_q8_0(x, Wq, N, K, *, out=None):
    """y = x @ W.T [N] float32, W given as quantize_q8_0 blocks (34 bytes per 32 values)."""
    return _gemv("q8_0", _core.gemv_q8_0, x, Wq, N, K, out, False)


def gemv_q4_0_batch(x, Wq, N, K, *, out=None):
    """Y = X @ W.T [M, N] for up to 8 rows of X [M, K]; row m equals gemv_q4_0(X[m], Wq, N, K)."""
    return _gemv("q4_0", _core.gemv_q4_0_batch, x, Wq, N, K, out, True)


def gemv_q8_0_batch(x, Wq, N, K, *, out=None):
    return _gemv("q8_0", _core.gemv_q8_0_batch, x, Wq, N, K, out, True)


def _silu_mul_gemv(fmt, gate, up, Wq, N, K, out):
    """The decode step's down projection, y = (silu(gate) * up) @ W.T, with the
    SwiGLU product formed once while x is quantized (CUDA tensors; gate and up [K]
    or [M, K], M <= 8; asynchronous on the current stream)."""
    t = _torch()
    if not (_is_cuda_tensor(gate) and _is_cuda_tensor(up)):
        raise ArgumentError("gate and up must be CUDA tensors")
    if up.shape != gate.shape or up.dtype != gate.dtype or not up.is_contiguous():
        raise ArgumentError("up must be a contiguous tensor of gate's shape and dtype")
    batched = gate.dim() == 2
    M = _check_dev_gemv(fmt, gate, Wq, N, K, out, batched)
    if out is None:
        out = t.empty((M, N) if batched else (N,), dtype=t.float32, device=gate.device)
    index = gate.device.index if gate.device.index is not None else t.cuda.current_device()
    _core._gemv_q_silu_mul_dev(0 if fmt == "q4_0" else 1, M, N, K, gate.data_ptr(), K, up.data_ptr(), K,
                               Wq.data_ptr(), out.data_ptr(), N, _current_stream(index), index)
    return out


def gemv_q4_0_silu_mul(gate, up, Wq, N, K, *, out=None):
    """y = (silu(gate) * up) @ W.T, W as quantize_q4_0 blocks: the reference
    decoder's w_down(silu(w_gate(h)) * w_up(h)) after the gate/up GEMV, with no
    separate SiLU pass: the product (silu(g) = g / (1 + exp(-g))) is formed
    once per call while x is quantized to Q8, and the GEMV reads those blocks."""
    return _silu_mul_gemv("q4_0", gate, up, Wq, N, K, out)


def gemv_q8_0_silu_mul(gate, up, Wq, N, K, *, out=None):
    return _silu_mul_gemv("q8_0", gate, up, Wq, N, K, out)


def silu_mul(gate, up, *, out=None):
    """silu(gate) * up on the device, the arithmetic gemv_*_silu_mul uses."""
    t = _torch()
    if not (_is_cuda_tensor(gate) and _is_cuda_tensor(up)) or gate.dtype != t.float32 or up.shape != gate.shape \
            or up.dtype != t.float32 or not gate.is_contiguous() or not up.is_contiguous():
        raise ArgumentError("gate and up must be contiguous float32 CUDA tensors of one shape")
    if out is None:
        out = t.empty_like(gate)
    index = gate.device.index if gate.device.index is not None else t.cuda.current_device()
    _core._silu_mul(gate.numel(), gate.data_ptr(), up.data_ptr(), out.data_ptr(), _current_stream(index), index)
    return out


def _quantize(core_fn, W, bpb, out):
    if _is_cuda_tensor(W):
        K = W.shape[-1]
        shape = tuple(W.shape[:-1]) + (K // 32 * bpb,)
        return _device_call(core_fn, (W,), shape, _torch().uint8, _wrap(W), out=out)
    return core_fn(W, out=out)


def quantize_q4_0(W, *, out=None):
    """ggml Q4_0 blocks of W [..., K] (K % 32 == 0): uint8 [..., K/32*18], byte-identical to
    ggml's quantize_row_q4_0_ref. Raises ArgumentError for NaN/Inf or |W| >= 524160."""
    return _quantize(_core.quantize_q4_0, W, 18, out)


def quantize_q8_0(W, *, out=None):
    """ggml Q8_0 blocks of W [..., K]: uint8 [..., K/32*34], byte-identical to quantize_row_q8_0_ref."""
    return _quantize(_core.quantize_q8_0, W, 34, out)


def _dense(core_fn, A, B, C, alpha, beta, trans_b, **kw):
    if _is_cuda_tensor(A) or _is_cuda_tensor(B):
        t = _torch()
        if C is None:
            C = t.zeros((A.shape[0], B.shape[0] if trans_b else B.shape[1]), dtype=t.float32, device=A.device)
        with t.cuda.device(A.device):
            _core._set_device(A.device.index)
            core_fn(_wrap(A), _wrap(B), C=_wrap(C), alpha=alpha, beta=beta, trans_b=trans_b,
                    stream=_stream_of(C), **kw)
        return C
    return core_fn(A, B, C=C, alpha=alpha, beta=beta, trans_b=trans_b, **kw)


def sgemm(A, B, C=None, alpha=1.0, beta=0.0, isa="", *, trans_a=False, trans_b=False):
    """C = alpha * A @ B.T + beta * C in float32 for the decode shape: trans_b=True and at most
    8 rows of A (x @ W.T with W [N, K] is sgemm(x, W, trans_b=True)). isa must be ''."""
    return _dense(_core.sgemm, A, B, C, alpha, beta, trans_b, isa=isa, trans_a=trans_a)


def sgemm_f16(A, B, alpha=1.0, beta=0.0, C=None, *, trans_b=False):
    """float16 A [M, K] and B [N, K] (trans_b=True, M <= 8), float32 accumulation and output."""
    return _dense(_core.sgemm_f16, A, B, C, alpha, beta, trans_b)


def sgemm_bf16(A, B, alpha=1.0, beta=0.0, C=None, *, trans_b=False):
    """bfloat16 A and B (uint16 bit patterns or ml_dtypes.bfloat16; torch.bfloat16 on the device),
    float32 accumulation and output; trans_b=True, M <= 8."""
    return _dense(_core.sgemm_bf16, A, B, C, alpha, beta, trans_b)


def sgemm_u8s8(A, B, a_scale, a_zero_point, b_scales, C=None, *, trans_b=False):
    """C = a_scale * b_scales[j] * sum_k (A[i, k] - a_zero_point) * B[j, k] in float32 for the
    decode shape: A uint8 [M, K] (M <= 8), B int8 [N, K] with trans_b=True, b_scales float32 [N].
    The integer sums are exact and each output is the reference's scalar-table value."""
    if any(_is_cuda_tensor(a) for a in (A, B, b_scales)):
        t = _torch()
        if C is None:
            C = t.empty((A.shape[0], B.shape[0] if trans_b else B.shape[1]), dtype=t.float32, device=A.device)
        with t.cuda.device(A.device):
            _core._set_device(A.device.index)
            _core.sgemm_u8s8(_wrap(A), _wrap(B), a_scale, a_zero_point, _wrap(b_scales), C=_wrap(C),
                             trans_b=trans_b, stream=_stream_of(C))
        return C
    return _core.sgemm_u8s8(A, B, a_scale, a_zero_point, b_scales, C=C, trans_b=trans_b)


def gemv_dense(x, W, *, wtype=None, out=None):
    """Y = X @ W.T [M, N] float32 for float32 X [M, K] (M <= 8) and W [N, K] in float32, float16
    or bfloat16 (wtype 'float32' | 'float16' | 'bfloat16'; inferred from torch dtypes)."""
    if _is_cuda_tensor(x) or _is_cuda_tensor(W):
        t = _torch()
        if wtype is None:
            wtype = {t.float32: "float32", t.float16: "float16", t.bfloat16: "bfloat16"}[W.dtype]
        return _device_call(_core.gemv_dense, (x, W), (x.shape[0], W.shape[0]), t.float32, _wrap(x), _wrap(W),
                            wtype, out=out)
    if wtype is None:
        import numpy as np
        wtype = {np.dtype(np.float32): "float32", np.dtype(np.float16): "float16"}.get(W.dtype, "bfloat16")
    return _core.gemv_dense(x, W, wtype, out=out)


# ---- runtime information and settings ----------------------------------------------

def set_pdl(enabled: bool, device: int = 0) -> None:
    """Launch GEMVs with programmatic dependent launch on `device`: a GEMV starts
    streaming its weights while the previous GEMV of the stream drains. Only
    valid when no kernel right before a GEMV in the stream writes its weights."""
    _core._set_device(device)
    _core._ctx_set(1, 1 if enabled else 0)


def set_num_threads(n: int) -> None:
    """Accepted for compatibility; the GPU path has no host thread team."""


def get_num_threads() -> int:
    return 1


def detected_isa() -> str:
    return "sm_100a"


def build_info() -> dict:
    """Build and device details (the reference's build_info keys where they apply)."""
    info = {"version": __version__, "library": _core.version(), "isa_compiled": "sm_100a", "isa_usable": "sm_100a",
            "runtime_isa": "sm_100a", "q8_0_path": "sm_100a dp4a", "openmp": False,
            "library_path": library_path()}
    t = _torch()
    if t is None:
        try:
            import torch as t  # noqa: F811
        except Exception:  # noqa: BLE001
            t = None
    if t is not None and t.cuda.is_available():
        p = t.cuda.get_device_properties(0)
        info.update(device=p.name, sm_count=p.multi_processor_count, capability=f"{p.major}.{p.minor}",
                    memory_bytes=p.total_memory, l2_cache_bytes=getattr(p, "L2_cache_size", None),
                    gpu_count=t.cuda.device_count(), nccl=".".join(map(str, t.cuda.nccl.version())))
    return info
