"""oracle.py — TEST INFRASTRUCTURE ONLY.

NumPy front end of the CPU restatement of the reference's decode-GEMV path
(smk_oracle.c, built into oracle/_build/liboracle.so) and of the reference
library itself compiled from its sources (oracle/_ref/libsmk_ref.so).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs import
this module, as the checker or as the timed CPU baseline; the shipped
package (simd-ml-kernels_b200/) never does.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libsmk_ref.so")

_P = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
_F = ctypes.c_float

_lib = None
_ref = None


def build() -> None:
    """Compile the restatement (and the reference, where its tree exists)."""
    subprocess.run(["make", "-s", "-C", HERE, "all"], check=True)


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(ORACLE_SO):
            build()
        L = ctypes.CDLL(ORACLE_SO)
        L.smko_fp32_to_fp16.restype = ctypes.c_uint16
        L.smko_fp32_to_fp16.argtypes = [_F]
        L.smko_fp16_to_fp32.restype = _F
        L.smko_fp16_to_fp32.argtypes = [ctypes.c_uint16]
        L.smko_fp32_to_fp16_n.argtypes = [_P, _P, _I64]
        for name in ("smko_quantize_q4_0", "smko_quantize_q8_0"):
            getattr(L, name).argtypes = [_P, _I64, _I, _P]
            getattr(L, name).restype = _I
        L.smko_quantize_x_q8.argtypes = [_P, _I, _P, _P]
        L.smko_quantize_x_q8.restype = _I
        for name in ("smko_gemv_q4_0", "smko_gemv_q8_0"):
            getattr(L, name).argtypes = [_I, _I, _P, _P, _P]
        for name in ("smko_block_sums_q4_0", "smko_block_sums_q8_0"):
            getattr(L, name).argtypes = [_I, _I, _P, _P, _P]
        for name in ("smko_ref64_q4_0", "smko_ref64_q8_0"):
            getattr(L, name).argtypes = [_I, _I, _P, _P, _P, _P, _P]
        L.smko_dense_ref64.argtypes = [_I, _I, _I, _P, _I, _P, _I, _P, _P]
        L.smko_dense_scalar.argtypes = [_I, _I, _I, _F, _P, _I, _P, _I, _F, _P]
        L.smko_gemv_slice.argtypes = [_I, _I, _I, ctypes.POINTER(_I), ctypes.POINTER(_I)]
        L.smko_sgemm_u8s8.argtypes = [_I, _I, _I, _I, _P, _I, _I, _P, _I, _F, _P, _P, _I]
        L.smko_u8s8_ref64.argtypes = [_I, _I, _I, _I, _P, _I, _P, _P, _P]
        _lib = L
    return _lib


BLOCK_BYTES = {"q4_0": 18, "q8_0": 34}


def fp32_to_fp16_bits(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(x.shape, np.uint16)
    lib().smko_fp32_to_fp16_n(_ptr(x), _ptr(out), x.size)
    return out


def quantize(fmt: str, W: np.ndarray) -> np.ndarray:
    """ggml Q4_0 / Q8_0 blocks of W [..., K] (shape [..., K/32*bytes]); raises ValueError when the
    reference would reject W (NaN/Inf or a scale that overflows binary16)."""
    W = np.ascontiguousarray(W, np.float32)
    K = W.shape[-1]
    rows = W.size // K if K else 0
    out = np.zeros(W.shape[:-1] + (K // 32 * BLOCK_BYTES[fmt],), np.uint8)
    fn = lib().smko_quantize_q4_0 if fmt == "q4_0" else lib().smko_quantize_q8_0
    if rows and not fn(_ptr(W), rows, K, _ptr(out)):
        raise ValueError("W must be finite with representable block scales")
    return out


def quantize_x(x: np.ndarray) -> tuple[np.ndarray, np.ndarray, bool]:
    """(int8 quants [K], float32 scales [K/32], ok) of one activation row."""
    x = np.ascontiguousarray(x, np.float32)
    K = x.shape[0]
    qs = np.zeros(K, np.int8)
    dx = np.zeros(K // 32, np.float32)
    ok = bool(lib().smko_quantize_x_q8(_ptr(x), K, _ptr(qs), _ptr(dx))) if K else True
    return qs, dx, ok


def gemv_scalar(fmt: str, x: np.ndarray, Wq: np.ndarray, N: int, K: int) -> np.ndarray:
    """The reference's scalar-table GEMV, same FP32 operation order (bitwise)."""
    x = np.ascontiguousarray(x, np.float32)
    Wq = np.ascontiguousarray(Wq, np.uint8)
    y = np.zeros(N, np.float32)
    fn = lib().smko_gemv_q4_0 if fmt == "q4_0" else lib().smko_gemv_q8_0
    fn(N, K, _ptr(x), _ptr(Wq), _ptr(y))
    return y


def block_sums(fmt: str, xq: np.ndarray, Wq: np.ndarray, N: int, K: int) -> np.ndarray:
    """Exact int32 sums [N, K/32] of every (row, block) of the quantized operands."""
    xq = np.ascontiguousarray(xq, np.int8)
    Wq = np.ascontiguousarray(Wq, np.uint8)
    out = np.zeros((N, K // 32), np.int32)
    fn = lib().smko_block_sums_q4_0 if fmt == "q4_0" else lib().smko_block_sums_q8_0
    fn(N, K, _ptr(xq), _ptr(Wq), _ptr(out))
    return out


def ref64(fmt: str, x: np.ndarray, Wq: np.ndarray, N: int, K: int) -> tuple[np.ndarray, np.ndarray]:
    """(y64, mag) for one activation row: the float64 result of the quantized operands and the
    magnitude of the reference's bound 2*(K/32+4)*2^-24*mag."""
    qs, dx, ok = quantize_x(x)
    Wq = np.ascontiguousarray(Wq, np.uint8)
    y64 = np.zeros(N, np.float64)
    mag = np.zeros(N, np.float64)
    if not ok:
        return np.full(N, np.nan), np.full(N, np.nan)
    fn = lib().smko_ref64_q4_0 if fmt == "q4_0" else lib().smko_ref64_q8_0
    fn(N, K, _ptr(qs), _ptr(dx), _ptr(Wq), _ptr(y64), _ptr(mag))
    return y64, mag


KIND = {"f32": 0, "f16": 1, "bf16": 2}


def _as_kind(a: np.ndarray, kind: str) -> np.ndarray:
    if kind == "f32":
        return np.ascontiguousarray(a, np.float32)
    return np.ascontiguousarray(a).view(np.uint16) if a.dtype.itemsize == 2 else np.ascontiguousarray(a, np.uint16)


def dense_ref64(A: np.ndarray, a_kind: str, B: np.ndarray, b_kind: str) -> tuple[np.ndarray, np.ndarray]:
    """(y64, mag) of A [M, K] · B [N, K]ᵀ on the exact input values."""
    A = _as_kind(A, a_kind)
    B = _as_kind(B, b_kind)
    M, K = A.shape
    N = B.shape[0]
    y64 = np.zeros((M, N), np.float64)
    mag = np.zeros((M, N), np.float64)
    lib().smko_dense_ref64(M, N, K, _ptr(A), KIND[a_kind], _ptr(B), KIND[b_kind], _ptr(y64), _ptr(mag))
    return y64, mag


def dense_scalar(A, a_kind, B, b_kind, alpha=1.0, beta=0.0, C=None) -> np.ndarray:
    A = _as_kind(A, a_kind)
    B = _as_kind(B, b_kind)
    M, K = A.shape
    N = B.shape[0]
    out = np.zeros((M, N), np.float32) if C is None else np.array(C, np.float32, copy=True)
    lib().smko_dense_scalar(M, N, K, alpha, _ptr(A), KIND[a_kind], _ptr(B), KIND[b_kind], beta, _ptr(out))
    return out


def gemv_slice(N: int, t: int, parts: int) -> tuple[int, int]:
    lo, hi = _I(), _I()
    lib().smko_gemv_slice(N, t, parts, ctypes.byref(lo), ctypes.byref(hi))
    return lo.value, hi.value


def _u8s8_shapes(A, B, trans_b):
    A = np.ascontiguousarray(A, np.uint8)
    B = np.ascontiguousarray(B, np.int8)
    M, K = A.shape
    N = B.shape[0] if trans_b else B.shape[1]
    return A, B, M, N, K


def sgemm_u8s8(A, B, a_scale, a_zero_point, b_scales, trans_b=False) -> np.ndarray:
    """The reference's scalar-table sgemm_u8s8 (exact int64 sums, one double epilogue)."""
    A, B, M, N, K = _u8s8_shapes(A, B, trans_b)
    bs = np.ascontiguousarray(b_scales, np.float32)
    C = np.zeros((M, N), np.float32)
    lib().smko_sgemm_u8s8(int(trans_b), M, N, K, _ptr(A), K, int(a_zero_point), _ptr(B), B.shape[1],
                          float(a_scale), _ptr(bs), _ptr(C), N)
    return C


def u8s8_ref64(A, B, a_zero_point, trans_b=False) -> tuple[np.ndarray, np.ndarray]:
    """Exact Σ (A − zp)·op(B) and the bound's Σ |A − zp|·|op(B)|, as float64 [M, N]."""
    A, B, M, N, K = _u8s8_shapes(A, B, trans_b)
    s64 = np.zeros((M, N), np.float64)
    mag = np.zeros((M, N), np.float64)
    lib().smko_u8s8_ref64(int(trans_b), M, N, K, _ptr(A), int(a_zero_point), _ptr(B), _ptr(s64), _ptr(mag))
    return s64, mag


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 bit patterns, round to nearest even (tests/test_precision.py:196-198)."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)


# ---- the reference itself (compiled from its sources) -------------------------

def ref_available() -> bool:
    return os.path.exists(REF_SO)


def ref() -> ctypes.CDLL:
    """oracle/_ref/libsmk_ref.so: the reference's own CPU kernels (ref_glue.cpp's C ABI)."""
    global _ref
    if _ref is None:
        R = ctypes.CDLL(REF_SO)
        R.smkref_q8_0_path.restype = ctypes.c_char_p
        R.smkref_active_isa.restype = ctypes.c_char_p
        R.smkref_isa_usable.argtypes = [_I]
        R.smkref_set_num_threads.argtypes = [_I]
        R.smkref_get_num_threads.restype = _I
        for name in ("smkref_gemv_q4_0", "smkref_gemv_q8_0"):
            getattr(R, name).argtypes = [_I, _I, _I, _P, _P, _P]
        for name in ("smkref_quantize_q4_0", "smkref_quantize_q8_0"):
            getattr(R, name).argtypes = [_P, _I, _I, _P]
            getattr(R, name).restype = _I
        R.smkref_quantize_x_q8.argtypes = [_P, _I, _P, _P]
        R.smkref_quantize_x_q8.restype = _I
        R.smkref_sgemm_tb.argtypes = [_I, _I, _I, _I, _F, _P, _P, _F, _P]
        R.smkref_sgemm_f16_tb.argtypes = [_I, _I, _I, _I, _F, _P, _P, _F, _P]
        R.smkref_sgemm_bf16_tb.argtypes = [_I, _I, _I, _I, _F, _P, _P, _F, _P]
        R.smkref_sgemm_u8s8.argtypes = [_I, _I, _I, _I, _I, _P, _I, _P, _F, _P, _P]
        R.smkref_u8s8_path.restype = ctypes.c_char_p
        _ref = R
    return _ref


def ref_gemv(fmt: str, x: np.ndarray, Wq: np.ndarray, N: int, K: int, isa: int = -1) -> np.ndarray:
    y = np.zeros(N, np.float32)
    fn = ref().smkref_gemv_q4_0 if fmt == "q4_0" else ref().smkref_gemv_q8_0
    fn(isa, N, K, _ptr(np.ascontiguousarray(x, np.float32)), _ptr(np.ascontiguousarray(Wq, np.uint8)), _ptr(y))
    return y


def ref_quantize(fmt: str, W: np.ndarray) -> np.ndarray | None:
    W = np.ascontiguousarray(W, np.float32)
    K = W.shape[-1]
    rows = W.size // K if K else 0
    out = np.zeros(W.shape[:-1] + (K // 32 * BLOCK_BYTES[fmt],), np.uint8)
    fn = ref().smkref_quantize_q4_0 if fmt == "q4_0" else ref().smkref_quantize_q8_0
    return out if (rows == 0 or fn(_ptr(W), rows, K, _ptr(out))) else None


def ref_sgemm_u8s8(A, B, a_scale, a_zero_point, b_scales, trans_b=False, isa: int = -1) -> np.ndarray:
    """The reference's own sgemm_u8s8 (table `isa`: -1 this CPU's, 0 scalar)."""
    A, B, M, N, K = _u8s8_shapes(A, B, trans_b)
    bs = np.ascontiguousarray(b_scales, np.float32)
    C = np.zeros((M, N), np.float32)
    ref().smkref_sgemm_u8s8(isa, int(trans_b), M, N, K, _ptr(A), int(a_zero_point), _ptr(B), float(a_scale),
                            _ptr(bs), _ptr(C))
    return C


def dequantize_rows(fmt: str, Wq: np.ndarray, K: int, rows) -> np.ndarray:
    """float32 rows of a Q4_0 / Q8_0 matrix [N, K/32 blocks]: fp16(d)·(q − 8)
    (Q4_0: value j in the low nibble of byte j, value 16 + j in the high one)
    or fp16(d)·q (Q8_0), as examples/llama/gguf_reader.py:113-129 computes it."""
    r = np.atleast_1d(np.asarray(rows))
    nb = K // 32
    blocks = np.ascontiguousarray(Wq, np.uint8).reshape(-1, nb, BLOCK_BYTES[fmt])[r]
    d = blocks[:, :, :2].copy().view("<f2").astype(np.float32)
    if fmt == "q8_0":
        q = blocks[:, :, 2:].view(np.int8).astype(np.float32)
    else:
        b = blocks[:, :, 2:]
        q = np.concatenate([b & 0x0F, b >> 4], axis=-1).astype(np.float32) - np.float32(8.0)
    return (d * q).reshape(len(r), K)
