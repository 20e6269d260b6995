"""Host-side behaviour that needs no GPU: the drop-in API rejects every input
the reference rejects, with the same error classes and messages (reference
tests/test_bindings_edge_cases.py:651-740), the C-ABI library loads and
exports every function include/smk_cuda.h declares, and the row-sharding
planner follows the reference's gemv_slice rules."""

from __future__ import annotations

import ctypes
import os
import re

import numpy as np
import pytest

import oracle as O
import simd_ml_kernels as sk
from simd_ml_kernels import shard

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _blocks(fmt, n, k):
    # Shape-correct zero blocks: these tests never reach a kernel.
    return np.zeros((n, k // 32 * (18 if fmt == "q4_0" else 34)), np.uint8)


@pytest.mark.parametrize("fmt", ["q4_0", "q8_0"])
def test_gemv_rejects(fmt):
    g = sk.gemv_q4_0 if fmt == "q4_0" else sk.gemv_q8_0
    x = np.ones(64, np.float32)
    wq = _blocks(fmt, 3, 64)
    with pytest.raises(sk.ArgumentError, match="multiple of 32"):
        g(np.ones(63, np.float32), wq, 3, 63)
    with pytest.raises(sk.ArgumentError, match="bytes"):
        g(x, wq, 4, 64)
    with pytest.raises(sk.ArgumentError, match="1-D"):
        g(x[None, :], wq, 3, 64)
    with pytest.raises(sk.ArgumentError, match="1-D"):
        g(np.ones(32, np.float32), wq, 3, 64)
    with pytest.raises(sk.ArgumentError, match=">= 0"):
        g(x, wq, -1, 64)
    with pytest.raises(sk.DTypeError, match="uint8"):
        g(x, wq.view(np.int8), 3, 64)
    with pytest.raises(sk.DTypeError):
        g(x.astype(np.float64), wq, 3, 64)
    with pytest.raises(sk.ArgumentError, match="C-contiguous"):
        g(x, np.ascontiguousarray(np.stack([wq, wq], axis=1))[:, 0], 3, 64)
    if fmt == "q4_0":
        with pytest.raises(sk.ArgumentError, match="bytes"):
            g(x, _blocks("q8_0", 3, 64), 3, 64)   # Q8_0 blocks given to the Q4_0 GEMV


def test_error_classes():
    assert issubclass(sk.ArgumentError, ValueError) and issubclass(sk.ArgumentError, RuntimeError)
    assert issubclass(sk.DTypeError, TypeError) and issubclass(sk.DTypeError, RuntimeError)


@pytest.mark.parametrize("q", ["quantize_q4_0", "quantize_q8_0"])
def test_quantize_rejects_before_the_device(q):
    fn = getattr(sk, q)
    with pytest.raises(sk.ArgumentError, match="multiple of 32"):
        fn(np.ones((2, 33), np.float32))
    with pytest.raises(sk.DTypeError):
        fn(np.ones((2, 32), np.float64))
    with pytest.raises(sk.ArgumentError, match="C-contiguous"):
        fn(np.ones((32, 64), np.float32).T)
    with pytest.raises(sk.ArgumentError, match="at least 1 dimension"):
        fn(np.array(1.0, np.float32))


def test_dense_rejects_before_the_device():
    A = np.ones((2, 16), np.float32)
    with pytest.raises(sk.ArgumentError, match="Shape mismatch"):
        sk.sgemm(A, np.ones((3, 8), np.float32), trans_b=True)
    with pytest.raises(sk.DTypeError, match="float16"):
        sk.sgemm_f16(A, A, trans_b=True)
    with pytest.raises(sk.DTypeError, match="BF16"):
        sk.sgemm_bf16(A.astype(np.float16), A.astype(np.float16), trans_b=True)
    with pytest.raises(sk.ArgumentError, match="isa must be one of"):
        sk.sgemm(A, A, isa="neon", trans_b=True)
    with pytest.raises(RuntimeError, match="does not include it"):
        sk.sgemm(A, A, isa="avx2", trans_b=True)
    with pytest.raises(sk.ArgumentError, match="decode"):
        sk.sgemm(np.ones((9, 16), np.float32), np.ones((4, 16), np.float32), trans_b=True)


def test_valid_call_fails_loudly_without_a_gpu():
    """No CPU fallback: with no usable device a valid call raises."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(RuntimeError, match="B200"):
        sk.gemv_q4_0(np.ones(64, np.float32), _blocks("q4_0", 3, 64), 3, 64)


def test_c_abi_exports_every_declared_symbol():
    header = open(os.path.join(REPO, "include", "smk_cuda.h")).read()
    declared = set(re.findall(r"^\s*(?:smk_status|const char\*)\s+(smk_\w+)\(", header, re.M))
    assert {"smk_gemv_q4_0", "smk_gemv_q8_0", "smk_gemv_q", "smk_gemv_dense", "smk_quantize",
            "smk_gemv_u8s8", "smk_gemv_u8s8_host", "smk_gemv_q_silu_mul"} <= declared
    lib = ctypes.CDLL(sk.library_path())
    missing = [name for name in sorted(declared) if not hasattr(lib, name)]
    assert not missing, f"declared but not exported: {missing}"
    lib.smk_version.restype = ctypes.c_char_p
    assert b"sm_100a" in lib.smk_version()


def test_sgemm_u8s8_argument_checks():
    """sgemm_u8s8 rejects what the reference rejects, in its order and with its
    messages (the reference's tests/test_bindings_edge_cases.py:190-258 restated),
    before any device work; shapes outside the decode contract raise
    ArgumentError naming it; empty outputs come back without a GPU."""
    A, B, s, zp, bs = np.ones((4, 6), np.uint8), np.ones((5, 6), np.int8), 0.5, 1, np.ones(5, np.float32)
    f = sk.sgemm_u8s8
    for dt in (np.int8, np.uint16, np.float32):
        with pytest.raises(sk.DTypeError, match="A must be uint8"):
            f(A.astype(dt), B, s, zp, bs, trans_b=True)
    for dt in (np.uint8, np.int16, np.float32):
        with pytest.raises(sk.DTypeError, match="B must be int8"):
            f(A, B.astype(dt), s, zp, bs, trans_b=True)
    with pytest.raises(sk.DTypeError, match="b_scales"):
        f(A, B, s, zp, bs.astype(np.float64), trans_b=True)
    with pytest.raises(sk.ArgumentError, match="b_scales must have N = 5"):
        f(A, B, s, zp, np.ones(4, np.float32), trans_b=True)
    with pytest.raises(sk.ArgumentError, match="1-D"):
        f(A, B, s, zp, np.ones((5, 1), np.float32), trans_b=True)
    for bad in (-1, 256):
        with pytest.raises(sk.ArgumentError, match=r"\[0, 255\]"):
            f(A, B, s, bad, bs, trans_b=True)
    with pytest.raises(sk.ArgumentError, match="finite"):
        f(A, B, float("nan"), zp, bs, trans_b=True)
    with pytest.raises(sk.ArgumentError, match="Shape mismatch"):
        f(A, np.ones((6, 5), np.int8), s, zp, bs, trans_b=True)
    with pytest.raises(sk.ArgumentError, match="C-contiguous"):
        f(np.asfortranarray(A), B, s, zp, bs, trans_b=True)
    with pytest.raises(sk.ArgumentError, match="trans_b=True"):
        f(A, np.ones((6, 5), np.int8), s, zp, bs)             # B as [K, N]: outside the decode path
    with pytest.raises(sk.ArgumentError, match="at most 8 rows"):
        f(np.ones((9, 6), np.uint8), B, s, zp, bs, trans_b=True)
    with pytest.raises(sk.DTypeError, match="C must be float32"):
        f(A, B, s, zp, bs, np.zeros((4, 5)), trans_b=True)
    for M, K, N in ((0, 3, 5), (4, 3, 0)):   # no outputs: any layout of B
        C = f(np.ones((M, K), np.uint8), np.ones((K, N), np.int8), 1.0, 0, np.ones(N, np.float32))
        assert C.shape == (M, N)


def test_row_slices_match_reference_rule():
    for N in (1, 7, 8, 9, 100, 1003, 8192, 28672, 128256):
        for parts in (1, 2, 3, 4, 8):
            assert [shard.row_slice(N, t, parts) for t in range(parts)] == \
                   [O.gemv_slice(N, t, parts) for t in range(parts)]
    assert shard.shard_sizes(128256, 8) == [16032] * 8


def test_stub_matches_extension():
    """simd_ml_kernels/_core.pyi names every public function of the extension
    with its parameter names, order, keyword-only markers and defaults, as
    pybind11 states them on the first docstring line (a stub that drifts
    from the module would mislead a type checker)."""
    import ast
    from simd_ml_kernels import _core
    stub = ast.parse(open(os.path.join(os.path.dirname(sk.__file__), "_core.pyi"), encoding="utf-8").read())
    stubs = {n.name: n for n in stub.body if isinstance(n, ast.FunctionDef)}
    public = sorted(n for n in dir(_core) if not n.startswith("_") and callable(getattr(_core, n))
                    and not isinstance(getattr(_core, n), type))
    assert sorted(stubs) == public

    def params(fn):
        a = fn.args
        pos = [p.arg for p in a.args]
        pos_def = [None] * (len(pos) - len(a.defaults)) + [ast.literal_eval(d) for d in a.defaults]
        kw = [p.arg for p in a.kwonlyargs]
        kw_def = [None if d is None else ast.literal_eval(d) for d in a.kw_defaults]
        return list(zip(pos, pos_def)), list(zip(kw, kw_def))

    for name in public:
        head = getattr(_core, name).__doc__.strip().splitlines()[0].split(") ->")[0] + ")"
        runtime = ast.parse(f"def {head}: ...").body[0]
        assert params(runtime) == params(stubs[name]), name
