"""smk_gemv_q_noalloc — the quantized decode GEMV for callers that cannot
allocate GPU memory (hosts whose memory pools own every device allocation,
servers that allocate nothing per request, plugins loaded into either). It
keeps its scratch in a fixed array inside the library instead of calling
cudaMalloc.

Called through the C ABI (ctypes on libsmk_cuda.so) with device pointers,
and compared with the regular entry point (smk_gemv_q, through the Python
API) within the tolerance the parity tests use, on two calls in a row with
different shapes (the second call reuses the scratch the first one left
behind). Collected last on purpose: a failure here leaves every other test
already run.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu

U = 2.0 ** -24


def _lib():
    import simd_ml_kernels as sk
    lib = ctypes.CDLL(sk.library_path())
    fn = lib.smk_gemv_q_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_int64,
                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p]
    lib.smk_last_error.restype = ctypes.c_char_p
    lib.smk_noalloc_device_error.restype = ctypes.c_int
    lib.smk_noalloc_device_error.argtypes = [ctypes.POINTER(ctypes.c_uint), ctypes.c_void_p]
    return lib, fn


def _device_error(lib, stream) -> int:
    code = ctypes.c_uint(0xFFFFFFFF)
    assert lib.smk_noalloc_device_error(ctypes.byref(code), stream) == 0, lib.smk_last_error().decode()
    return code.value


def _check(lib, noalloc, sk, torch, fmt, M, N, K, f, seed, stream):
    """One no-alloc call against smk_gemv_q (Python API) and the oracle."""
    X, Wq = _case(seed, M, N, K, fmt)
    xd = torch.from_numpy(X).cuda()
    wd = torch.from_numpy(Wq.reshape(-1)).cuda()
    y = torch.full((M, N), float("nan"), device="cuda")
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    st = noalloc(f, M, N, K, xd.data_ptr(), K, wd.data_ptr(), y.data_ptr(), N, stream.cuda_stream)
    assert st == 0, lib.smk_last_error().decode()
    torch.cuda.synchronize()
    free1 = torch.cuda.mem_get_info()[0]
    got = y.cpu().numpy()
    batch = sk.gemv_q4_0_batch if fmt == "q4_0" else sk.gemv_q8_0_batch
    want = batch(xd, wd, N, K).cpu().numpy()
    bound_scale = min(2 * (K // 32 + 4) * U, 1e-5)
    for m in range(M):
        y64, mag = O.ref64(fmt, X[m], Wq, N, K)
        bound = bound_scale * mag + 1e-300
        assert (np.abs(got[m].astype(np.float64) - want[m]) <= bound).all(), f"{fmt} K={K} row {m}: vs smk_gemv_q"
        assert (np.abs(got[m].astype(np.float64) - y64) <= bound).all(), f"{fmt} K={K} row {m}: vs the oracle"
    return free0, free1


def _case(seed, M, N, K, fmt):
    rng = np.random.default_rng(seed)
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    X = rng.standard_normal((M, K)).astype(np.float32)
    return X, O.quantize(fmt, W)


def test_noalloc_matches_regular_entry_point(cuda_device):
    import torch
    import simd_ml_kernels as sk

    lib, noalloc = _lib()
    torch.cuda.set_device(cuda_device)
    stream = torch.cuda.current_stream()
    cases = [("q4_0", 1, 4096, 2048, 0), ("q8_0", 3, 1000, 4096, 1)]   # two calls in a row
    frees = []
    for fmt, M, N, K, f in cases:
        frees.append(_check(lib, noalloc, sk, torch, fmt, M, N, K, f, 7 + M + N + K, stream))
    # The second call (set-up already done by the first) leaves device memory as it was.
    assert frees[1][0] == frees[1][1], "smk_gemv_q_noalloc changed the free device memory"
    assert _device_error(lib, stream.cuda_stream) == 0


def test_noalloc_generic_kernel_and_limit(cuda_device):
    """K % 256 != 0 (the generic kernel, which reads x from the same array), and
    a call exactly at the array's limit: M * ceil(K/8192) = 102."""
    import torch
    import simd_ml_kernels as sk

    lib, noalloc = _lib()
    torch.cuda.set_device(cuda_device)
    stream = torch.cuda.current_stream()
    _check(lib, noalloc, sk, torch, "q4_0", 2, 777, 2080, 0, 11, stream)
    _check(lib, noalloc, sk, torch, "q8_0", 1, 300, 2080, 1, 12, stream)
    free0, free1 = _check(lib, noalloc, sk, torch, "q4_0", 1, 40, 102 * 8192, 0, 13, stream)
    assert free0 == free1
    assert _device_error(lib, stream.cuda_stream) == 0


def test_noalloc_rejects_beyond_its_scratch(cuda_device):
    import torch

    lib, noalloc = _lib()
    for M, K in ((8, 131072), (1, 102 * 8192 + 256)):   # 8 * 16 and 1 * 103 k-steps of 10 KiB
        st = noalloc(0, M, 4, K, None, K, None, None, 4, None)
        assert st == 1                  # SMK_ERR_ARGUMENT, before any device work
        assert b"scratch" in lib.smk_last_error()
    torch.cuda.synchronize()
