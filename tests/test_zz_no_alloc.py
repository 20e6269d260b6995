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
    return lib, fn


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
    for fmt, M, N, K, f in cases:
        X, Wq = _case(7 + M + N + K, M, N, K, fmt)
        xd = torch.from_numpy(X).cuda()
        wd = torch.from_numpy(Wq.reshape(-1)).cuda()
        y = torch.full((M, N), float("nan"), device="cuda")
        st = noalloc(f, M, N, K, xd.data_ptr(), K, wd.data_ptr(), y.data_ptr(), N, stream.cuda_stream)
        assert st == 0, lib.smk_last_error().decode()
        torch.cuda.synchronize()
        got = y.cpu().numpy()
        batch = sk.gemv_q4_0_batch if fmt == "q4_0" else sk.gemv_q8_0_batch
        want = batch(xd, wd, N, K).cpu().numpy()
        bound_scale = min(2 * (K // 32 + 4) * U, 1e-5)
        for m in range(M):
            y64, mag = O.ref64(fmt, X[m], Wq, N, K)
            bound = bound_scale * mag + 1e-300
            assert (np.abs(got[m].astype(np.float64) - want[m]) <= bound).all(), f"{fmt} row {m}: vs smk_gemv_q"
            assert (np.abs(got[m].astype(np.float64) - y64) <= bound).all(), f"{fmt} row {m}: vs the oracle"


def test_noalloc_rejects_beyond_its_scratch(cuda_device):
    import torch

    lib, noalloc = _lib()
    M, N, K = 8, 4, 131072          # 8 rows * 16 k-steps * 10 KiB = 1.25 MiB > 1 MiB
    st = noalloc(0, M, N, K, None, K, None, None, N, None)
    assert st == 1                  # SMK_ERR_ARGUMENT, before any device work
    assert b"scratch" in lib.smk_last_error()
    torch.cuda.synchronize()
