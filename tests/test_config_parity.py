"""GPU parity on BASELINE's own workloads: the exact bytes bench.py times.

Each config's inputs come from bench.py's generators (numpy default_rng with the
BASELINE seeds, weights in 8192-row chunks, then x). They are quantized by the
device quantizer, and the bytes must equal the SHA-256 pins that
tests/golden/make_config_pins.py computed with the reference's own quantizer.
The GEMVs the bench times then run on those bytes and every output row must
satisfy the parity bar of the other GPU tests:
    |y - y64| <= min(2*(K/32+4)*2^-24, 1e-5) * mag  and  ||y - y64|| / ||y64|| <= 1e-5,
y64 and mag from the oracle (the float64 sums of the same quantized operands,
the reference's _cli.py:157-189). Dense config 3 meets the reference's
2*(K+2)*2^-24*|x|.|W| bound (tests/test_precision.py:212-221 there).

Covered: config 0 (8192x2048 Q4_0, M = 1), config 1 (Q8_0, four shapes), config 2
(all 113 Llama-3.2-1B matrices at M = 1, its 128256x2048 LM head at M = 8 too),
config 3 (4096x4096 and 14336x4096, float32 / bfloat16 / float16 weights,
M = 1, 4, 8) and config 4 (28672x8192, 8192x28672, 128256x8192 Q4_0 at M = 1
and 8).
"""

from __future__ import annotations

import concurrent.futures as cf
import hashlib
import json
import os

import numpy as np
import pytest

import bench
import oracle as O

pytestmark = pytest.mark.gpu

U = 2.0 ** -24
PINS = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "config_pins.json")))


@pytest.fixture(scope="module")
def sk(cuda_device):
    import simd_ml_kernels
    return simd_ml_kernels


@pytest.fixture(scope="module")
def torch(cuda_device):
    import torch as t
    return t


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def device_weights(sk, torch, fmt: str, wl: bench.Workload):
    """(device bytes [N, row bytes], host copy, SHA-256 of the bytes, x) of wl,
    quantized by the device quantizer chunk by chunk."""
    quant = sk.quantize_q4_0 if fmt == "q4_0" else sk.quantize_q8_0
    rb = wl.K // 32 * O.BLOCK_BYTES[fmt]
    wd = torch.empty((wl.N, rb), dtype=torch.uint8, device="cuda")
    h = hashlib.sha256()
    for r0, c in wl.chunks():
        quant(torch.from_numpy(c).cuda(), out=wd[r0:r0 + c.shape[0]])
        h.update(wd[r0:r0 + c.shape[0]].cpu().numpy().tobytes())
    return wd, wd.cpu().numpy(), h.hexdigest(), wl.x


def check_rows(fmt, Y, X, Wq, N, K, what):
    """Every row of Y against the oracle."""
    bound_scale = min(2 * (K // 32 + 4) * U, 1e-5)
    for m in range(len(X)):
        y64, mag = O.ref64(fmt, X[m], Wq, N, K)
        y = np.asarray(Y[m], np.float64)
        assert np.isfinite(y).all(), f"{what} row {m}: non-finite"
        err = np.abs(y - y64)
        bound = bound_scale * mag + 1e-300
        assert (err <= bound).all(), f"{what} row {m}: max err/bound {np.max(err / bound):.3g}"
        assert np.linalg.norm(y - y64) / np.linalg.norm(y64) <= 1e-5, f"{what} row {m}: norm-wise"


def test_config0_bytes_and_gemv(sk, torch):
    wd, wq, digest, x = device_weights(sk, torch, "q4_0", bench.config0())
    pin = PINS["config0"]
    assert digest == pin["w_sha256"] and sha(x) == pin["x_sha256"]
    y = sk.gemv_q4_0(torch.from_numpy(x[0]).cuda(), wd.reshape(-1), bench.N_ROWS, bench.K_COLS).cpu().numpy()
    check_rows("q4_0", y[None], x, wq, bench.N_ROWS, bench.K_COLS, "config 0")


@pytest.mark.parametrize("i", range(len(bench.CFG1_SHAPES)))
def test_config1_bytes_and_gemv(sk, torch, i):
    N, K = bench.CFG1_SHAPES[i]
    wd, wq, digest, x = device_weights(sk, torch, "q8_0", bench.config1(N, K))
    pin = PINS["config1"][i]
    assert (pin["N"], pin["K"]) == (N, K) and digest == pin["w_sha256"] and sha(x) == pin["x_sha256"]
    y = sk.gemv_q8_0(torch.from_numpy(x[0]).cuda(), wd.reshape(-1), N, K).cpu().numpy()
    check_rows("q8_0", y[None], x, wq, N, K, f"config 1 {N}x{K}")


@pytest.mark.parametrize("i", range(len(bench.CFG4_SHAPES)))
def test_config4_bytes_and_gemv(sk, torch, i):
    """Config 4 at M = 1 (the one-row kernels) and M = 8 (the tensor-core kernel,
    K split into parts across CTAs where x outgrows shared memory)."""
    N, K = bench.CFG4_SHAPES[i]
    wd, wq, digest, X = device_weights(sk, torch, "q4_0", bench.config4(N, K))
    pin = PINS["config4"][i]
    assert (pin["N"], pin["K"]) == (N, K) and digest == pin["w_sha256"] and sha(X) == pin["x_sha256"]
    w = wd.reshape(-1)
    Xd = torch.from_numpy(X).cuda()
    y1 = sk.gemv_q4_0(Xd[0], w, N, K).cpu().numpy()
    check_rows("q4_0", y1[None], X[:1], wq, N, K, f"config 4 {N}x{K} M=1")
    Y8 = sk.gemv_q4_0_batch(Xd, w, N, K).cpu().numpy()
    check_rows("q4_0", Y8, X, wq, N, K, f"config 4 {N}x{K} M=8")


def test_config2_llama_stack_bytes_and_gemvs(sk, torch):
    """All 113 matrices of a Llama-3.2-1B decode step (generator (2, i) each),
    one GEMV each on x ~ N(0, 1) from generator (2, 1000 + i); the 128256x2048
    LM head (the K = 2048 large launch shape) also with 8 rows of x."""
    pins = PINS["config2"]
    n = len(bench.LLAMA_MATRICES)

    def draw(i):
        wl = bench.config2(i)
        return [c for _, c in wl.chunks()]

    with cf.ThreadPoolExecutor(max_workers=8) as pool:   # numpy releases the GIL while it draws
        ahead = {i: pool.submit(draw, i) for i in range(min(8, n))}
        for i in range(n):
            cs = ahead.pop(i).result()
            if i + 8 < n:
                ahead[i + 8] = pool.submit(draw, i + 8)
            N, K = bench.LLAMA_MATRICES[i]
            wd = torch.cat([sk.quantize_q4_0(torch.from_numpy(c).cuda()) for c in cs])
            del cs
            wq = wd.cpu().numpy()
            assert (pins[i]["N"], pins[i]["K"]) == (N, K) and sha(wq) == pins[i]["w_sha256"], f"matrix {i}"
            M = 8 if i == n - 1 else 1
            X = np.random.default_rng([2, 1000 + i]).standard_normal((M, K)).astype(np.float32)
            Xd = torch.from_numpy(X).cuda()
            y1 = sk.gemv_q4_0(Xd[0], wd.reshape(-1), N, K).cpu().numpy()
            check_rows("q4_0", y1[None], X[:1], wq, N, K, f"config 2 matrix {i} {N}x{K} M=1")
            if M > 1:
                Y = sk.gemv_q4_0_batch(Xd, wd.reshape(-1), N, K).cpu().numpy()
                check_rows("q4_0", Y, X, wq, N, K, f"config 2 LM head M={M}")
            del wd


@pytest.mark.parametrize("i", range(len(bench.CFG3_SHAPES)))
@pytest.mark.parametrize("kind", ["float32", "bfloat16", "float16"])
def test_config3_dense_bytes_and_gemv(sk, torch, i, kind):
    """Config 3: float32 x against float32 / bfloat16 / float16 W (W rounded to
    nearest even on the device), M = 1, 4, 8."""
    N, K = bench.CFG3_SHAPES[i]
    W32, X = bench.config3(N, K).full()
    pin = PINS["config3"][i]
    assert (pin["N"], pin["K"]) == (N, K) and sha(W32) == pin["float32_sha256"] and sha(X) == pin["x_sha256"]
    Wd = torch.from_numpy(W32).cuda().to(getattr(torch, kind))
    Wh = Wd.cpu()
    bits = Wh.numpy() if kind == "float32" else Wh.view(torch.int16).numpy().view(np.uint16)
    assert sha(bits) == pin[f"{kind}_sha256"], f"{kind} rounding of the weights"
    ok = {"float32": "f32", "bfloat16": "bf16", "float16": "f16"}[kind]
    for M in bench.CFG3_ROWS:
        Y = sk.gemv_dense(torch.from_numpy(X[:M]).cuda(), Wd).cpu().numpy()
        y64, mag = O.dense_ref64(X[:M], "f32", bits, ok)
        bound = 2 * (K + 2) * U * mag + 1e-300
        err = np.abs(Y - y64)
        assert (err <= bound).all(), f"{kind} {N}x{K} M={M}: max err/bound {np.max(err / bound):.3g}"
