"""GPU parity: the sm_100a kernels against the oracle (oracle/smk_oracle.c,
pinned to the reference by test_oracle_golden.py) and the golden vectors.

Bars (made precise where the reference itself needs it):
  * activation quantization (Q8 quants and FP32 scales): bit-exact;
  * per-block integer sums of every (row, block): bit-exact (int32);
  * weight quantization (quantize_q4_0 / quantize_q8_0): byte-exact;
  * GEMV outputs: |y - y64| <= min(2*(K/32+4)*2^-24, 1e-5) * mag per row,
    y64 the float64 sum of the same quantized operands and mag the
    reference's bound magnitude sum_b |dw*dx| * sum_i |qw*qx|
    (reference q4_0.hpp:23-30); and ||y - y64|| / ||y64|| <= 1e-5;
  * dense: |C - C64| <= 2*(K+2)*2^-24 * |alpha|*(|x| @ |W|.T) + |beta*C0| terms
    (reference tests/test_precision.py:212-221);
  * NaN/±Inf in x -> the row's outputs NaN; K = 0 -> zeros; N = 0 -> empty.
"""

from __future__ import annotations

import hashlib
import os

import numpy as np
import pytest

import oracle as O
import make_golden as G

pytestmark = pytest.mark.gpu

U = 2.0 ** -24
GOLD = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def sk(cuda_device):
    import simd_ml_kernels
    return simd_ml_kernels


@pytest.fixture(scope="module")
def torch(cuda_device):
    import torch as t
    return t


def q_bound(K):
    return min(2 * (K // 32 + 4) * U, 1e-5)


def assert_gemv_close(y, y64, mag, K, what=""):
    y = np.asarray(y, np.float64)
    bound = q_bound(K) * mag + 1e-300
    err = np.abs(y - y64)
    assert np.isfinite(y).all(), f"{what}: non-finite output"
    assert (err <= bound).all(), f"{what}: max err/bound {np.max(err / bound):.3g}"
    n = np.linalg.norm(y64)
    if n > 0:
        assert np.linalg.norm(y - y64) / n <= 1e-5, f"{what}: norm-wise error {np.linalg.norm(y - y64) / n:.3g}"


def make_case(seed, N, K, fmt, scale=1.0):
    rng = np.random.default_rng(seed)
    W = (rng.standard_normal((N, K)) * scale).astype(np.float32)
    x = (rng.standard_normal(K) * 4).astype(np.float32)
    return x, O.quantize(fmt, W)


# ---- quantization ------------------------------------------------------------------

def test_quantize_x_bit_exact(sk, torch):
    from simd_ml_kernels import _core
    g = np.load(os.path.join(GOLD, "ref_quantize_x.npz"))
    xs = [g["x0"], g["x1"], g["x2"], (np.random.default_rng(1).standard_normal(8 * 4096) * 3).astype(np.float32)]
    for x in xs:
        K = x.shape[0]
        xd = torch.from_numpy(x).cuda()
        qs = torch.empty(K, dtype=torch.int8, device="cuda")
        dx = torch.empty(K // 32, dtype=torch.float32, device="cuda")
        _core._quantize_x(xd.data_ptr(), 1, K, qs.data_ptr(), dx.data_ptr(), torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        want_qs, want_dx, ok = O.quantize_x(x)
        assert ok
        np.testing.assert_array_equal(qs.cpu().numpy(), want_qs)
        np.testing.assert_array_equal(dx.cpu().numpy().view(np.uint32), want_dx.view(np.uint32))


def test_x_quantizer_arithmetic_exhaustive(sk):
    """The activation quantizer's shortened steps are CUDA's correctly rounded
    operations over their whole domains: RN(a/127) for every finite a >= 0,
    RN(1/d) for every 2^-126 <= d <= 2^126, and round half away from zero for
    every |t| <= 128 (the range v·(1/d) spans for a finite block), bit for bit."""
    from simd_ml_kernels import _core
    div, rcp, rnd = _core._check_x_arith()
    assert (div, rcp, rnd) == (0, 0, 0), f"mismatches: divide {div}, reciprocal {rcp}, round {rnd}"


@pytest.mark.parametrize("fmt", ["q4_0", "q8_0"])
def test_quantize_weights_byte_exact(sk, fmt):
    g = np.load(os.path.join(GOLD, "ref_quantize.npz"))
    fn = sk.quantize_q4_0 if fmt == "q4_0" else sk.quantize_q8_0
    for i in range(4):
        np.testing.assert_array_equal(fn(g[f"w{i}"]), g[f"{fmt}_{i}"])
    np.testing.assert_array_equal(fn(g["w_special"]), g[f"{fmt}_special"])
    rej = g["w_reject"]
    for i in range(rej.shape[0]):
        if g[f"{fmt}_reject_ok"][i]:
            fn(rej[i:i + 1])
        else:
            with pytest.raises(sk.ArgumentError, match="finite"):
                fn(rej[i:i + 1])


def test_quantize_llama_cpp_fixture(sk):
    fx = np.load(os.path.join(GOLD, "q4_0_llama_cpp_fixture.npz"))
    np.testing.assert_array_equal(sk.quantize_q4_0(fx["w"]), fx["blocks"])


def test_quantize_large_matches_oracle(sk, torch):
    """Device quantization of a config-sized matrix, on torch tensors."""
    rng = np.random.default_rng(0)
    W = (rng.standard_normal((2048, 2048)) * 0.02).astype(np.float32)
    for fmt, fn in (("q4_0", sk.quantize_q4_0), ("q8_0", sk.quantize_q8_0)):
        got = fn(torch.from_numpy(W).cuda()).cpu().numpy()
        np.testing.assert_array_equal(got, O.quantize(fmt, W))


# ---- integer block sums -----------------------------------------------------------

@pytest.mark.parametrize("fmt", ["q4_0", "q8_0"])
@pytest.mark.parametrize("M,N,K", [(1, 7, 256), (1, 33, 2048), (1, 5, 8192), (3, 17, 512), (8, 9, 2048),
                                   (1, 13, 4128), (2, 11, 160), (1, 3, 28672)])
def test_block_sums_bit_exact(sk, torch, fmt, M, N, K):
    from simd_ml_kernels import _core
    rng = np.random.default_rng(M * 1000 + N + K)
    W = rng.standard_normal((N, K)).astype(np.float32)
    X = (rng.standard_normal((M, K)) * 3).astype(np.float32)
    Wq = O.quantize(fmt, W)
    xd = torch.from_numpy(X).cuda()
    wd = torch.from_numpy(Wq.reshape(-1)).cuda()
    out = torch.zeros((M, N, K // 32), dtype=torch.int32, device="cuda")
    _core._block_sums(0 if fmt == "q4_0" else 1, xd.data_ptr(), M, N, K, wd.data_ptr(), out.data_ptr(),
                      torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    for m in range(M):
        qs, dx, ok = O.quantize_x(X[m])
        np.testing.assert_array_equal(got[m], O.block_sums(fmt, qs, Wq, N, K), err_msg=f"row {m}")


# ---- GEMV outputs ---------------------------------------------------------------------

@pytest.mark.parametrize("fmt", ["q4_0", "q8_0"])
def test_gemv_golden_cases(sk, fmt):
    """Every golden case: within the bound of the float64 sum, and (scalar order)
    oracle == the reference's scalar table, so this is parity with the reference."""
    g = np.load(os.path.join(GOLD, "ref_gemv.npz"))
    fn = sk.gemv_q4_0 if fmt == "q4_0" else sk.gemv_q8_0
    for s, n, k, extreme in g["cases"]:
        W, x = G.gemv_case_inputs(int(s), int(n), int(k), "extreme" if extreme else "normal")
        Wq = O.quantize(fmt, W)
        assert hashlib.sha256(Wq.tobytes()).hexdigest() == str(g[f"{fmt}_{s}_sha"])
        y = fn(x, Wq, int(n), int(k))
        assert y.dtype == np.float32 and y.shape == (n,)
        y64, mag = O.ref64(fmt, x, Wq, int(n), int(k))
        assert_gemv_close(y, y64, mag, int(k), f"{fmt} case {s} N={n} K={k}")
        # Same bound on the reference's own outputs (scalar and SIMD tables).
        assert_gemv_close(g[f"{fmt}_{s}_scalar"], y64, mag, int(k), "reference scalar")


@pytest.mark.parametrize("fmt", ["q4_0", "q8_0"])
@pytest.mark.parametrize("N,K", [(1, 32), (2, 64), (7, 64), (8, 96), (9, 128), (17, 352), (100, 4096),
                                 (33, 11008), (31, 256), (257, 512), (1000, 1024), (3, 28672), (513, 2048)])
def test_gemv_shapes(sk, fmt, N, K):
    x, Wq = make_case(N * 37 + K, N, K, fmt)
    fn = sk.gemv_q4_0 if fmt == "q4_0" else sk.gemv_q8_0
    y = fn(x, Wq, N, K)
    y64, mag = O.ref64(fmt, x, Wq, N, K)
    assert_gemv_close(y, y64, mag, K, f"{fmt} {N}x{K}")


@pytest.mark.parametrize("fmt", ["q4_0", "q8_0"])
@pytest.mark.parametrize("N,K", [(8192, 2048), (2048, 8192), (512, 2048), (28672, 8192)])
def test_gemv_config_shapes(sk, torch, fmt, N, K):
    """BASELINE configs 0/1/2/4 shapes (seeded synthetic weights, device-resident)."""
    rng = np.random.default_rng(N + K)
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    x = rng.standard_normal(K).astype(np.float32)
    Wq = O.quantize(fmt, W)
    fn = sk.gemv_q4_0 if fmt == "q4_0" else sk.gemv_q8_0
    y = fn(torch.from_numpy(x).cuda(), torch.from_numpy(Wq.reshape(-1)).cuda(), N, K).cpu().numpy()
    y64, mag = O.ref64(fmt, x, Wq, N, K)
    assert_gemv_close(y, y64, mag, K, f"{fmt} {N}x{K}")


@pytest.mark.parametrize("fmt", ["q4_0", "q8_0"])
@pytest.mark.parametrize("M,N,K", [(2, 100, 2048), (4, 33, 4096), (8, 257, 2048), (8, 64, 8192), (5, 19, 160),
                                   (8, 96, 28672)])
def test_gemv_batch_rows_equal_single_rows(sk, fmt, M, N, K):
    """M rows against one read of W: every row within the bound, and (x in
    shared or global memory alike) equal to its own single-row call."""
    rng = np.random.default_rng(M + N + K)
    W = rng.standard_normal((N, K)).astype(np.float32)
    X = (rng.standard_normal((M, K)) * 2).astype(np.float32)
    Wq = O.quantize(fmt, W)
    bfn = sk.gemv_q4_0_batch if fmt == "q4_0" else sk.gemv_q8_0_batch
    Y = bfn(X, Wq, N, K)
    assert Y.shape == (M, N)
    for m in range(M):
        y64, mag = O.ref64(fmt, X[m], Wq, N, K)
        assert_gemv_close(Y[m], y64, mag, K, f"{fmt} row {m}")


@pytest.mark.parametrize("fmt", ["q4_0", "q8_0"])
@pytest.mark.parametrize("bad", [np.nan, np.inf, -np.inf])
def test_gemv_nonfinite_x_gives_nan(sk, fmt, bad):
    for N, K in ((9, 64), (40, 2048)):
        W = np.full((N, K), 0.25, np.float32)
        x = np.ones(K, np.float32)
        x[37] = bad
        fn = sk.gemv_q4_0 if fmt == "q4_0" else sk.gemv_q8_0
        q = sk.quantize_q4_0 if fmt == "q4_0" else sk.quantize_q8_0
        assert np.isnan(fn(x, q(W), N, K)).all()


def test_gemv_batch_nan_row_only(sk):
    N, K = 24, 2048
    W = np.random.default_rng(2).standard_normal((N, K)).astype(np.float32)
    X = np.ones((3, K), np.float32)
    X[1, 100] = np.nan
    Y = sk.gemv_q4_0_batch(X, sk.quantize_q4_0(W), N, K)
    assert np.isnan(Y[1]).all() and np.isfinite(Y[0]).all() and np.isfinite(Y[2]).all()


def _mma_case(fmt, M, N, K):
    rng = np.random.default_rng(M * 100003 + N + K)
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    X = (rng.standard_normal((M, K)) * 3).astype(np.float32)
    X[M - 1, K // 3] = np.nan
    return X, O.quantize(fmt, W)


@pytest.mark.parametrize("fmt", ["q4_0", "q8_0"])
@pytest.mark.parametrize("M,N,K", [(3, 28500, 256), (8, 30000, 512), (5, 29001, 2048)])
def test_mma_rows_bitwise_equal_reference_scalar(sk, torch, fmt, M, N, K):
    """3..8 rows of x take the integer tensor-core kernel. When its 16-row
    tiles alone fill the GPU (N >= ~28.4K on 148 SMs), each row's blocks are
    accumulated in order with the reference scalar kernel's roundings: every
    output equals the reference's scalar GEMV (the oracle, pinned to it
    bitwise) bit for bit; a non-finite value makes only its row NaN."""
    X, Wq = _mma_case(fmt, M, N, K)
    batch = sk.gemv_q4_0_batch if fmt == "q4_0" else sk.gemv_q8_0_batch
    Y = batch(torch.from_numpy(X).cuda(), torch.from_numpy(Wq.ravel()).cuda(), N, K).cpu().numpy()
    for m in range(M - 1):
        want = O.gemv_scalar(fmt, X[m], Wq, N, K)
        np.testing.assert_array_equal(Y[m].view(np.uint32), want.view(np.uint32), err_msg=f"row {m}")
    assert np.isnan(Y[M - 1]).all()


@pytest.mark.parametrize("fmt", ["q4_0", "q8_0"])
@pytest.mark.parametrize("M,N,K", [(3, 1000, 2048), (8, 4099, 256), (5, 17, 8192), (8, 16, 512), (4, 2048, 28672),
                                   (6, 31, 768), (8, 8192, 28672), (5, 1000, 57344)])
def test_mma_rows_split_k(sk, torch, fmt, M, N, K):
    """Fewer tiles than the GPU holds, or x larger than shared memory: K is
    split into parts (within a CTA, and for K = 28672 / 57344 across CTAs,
    each holding its slice of x) whose sums are added in order: within the
    reference's bound of the float64 sums, identical from call to call, NaN
    rows as the reference."""
    X, Wq = _mma_case(fmt, M, N, K)
    batch = sk.gemv_q4_0_batch if fmt == "q4_0" else sk.gemv_q8_0_batch
    xd, wd = torch.from_numpy(X).cuda(), torch.from_numpy(Wq.ravel()).cuda()
    Y = batch(xd, wd, N, K).cpu().numpy()
    np.testing.assert_array_equal(batch(xd, wd, N, K).cpu().numpy().view(np.uint32), Y.view(np.uint32))
    for m in range(M - 1):
        y64, mag = O.ref64(fmt, X[m], Wq, N, K)
        assert_gemv_close(Y[m], y64, mag, K, f"{fmt} row {m}")
    assert np.isnan(Y[M - 1]).all()


def test_silu_mul_values(sk, torch):
    """silu(g) * u on the device against the float64 definition, within the
    reference's own SiLU tolerance 1e-35 + 1e-6·|ref| (its tests hold every
    SiLU table to it), plus one rounding of the product; and the reference's
    special values: silu(-inf) = NaN, silu(+inf) = +inf, x < -88 gives -0."""
    rng = np.random.default_rng(3)
    g = np.concatenate([rng.standard_normal(100000).astype(np.float32) * 8,
                        np.array([0.0, -0.0, 1e-30, -1e-30, 88.0, -88.0, -100.0, 100.0, -1e4, 3.4e38, -3.4e38],
                                 np.float32)])
    u = rng.standard_normal(g.size).astype(np.float32)
    got = sk.silu_mul(torch.from_numpy(g).cuda(), torch.from_numpy(u).cuda()).cpu().numpy().astype(np.float64)
    g64 = g.astype(np.float64)
    with np.errstate(over="ignore"):
        want = g64 / (1.0 + np.exp(-g64)) * u.astype(np.float64)
    assert (np.abs(got - want) <= 1e-35 + 1.2e-6 * np.abs(want)).all()
    sp = np.array([-np.inf, np.inf, -90.0], np.float32)
    r = sk.silu_mul(torch.from_numpy(sp).cuda(), torch.ones(3, device="cuda")).cpu().numpy()
    assert np.isnan(r[0]) and r[1] == np.inf and r[2] == 0.0 and np.signbit(r[2])


@pytest.mark.parametrize("fmt", ["q4_0", "q8_0"])
@pytest.mark.parametrize("M,N,K", [(1, 2048, 8192), (1, 1000, 2048), (3, 517, 4096), (8, 64, 256), (2, 33, 160)])
def test_gemv_silu_mul_equals_unfused(sk, torch, fmt, M, N, K):
    """The fused down projection (SwiGLU product formed while quantizing x)
    equals silu_mul followed by the plain GEMV bit for bit — fast, tensor-core
    and generic kernels alike."""
    rng = np.random.default_rng(M + N + K)
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    Wq = torch.from_numpy(O.quantize(fmt, W).ravel()).cuda()
    g = torch.from_numpy((rng.standard_normal((M, K)) * 3).astype(np.float32)).cuda()
    u = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32)).cuda()
    fused = (sk.gemv_q4_0_silu_mul if fmt == "q4_0" else sk.gemv_q8_0_silu_mul)(g, u, Wq, N, K)
    plain = (sk.gemv_q4_0_batch if fmt == "q4_0" else sk.gemv_q8_0_batch)(sk.silu_mul(g, u), Wq, N, K)
    assert torch.equal(fused.view(torch.int32), plain.view(torch.int32))
    fused1 = (sk.gemv_q4_0_silu_mul if fmt == "q4_0" else sk.gemv_q8_0_silu_mul)(g[0], u[0], Wq, N, K)
    plain1 = (sk.gemv_q4_0 if fmt == "q4_0" else sk.gemv_q8_0)(sk.silu_mul(g[0], u[0]), Wq, N, K)
    assert torch.equal(fused1.view(torch.int32), plain1.view(torch.int32))


@pytest.mark.parametrize("fmt", ["q4_0", "q8_0"])
@pytest.mark.parametrize("K", [8192, 12288])
def test_x_in_global_equals_x_in_shared(sk, torch, fmt, K):
    """With K >= 8192 and at most 16384 rows, x is quantized once into global
    scratch; with more rows each CTA quantizes it into shared memory. (At
    K >= 16384 so few rows take the split-K kernel, test_q4_0_split_k_rows.) A row's
    arithmetic is the same either way: the first 2048 rows of a 16392-row
    GEMV equal a 2048-row GEMV over the same rows, bit for bit, and stay
    within the bound of the float64 sums."""
    N_big, N_small = 16392, 2048
    g = torch.Generator(device="cuda")
    g.manual_seed(K + (fmt == "q8_0"))
    quant = sk.quantize_q4_0 if fmt == "q4_0" else sk.quantize_q8_0
    wd = quant(torch.randn((N_big, K), generator=g, device="cuda") * 0.02).reshape(-1)
    xd = torch.randn(K, generator=g, device="cuda")
    fn = sk.gemv_q4_0 if fmt == "q4_0" else sk.gemv_q8_0
    big = fn(xd, wd, N_big, K)
    small_bytes = N_small * (K // 32) * O.BLOCK_BYTES[fmt]
    small = fn(xd, wd[:small_bytes], N_small, K)
    assert torch.equal(big[:N_small].view(torch.int32), small.view(torch.int32))
    y64, mag = O.ref64(fmt, xd.cpu().numpy(), wd[:small_bytes].cpu().numpy().reshape(N_small, -1), N_small, K)
    assert_gemv_close(small.cpu().numpy(), y64, mag, K, f"{fmt} K={K}")


def test_gemv_silu_mul_first_call_inside_capture(sk, torch):
    """The fused down projection keeps its quantized activations in a scratch
    buffer per stream. Its first call on a fresh stream may come inside a
    CUDA-graph capture (the allocation is made there), and a later, larger
    call in the same capture grows the buffer without invalidating the first:
    replays equal the unfused results bit for bit."""
    rng = np.random.default_rng(11)
    shapes = [(2048, 8192), (1024, 16384)]   # the second needs a larger scratch
    cases = []
    for N, K in shapes:
        W = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
        Wq = torch.from_numpy(O.quantize("q4_0", W).ravel()).cuda()
        g = torch.from_numpy((rng.standard_normal(K) * 3).astype(np.float32)).cuda()
        u = torch.from_numpy(rng.standard_normal(K).astype(np.float32)).cuda()
        cases.append((N, K, Wq, g, u, torch.empty(N, device="cuda")))
    stream = torch.cuda.Stream()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(graph, stream=stream):
            for N, K, Wq, g, u, y in cases:
                sk.gemv_q4_0_silu_mul(g, u, Wq, N, K, out=y)
    for _, _, _, _, _, y in cases:
        y.fill_(float("nan"))
    graph.replay()
    torch.cuda.synchronize()
    for N, K, Wq, g, u, y in cases:
        want = sk.gemv_q4_0(sk.silu_mul(g, u), Wq, N, K)
        assert torch.equal(y.view(torch.int32), want.view(torch.int32))
    del graph


@pytest.mark.parametrize("fmt", ["q4_0", "q8_0"])
def test_gemv_k0_and_n0(sk, fmt):
    fn = sk.gemv_q4_0 if fmt == "q4_0" else sk.gemv_q8_0
    assert (fn(np.ones(0, np.float32), np.zeros(0, np.uint8), 5, 0) == 0).all()
    assert fn(np.ones(32, np.float32), np.zeros(0, np.uint8), 0, 32).shape == (0,)


@pytest.mark.parametrize("fmt", ["q4_0", "q8_0"])
def test_gemv_unaligned(sk, torch, fmt):
    """Wq at an odd address and x at a 4-byte offset (reference test_precision.py:800-814):
    host operands are staged to aligned device memory, so the result is bitwise the
    aligned one; an unaligned device pointer takes the generic kernel (within the bound)."""
    for N, K in ((13, 160), (21, 2048)):
        x, Wq = make_case(4 + K, N, K, fmt)
        Wq = Wq.ravel()
        buf = np.empty(Wq.size + 1, np.uint8)
        buf[1:] = Wq
        xbuf = np.empty(K + 1, np.float32)
        xbuf[1:] = x
        fn = sk.gemv_q4_0 if fmt == "q4_0" else sk.gemv_q8_0
        want = fn(x, Wq, N, K)
        np.testing.assert_array_equal(fn(xbuf[1:], buf[1:], N, K), want)
        dbuf = torch.from_numpy(buf).cuda()
        got = fn(torch.from_numpy(x).cuda(), dbuf[1:], N, K).cpu().numpy()
        y64, mag = O.ref64(fmt, x, Wq, N, K)
        assert_gemv_close(got, y64, mag, K, "unaligned device Wq")


@pytest.mark.parametrize("fmt", ["q4_0", "q8_0"])
def test_gemv_deterministic_pdl_and_streams(sk, torch, fmt):
    """Bitwise identical across repeated calls, with and without programmatic
    dependent launch, and between the NumPy path and the torch stream path."""
    N, K = 4096, 2048
    x, Wq = make_case(11, N, K, fmt)
    fn = sk.gemv_q4_0 if fmt == "q4_0" else sk.gemv_q8_0
    ref = fn(x, Wq, N, K)
    xd, wd = torch.from_numpy(x).cuda(), torch.from_numpy(Wq.ravel()).cuda()
    outs = [fn(xd, wd, N, K) for _ in range(5)]
    sk.set_pdl(True)
    try:
        outs += [fn(xd, wd, N, K) for _ in range(5)]
    finally:
        sk.set_pdl(False)
    for o in outs:
        np.testing.assert_array_equal(o.cpu().numpy().view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("fmt", ["q4_0", "q8_0"])
def test_launch_settings_bitwise_equal(sk, torch, fmt):
    """Outputs do not depend on the launch shape of the fast kernel (warps per
    CTA, shared-memory stages per warp, CTAs per SM, tile order, programmatic
    dependent launch): bitwise identical."""
    from simd_ml_kernels import _core
    cases = [(28672, 8192), (8192, 2048), (1000, 28672), (300, 256)]
    ref = {}
    for N, K in cases:
        x, Wq = make_case(N + K, N, K, fmt)
        ref[(N, K)] = (torch.from_numpy(x).cuda(), torch.from_numpy(Wq.ravel()).cuda(), x, Wq)
    base = {key: (sk.gemv_q4_0 if fmt == "q4_0" else sk.gemv_q8_0)(v[0], v[1], *key).cpu().numpy()
            for key, v in ref.items()}
    for key, y in base.items():
        y64, mag = O.ref64(fmt, ref[key][2], ref[key][3], *key)
        assert_gemv_close(y, y64, mag, key[1], f"{fmt} {key}")
    settings = [(16, 2, 1, False, 1), (8, 3, 1, True, 2), (2, 8, 1, False, 1), (4, 2, 2, True, 1),
                (12, 1, 3, False, 2), (16, 1, 2, True, 1)]
    try:
        for warps, stages, ctas, pdl, order in settings:
            _core._ctx_set(2, warps)
            _core._ctx_set(3, stages)
            _core._ctx_set(4, ctas)
            _core._ctx_set(5, order)
            sk.set_pdl(pdl)
            for key, v in ref.items():
                fn = sk.gemv_q4_0 if fmt == "q4_0" else sk.gemv_q8_0
                for _ in range(2):
                    got = fn(v[0], v[1], *key).cpu().numpy()
                    np.testing.assert_array_equal(got.view(np.uint32), base[key].view(np.uint32),
                                                  err_msg=f"{fmt} {key} warps={warps} stages={stages} ctas={ctas} "
                                                          f"order={order}")
    finally:
        for opt in (2, 3, 4, 5):
            _core._ctx_set(opt, 0)
        sk.set_pdl(False)


@pytest.mark.parametrize("fmt", ["q4_0", "q8_0"])
def test_dependent_chain_under_pdl(sk, torch, fmt):
    """A chain of GEMVs where each output is the next input, queued back to
    back on one stream with programmatic dependent launch: every GEMV must
    see its predecessor's finished output. Equal, bit for bit, to the chain
    run with a host synchronisation between the calls."""
    K, links = 2048, 12
    rng = np.random.default_rng(21)
    quant = sk.quantize_q4_0 if fmt == "q4_0" else sk.quantize_q8_0
    fn = sk.gemv_q4_0 if fmt == "q4_0" else sk.gemv_q8_0
    Ws = [quant(torch.from_numpy((rng.standard_normal((K, K)) * 0.03).astype(np.float32)).cuda()).reshape(-1)
          for _ in range(3)]
    x0 = torch.from_numpy(rng.standard_normal(K).astype(np.float32)).cuda()
    ys = [torch.empty(K, device="cuda") for _ in range(links)]
    want = []
    x = x0
    for i in range(links):
        x = fn(x, Ws[i % 3], K, K)
        torch.cuda.synchronize()
        want.append(x.cpu().numpy())
    sk.set_pdl(True)
    try:
        for trial in range(3):
            x = x0
            for i in range(links):
                fn(x, Ws[i % 3], K, K, out=ys[i])
                x = ys[i]
            torch.cuda.synchronize()
            for i in range(links):
                np.testing.assert_array_equal(ys[i].cpu().numpy().view(np.uint32), want[i].view(np.uint32),
                                              err_msg=f"{fmt} link {i} trial {trial}")
    finally:
        sk.set_pdl(False)


@pytest.mark.parametrize("fmt", ["q4_0", "q8_0"])
def test_host_io_paths_bitwise_equal(sk, torch, fmt):
    """The synchronous host-memory contract in every combination — x pageable
    or page-locked, weights in host or device memory, y returned or written
    into a given pageable / page-locked array — gives bitwise the result of
    the all-device path; so does the batched call with device weights, and
    its argument errors are the reference's."""
    N, K = 3000, 2048
    x, Wq = make_case(31, N, K, fmt)
    fn = sk.gemv_q4_0 if fmt == "q4_0" else sk.gemv_q8_0
    wd = torch.from_numpy(Wq.ravel()).cuda()
    want = fn(torch.from_numpy(x).cuda(), wd, N, K).cpu().numpy()
    x_pinned = torch.from_numpy(x).pin_memory().numpy()
    y_pinned = torch.empty(N).pin_memory().numpy()
    for xs in (x, x_pinned):
        for ws in (Wq.ravel(), wd):
            np.testing.assert_array_equal(fn(xs, ws, N, K).view(np.uint32), want.view(np.uint32))
            y_page = np.empty(N, np.float32)
            fn(xs, ws, N, K, out=y_page)
            np.testing.assert_array_equal(y_page.view(np.uint32), want.view(np.uint32))
            y_pinned[:] = np.nan
            fn(xs, ws, N, K, out=y_pinned)
            np.testing.assert_array_equal(y_pinned.view(np.uint32), want.view(np.uint32))
    # Results come back in page-locked arrays recycled from a pool: live
    # results never share memory, and a recycled block holds the new result.
    ya, yb = fn(x_pinned, wd, N, K), fn(-x_pinned, wd, N, K)
    assert torch.from_numpy(ya).is_pinned() and not np.shares_memory(ya, yb)
    np.testing.assert_array_equal(ya.view(np.uint32), want.view(np.uint32))
    np.testing.assert_array_equal(yb, -want)
    del ya
    yc = fn(x_pinned, wd, N, K)
    np.testing.assert_array_equal(yc.view(np.uint32), want.view(np.uint32))
    np.testing.assert_array_equal(yb, -want)
    batch = sk.gemv_q4_0_batch if fmt == "q4_0" else sk.gemv_q8_0_batch
    X = np.stack([x, -x, 0.5 * x])
    wantM = batch(torch.from_numpy(X).cuda(), wd, N, K).cpu().numpy()
    np.testing.assert_array_equal(batch(X, wd, N, K).view(np.uint32), wantM.view(np.uint32))
    with pytest.raises(sk.DTypeError, match="x must be float32"):
        fn(x.astype(np.float64), wd, N, K)
    with pytest.raises(sk.DTypeError, match="Wq must be uint8"):
        fn(x, wd.view(torch.int8), N, K)
    with pytest.raises(sk.ArgumentError, match="Wq must hold"):
        fn(x, wd[:-1], N, K)
    with pytest.raises(sk.ArgumentError, match="x must be 1-D"):
        fn(x[:-32], wd, N, K)


@pytest.mark.parametrize("M", [1, 3])
def test_host_call_graph_replay_tracks_operands(sk, torch, M):
    """A synchronous call that repeats its operands' addresses and shape replays
    a captured CUDA graph (from the second call on). Every call must still use
    that call's values: x is rewritten in place and the weights on the device
    change between calls, for pageable and page-locked x and y. Each result
    equals the all-device call bitwise, with the graphs on (the default) and
    off (SMK_OPT_HOST_GRAPHS = 0)."""
    from simd_ml_kernels import _core
    N, K = 4096, 2048
    rng = np.random.default_rng(90 + M)
    W = (rng.standard_normal((2, N, K)) * 0.02).astype(np.float32)
    wq = [torch.from_numpy(O.quantize("q4_0", W[i]).ravel()).cuda() for i in range(2)]
    wd = wq[0].clone()
    xs_pinned = torch.empty((M, K)).pin_memory().numpy()
    xs_page = np.empty((M, K), np.float32)
    y_pinned = torch.empty((M, N)).pin_memory().numpy()
    y_page = np.empty((M, N), np.float32)
    try:
        for graphs in (1, 0):
            _core._ctx_set(6, graphs)
            for xs in (xs_page, xs_pinned):
                for ys in (y_page, y_pinned):
                    for call in range(5):
                        xs[:] = rng.standard_normal((M, K)).astype(np.float32)
                        wd.copy_(wq[call % 2])
                        want = sk.gemv_q4_0_batch(torch.from_numpy(xs.copy()).cuda(), wd, N, K).cpu().numpy()
                        ys[:] = np.nan
                        sk.gemv_q4_0_batch(xs, wd, N, K, out=ys)
                        np.testing.assert_array_equal(ys.view(np.uint32), want.view(np.uint32),
                                                      err_msg=f"graphs={graphs} call {call}")
                        y = sk.gemv_q4_0_batch(xs, wd, N, K)
                        np.testing.assert_array_equal(y.view(np.uint32), want.view(np.uint32))
    finally:
        _core._ctx_set(6, 1)
    assert _core._device_error(torch.cuda.current_stream().cuda_stream) == 0


def test_prefetch_delay_option_changes_no_result(sk, torch):
    """SMK_OPT_PREFETCH_DELAY (8) only moves the four-row kernel's first weight
    copies in time: outputs are bitwise equal for every setting, chained under
    programmatic dependent launch or not; out-of-range values are refused."""
    from simd_ml_kernels import _core
    N, K = 8192, 2048
    rng = np.random.default_rng(95)
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    wd = torch.from_numpy(O.quantize("q4_0", W).ravel()).cuda()
    x = torch.from_numpy(rng.standard_normal((4, K)).astype(np.float32)).cuda()
    ys = {}
    try:
        for pdl in (False, True):
            sk.set_pdl(pdl, 0)
            for delay in (0, 1, 100, 5000, 100000):
                _core._ctx_set(8, delay)
                y = torch.empty((4, N), device="cuda")
                for i in range(4):   # chained launches on one stream
                    sk.gemv_q4_0(x[i], wd, N, K, out=y[i])
                ys[(pdl, delay)] = y.cpu().numpy()
        with pytest.raises(sk.ArgumentError, match="prefetch delay"):
            _core._ctx_set(8, -1)
        with pytest.raises(sk.ArgumentError, match="prefetch delay"):
            _core._ctx_set(8, 100001)
    finally:
        _core._ctx_set(8, 100)
        sk.set_pdl(False, 0)
    want = ys[(False, 0)]
    for k, y in ys.items():
        np.testing.assert_array_equal(y.view(np.uint32), want.view(np.uint32), err_msg=str(k))
    assert _core._device_error(torch.cuda.current_stream().cuda_stream) == 0


@pytest.mark.parametrize("N,K", [(1003, 2048), (8192, 2048), (517, 2080), (4096, 4096)])
def test_host_output_copy_bitwise_equal(sk, torch, N, K):
    """Host outputs from the fast kernel are copied to page-locked memory by
    the CTA that finishes last: odd N and a page-locked output 4 bytes off a
    16-byte boundary take its scalar copy, one and two rows the fast kernel,
    three rows the tensor-core kernel and K % 256 != 0 the generic kernel
    (both write host memory directly). Each agrees bitwise with the
    all-device call, over repeated calls (the finish counter starts from zero
    each launch)."""
    x, Wq = make_case(77, N, K, "q4_0")
    wd = torch.from_numpy(Wq.ravel()).cuda()
    X = np.stack([x, -0.5 * x, 0.25 * x])
    for M in (1, 2, 3):
        want = sk.gemv_q4_0_batch(torch.from_numpy(X[:M]).cuda(), wd, N, K).cpu().numpy()
        pool = torch.empty(M * N + 8).pin_memory().numpy()
        for off in (0, 1, 4):
            out = pool[off:off + M * N].reshape(M, N)
            for rep in range(3):
                out[:] = np.nan
                sk.gemv_q4_0_batch(X[:M], wd, N, K, out=out)
                np.testing.assert_array_equal(out.view(np.uint32), want.view(np.uint32))
        y1 = sk.gemv_q4_0_batch(X[:M], wd, N, K)
        np.testing.assert_array_equal(y1.view(np.uint32), want.view(np.uint32))
    from simd_ml_kernels import _core
    assert _core._device_error(0) == 0


@pytest.mark.parametrize("N,K", [(1, 16384), (3, 28672), (1000, 16384), (2048, 28672), (4095, 16384), (4733, 28672),
                                 (1024, 57344)])
def test_q4_0_split_k_rows(sk, torch, N, K):
    """Q4_0, one row of x, K a multiple of 2048 from 16384 and fewer than 8
    four-row tiles per SM: the kernel that splits each tile's k-steps over
    several warps. Outputs within the bound of the float64 sum; the host-memory
    call (NumPy in and out, y copied to page-locked memory by the kernel's last
    CTA) equals the device call bitwise, on two calls in a row."""
    x, Wq = make_case(7 * N + K, N, K, "q4_0", scale=0.02)
    y64, mag = O.ref64("q4_0", x, Wq, N, K)
    wd = torch.from_numpy(Wq.ravel()).cuda()
    yd = sk.gemv_q4_0(torch.from_numpy(x).cuda(), wd, N, K).cpu().numpy()
    assert_gemv_close(yd, y64, mag, K, f"N={N} K={K}")
    for _ in range(2):
        yh = sk.gemv_q4_0(x, wd, N, K)
        np.testing.assert_array_equal(yh.view(np.uint32), yd.view(np.uint32))
    from simd_ml_kernels import _core
    assert _core._device_error(torch.cuda.current_stream().cuda_stream) == 0


def test_row_shards_bitwise_equal_full(sk, torch):
    """Row-sharding (the multi-GPU plan, 8-row groups as the reference's
    gemv_slice): every shard's outputs bitwise equal the unsharded call."""
    from simd_ml_kernels import shard
    N, K = 1003, 2048
    x, Wq = make_case(5, N, K, "q4_0")
    full = sk.gemv_q4_0(x, Wq, N, K)
    rb = K // 32 * 18
    for parts in (2, 3, 4, 8):
        pieces = []
        for t in range(parts):
            lo, hi = shard.row_slice(N, t, parts)
            assert (lo, hi) == O.gemv_slice(N, t, parts)
            pieces.append(sk.gemv_q4_0(x, Wq.ravel()[lo * rb:hi * rb], hi - lo, K))
        np.testing.assert_array_equal(np.concatenate(pieces).view(np.uint32), full.view(np.uint32))


# ---- dense ---------------------------------------------------------------------------

def _dense_operands(kind, A, B):
    return G.dense_operands(kind, A, B)


@pytest.mark.parametrize("kind", ["f32", "f16", "bf16"])
def test_dense_golden_cases(sk, kind):
    g = np.load(os.path.join(GOLD, "ref_dense.npz"))
    fn = {"f32": sk.sgemm, "f16": sk.sgemm_f16, "bf16": sk.sgemm_bf16}[kind]
    for i, (m, n, k) in enumerate(g["cases"]):
        A, B, C0, alpha, beta = G.dense_case_inputs(i, int(m), int(n), int(k))
        a, b = _dense_operands(kind, A, B)
        if kind == "f16":
            a, b = a.view(np.float16), b.view(np.float16)
        C = C0.copy()
        fn(a, b, C=C, alpha=alpha, beta=beta, trans_b=True)
        y64, mag = O.dense_ref64(a.view(np.uint16) if kind != "f32" else a, kind,
                                 b.view(np.uint16) if kind != "f32" else b, kind)
        want = alpha * y64 + beta * C0.astype(np.float64)
        bound = 2 * (k + 2) * U * (abs(alpha) * mag + abs(beta) * np.abs(C0)) + 1e-300
        assert (np.abs(C - want) <= bound).all(), f"{kind} case {i}"
        assert (np.abs(g[f"{kind}_{i}_simd"] - want) <= bound).all()


@pytest.mark.parametrize("wtype", ["float32", "float16", "bfloat16"])
@pytest.mark.parametrize("M,N,K", [(1, 4096, 4096), (4, 4096, 4096), (8, 1000, 4096), (1, 37, 33), (3, 64, 4099),
                                   (8, 14336, 4096)])
def test_dense_fp32_x(sk, torch, wtype, M, N, K):
    """fp32 activations against fp32/f16/bf16 weights."""
    rng = np.random.default_rng(M + N + K)
    W32 = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    X = rng.standard_normal((M, K)).astype(np.float32)
    if wtype == "float32":
        Wt, Wk, kind = torch.from_numpy(W32), W32, "f32"
    elif wtype == "float16":
        Wt, Wk, kind = torch.from_numpy(W32.astype(np.float16)), W32.astype(np.float16).view(np.uint16), "f16"
    else:
        Wt, Wk, kind = torch.from_numpy(W32).to(torch.bfloat16), O.bf16_bits(W32), "bf16"
    Y = sk.gemv_dense(torch.from_numpy(X).cuda(), Wt.cuda()).cpu().numpy()
    y64, mag = O.dense_ref64(X, "f32", Wk, kind)
    bound = 2 * (K + 2) * U * mag + 1e-300
    assert (np.abs(Y - y64) <= bound).all(), f"max err/bound {np.max(np.abs(Y - y64) / bound):.3g}"


@pytest.mark.parametrize("kind", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("M,N,K", [(1, 1001, 1000), (5, 7, 8), (7, 33, 2056), (2, 3, 16), (8, 13, 520)])
def test_dense_streaming_edges(sk, kind, M, N, K):
    """The TMA-streaming dense kernel's edges: rows not a multiple of the
    4-row item, a last K chunk shorter than 1 KB, K below one chunk, every M,
    and the alpha/beta epilogue."""
    rng = np.random.default_rng(7 * M + N + K)
    A = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    B = rng.uniform(-1, 1, (N, K)).astype(np.float32)
    C0 = rng.uniform(-1, 1, (M, N)).astype(np.float32)
    a, b = _dense_operands(kind, A, B)
    fn = {"f32": sk.sgemm, "f16": sk.sgemm_f16, "bf16": sk.sgemm_bf16}[kind]
    if kind == "f16":
        a, b = a.view(np.float16), b.view(np.float16)
    for alpha, beta in ((1.0, 0.0), (-1.5, 0.5)):
        C = C0.copy()
        fn(a, b, C=C, alpha=alpha, beta=beta, trans_b=True)
        y64, mag = O.dense_ref64(a.view(np.uint16) if kind != "f32" else a, kind,
                                 b.view(np.uint16) if kind != "f32" else b, kind)
        want = alpha * y64 + beta * C0.astype(np.float64)
        bound = 2 * (K + 2) * U * (abs(alpha) * mag + abs(beta) * np.abs(C0)) + 1e-300
        assert (np.abs(C - want) <= bound).all(), f"{kind} alpha={alpha}: max err/bound {np.max(np.abs(C - want) / bound):.3g}"


def test_dense_bf16_special_values(sk, torch):
    """bfloat16 weights with several rows of fp32 x: an infinity in x gives
    infinities of the right signs, a NaN gives NaN (IEEE arithmetic, as the
    reference's fp32 loops), and a value near the fp32 maximum or tiny values
    stay within the bound of the float64 sums."""
    M, N, K = 6, 64, 256
    rng = np.random.default_rng(21)
    W32 = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    Wb = O.bf16_bits(W32)
    X = rng.standard_normal((M, K)).astype(np.float32)
    X[1, 17] = np.inf
    X[2, 100] = np.nan
    X[3, 5] = 3.0e38
    X[4] *= np.float32(1e-30)
    X[5, 200] = -np.inf
    Y = sk.gemv_dense(torch.from_numpy(X).cuda(), torch.from_numpy(W32).to(torch.bfloat16).cuda()).cpu().numpy()
    Wf = O.bf16_to_f32(Wb).astype(np.float64)
    with np.errstate(invalid="ignore", over="ignore"):
        want = X.astype(np.float64) @ Wf.T
    for m in (1, 5):
        assert np.isinf(Y[m]).all() and (np.sign(Y[m]) == np.sign(want[m])).all(), f"row {m}"
    assert np.isnan(Y[2]).all()
    for m in (0, 3, 4):
        y64, mag = O.dense_ref64(X[m:m + 1], "f32", Wb, "bf16")
        bound = 2 * (K + 2) * U * mag + 1e-300
        assert (np.abs(Y[m:m + 1] - y64) <= bound).all(), f"row {m}"


@pytest.mark.parametrize("xtype", ["float32", "bfloat16"])
@pytest.mark.parametrize("M,N,K", [(4, 4096, 4096), (8, 1003, 512), (5, 37, 128), (8, 14336, 1024), (6, 200, 8192)])
def test_dense_bf16_tensor_core_kernel(sk, torch, xtype, M, N, K):
    """bfloat16 weights with 4..8 rows of x take the tensor-core kernel (x split
    exactly into bf16 parts; one part when x is bfloat16 itself). Against the
    float64 sums within the reference's dense bound, for tile counts that split
    K over the warps (small N) and N not a multiple of 16, and the same call on
    the CUDA-core kernel (SMK_OPT_DENSE_MMA = 0) within the same bound."""
    from simd_ml_kernels import _core
    rng = np.random.default_rng(M * 7 + N + K)
    W32 = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    X = rng.standard_normal((M, K)).astype(np.float32)
    Wbits = O.bf16_bits(W32)
    if xtype == "float32":   # the device entry: fp32 x, bf16 W (torch tensors)
        run = lambda: sk.gemv_dense(torch.from_numpy(X).cuda(), torch.from_numpy(W32).to(torch.bfloat16).cuda())  # noqa: E731
        want, mag = O.dense_ref64(X, "f32", Wbits, "bf16")
    else:   # the reference's sgemm_bf16: both operands bf16 (host arrays)
        Xbits = O.bf16_bits(X)

        def run():
            C = np.zeros((M, N), np.float32)
            sk.sgemm_bf16(Xbits, Wbits, C=C, trans_b=True)
            return C
        want, mag = O.dense_ref64(Xbits, "bf16", Wbits, "bf16")
    bound = 2 * (K + 2) * U * mag + 1e-300
    try:
        for mma in (1, 0):
            _core._ctx_set(7, mma)
            got = run()
            got = got.cpu().numpy() if hasattr(got, "cpu") else got
            assert (np.abs(got - want) <= bound).all(), f"mma={mma}: max err/bound {np.max(np.abs(got - want) / bound):.3g}"
    finally:
        _core._ctx_set(7, 1)
    assert _core._device_error(torch.cuda.current_stream().cuda_stream) == 0


def test_dense_bf16_tensor_core_infinite_weight(sk, torch):
    """An infinite weight meets x values whose lower bf16 parts are zero (x = 1,
    2, 0.5 ...): the reference's single product gives ±inf, the tensor-core
    kernel's low-part product 0·inf would give NaN, so that output is recomputed
    in plain fp32 and comes out ±inf; a zero x next to an infinite weight gives
    NaN in both."""
    M, N, K = 4, 64, 256
    rng = np.random.default_rng(5)
    W32 = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    W32[3, 10] = np.inf
    W32[7, 20] = -np.inf
    X = np.round(rng.standard_normal((M, K)) * 4).astype(np.float32) / 4   # few significant bits
    X[:, 10] = 2.0
    X[:, 20] = 0.5
    X[2, 20] = 0.0
    Y = sk.gemv_dense(torch.from_numpy(X).cuda(), torch.from_numpy(W32).to(torch.bfloat16).cuda()).cpu().numpy()
    assert (Y[:, 3] == np.inf).all()
    assert (Y[[0, 1, 3], 7] == -np.inf).all() and np.isnan(Y[2, 7])
    fin = np.ones(N, bool)
    fin[[3, 7]] = False
    y64, mag = O.dense_ref64(X, "f32", O.bf16_bits(W32[fin]), "bf16")
    assert (np.abs(Y[:, fin] - y64) <= 2 * (K + 2) * U * mag + 1e-300).all()


@pytest.mark.parametrize("M,N,K", [(6, 4096, 4096), (8, 1003, 512), (7, 37, 128), (8, 14336, 1024), (6, 200, 8192)])
def test_dense_f16_tensor_core_kernel(sk, torch, M, N, K):
    """float16 weights with 6..8 rows of float32 x take the tensor-core kernel:
    each weight split exactly into two bf16 parts (hi, and a lo of at most 3
    significant bits), x into three, every product exact. Weights with a wide
    spread of magnitudes (fp16 subnormals included) against the float64 sums
    within the reference's dense bound, on the tensor-core kernel and on the
    CUDA-core kernel (SMK_OPT_DENSE_MMA = 0)."""
    from simd_ml_kernels import _core
    rng = np.random.default_rng(M * 11 + N + K)
    W16 = (rng.standard_normal((N, K)) * 0.02 * np.exp2(rng.integers(-14, 6, (N, K)))).astype(np.float16)
    X = rng.standard_normal((M, K)).astype(np.float32)
    want, mag = O.dense_ref64(X, "f32", W16.view(np.uint16), "f16")
    bound = 2 * (K + 2) * U * mag + 1e-300
    wd = torch.from_numpy(W16).cuda()
    try:
        for mma in (1, 0):
            _core._ctx_set(7, mma)
            got = sk.gemv_dense(torch.from_numpy(X).cuda(), wd).cpu().numpy()
            assert (np.abs(got - want) <= bound).all(), f"mma={mma}: max err/bound {np.max(np.abs(got - want) / bound):.3g}"
    finally:
        _core._ctx_set(7, 1)
    assert _core._device_error(torch.cuda.current_stream().cuda_stream) == 0


def test_dense_f16_tensor_core_infinite_weight(sk, torch):
    """An infinite fp16 weight makes its lo part NaN in the tensor-core kernel;
    the output is recomputed in plain fp32: ±inf as the reference's single
    product gives, NaN where the weight meets a zero x."""
    M, N, K = 6, 64, 256
    rng = np.random.default_rng(6)
    W16 = (rng.standard_normal((N, K)) * 0.02).astype(np.float16)
    W16[3, 10] = np.inf
    W16[7, 20] = -np.inf
    X = rng.standard_normal((M, K)).astype(np.float32)
    X[:, 10] = 2.0
    X[:, 20] = 0.5
    X[2, 20] = 0.0
    Y = sk.gemv_dense(torch.from_numpy(X).cuda(), torch.from_numpy(W16).cuda()).cpu().numpy()
    assert (Y[:, 3] == np.inf).all()
    assert (Y[[0, 1, 3], 7] == -np.inf).all() and np.isnan(Y[2, 7])
    fin = np.ones(N, bool)
    fin[[3, 7]] = False
    y64, mag = O.dense_ref64(X, "f32", W16[fin].view(np.uint16), "f16")
    assert (np.abs(Y[:, fin] - y64) <= 2 * (K + 2) * U * mag + 1e-300).all()


def test_dense_rejects_non_decode(sk):
    A = np.ones((9, 16), np.float32)
    B = np.ones((4, 16), np.float32)
    with pytest.raises(sk.ArgumentError, match="decode"):
        sk.sgemm(A, B, trans_b=True)
    with pytest.raises(sk.ArgumentError, match="decode"):
        sk.sgemm(A[:2], B.T.copy())


# ---- INT8 sgemm_u8s8 (trans_b, M <= 8) ------------------------------------------------

def test_u8s8_golden_bitwise(sk, torch):
    """Every golden case, through host arrays and through CUDA tensors:
    bitwise the reference's scalar table (exact sums and its epilogue)."""
    g = np.load(os.path.join(GOLD, "ref_u8s8.npz"))
    for i, (m, n, k, zp) in enumerate(g["cases"]):
        A, W, scales, a_scale = G.u8s8_case_inputs(i, int(m), int(n), int(k))
        want = g[f"tb1_{i}_scalar"]
        got = sk.sgemm_u8s8(A, W, a_scale, int(zp), scales, trans_b=True)
        assert got.dtype == np.float32 and got.shape == (m, n)
        np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32), err_msg=f"case {i}")
        dev = sk.sgemm_u8s8(torch.from_numpy(A).cuda(), torch.from_numpy(W).cuda(), a_scale, int(zp),
                            torch.from_numpy(scales).cuda(), trans_b=True)
        np.testing.assert_array_equal(dev.cpu().numpy().view(np.uint32), want.view(np.uint32), err_msg=f"case {i}")


def _u8s8_case(seed, M, N, K):
    rng = np.random.default_rng(seed)
    A = rng.integers(0, 256, (M, K), dtype=np.uint8)
    W = rng.integers(-128, 128, (N, K), dtype=np.int8)
    return A, W, rng.uniform(-0.1, 0.1, N).astype(np.float32)


@pytest.mark.parametrize("M,N,K,zp", [
    (1, 4096, 4096, 128),      # the row path's shape; A in shared memory
    (8, 4096, 4096, 0),        # zero point 0: no column sums
    (4, 1003, 2048, 255),      # ragged N
    (1, 333, 1040, 3),         # K tail inside an item
    (8, 2048, 28672, 77),      # A too large for shared memory: read through L1
    (3, 17, 40, 9),            # K % 16 != 0: the per-byte kernel
    (1, 8, 1049600, 128),      # more than 1024 items per row: the per-byte kernel's int64 sums
    (8, 3000, 4096, 77),       # tensor-core kernel: 8 rows, Σ W by an extra MMA, ragged N, K split
    (5, 777, 1040, 200),       # tensor-core kernel: Σ W from a row of ones, K tail inside an item
])
def test_u8s8_shapes_bitwise_oracle(sk, torch, M, N, K, zp):
    A, W, scales = _u8s8_case(M * 131 + N + K, M, N, K)
    want = O.sgemm_u8s8(A, W, 0.0173, zp, scales, True)
    got = sk.sgemm_u8s8(torch.from_numpy(A).cuda(), torch.from_numpy(W).cuda(), 0.0173, zp,
                        torch.from_numpy(scales).cuda(), trans_b=True).cpu().numpy()
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))


def test_u8s8_unaligned_and_extreme(sk, torch):
    """Views of A and W at odd byte offsets (A staged byte by byte, W through
    the per-byte kernel) give the same bits; A = 255, W = -128, zp = 0 is
    exact (the largest sums: -255·128·K)."""
    M, N, K, zp = 3, 257, 2048, 100
    A, W, scales = _u8s8_case(5, M, N, K)
    want = O.sgemm_u8s8(A, W, 0.25, zp, scales, True)
    abuf = torch.zeros(M * K + 16, dtype=torch.uint8, device="cuda")
    wbuf = torch.zeros(N * K + 16, dtype=torch.int8, device="cuda")
    for ao, wo in ((3, 0), (0, 1), (5, 7)):
        a = abuf[ao:ao + M * K].view(M, K)
        w = wbuf[wo:wo + N * K].view(N, K)
        a.copy_(torch.from_numpy(A))
        w.copy_(torch.from_numpy(W))
        got = sk.sgemm_u8s8(a, w, 0.25, zp, torch.from_numpy(scales).cuda(), trans_b=True).cpu().numpy()
        np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32), err_msg=f"offsets {ao}, {wo}")
    K = 4096
    got = sk.sgemm_u8s8(np.full((8, K), 255, np.uint8), np.full((33, K), -128, np.int8), 1.0, 0,
                        np.ones(33, np.float32), trans_b=True)
    np.testing.assert_array_equal(got, np.full((8, 33), -255.0 * 128 * K, np.float32))


def test_u8s8_in_cuda_graph(sk, torch):
    """The CUDA-tensor path only launches on torch's current stream: it
    captures into a CUDA graph, and replays give the oracle's bits."""
    M, N, K, zp = 2, 1536, 3072, 17
    A, W, scales = _u8s8_case(9, M, N, K)
    a, w, s = torch.from_numpy(A).cuda(), torch.from_numpy(W).cuda(), torch.from_numpy(scales).cuda()
    C = torch.empty((M, N), device="cuda")
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        sk.sgemm_u8s8(a, w, 0.5, zp, s, C, trans_b=True)   # warm-up outside capture
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            sk.sgemm_u8s8(a, w, 0.5, zp, s, C, trans_b=True)
    C.zero_()
    g.replay()
    torch.cuda.synchronize()
    np.testing.assert_array_equal(C.cpu().numpy().view(np.uint32),
                                  O.sgemm_u8s8(A, W, 0.5, zp, scales, True).view(np.uint32))
    del g


def test_no_device_errors(sk):
    from simd_ml_kernels import _core
    assert _core._device_error(0) == 0
