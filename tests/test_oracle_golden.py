"""The oracle (oracle/smk_oracle.c) against the golden vectors the reference
itself produced (tests/golden/, written by make_golden.py from the reference
compiled from its sources, and the llama.cpp fixture of the reference's
tests). CPU only. This is what makes the oracle trustworthy as the checker of
the GPU parity tests."""

from __future__ import annotations

import hashlib
import os

import numpy as np
import pytest

import oracle as O
import make_golden as G

GOLD = os.path.join(os.path.dirname(__file__), "golden")
U = 2.0 ** -24


def load(name):
    return np.load(os.path.join(GOLD, name))


def sha(b):
    return hashlib.sha256(np.ascontiguousarray(b).tobytes()).hexdigest()


def test_llama_cpp_fixture_byte_exact():
    """quantize_q4_0 byte for byte against llama.cpp v0.7.0's blocks
    (reference tests/test_precision.py:705-719)."""
    fx = load("q4_0_llama_cpp_fixture.npz")
    assert fx["w"].shape == (20, 256)
    np.testing.assert_array_equal(O.quantize("q4_0", fx["w"]), fx["blocks"])
    blk = fx["blocks"].reshape(20, 8, 18)
    assert blk[14, 0, :2].view("<u2")[0] == 0x8000          # zero block: d = -0.0
    assert (blk[14, 0, 2:] == 0x88).all()


@pytest.mark.parametrize("fmt", ["q4_0", "q8_0"])
def test_quantize_matches_reference(fmt):
    g = load("ref_quantize.npz")
    for i in range(4):
        np.testing.assert_array_equal(O.quantize(fmt, g[f"w{i}"]), g[f"{fmt}_{i}"])
    np.testing.assert_array_equal(O.quantize(fmt, g["w_special"]), g[f"{fmt}_special"])
    rej = g["w_reject"]
    for i in range(rej.shape[0]):
        ok = True
        try:
            O.quantize(fmt, rej[i:i + 1])
        except ValueError:
            ok = False
        assert ok == bool(g[f"{fmt}_reject_ok"][i]), (fmt, i)


def test_quantize_x_matches_reference():
    g = load("ref_quantize_x.npz")
    for i in range(3):
        qs, dx, ok = O.quantize_x(g[f"x{i}"])
        assert ok == bool(g[f"ok{i}"])
        np.testing.assert_array_equal(qs, g[f"qs{i}"])
        np.testing.assert_array_equal(dx.view(np.uint32), g[f"dx{i}"].view(np.uint32))
    assert not O.quantize_x(g["x_bad"])[2] and not g["ok_bad"]


@pytest.mark.parametrize("fmt", ["q4_0", "q8_0"])
def test_gemv_matches_reference(fmt):
    """Scalar-order oracle bit for bit against the reference's scalar table;
    the reference's SIMD table within its documented bound of the float64 sum."""
    g = load("ref_gemv.npz")
    for s, n, k, extreme in g["cases"]:
        W, x = G.gemv_case_inputs(int(s), int(n), int(k), "extreme" if extreme else "normal")
        Wq = O.quantize(fmt, W)
        assert sha(Wq) == str(g[f"{fmt}_{s}_sha"]), f"input drift at case {s}"
        y = O.gemv_scalar(fmt, x, Wq, int(n), int(k))
        np.testing.assert_array_equal(y.view(np.uint32), g[f"{fmt}_{s}_scalar"].view(np.uint32))
        y64, mag = O.ref64(fmt, x, Wq, int(n), int(k))
        bound = 2 * (k // 32 + 4) * U * mag + 1e-300
        assert (np.abs(g[f"{fmt}_{s}_simd"].astype(np.float64) - y64) <= bound).all()
        assert (np.abs(y.astype(np.float64) - y64) <= bound).all()


@pytest.mark.parametrize("fmt", ["q4_0", "q8_0"])
def test_block_sums_consistent(fmt):
    """The oracle's per-block int sums reproduce its float64 result."""
    rng = np.random.default_rng(3)
    N, K = 9, 320
    W = rng.standard_normal((N, K)).astype(np.float32)
    x = rng.standard_normal(K).astype(np.float32)
    Wq = O.quantize(fmt, W)
    qs, dx, ok = O.quantize_x(x)
    sums = O.block_sums(fmt, qs, Wq, N, K)
    bpb = O.BLOCK_BYTES[fmt]
    d = np.ascontiguousarray(Wq.reshape(N, K // 32, bpb)[:, :, :2]).view("<f2")[:, :, 0].astype(np.float64)
    y64 = (sums.astype(np.float64) * d * dx.astype(np.float64)[None, :]).sum(axis=1)
    ref, _ = O.ref64(fmt, x, Wq, N, K)
    np.testing.assert_allclose(y64, ref, rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("kind", ["f32", "f16", "bf16"])
def test_dense_matches_reference(kind):
    g = load("ref_dense.npz")
    for i, (m, n, k) in enumerate(g["cases"]):
        A, B, C0, alpha, beta = G.dense_case_inputs(i, int(m), int(n), int(k))
        assert sha(np.concatenate([A.ravel(), B.ravel(), C0.ravel()])) == str(g[f"sha{i}"])
        a, b = G.dense_operands(kind, A, B)
        got = O.dense_scalar(a, kind, b, kind, alpha, beta, C0)
        np.testing.assert_array_equal(got.view(np.uint32), g[f"{kind}_{i}_scalar"].view(np.uint32))
        y64, mag = O.dense_ref64(a, kind, b, kind)
        want = alpha * y64 + beta * C0.astype(np.float64)
        bound = 2 * (k + 2) * U * (abs(alpha) * mag + abs(beta) * np.abs(C0)) + 1e-300
        assert (np.abs(g[f"{kind}_{i}_simd"] - want) <= bound).all()


def test_u8s8_matches_reference():
    """sgemm_u8s8: the restatement is bitwise the reference's scalar table for
    both B layouts, and the reference's table for this CPU is within the
    documented bound 2(K+2)u·|a_scale·b_j|·Σ|A − zp||B| of the exact sums
    (int8_gemm.hpp:23-24, tests/test_precision.py:262-280 there)."""
    g = load("ref_u8s8.npz")
    for i, (m, n, k, zp) in enumerate(g["cases"]):
        A, W, scales, a_scale = G.u8s8_case_inputs(i, int(m), int(n), int(k))
        assert sha(np.concatenate([A.view(np.uint8).ravel(), W.view(np.uint8).ravel(),
                                   scales.view(np.uint8)])) == str(g[f"sha{i}"])
        sc = np.float64(a_scale) * scales.astype(np.float64)
        for tb in (1, 0):
            B = W if tb else np.ascontiguousarray(W.T)
            got = O.sgemm_u8s8(A, B, a_scale, int(zp), scales, bool(tb))
            np.testing.assert_array_equal(got.view(np.uint32), g[f"tb{tb}_{i}_scalar"].view(np.uint32))
            s64, mag = O.u8s8_ref64(A, B, int(zp), bool(tb))
            bound = 2 * (int(k) + 2) * U * mag * np.abs(sc) + 1e-30
            assert (np.abs(g[f"tb{tb}_{i}_simd"] - s64 * sc) <= bound).all()
    # The all-extreme case is exact: -255·128·K.
    m, n, k, _ = g["cases"][G.U8S8_EXTREME]
    np.testing.assert_array_equal(g[f"tb1_{G.U8S8_EXTREME}_scalar"], np.full((m, n), -255.0 * 128 * k, np.float32))


def test_fp16_conversion_sample():
    """binary32 -> binary16 RNE on every half-way point between consecutive
    halves, their neighbours, and a random sample (the reference's exhaustive
    fp32_to_fp16 test restated, test_q8_0.cpp:40-67)."""
    h = np.arange(0, 0x7c00, dtype=np.uint32)
    lo = h.astype(np.uint16).view(np.float16).astype(np.float32)
    hi = (h + 1).astype(np.uint16).view(np.float16).astype(np.float32)
    mid = ((lo.astype(np.float64) + hi.astype(np.float64)) / 2).astype(np.float32)
    mids = mid.view(np.uint32)
    xs = np.concatenate([mids, mids - 1, mids + 1, lo.view(np.uint32)])
    xs = np.concatenate([xs, xs | 0x80000000, np.random.default_rng(0).integers(0, 2**32, 2_000_000, dtype=np.uint64).astype(np.uint32)])
    f = xs.view(np.float32)
    with np.errstate(over="ignore", invalid="ignore"):
        want = f.astype(np.float16).view(np.uint16).copy()
    nan = np.isnan(f)
    want[nan] = (0x7E00 | ((xs[nan] >> 16) & 0x8000)).astype(np.uint16)
    np.testing.assert_array_equal(O.fp32_to_fp16_bits(f), want)


def test_gemv_slice_rules():
    """Contiguous whole 8-row groups, sizes within one group of each other
    (reference dispatch.cpp:373-379)."""
    for N in (1, 7, 8, 9, 100, 1003, 128256):
        for parts in (1, 2, 3, 4, 8):
            edges = [O.gemv_slice(N, t, parts) for t in range(parts)]
            assert edges[0][0] == 0 and edges[-1][1] == N
            for (a, b), (c, d) in zip(edges, edges[1:]):
                assert b == c
            for lo, hi in edges:
                assert lo % 8 == 0 and lo <= hi


def test_config_pins_reproduce_on_cpu():
    """bench.py's generators give, on any host, the bytes the GPU tests pin
    (tests/golden/config_pins.json, written with the reference's quantizer):
    config 0's Q4_0 weights through the oracle's quantizer, config 3's
    float32 weights and their bfloat16 / float16 roundings."""
    import hashlib
    import json

    import bench

    pins = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "config_pins.json")))
    sha = lambda a: hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()  # noqa: E731
    W, x = bench.config0().full()
    assert sha(O.quantize("q4_0", W)) == pins["config0"]["w_sha256"] and sha(x) == pins["config0"]["x_sha256"]
    N, K = bench.CFG3_SHAPES[0]
    W, X = bench.config3(N, K).full()
    p3 = pins["config3"][0]
    assert sha(W) == p3["float32_sha256"] and sha(X) == p3["x_sha256"]
    assert sha(O.bf16_bits(W)) == p3["bfloat16_sha256"]
    assert sha(W.astype(np.float16).view(np.uint16)) == p3["float16_sha256"]
