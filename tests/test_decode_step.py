"""The rest of a Llama decode step on the GPU (simd_ml_kernels.decode): residual
add + RMSNorm, RoPE + KV-cache write, grouped-query attention, and the whole
token step of LlamaDecoder.

Checkers: the reference's own functions (rope_inv_freq, rope_cos_sin,
apply_rope, Llama._rope, rms_norm of examples/llama/llama.py, evaluated by
tests/golden/make_decode_golden.py into ref_decode.npz) and the float64
restatements of oracle/decode_oracle.py, which the CPU tests here pin to those
golden vectors. Tolerances: a few float32 ulps of the values' magnitudes for
RMSNorm and RoPE (CUDA's cosf/sinf against NumPy's float32 cos/sin differ by an
ulp or two), 1e-5 of the output magnitude for attention (float32 sums in
another order); the end-to-end logits within 1e-3 (L2, relative) of the
float64 step, where an activation that lands on a Q8 rounding boundary may
round the other way.
"""

from __future__ import annotations

import math
import os

import numpy as np
import pytest

import decode_oracle as D
import oracle as O
from simd_ml_kernels import decode as dec

GOLD = np.load(os.path.join(os.path.dirname(__file__), "golden", "ref_decode.npz"))
LLAMA3 = {"factor": 32.0, "high_freq_factor": 4.0, "low_freq_factor": 1.0, "original_max_position_embeddings": 8192,
          "rope_type": "llama3"}
ROPE = {"llama3": (64, 500000.0, LLAMA3), "default": (128, 10000.0, None)}
U = 2.0 ** -24


# ---- CPU: the host math and the oracle against the reference --------------------------

@pytest.mark.parametrize("name", sorted(ROPE))
def test_rope_inv_freq_bitwise_reference(name):
    hd, theta, scaling = ROPE[name]
    got = dec.rope_inv_freq(hd, theta, scaling)
    assert np.array_equal(got.view(np.uint32), GOLD[f"{name}:inv_freq"].view(np.uint32))


@pytest.mark.parametrize("name", sorted(ROPE))
def test_oracle_rope_matches_reference(name):
    """rope64 against the reference's apply_rope and interleaved Llama._rope."""
    inv = GOLD[f"{name}:inv_freq"]
    for pos in (0, 1, 77, 4000):
        x = GOLD[f"{name}:{pos}:x"]
        bound = 4 * U * (np.abs(x) + np.abs(x[:, ::-1])).max() + 1e-30
        for layout, il in (("hf", False), ("interleaved", True)):
            got = D.rope64(x, inv, pos, il)
            assert np.abs(got - GOLD[f"{name}:{pos}:{layout}"]).max() <= bound, (name, pos, layout)


def test_oracle_rms_norm_matches_reference():
    for i in range(2):
        x, w, h = GOLD[f"rms:{i}:x"], GOLD[f"rms:{i}:w"], GOLD[f"rms:{i}:h"]
        got = D.rms_norm64(x, w, 1e-5)
        assert (np.abs(got - h) <= 8 * U * np.abs(got) + 1e-30).all()


# ---- GPU kernels ----------------------------------------------------------------

@pytest.fixture(scope="module")
def torch(cuda_device):
    import torch as t
    return t


@pytest.mark.gpu
def test_add_rmsnorm(torch):
    """x += delta in place (bitwise the float32 sum), h within 16 ulps of the
    float64 RMSNorm; against the reference's own rms_norm within the same."""
    rng = np.random.default_rng(1)
    for M, n in ((1, 2048), (3, 2048), (2, 8192), (1, 333), (4, 1)):
        x = (rng.standard_normal((M, n)) * 2).astype(np.float32)
        dl = rng.standard_normal((M, n)).astype(np.float32)
        w = (1 + 0.1 * rng.standard_normal(n)).astype(np.float32)
        xd, dd, wd = (torch.from_numpy(a).cuda() for a in (x, dl, w))
        h = dec.add_rmsnorm(xd, wd, 1e-5, delta=dd).cpu().numpy()
        xs = x + dl
        np.testing.assert_array_equal(xd.cpu().numpy().view(np.uint32), xs.view(np.uint32))
        for m in range(M):
            want = D.rms_norm64(xs[m], w, 1e-5)
            assert (np.abs(h[m] - want) <= 16 * U * np.abs(want) + 1e-30).all(), (M, n, m)
    for i in range(2):
        x, w, want = GOLD[f"rms:{i}:x"], GOLD[f"rms:{i}:w"], GOLD[f"rms:{i}:h"]
        got = dec.add_rmsnorm(torch.from_numpy(x.copy()).cuda(), torch.from_numpy(w).cuda(), 1e-5).cpu().numpy()
        assert (np.abs(got - want) <= 16 * U * np.abs(want) + 1e-30).all()


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(ROPE))
@pytest.mark.parametrize("interleaved", [False, True])
def test_rope_kv(torch, name, interleaved):
    """q and k rotated as the reference (its golden outputs and the float64
    rotation), k and v written to row pos of the caches, other rows untouched."""
    hd, theta, scaling = ROPE[name]
    inv = dec.rope_inv_freq(hd, theta, scaling)
    nh, nkv, cap = 6, 2, 4096 + 8
    rng = np.random.default_rng(hd)
    for pos in (0, 1, 77, 4000):
        qkv = rng.standard_normal((nh + 2 * nkv) * hd).astype(np.float32)
        x = GOLD[f"{name}:{pos}:x"]   # 6 rows: the q heads take the reference's inputs
        qkv[:nh * hd] = x.reshape(-1)
        kc = torch.full((nkv, cap, hd), 7.0, device="cuda")
        vc = torch.full((nkv, cap, hd), 7.0, device="cuda")
        q = dec.rope_kv(torch.from_numpy(qkv).cuda(), torch.from_numpy(inv).cuda(), pos, nh, nkv, hd, kc, vc,
                        interleaved=interleaved).cpu().numpy()
        ref = GOLD[f"{name}:{pos}:{'interleaved' if interleaved else 'hf'}"]
        mag = 2 * np.abs(x).max()   # |a| + |b| of any pair
        assert np.abs(q - ref).max() <= 8 * U * mag, (name, pos)
        k_want = D.rope64(qkv[nh * hd:(nh + nkv) * hd].reshape(nkv, hd), inv, pos, interleaved)
        kh, vh = kc.cpu().numpy(), vc.cpu().numpy()
        assert np.abs(kh[:, pos] - k_want).max() <= 8 * U * np.abs(qkv).max()
        np.testing.assert_array_equal(vh[:, pos], qkv[(nh + nkv) * hd:].reshape(nkv, hd))
        others = np.delete(kh, pos, axis=1)
        assert (others == 7.0).all() and (np.delete(vh, pos, axis=1) == 7.0).all()


@pytest.mark.gpu
@pytest.mark.parametrize("nh,nkv,hd", [(32, 8, 64), (8, 8, 128), (16, 2, 32)])
@pytest.mark.parametrize("length", [1, 7, 256, 300, 1000, 2049])
def test_attention_decode(torch, nh, nkv, hd, length):
    """GQA attention of one token over `length` cached positions against the
    float64 softmax attention; beyond 256 positions the chunks are combined
    by the last CTA of each KV head (the tickets reset for the next call)."""
    cap = 2112
    rng = np.random.default_rng(length + nh)
    q = rng.standard_normal((nh, hd)).astype(np.float32)
    k = rng.standard_normal((nkv, cap, hd)).astype(np.float32)
    v = rng.standard_normal((nkv, cap, hd)).astype(np.float32)
    qd, kd, vd = (torch.from_numpy(a).cuda() for a in (q, k, v))
    want = D.attention64(q, k, v, length)
    for _ in range(2):   # twice: the combine tickets start from zero again
        got = dec.attention_decode(qd, kd, vd, length, nkv, max_len=cap).cpu().numpy()
        assert np.abs(got - want).max() <= 1e-5 * np.abs(want).max(), (nh, nkv, hd, length)
    from simd_ml_kernels import _core
    assert _core._device_error(torch.cuda.current_stream().cuda_stream) == 0


@pytest.mark.gpu
@pytest.mark.parametrize("nh,nkv,hd,interleaved", [(32, 8, 64, False), (8, 8, 128, True), (16, 2, 32, False)])
@pytest.mark.parametrize("pos,max_len", [(0, 1), (6, 300), (255, 256), (256, 600), (1500, 2112)])
def test_rope_attention_equals_unfused(torch, nh, nkv, hd, interleaved, pos, max_len):
    """The fused kernel (RoPE, cache write and attention in one launch) gives the
    bits of rope_kv followed by attention_decode: the same attention output,
    the same k and v rows at pos, and nothing else of the caches touched; with
    one chunk and with several (the position in the first, a middle or the
    last chunk)."""
    cap = 2112
    rng = np.random.default_rng(pos + nh + hd)
    inv = torch.from_numpy(dec.rope_inv_freq(hd, 500000.0, LLAMA3)).cuda()
    qkv = torch.from_numpy(rng.standard_normal((nh + 2 * nkv) * hd).astype(np.float32)).cuda()
    k0 = rng.standard_normal((nkv, cap, hd)).astype(np.float32)
    v0 = rng.standard_normal((nkv, cap, hd)).astype(np.float32)
    kc1, vc1 = torch.from_numpy(k0).cuda(), torch.from_numpy(v0).cuda()
    kc2, vc2 = kc1.clone(), vc1.clone()
    q = dec.rope_kv(qkv, inv, pos, nh, nkv, hd, kc1, vc1, interleaved=interleaved)
    want = dec.attention_decode(q, kc1, vc1, pos + 1, nkv, max_len=max_len).cpu().numpy()
    for _ in range(2):   # twice: the combine tickets start from zero again
        got = dec.rope_attention(qkv, inv, pos, nh, nkv, hd, kc2, vc2, interleaved=interleaved,
                                 max_len=max_len).cpu().numpy()
        np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
    assert torch.equal(kc1.view(torch.int32), kc2.view(torch.int32))
    assert torch.equal(vc1.view(torch.int32), vc2.view(torch.int32))
    from simd_ml_kernels import _core
    assert _core._device_error(torch.cuda.current_stream().cuda_stream) == 0


@pytest.mark.gpu
def test_rope_attention_host_errors(torch):
    """A position outside 0 .. max_len-1 is refused on the host, before a launch."""
    qkv = torch.zeros(6 * 32, device="cuda")
    inv = torch.ones(16, device="cuda")
    kc = torch.zeros((1, 8, 32), device="cuda")
    with pytest.raises(Exception, match="outside"):
        dec.rope_attention(qkv, inv, 5, 4, 1, 32, kc, kc.clone(), max_len=4)


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", ["q4_0", "q8_0"])
@pytest.mark.parametrize("N,K", [(3072, 2048), (2048, 2048), (1000, 4096), (2048, 8192), (128256, 2048)])
def test_gemv_rmsnorm_equals_unfused(torch, fmt, N, K):
    """The RMSNorm fused into the GEMV's x quantization gives the bits of
    add_rmsnorm followed by the GEMV. x holds small integers, so the sum of
    squares is exact in any order and both paths see the same normalised row;
    the shapes reach the four-row kernel (K = 2048), the superblock kernel and x
    quantized once in global memory (K = 8192)."""
    import simd_ml_kernels as sk
    rng = np.random.default_rng(N + K)
    x = rng.integers(-8, 9, K).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(K)).astype(np.float32)
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    quant = sk.quantize_q4_0 if fmt == "q4_0" else sk.quantize_q8_0
    gemv = sk.gemv_q4_0 if fmt == "q4_0" else sk.gemv_q8_0
    Wq = quant(torch.from_numpy(W).cuda()).reshape(-1)
    xd, wd = torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda()
    got = dec.gemv_rmsnorm(xd, wd, 1e-5, Wq, N, K, fmt).cpu().numpy()
    h = dec.add_rmsnorm(xd.clone(), wd, 1e-5)
    want = gemv(h, Wq, N, K).cpu().numpy()
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
    assert torch.equal(xd, torch.from_numpy(x).cuda())   # x is not modified


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", ["q4_0", "q8_0"])
@pytest.mark.parametrize("N,K", [(2048, 2048), (2048, 8192), (1000, 4096)])
def test_gemv_residual_equals_unfused(torch, fmt, N, K):
    """The residual add fused into the GEMV's store: r += x @ W.T in place,
    and r += (silu(gate) * up) @ W.T, each bitwise fl(r + the plain GEMV)."""
    import simd_ml_kernels as sk
    rng = np.random.default_rng(3 * N + K)
    x = rng.standard_normal(K).astype(np.float32)
    up = rng.standard_normal(K).astype(np.float32)
    r0 = rng.standard_normal(N).astype(np.float32)
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    quant = sk.quantize_q4_0 if fmt == "q4_0" else sk.quantize_q8_0
    gemv = sk.gemv_q4_0 if fmt == "q4_0" else sk.gemv_q8_0
    silu = sk.gemv_q4_0_silu_mul if fmt == "q4_0" else sk.gemv_q8_0_silu_mul
    Wq = quant(torch.from_numpy(W).cuda()).reshape(-1)
    xd, ud = torch.from_numpy(x).cuda(), torch.from_numpy(up).cuda()
    r = torch.from_numpy(r0).cuda()
    dec.gemv_residual(xd, Wq, N, K, r, fmt)
    want = torch.from_numpy(r0).cuda() + gemv(xd, Wq, N, K)
    assert torch.equal(r.view(torch.int32), want.view(torch.int32))
    r2 = torch.from_numpy(r0).cuda()
    dec.gemv_residual(xd, Wq, N, K, r2, fmt, up=ud)
    want2 = torch.from_numpy(r0).cuda() + silu(xd, ud, Wq, N, K)
    assert torch.equal(r2.view(torch.int32), want2.view(torch.int32))


def _small_model(torch, fmt, seed=11, interleaved=False):
    import simd_ml_kernels as sk
    sh = dec.LlamaShape(hidden=256, layers=2, heads=4, kv_heads=2, head_dim=64, ffn=512, vocab=512, eps=1e-5)
    rng = np.random.default_rng(seed)
    quant = sk.quantize_q4_0 if fmt == "q4_0" else sk.quantize_q8_0

    def q(n, k, sigma=0.05):
        w = (rng.standard_normal((n, k)) * sigma).astype(np.float32)
        return quant(torch.from_numpy(w).cuda())

    def norm(n):
        return torch.from_numpy((1 + 0.1 * rng.standard_normal(n)).astype(np.float32)).cuda()

    H, nh, nkv, hd, F = sh.hidden, sh.heads, sh.kv_heads, sh.head_dim, sh.ffn
    layers = [dec.LlamaLayerWeights(attn_norm=norm(H), qkv=q((nh + 2 * nkv) * hd, H), o=q(H, nh * hd),
                                    mlp_norm=norm(H), gate_up=q(2 * F, H), down=q(H, F))
              for _ in range(sh.layers)]
    embed = q(sh.vocab, H, 1.0)
    w = dec.LlamaWeights(layers=layers, norm=norm(H), embed=embed, lm_head=embed, fmt=fmt)
    inv = dec.rope_inv_freq(hd, 500000.0, LLAMA3)
    host = {"hidden": H, "layers": sh.layers, "heads": nh, "kv_heads": nkv, "head_dim": hd, "ffn": F,
            "vocab": sh.vocab, "eps": sh.eps, "fmt": fmt, "inv_freq": inv, "interleaved": interleaved,
            "embed": embed.cpu().numpy(), "lm_head": embed.cpu().numpy(), "norm": w.norm.cpu().numpy(),
            "layer_weights": [{k: getattr(L, k).cpu().numpy() for k in ("attn_norm", "qkv", "o", "mlp_norm",
                                                                        "gate_up", "down")} for L in layers]}
    return sh, w, inv, host


@pytest.mark.gpu
@pytest.mark.parametrize("fmt,interleaved", [("q4_0", False), ("q8_0", True)])
def test_llama_decoder_matches_float64_step(torch, fmt, interleaved):
    """A 2-layer GQA model, 6 tokens: every step's logits within 1e-3 (L2,
    relative) of the float64 restatement of the reference's Llama.step on the
    same quantized weights, and the same logits when the steps are captured in
    a CUDA graph and replayed from a reset cache."""
    sh, w, inv, host = _small_model(torch, fmt, interleaved=interleaved)
    tokens = [3, 141, 59, 265, 358, 97]
    cap = 16
    d = dec.LlamaDecoder(sh, w, inv, capacity=cap, interleaved=interleaved)
    got = [d.step(t).cpu().numpy().copy() for t in tokens]
    want = D.step64(host, tokens, cap)
    for i, (g, ww) in enumerate(zip(got, want)):
        assert np.isfinite(g).all()
        rel = np.linalg.norm(g - ww) / np.linalg.norm(ww)
        assert rel <= 1e-3, f"token {i}: relative L2 error {rel:.3g}"
    # The same steps, captured once and replayed.
    d.reset()
    graph = torch.cuda.CUDAGraph()
    outs = [torch.empty(sh.vocab, device="cuda") for _ in tokens]
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        d.step(tokens[0])   # first-use set-up outside the capture
        d.reset()
        with torch.cuda.graph(graph, stream=s):
            for t, o in zip(tokens, outs):
                o.copy_(d.step(t))
    d.reset()
    graph.replay()
    torch.cuda.synchronize()
    for g, o in zip(got, outs):
        np.testing.assert_array_equal(o.cpu().numpy().view(np.uint32), g.view(np.uint32))
    from simd_ml_kernels import _core
    assert _core._device_error(torch.cuda.current_stream().cuda_stream) == 0


def test_decode_host_errors():
    """Argument checks happen on the host, before any launch (no GPU needed)."""
    with pytest.raises(ValueError, match="llama3 and default"):
        dec.rope_inv_freq(64, 10000.0, {"rope_type": "yarn"})
