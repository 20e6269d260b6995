"""decode_oracle.py — TEST INFRASTRUCTURE ONLY.

Float64 restatements of the decode-step math of the reference's Llama example
(examples/llama/llama.py of Mattral/simd-ml-kernels 0.3.0), the checker of the
GPU decode kernels (simd_ml_kernels.decode). Each function takes the float32
inputs the reference's code would see, computes in float64 and returns float64:

  rms_norm64      llama.py:184-188   weight * x / sqrt(mean(x^2) + eps)
  rope64          llama.py:160-178 and Llama._rope: x*cos + rotate_half(x)*sin
                  (pairs (i, i + d/2)) or, interleaved, pairs (2i, 2i+1); the
                  angles f32(pos) * inv_freq rounded to float32 as rope_cos_sin
  attention64     Llama._attention (:398-412): per query head h on KV head
                  h // (nh / nkv), softmax(q.K^T / sqrt(d)) . V
  step64          Llama.step (:414-439) with float32 values between the
                  operations, as the reference passes them, and the GEMVs as
                  the float64 sums of the quantized operands (oracle.ref64)

Only tests/ import this module.
"""

from __future__ import annotations

import math

import numpy as np

import oracle as O


def rms_norm64(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x = np.asarray(x, np.float64)
    return np.asarray(w, np.float64) * x / math.sqrt(float(np.mean(x * x)) + eps)


def angles32(inv_freq: np.ndarray, pos: int) -> np.ndarray:
    return (np.float32(pos) * np.asarray(inv_freq, np.float32)).astype(np.float32)


def rope64(x: np.ndarray, inv_freq: np.ndarray, pos: int, interleaved: bool = False) -> np.ndarray:
    """x [heads, d] rotated at position pos."""
    x = np.asarray(x, np.float64)
    ang = angles32(inv_freq, pos).astype(np.float64)
    c, s = np.cos(ang), np.sin(ang)
    half = x.shape[-1] // 2
    out = np.empty_like(x)
    if interleaved:
        a, b = x[:, 0::2], x[:, 1::2]
        out[:, 0::2] = a * c - b * s
        out[:, 1::2] = b * c + a * s
    else:
        a, b = x[:, :half], x[:, half:]
        out[:, :half] = a * c - b * s
        out[:, half:] = b * c + a * s
    return out


def attention64(q: np.ndarray, k: np.ndarray, v: np.ndarray, length: int, scale: float | None = None) -> np.ndarray:
    """q [nh, d], k / v [nkv, >= length, d]: out [nh, d]."""
    q = np.asarray(q, np.float64)
    nh, d = q.shape
    nkv = k.shape[0]
    rep = nh // nkv
    sc = float(np.float32(1.0 / math.sqrt(d))) if scale is None else scale
    out = np.empty((nh, d))
    for h in range(nh):
        g = h // rep
        kk = np.asarray(k[g, :length], np.float64)
        vv = np.asarray(v[g, :length], np.float64)
        s = sc * (kk @ q[h])
        p = np.exp(s - s.max())
        out[h] = (p / p.sum()) @ vv
    return out


def silu_mul64(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    g = np.asarray(g, np.float64)
    return g / (1.0 + np.exp(-g)) * np.asarray(u, np.float64)


def gemv64(fmt: str, x32: np.ndarray, Wq: np.ndarray, N: int, K: int) -> np.ndarray:
    y64, _ = O.ref64(fmt, np.asarray(x32, np.float32), Wq, N, K)
    return y64


def step64(model: dict, tokens, capacity: int) -> list[np.ndarray]:
    """Logits (float64) of each token of `tokens` run through the decoder whose
    host copies `model` holds: shape entries (hidden, layers, heads, kv_heads,
    head_dim, ffn, vocab, eps), fmt, inv_freq, interleaved, embed / lm_head
    blocks, and per layer attn_norm, qkv, o, mlp_norm, gate_up, down."""
    f32 = np.float32
    H, nh, nkv, hd, F, V = (model[k] for k in ("hidden", "heads", "kv_heads", "head_dim", "ffn", "vocab"))
    fmt, eps = model["fmt"], model["eps"]
    kc = np.zeros((model["layers"], nkv, capacity, hd), f32)
    vc = np.zeros_like(kc)
    out = []
    for pos, tok in enumerate(tokens):
        x = O.dequantize_rows(fmt, model["embed"], H, [tok])[0].astype(f32)
        for li, L in enumerate(model["layer_weights"]):
            h = rms_norm64(x, L["attn_norm"], eps).astype(f32)
            qkv = gemv64(fmt, h, L["qkv"], (nh + 2 * nkv) * hd, H).astype(f32)
            q = rope64(qkv[:nh * hd].reshape(nh, hd), model["inv_freq"], pos, model["interleaved"]).astype(f32)
            k = rope64(qkv[nh * hd:(nh + nkv) * hd].reshape(nkv, hd), model["inv_freq"], pos,
                       model["interleaved"]).astype(f32)
            kc[li, :, pos] = k
            vc[li, :, pos] = qkv[(nh + nkv) * hd:].reshape(nkv, hd)
            a = attention64(q, kc[li], vc[li], pos + 1).astype(f32).reshape(-1)
            x = (x.astype(np.float64) + gemv64(fmt, a, L["o"], H, nh * hd)).astype(f32)
            h = rms_norm64(x, L["mlp_norm"], eps).astype(f32)
            gu = gemv64(fmt, h, L["gate_up"], 2 * F, H).astype(f32)
            m = silu_mul64(gu[:F], gu[F:]).astype(f32)
            x = (x.astype(np.float64) + gemv64(fmt, m, L["down"], H, F)).astype(f32)
        h = rms_norm64(x, model["norm"], eps).astype(f32)
        out.append(gemv64(fmt, h, model["lm_head"], V, H))
    return out
