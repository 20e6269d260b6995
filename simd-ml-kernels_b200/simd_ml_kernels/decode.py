"""A Llama decode step on the GPU: the GEMVs of this package plus the kernels
the reference's decoder runs in NumPy around them (examples/llama/llama.py):
RMSNorm with the residual add before it (rms_norm :184-188, step :414-439),
RoPE with the KV-cache write (rope_cos_sin / apply_rope :131-178, Llama._rope)
and grouped-query attention over the cache (Llama._attention :398-412).

Functions (CUDA tensors, queued on torch's current stream):

    add_rmsnorm(x, w, eps, delta=None, out=None)     x += delta; out = RMSNorm(x) * w
    rope_kv(qkv, inv_freq, pos, nh, nkv, hd, k_cache, v_cache, q_out=None, interleaved=False)
    attention_decode(q, k_cache, v_cache, length, nkv, out=None)
    rope_attention(qkv, inv_freq, pos, nh, nkv, hd, k_cache, v_cache, out=None, interleaved=False)
                                                     the two above as one kernel
    gemv_rmsnorm(x, w_norm, eps, Wq, N, K, fmt="q4_0", out=None)
                                                     (RMSNorm(x) * w_norm) @ W.T in one GEMV
    gemv_residual(x, Wq, N, K, r, fmt="q4_0", up=None)
                                                     r += x @ W.T (or silu(x) * up) in one GEMV
    rope_inv_freq(head_dim, theta, scaling=None)     the frequencies (float32, host)

`LlamaDecoder` holds one model's weights on the device (Q4_0 or Q8_0 blocks,
q/k/v and gate/up as concatenated row groups), its KV cache and buffers, and
runs `step(token)`: the embedding row, then per layer five launches: the q/k/v
GEMV with the attention RMSNorm in its x quantization, RoPE + cache write +
attention, the o GEMV adding into the residual stream, the gate/up GEMV with
the MLP RMSNorm, and the down GEMV on silu(gate)*up adding into the residual
stream; then the LM-head GEMV with the final norm. Every launch is
asynchronous, so a run of steps can be captured in a CUDA graph.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

from . import _core


def _torch():
    import torch
    return torch


def _dev(t) -> int:
    return t.device.index if t.device.index is not None else _torch().cuda.current_device()


def _stream(t) -> int:
    return _torch().cuda.current_stream(t.device).cuda_stream


def _check(t, name, dtype=None):
    torch = _torch()
    if not (isinstance(t, torch.Tensor) and t.is_cuda):
        raise ValueError(f"{name} must be a CUDA tensor")
    if dtype is not None and t.dtype != dtype:
        raise ValueError(f"{name} must be {dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def add_rmsnorm(x, w, eps: float, delta=None, out=None):
    """Rows of x [M, n] (or one row [n]): x += delta (in place, when given), then
    out = w * (x * f32(1 / sqrt(mean(x^2) + eps))), the reference's rms_norm."""
    torch = _torch()
    _check(x, "x", torch.float32)
    _check(w, "w", torch.float32)
    n = x.shape[-1]
    M = x.numel() // n if n else 0
    if w.numel() != n:
        raise ValueError("w must hold one weight per value of a row")
    if delta is not None:
        _check(delta, "delta", torch.float32)
        if delta.numel() != x.numel():
            raise ValueError("delta must match x")
    if out is None:
        out = torch.empty_like(x)
    _check(out, "out", torch.float32)
    _core._add_rmsnorm(M, n, x.data_ptr(), n, 0 if delta is None else delta.data_ptr(), n, w.data_ptr(), float(eps),
                       out.data_ptr(), n, _stream(x), _dev(x))
    return out


def rope_kv(qkv, inv_freq, pos: int, nh: int, nkv: int, hd: int, k_cache, v_cache, q_out=None,
            interleaved: bool = False):
    """Rotates one token's q and k (qkv = [q | k | v]) at position pos, writes
    k and v to row pos of the caches [nkv, capacity, hd]; returns q [nh, hd]."""
    torch = _torch()
    for t, nm in ((qkv, "qkv"), (inv_freq, "inv_freq"), (k_cache, "k_cache"), (v_cache, "v_cache")):
        _check(t, nm, torch.float32)
    if qkv.numel() != (nh + 2 * nkv) * hd or inv_freq.numel() != hd // 2:
        raise ValueError("qkv must hold (nh + 2*nkv) * hd values and inv_freq hd/2")
    cap = k_cache.shape[-2]
    if k_cache.numel() != nkv * cap * hd or v_cache.numel() != k_cache.numel():
        raise ValueError("caches must be [nkv, capacity, hd]")
    if q_out is None:
        q_out = torch.empty((nh, hd), dtype=torch.float32, device=qkv.device)
    _core._rope_kv(qkv.data_ptr(), inv_freq.data_ptr(), 0, int(pos), nh, nkv, hd, int(interleaved), q_out.data_ptr(),
                   k_cache.data_ptr(), v_cache.data_ptr(), cap, _stream(qkv), _dev(qkv))
    return q_out


def attention_decode(q, k_cache, v_cache, length: int, nkv: int, out=None, max_len: int | None = None,
                     scale: float | None = None):
    """softmax(scale * q . K[:length]) . V[:length] per query head, query head h on
    KV head h // (nh / nkv); q [nh, hd], caches [nkv, capacity, hd]. scale
    defaults to float32(1 / sqrt(hd)), the reference's."""
    torch = _torch()
    for t, nm in ((q, "q"), (k_cache, "k_cache"), (v_cache, "v_cache")):
        _check(t, nm, torch.float32)
    nh, hd = q.shape[-2], q.shape[-1]
    cap = k_cache.shape[-2]
    if out is None:
        out = torch.empty_like(q)
    s = float(np.float32(1.0 / math.sqrt(hd))) if scale is None else float(scale)
    _core._attention_decode(q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), out.data_ptr(), 0, int(length),
                            int(max_len or length), nh, nkv, hd, cap, s, _stream(q), _dev(q))
    return out


def rope_attention(qkv, inv_freq, pos: int, nh: int, nkv: int, hd: int, k_cache, v_cache, out=None,
                   interleaved: bool = False, max_len: int | None = None, scale: float | None = None):
    """rope_kv and attention_decode in one kernel: rotates this token's q and k
    (qkv = [q | k | v], not rotated) at position pos, writes k and v to row pos
    of the caches [nkv, capacity, hd] and returns the attention of q over
    positions 0 .. pos, [nh, hd]. The same values as the two calls."""
    torch = _torch()
    for t, nm in ((qkv, "qkv"), (inv_freq, "inv_freq"), (k_cache, "k_cache"), (v_cache, "v_cache")):
        _check(t, nm, torch.float32)
    if qkv.numel() != (nh + 2 * nkv) * hd or inv_freq.numel() != hd // 2:
        raise ValueError("qkv must hold (nh + 2*nkv) * hd values and inv_freq hd/2")
    cap = k_cache.shape[-2]
    if k_cache.numel() != nkv * cap * hd or v_cache.numel() != k_cache.numel():
        raise ValueError("caches must be [nkv, capacity, hd]")
    if out is None:
        out = torch.empty((nh, hd), dtype=torch.float32, device=qkv.device)
    _check(out, "out", torch.float32)
    s = float(np.float32(1.0 / math.sqrt(hd))) if scale is None else float(scale)
    _core._rope_attention(qkv.data_ptr(), inv_freq.data_ptr(), 0, int(pos), int(max_len or pos + 1), nh, nkv, hd,
                          int(interleaved), k_cache.data_ptr(), v_cache.data_ptr(), cap, s, out.data_ptr(),
                          _stream(qkv), _dev(qkv))
    return out


def _fmt_code(fmt: str) -> int:
    if fmt not in ("q4_0", "q8_0"):
        raise ValueError("fmt must be 'q4_0' or 'q8_0'")
    return 0 if fmt == "q4_0" else 1


def gemv_rmsnorm(x, w_norm, eps: float, Wq, N: int, K: int, fmt: str = "q4_0", out=None):
    """y = (RMSNorm(x) * w_norm) @ W.T for x [K] or [M, K]: the reference's
    rms_norm applied to each row inside the GEMV's x quantization (one launch,
    x unchanged). y [N] or [M, N]."""
    torch = _torch()
    _check(x, "x", torch.float32)
    _check(w_norm, "w_norm", torch.float32)
    M = 1 if x.dim() == 1 else x.shape[0]
    if x.shape[-1] != K or w_norm.numel() != K:
        raise ValueError("x rows and w_norm must hold K values")
    if out is None:
        out = torch.empty((N,) if x.dim() == 1 else (M, N), dtype=torch.float32, device=x.device)
    _check(out, "out", torch.float32)
    _core._gemv_q_fused(_fmt_code(fmt), M, N, K, x.data_ptr(), K, 0, 0, w_norm.data_ptr(), float(eps),
                        Wq.data_ptr(), 0, 0, out.data_ptr(), N, _stream(x), _dev(x))
    return out


def gemv_residual(x, Wq, N: int, K: int, r, fmt: str = "q4_0", up=None):
    """r += x @ W.T (or (silu(x) * up) @ W.T when up is given) for x [K] or
    [M, K] and r [N] or [M, N]: the residual add of the reference's decoder
    step fused into the GEMV's store, in place. Returns r."""
    torch = _torch()
    _check(x, "x", torch.float32)
    _check(r, "r", torch.float32)
    M = 1 if x.dim() == 1 else x.shape[0]
    if x.shape[-1] != K or r.numel() != M * N:
        raise ValueError("x rows must hold K values and r M * N")
    if up is not None:
        _check(up, "up", torch.float32)
        if up.shape != x.shape:
            raise ValueError("up must match x")
    _core._gemv_q_fused(_fmt_code(fmt), M, N, K, x.data_ptr(), K, 0 if up is None else up.data_ptr(), K, 0, 0.0,
                        Wq.data_ptr(), r.data_ptr(), N, r.data_ptr(), N, _stream(x), _dev(x))
    return r


def rope_inv_freq(head_dim: int, theta: float, scaling: dict | None = None) -> np.ndarray:
    """RoPE inverse frequencies in float32, as the Llama configs define them:
    1 / theta^(2i / d) for i < d/2, and with rope_scaling of type "llama3"
    (factor, low_freq_factor, high_freq_factor, original_max_position_embeddings)
    the long wavelengths divided by factor, the short ones kept and the band
    between blended linearly in 1/wavelength. Each step rounds to float32, the
    precision the reference and transformers compute these in
    (examples/llama/llama.py:131-157)."""
    f32 = np.float32
    i2 = np.arange(0, head_dim, 2, dtype=np.int64).astype(f32)
    base = (f32(1.0) / (f32(theta) ** (i2 / f32(head_dim)))).astype(f32)
    kind = None if scaling is None else scaling.get("rope_type", scaling.get("type"))
    if kind in (None, "default"):
        return base
    if kind != "llama3":
        raise ValueError(f"rope_scaling type {kind!r} is not implemented (llama3 and default are)")
    factor = scaling["factor"]
    lo, hi = scaling["low_freq_factor"], scaling["high_freq_factor"]
    ctx = scaling["original_max_position_embeddings"]
    wave = (f32(2 * math.pi) / base).astype(f32)
    long_wave = ctx / lo
    short_wave = ctx / hi
    shrunk = np.where(wave > long_wave, base / f32(factor), base).astype(f32)
    t = ((f32(ctx) / wave - f32(lo)) / f32(hi - lo)).astype(f32)
    blend = ((1 - t) * shrunk / f32(factor) + t * shrunk).astype(f32)
    between = ~(wave < short_wave) & ~(wave > long_wave)
    return np.where(between, blend, shrunk).astype(f32)


# ---- the decoder ------------------------------------------------------------------

@dataclass
class LlamaShape:
    hidden: int
    layers: int
    heads: int
    kv_heads: int
    head_dim: int
    ffn: int
    vocab: int
    eps: float = 1e-5


@dataclass
class LlamaLayerWeights:
    attn_norm: object       # [hidden] float32
    qkv: object             # blocks of [q rows | k rows | v rows] x hidden
    o: object               # blocks of hidden x (heads * head_dim)
    mlp_norm: object
    gate_up: object         # blocks of [gate rows | up rows] x hidden
    down: object            # blocks of hidden x ffn


@dataclass
class LlamaWeights:
    layers: list
    norm: object            # [hidden] float32
    embed: object           # blocks of vocab x hidden (the token embedding)
    lm_head: object         # blocks of vocab x hidden (the embedding itself when tied)
    fmt: str = "q4_0"


@dataclass
class _Buffers:
    x: object
    h: object
    qkv: object
    q: object
    att: object
    delta: object
    gate_up: object
    logits: object
    tok: object
    k_cache: object
    v_cache: object
    extra: dict = field(default_factory=dict)


class LlamaDecoder:
    """One sequence of a Llama-architecture decoder on the GPU (the reference's
    Llama.step). The GEMVs use this package's quantized kernels: q/k/v and
    gate/up read their shared input once as concatenated row groups, the down
    projection forms silu(gate)*up while quantizing its input. RoPE uses the
    Hugging Face pair layout unless `interleaved` (GGUF files)."""

    def __init__(self, shape: LlamaShape, weights: LlamaWeights, inv_freq: np.ndarray, capacity: int,
                 interleaved: bool = False, device=None):
        torch = _torch()
        import simd_ml_kernels as sk
        self.sk, self.shape, self.w, self.cap, self.interleaved = sk, shape, weights, capacity, interleaved
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        s = shape
        if s.heads % s.kv_heads or s.head_dim % 32 or s.heads * s.head_dim != s.hidden:
            raise ValueError("heads must be a multiple of kv_heads, head_dim a multiple of 32, heads*head_dim = hidden")
        f32 = dict(dtype=torch.float32, device=self.device)
        self.inv_freq = torch.as_tensor(np.asarray(inv_freq, np.float32), **f32)
        qkv_rows = (s.heads + 2 * s.kv_heads) * s.head_dim
        self.buf = _Buffers(
            x=torch.zeros(s.hidden, **f32), h=torch.empty(s.hidden, **f32), qkv=torch.empty(qkv_rows, **f32),
            q=torch.empty((s.heads, s.head_dim), **f32), att=torch.empty((s.heads, s.head_dim), **f32),
            delta=torch.zeros(s.hidden, **f32), gate_up=torch.empty(2 * s.ffn, **f32),
            logits=torch.empty(s.vocab, **f32), tok=torch.arange(s.vocab, dtype=torch.int32, device=self.device),
            k_cache=torch.zeros((s.layers, s.kv_heads, capacity, s.head_dim), **f32),
            v_cache=torch.zeros((s.layers, s.kv_heads, capacity, s.head_dim), **f32))
        self.pos = 0
        self._gemv = sk.gemv_q4_0 if weights.fmt == "q4_0" else sk.gemv_q8_0
        self._gemv_silu = sk.gemv_q4_0_silu_mul if weights.fmt == "q4_0" else sk.gemv_q8_0_silu_mul
        self._fmt = 0 if weights.fmt == "q4_0" else 1

    def reset(self) -> None:
        self.pos = 0
        self.buf.k_cache.zero_()
        self.buf.v_cache.zero_()

    def _embed(self, token) -> None:
        """x = the token's embedding row. A host token id selects its entry of
        the device table tok = 0 .. vocab-1 (no copy or fill kernel); a device
        tensor is passed through as the row index."""
        torch = _torch()
        s, b = self.shape, self.buf
        if isinstance(token, torch.Tensor):
            rows = token.reshape(1).to(torch.int32)
            b.extra["tok"] = rows   # alive until the launch has read it
            ptr = rows.data_ptr()
        else:
            t = int(token)
            if not 0 <= t < s.vocab:
                raise IndexError(f"token {t} outside the vocabulary ({s.vocab})")
            ptr = b.tok.data_ptr() + 4 * t
        _core._dequantize_rows(self._fmt, s.vocab, s.hidden, self.w.embed.data_ptr(), ptr, 1,
                               b.x.data_ptr(), s.hidden, _stream(b.x), _dev(b.x))

    def step(self, token, logits: bool = True):
        """One token at position self.pos: logits [vocab] (a CUDA tensor, the
        decoder's buffer) or None when logits is False."""
        s, b, w = self.shape, self.buf, self.w
        pos = self.pos
        if pos >= self.cap:
            raise ValueError(f"KV cache full ({self.cap} positions)")
        nh, nkv, hd = s.heads, s.kv_heads, s.head_dim
        self._embed(token)
        fmt, H, F = w.fmt, s.hidden, s.ffn
        for li, L in enumerate(w.layers):
            gemv_rmsnorm(b.x, L.attn_norm, s.eps, L.qkv, b.qkv.numel(), H, fmt, out=b.qkv)
            rope_attention(b.qkv, self.inv_freq, pos, nh, nkv, hd, b.k_cache[li], b.v_cache[li], out=b.att,
                           interleaved=self.interleaved, max_len=self.cap)
            gemv_residual(b.att.reshape(-1), L.o, H, nh * hd, b.x, fmt)
            gemv_rmsnorm(b.x, L.mlp_norm, s.eps, L.gate_up, 2 * F, H, fmt, out=b.gate_up)
            gemv_residual(b.gate_up[:F], L.down, H, F, b.x, fmt, up=b.gate_up[F:])
        self.pos = pos + 1
        if not logits:
            return None
        gemv_rmsnorm(b.x, w.norm, s.eps, w.lm_head, s.vocab, H, fmt, out=b.logits)
        return b.logits

    def launches_per_token(self) -> int:
        # The embedding row; per layer five GEMV-side launches plus the kernel
        # that forms and quantizes silu(gate) * up for the down projection; the
        # LM head.
        return 1 + 6 * self.shape.layers + 1
