"""make_gguf.py — writes the GGUF fixtures under tests/golden/ and the
reference's reading of them.

Two small model files in llama.cpp's GGUF format, with llama-style tensor
names and every tensor type the reference's reader takes (Q4_0, Q8_0, F32,
F16, BF16) and metadata of every value kind:

    tiny_v3.gguf             version 3, default alignment (32)
    tiny_v2_align64.gguf     version 2, general.alignment = 64

Quantized tensors hold the reference's blocks of seeded weights (oracle/_ref,
the reference compiled from its sources). The files are read back with the
reference's own reader (examples/llama/gguf_reader.py, imported from the
reference tree, which only this container has), and what it returns is stored
in ref_gguf.npz: each tensor's type, shape and SHA-256 of its bytes, the
metadata, and dequantize_rows of a few rows. The tests compare the B200
build's reader, device upload and dequantization kernel against that.

    make -C oracle all && python tests/golden/make_gguf.py
"""

from __future__ import annotations

import hashlib
import json
import os
import struct
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "oracle"))
import oracle as O  # noqa: E402



def ref_tree() -> str:
    """The reference's source tree, from SMK_REFERENCE_TREE (no default)."""
    t = os.environ.get("SMK_REFERENCE_TREE")
    if not t or not os.path.isdir(t):
        raise SystemExit("set SMK_REFERENCE_TREE to the reference's source tree (Mattral/simd-ml-kernels 0.3.0)")
    return t

F32, F16, Q4_0, Q8_0, BF16 = 0, 1, 2, 8, 30
FILES = {"tiny_v3.gguf": (3, None), "tiny_v2_align64.gguf": (2, 64)}


def tensors() -> list[tuple[str, int, tuple[int, ...], bytes]]:
    """(name, ggml type, shape outermost first, data bytes) of the fixture."""
    rng = np.random.default_rng(1234)
    out = []

    def q(name, fmt, n, k, scale):
        W = (rng.standard_normal((n, k)) * scale).astype(np.float32)
        out.append((name, Q4_0 if fmt == "q4_0" else Q8_0, (n, k), O.ref_quantize(fmt, W).tobytes()))

    q("token_embd.weight", "q4_0", 64, 256, 0.05)
    q("blk.0.attn_q.weight", "q8_0", 128, 256, 0.02)
    q("blk.0.ffn_down.weight", "q4_0", 96, 512, 0.02)
    out.append(("blk.0.attn_norm.weight", F32, (256,), rng.standard_normal(256).astype("<f4").tobytes()))
    out.append(("blk.0.attn_k.weight", F16, (8, 64), rng.standard_normal((8, 64)).astype("<f2").tobytes()))
    bf = O.bf16_bits(rng.standard_normal((4, 32)).astype(np.float32))
    out.append(("blk.0.attn_v.weight", BF16, (4, 32), bf.astype("<u2").tobytes()))
    out.append(("output_norm.weight", F32, (256,), rng.standard_normal(256).astype("<f4").tobytes()))
    return out


def _str(s: str) -> bytes:
    b = s.encode("utf-8")
    return struct.pack("<Q", len(b)) + b


def metadata(align) -> list[tuple[str, int, object]]:
    """(key, GGUF value type, value): strings, integers of each width, floats,
    a bool, and arrays of numbers and of strings."""
    md = [("general.architecture", 8, "llama"), ("general.name", 8, "tiny fixture"),
          ("llama.block_count", 4, 1), ("llama.embedding_length", 4, 256),
          ("llama.rope.freq_base", 6, 500000.0), ("llama.attention.layer_norm_rms_epsilon", 6, 1e-5),
          ("tiny.u8", 0, 200), ("tiny.i8", 1, -7), ("tiny.u16", 2, 65000), ("tiny.i16", 3, -300),
          ("tiny.i32", 5, -123456), ("tiny.bool", 7, True), ("tiny.u64", 10, 2 ** 40 + 3),
          ("tiny.i64", 11, -(2 ** 40)), ("tiny.f64", 12, 0.1),
          ("tokenizer.ggml.scores", 9, (6, [0.5, -1.25, 3.0, 0.0, -0.0, 7.75])),
          ("tokenizer.ggml.token_type", 9, (5, [1, 1, 3, 6, 1])),
          ("tokenizer.ggml.tokens", 9, (8, ["<s>", "</s>", "hello", "wörld"]))]
    if align is not None:
        md.insert(0, ("general.alignment", 4, align))
    return md


_PACK = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q", 12: "<d"}


def _value(vtype: int, v) -> bytes:
    if vtype in _PACK:
        return struct.pack(_PACK[vtype], v)
    if vtype == 8:
        return _str(v)
    etype, items = v
    return struct.pack("<IQ", etype, len(items)) + b"".join(_value(etype, x) for x in items)


def write(path: str, version: int, align) -> None:
    ts = tensors()
    md = metadata(align)
    a = align or 32
    head = b"GGUF" + struct.pack("<IQQ", version, len(ts), len(md))
    for key, vtype, v in md:
        head += _str(key) + struct.pack("<I", vtype) + _value(vtype, v)
    offsets, pos = [], 0
    for _, _, _, data in ts:
        offsets.append(pos)
        pos += (len(data) + a - 1) // a * a
    for (name, ttype, shape, _), off in zip(ts, offsets):
        dims = list(reversed(shape))
        head += _str(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        head += struct.pack("<IQ", ttype, off)
    start = (len(head) + a - 1) // a * a
    body = bytearray(pos)
    for (_, _, _, data), off in zip(ts, offsets):
        body[off:off + len(data)] = data
    with open(path, "wb") as f:
        f.write(head + b"\0" * (start - len(head)) + bytes(body))


def _json_value(v):
    if isinstance(v, np.ndarray):
        return {"array": v.tolist(), "dtype": str(v.dtype)}
    if isinstance(v, list):
        return [_json_value(x) for x in v]
    return v


def main() -> None:
    sys.path.insert(0, os.path.join(ref_tree(), "examples", "llama"))
    from gguf_reader import GGUF, dequantize_rows   # the reference's reader

    out = {}
    for fname, (version, align) in FILES.items():
        path = os.path.join(HERE, fname)
        write(path, version, align)
        g = GGUF(path)
        out[f"{fname}:version"] = np.array(g.version)
        out[f"{fname}:metadata"] = np.array(json.dumps({k: _json_value(v) for k, v in g.metadata.items()}))
        names = list(g.tensors)
        out[f"{fname}:names"] = np.array(names)
        for n in names:
            t = g.tensors[n]
            out[f"{fname}:{n}:type"] = np.array(t.type)
            out[f"{fname}:{n}:shape"] = np.array(t.shape)
            out[f"{fname}:{n}:sha"] = np.array(hashlib.sha256(np.ascontiguousarray(t.data).tobytes()).hexdigest())
            if len(t.shape) == 2:
                rows = [0, 3, t.shape[0] - 1]
                out[f"{fname}:{n}:rows"] = np.array(rows)
                out[f"{fname}:{n}:dequant"] = dequantize_rows(t, np.array(rows))
    np.savez_compressed(os.path.join(HERE, "ref_gguf.npz"), **out)
    for name in ("tiny_v3.gguf", "tiny_v2_align64.gguf", "ref_gguf.npz"):
        print(f"{name}: {os.path.getsize(os.path.join(HERE, name))} bytes")


if __name__ == "__main__":
    main()
