"""make_decode_golden.py — golden vectors of the decode step's host-side math
from the reference itself: rope_inv_freq, rope_cos_sin, apply_rope, the
interleaved rotation of Llama._rope, and rms_norm of the reference's
examples/llama/llama.py (Mattral/simd-ml-kernels 0.3.0), for the Llama-3.2-1B
RoPE configuration (llama3 scaling) and the default one.

    SMK_REFERENCE_TREE=<reference tree> python tests/golden/make_decode_golden.py

llama.py imports the reference's package at module level for its GEMV calls;
none of the functions used here calls it, so a stand-in module takes its name
while llama.py loads. Writes tests/golden/ref_decode.npz.
"""

from __future__ import annotations

import importlib.util
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def ref_tree() -> str:
    t = os.environ.get("SMK_REFERENCE_TREE")
    if not t or not os.path.isdir(t):
        raise SystemExit("set SMK_REFERENCE_TREE to the reference's source tree (Mattral/simd-ml-kernels 0.3.0)")
    return t


def load_llama():
    saved = sys.modules.get("simd_ml_kernels")
    sys.modules["simd_ml_kernels"] = types.ModuleType("simd_ml_kernels")
    try:
        path = os.path.join(ref_tree(), "examples", "llama", "llama.py")
        spec = importlib.util.spec_from_file_location("ref_llama", path)
        mod = importlib.util.module_from_spec(spec)
        sys.modules["ref_llama"] = mod   # its dataclasses look their module up by name
        spec.loader.exec_module(mod)
        return mod
    finally:
        if saved is None:
            del sys.modules["simd_ml_kernels"]
        else:
            sys.modules["simd_ml_kernels"] = saved


def main() -> None:
    L = load_llama()
    out = {}
    llama3 = {"factor": 32.0, "high_freq_factor": 4.0, "low_freq_factor": 1.0,
              "original_max_position_embeddings": 8192, "rope_type": "llama3"}
    cfgs = {"llama3": (64, 500000.0, llama3), "default": (128, 10000.0, None)}
    rng = np.random.default_rng(5)
    for name, (hd, theta, scaling) in cfgs.items():
        cfg = types.SimpleNamespace(head_dim=hd, rope_theta=theta, rope_scaling=scaling)
        inv = L.rope_inv_freq(cfg)
        out[f"{name}:inv_freq"] = inv
        out[f"{name}:head_dim"] = np.int64(hd)
        for pos in (0, 1, 77, 4000):
            cos, sin = L.rope_cos_sin(inv, pos)
            x = rng.standard_normal((6, hd)).astype(np.float32)
            out[f"{name}:{pos}:x"] = x
            out[f"{name}:{pos}:hf"] = L.apply_rope(x, cos, sin)
            # Llama._rope with rope_interleaved set (the layout of GGUF files)
            out[f"{name}:{pos}:interleaved"] = L.Llama._rope(types.SimpleNamespace(rope_interleaved=True), x, cos, sin)
    for i, n in enumerate((2048, 333)):
        x = (rng.standard_normal(n) * 3).astype(np.float32)
        w = (1 + 0.1 * rng.standard_normal(n)).astype(np.float32)
        out[f"rms:{i}:x"], out[f"rms:{i}:w"] = x, w
        out[f"rms:{i}:h"] = L.rms_norm(x, w, 1e-5)
    np.savez_compressed(os.path.join(HERE, "ref_decode.npz"), **out)
    print("wrote tests/golden/ref_decode.npz")


if __name__ == "__main__":
    main()
