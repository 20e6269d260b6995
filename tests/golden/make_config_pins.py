"""make_config_pins.py — SHA-256 pins of the exact inputs bench.py times for
every BASELINE config, quantized by the reference itself (Mattral/simd-ml-kernels
0.3.0 compiled from its sources by oracle/Makefile into oracle/_ref/libsmk_ref.so).

    python tests/golden/make_config_pins.py      # writes tests/golden/config_pins.json

The inputs come from bench.py's generators (numpy default_rng with the
BASELINE seeds, weights drawn in 8192-row chunks, then x): config 0 (seed 0),
config 1 (seed 1, each shape its own generator), config 3 (seed 3, each N;
float32 weights and their bfloat16 / float16 roundings to nearest even),
config 4 (seed 4, each shape) and the 113 matrices of config 2 (generator
seeded (2, i) for matrix i). The GPU tests (tests/test_config_parity.py)
regenerate the same inputs, quantize them on the device, compare the bytes
with these pins and check every GEMV output against the oracle. Needs only
the prebuilt reference library, not the reference tree.
"""

from __future__ import annotations

import concurrent.futures as cf
import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
for p in (REPO, os.path.join(REPO, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)
import bench  # noqa: E402
import oracle as O  # noqa: E402

OUT = os.path.join(HERE, "config_pins.json")


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def q_pin(fmt: str, wl: bench.Workload) -> dict:
    """Quantize wl's weights chunk by chunk with the reference; hash the bytes and x."""
    h = hashlib.sha256()
    for _, c in wl.chunks():
        q = O.ref_quantize(fmt, c)
        assert q is not None, "the reference rejected a chunk"
        h.update(q.tobytes())
    out = {"N": wl.N, "K": wl.K, "fmt": fmt, "w_sha256": h.hexdigest()}
    if wl.M:
        out["x_sha256"] = sha(wl.x)
    return out


def f16_bits(W: np.ndarray, kind: str) -> np.ndarray:
    if kind == "float16":
        return W.astype(np.float16).view(np.uint16)
    return O.bf16_bits(W)


def main() -> None:
    if not O.ref_available():
        raise SystemExit("oracle/_ref/libsmk_ref.so is missing: make -C oracle all REF=<reference tree>")
    pins: dict = {"generator": "bench.Workload: numpy default_rng(entropy), W = standard_normal * sigma in "
                               "8192-row chunks (float64 -> float32), then x = standard_normal((M, K))",
                  "quantizer": "the reference's quantize_q4_0_rows / quantize_q8_0_rows (oracle/_ref)"}
    pins["config0"] = q_pin("q4_0", bench.config0())
    pins["config1"] = [q_pin("q8_0", bench.config1(N, K)) for N, K in bench.CFG1_SHAPES]
    c3 = []
    for N, K in bench.CFG3_SHAPES:
        W, X = bench.config3(N, K).full()
        c3.append({"N": N, "K": K, "x_sha256": sha(X), "float32_sha256": sha(W),
                   "bfloat16_sha256": sha(f16_bits(W, "bfloat16")), "float16_sha256": sha(f16_bits(W, "float16"))})
    pins["config3"] = c3
    with cf.ThreadPoolExecutor(max_workers=8) as ex:
        c4 = [ex.submit(q_pin, "q4_0", bench.config4(N, K)) for N, K in bench.CFG4_SHAPES]
        c2 = [ex.submit(q_pin, "q4_0", bench.config2(i)) for i in range(len(bench.LLAMA_MATRICES))]
        pins["config4"] = [f.result() for f in c4]
        pins["config2"] = [f.result() for f in c2]
    with open(OUT, "w") as f:
        json.dump(pins, f, indent=1)
        f.write("\n")
    print(f"wrote {os.path.relpath(OUT, REPO)}")


if __name__ == "__main__":
    main()
