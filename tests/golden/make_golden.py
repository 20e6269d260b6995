"""make_golden.py — writes the golden vectors under tests/golden/ from the
reference itself (Mattral/simd-ml-kernels 0.3.0 compiled from its sources
by oracle/Makefile into oracle/_ref/libsmk_ref.so) and from the llama.cpp
fixture the reference's tests hold (tests/data/q4_0_ggml_v0.7.0.npz,
checked by tests/test_precision.py:705-719 there).

Run in a container that has the reference tree (it reads it; the GPU box
does not have it and only reads the .npz files written here):

    make -C oracle all && python tests/golden/make_golden.py
    python tests/golden/make_golden.py u8s8     # only ref_u8s8.npz

Large weight matrices are not stored: each case keeps its seed and shape, the
SHA-256 of the reference's quantized bytes and the reference's outputs; the
tests regenerate W from the seed and check the hash before comparing.
"""

from __future__ import annotations

import hashlib
import os
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
ISA_SCALAR = 0


def sha(b: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(b).tobytes()).hexdigest()


def ref_quant_x(x: np.ndarray) -> tuple[np.ndarray, np.ndarray, int]:
    K = x.shape[0]
    qs = np.zeros(K, np.int8)
    dx = np.zeros(K // 32, np.float32)
    ok = O.ref().smkref_quantize_x_q8(x.ctypes.data, K, qs.ctypes.data, dx.ctypes.data)
    return qs, dx, int(ok)


def ref_dense(kind: str, isa: int, A: np.ndarray, B: np.ndarray, alpha: float, beta: float,
              C: np.ndarray) -> np.ndarray:
    M, K = A.shape
    N = B.shape[0]
    out = np.array(C, np.float32, copy=True)
    fn = {"f32": O.ref().smkref_sgemm_tb, "f16": O.ref().smkref_sgemm_f16_tb,
          "bf16": O.ref().smkref_sgemm_bf16_tb}[kind]
    fn(isa, M, N, K, alpha, A.ctypes.data, B.ctypes.data, beta, out.ctypes.data)
    return out


# Input generators, imported by the tests too (they regenerate W from the seed
# and check the SHA-256 of its quantized bytes before comparing outputs).
def gemv_case_inputs(seed: int, N: int, K: int, kind: str) -> tuple[np.ndarray, np.ndarray]:
    """W [N, K] and x [K] of a golden GEMV case. kind: 'normal' (standard normal, W scaled by
    1 + seed % 3), 'extreme' (every quant 0/15 or ±127, as test_q4_0.cpp:136-140)."""
    rng = np.random.default_rng(seed)
    if kind == "extreme":
        W = np.where(rng.integers(0, 2, (N, K)) == 1, np.float32(7.0), np.float32(-8.0)).astype(np.float32)
        W[:, ::32] = -8.0
        x = np.where(rng.integers(0, 2, K) == 1, np.float32(2.0), np.float32(-2.0)).astype(np.float32)
    else:
        W = (rng.standard_normal((N, K)) * (1 + seed % 3)).astype(np.float32)
        x = (rng.standard_normal(K) * 4).astype(np.float32)
    return W, x


GEMV_CASES = (
    [(100 + n, n, 64, "normal") for n in (1, 2, 7, 8, 9, 15, 16, 17, 31, 100)]
    + [(200 + k, 13, k, "normal") for k in (32, 96, 128, 160, 256, 1024, 4128)]
    + [(301, 11, 160, "normal"), (302, 9, 4096, "extreme"), (303, 33, 11008, "normal"),
       (304, 257, 2048, "normal"), (305, 64, 8192, "normal")]
)


DENSE_CASES = [(1, 37, 33), (1, 64, 4099), (1, 17, 70), (4, 33, 1027), (8, 45, 133), (1, 21, 77)]


def dense_case_inputs(i: int, m: int, n: int, k: int):
    """A [m, k], B [n, k], C0 [m, n] uniform in [-1, 1) and (alpha, beta) of dense case i."""
    rng = np.random.default_rng(900 + i)
    A = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    B = rng.uniform(-1, 1, (n, k)).astype(np.float32)
    C0 = rng.uniform(-1, 1, (m, n)).astype(np.float32)
    alpha, beta = (1.0, 0.0) if i % 2 == 0 else (-1.5, 0.5)
    return A, B, C0, alpha, beta


def dense_operands(kind: str, A: np.ndarray, B: np.ndarray):
    """The operands sgemm / sgemm_f16 / sgemm_bf16 take: float32, float16 bits, bfloat16 bits (RNE)."""
    if kind == "f32":
        return A, B
    if kind == "f16":
        return A.astype(np.float16).view(np.uint16), B.astype(np.float16).view(np.uint16)
    return O.bf16_bits(A), O.bf16_bits(B)


# sgemm_u8s8 cases (M, N, K, zero point): decode shapes M <= 8 with ragged N
# and K, the shapes of the reference's own parameter list
# (tests/test_precision.py:256-258) that have M <= 8, and one case of all-extreme
# operands (A = 255, B = -128, zp = 0: tests/test_precision.py:282-288).
U8S8_CASES = [(1, 1, 1, 0), (7, 9, 8, 128), (1, 4096, 128, 255), (5, 15, 3, 3), (8, 33, 385, 128),
              (1, 300, 257, 77), (4, 33, 1027, 200), (2, 64, 4096, 0), (1, 257, 1024, 128), (3, 33, 4096, 0),
              (1, 2048, 2048, 128), (8, 1000, 2080, 31)]
U8S8_EXTREME = 9   # index of the all-extreme case


def u8s8_case_inputs(i: int, m: int, n: int, k: int):
    """A uint8 [m, k], W int8 [n, k] (the trans_b layout), b_scales [n], a_scale of u8s8 case i."""
    rng = np.random.default_rng(700 + i)
    if i == U8S8_EXTREME:
        A = np.full((m, k), 255, np.uint8)
        W = np.full((n, k), -128, np.int8)
        return A, W, np.ones(n, np.float32), np.float32(1.0)
    A = rng.integers(0, 256, (m, k), dtype=np.uint8)
    W = rng.integers(-128, 128, (n, k), dtype=np.int8)
    scales = rng.uniform(-0.1, 0.1, n).astype(np.float32)
    return A, W, scales, np.float32(0.0173)


def write_u8s8() -> None:
    """sgemm_u8s8 outputs of the reference's scalar table and its table for
    this CPU, with B as [N, K] (trans_b) and as [K, N]."""
    uo = {"cases": np.array(U8S8_CASES, np.int64), "u8s8_path": np.array(O.ref().smkref_u8s8_path().decode())}
    for i, (m, n, k, zp) in enumerate(U8S8_CASES):
        A, W, scales, a_scale = u8s8_case_inputs(i, m, n, k)
        uo[f"sha{i}"] = np.array(sha(np.concatenate([A.view(np.uint8).ravel(), W.view(np.uint8).ravel(),
                                                    scales.view(np.uint8)])))
        for tb in (1, 0):
            B = W if tb else np.ascontiguousarray(W.T)
            uo[f"tb{tb}_{i}_scalar"] = O.ref_sgemm_u8s8(A, B, a_scale, zp, scales, bool(tb), isa=ISA_SCALAR)
            uo[f"tb{tb}_{i}_simd"] = O.ref_sgemm_u8s8(A, B, a_scale, zp, scales, bool(tb), isa=-1)
    np.savez_compressed(os.path.join(HERE, "ref_u8s8.npz"), **uo)


def special_quant_rows() -> np.ndarray:
    """Rows that exercise every rule of the two quantizers (test_q4_0.cpp:92-109,
    test_precision.py:501-512)."""
    rng = np.random.default_rng(11)
    w = (rng.standard_normal((10, 128)) * 0.5).astype(np.float32)
    w[0, :32] = -8.0 + 0.5 * np.arange(32)        # max -8: w + 8.5 on k + 0.5 and k
    w[0, 32:64] = 8.0 - 0.5 * np.arange(32)       # max +8: d = -1
    w[0, 64:96] = 0.0                             # zero block
    w[1, 5], w[1, 9], w[1, 35], w[1, 62] = 2.0, -2.0, -2.0, 2.0   # opposite-sign ties
    w[2, :32] = (np.arange(32) * 977 + 0x00800000).astype(np.uint32).view(np.float32)  # ~1.2e-38
    w[2, 32:64] = rng.uniform(-1e-5, 1e-5, 32)   # binary16-subnormal scales
    w[2, 64:96] = rng.uniform(-5.2e5, 5.2e5, 32)  # large, below the Q4_0 overflow
    w[3, :32] = np.arange(-16, 16) + 0.5          # exact halves (Q8_0 rounding)
    w[3, 31] = 127.0
    w[4, :32] = 1.0                               # constant block
    w[5, :32] = np.where(np.arange(32) % 2, 1e-44, -1e-44)   # 1/d overflows: q = 8 / 0
    w[6, :] = -np.abs(w[6, :])
    w[7, ::2] = 7.0
    w[7, ::32] = -8.0
    w[8, :] = np.round(rng.uniform(-8, 8, 128)) * 0.5
    w[9, :64] = -0.0
    return w.astype(np.float32)


def main() -> None:
    if not O.ref_available():
        sys.exit("oracle/_ref/libsmk_ref.so missing: run `make -C oracle all` where the reference tree is")
    R = O.ref()
    R.smkref_set_num_threads(1)
    meta = {"reference": "Mattral/simd-ml-kernels 0.3.0 (oracle/_ref, compiled from its sources)",
            "q8_0_path": R.smkref_q8_0_path().decode(), "active_isa": R.smkref_active_isa().decode()}
    print(meta)

    # 1. The llama.cpp fixture of the reference's tests (ggml_quantize_chunk output).
    fx = np.load(os.path.join(ref_tree(), "tests", "data", "q4_0_ggml_v0.7.0.npz"))
    np.savez_compressed(os.path.join(HERE, "q4_0_llama_cpp_fixture.npz"), w=fx["w"], blocks=fx["blocks"],
                        source=fx["source"])

    # 2. Quantizer bytes from the reference.
    out = {}
    rng = np.random.default_rng(7)
    shapes = [(1, 32), (3, 64), (17, 4096), (64, 352)]
    for i, (n, k) in enumerate(shapes):
        w = (rng.uniform(-1, 1, (n, k)) * 3).astype(np.float32)
        out[f"w{i}"] = w
        for fmt in ("q4_0", "q8_0"):
            out[f"{fmt}_{i}"] = O.ref_quantize(fmt, w)
    sp = special_quant_rows()
    out["w_special"] = sp
    for fmt in ("q4_0", "q8_0"):
        out[f"{fmt}_special"] = O.ref_quantize(fmt, sp)
    # Rejections: NaN, ±Inf, and scales that overflow binary16 (accepted at the largest finite scale).
    rej = np.ones((6, 64), np.float32)
    rej[0, 40], rej[1, 40], rej[2, 40] = np.nan, np.inf, -np.inf
    rej[3, 3] = 8.0 * 65520.0
    rej[4, 3] = 127.0 * 65520.0
    rej[5, 3] = -8.0 * 65504.0
    out["w_reject"] = rej
    out["q4_0_reject_ok"] = np.array([O.ref_quantize("q4_0", rej[i:i + 1]) is not None for i in range(6)])
    out["q8_0_reject_ok"] = np.array([O.ref_quantize("q8_0", rej[i:i + 1]) is not None for i in range(6)])
    np.savez_compressed(os.path.join(HERE, "ref_quantize.npz"), **out)

    # 3. Activation quantization (quantize_x_q8): random rows and special blocks.
    xs = []
    rng = np.random.default_rng(8)
    xs.append((rng.standard_normal(4096) * 4).astype(np.float32))
    xs.append(np.concatenate([sp[i] for i in range(10)]).astype(np.float32))          # 1280 values
    tiny = rng.uniform(-1, 1, 256).astype(np.float32) * np.float32(1e-30)
    huge = rng.uniform(-1, 1, 256).astype(np.float32) * np.float32(3e38)
    xs.append(np.concatenate([tiny, huge]))
    xo = {}
    for i, x in enumerate(xs):
        qs, dx, ok = ref_quant_x(x)
        xo[f"x{i}"], xo[f"qs{i}"], xo[f"dx{i}"], xo[f"ok{i}"] = x, qs, dx, ok
    bad = np.ones(64, np.float32)
    bad[45] = np.nan
    xo["x_bad"] = bad
    xo["ok_bad"] = ref_quant_x(bad)[2]
    np.savez_compressed(os.path.join(HERE, "ref_quantize_x.npz"), **xo)

    # 4. GEMV outputs of the reference's scalar table and its SIMD table for this CPU.
    go = {"cases": np.array([[s, n, k, 1 if kind == "extreme" else 0] for s, n, k, kind in GEMV_CASES], np.int64)}
    for s, n, k, kind in GEMV_CASES:
        W, x = gemv_case_inputs(s, n, k, kind)
        for fmt in ("q4_0", "q8_0"):
            Wq = O.ref_quantize(fmt, W)
            go[f"{fmt}_{s}_sha"] = np.array(sha(Wq))
            go[f"{fmt}_{s}_scalar"] = O.ref_gemv(fmt, x, Wq, n, k, isa=ISA_SCALAR)
            go[f"{fmt}_{s}_simd"] = O.ref_gemv(fmt, x, Wq, n, k, isa=-1)
    np.savez_compressed(os.path.join(HERE, "ref_gemv.npz"), **go)

    # 5. Dense x·Wᵀ (sgemm / sgemm_f16 / sgemm_bf16 with trans_b=True), M <= 8.
    do = {"cases": np.array(DENSE_CASES, np.int64)}
    for i, (m, n, k) in enumerate(DENSE_CASES):
        A, B, C0, alpha, beta = dense_case_inputs(i, m, n, k)
        do[f"sha{i}"] = np.array(sha(np.concatenate([A.ravel(), B.ravel(), C0.ravel()])))
        for kind in ("f32", "f16", "bf16"):
            a, b = dense_operands(kind, A, B)
            do[f"{kind}_{i}_scalar"] = ref_dense(kind, ISA_SCALAR, a, b, alpha, beta, C0)
            do[f"{kind}_{i}_simd"] = ref_dense(kind, -1, a, b, alpha, beta, C0)
    np.savez_compressed(os.path.join(HERE, "ref_dense.npz"), **do)

    # 6. INT8 sgemm_u8s8.
    write_u8s8()

    with open(os.path.join(HERE, "PROVENANCE.txt"), "w") as f:
        f.write("Golden vectors written by tests/golden/make_golden.py from\n")
        for key, val in meta.items():
            f.write(f"  {key}: {val}\n")
        f.write(f"  llama.cpp fixture: {fx['source']}\n")
    for name in sorted(os.listdir(HERE)):
        print(f"{name}: {os.path.getsize(os.path.join(HERE, name))} bytes")


if __name__ == "__main__":
    if sys.argv[1:] == ["u8s8"]:   # only the sgemm_u8s8 vectors
        write_u8s8()
    else:
        main()
