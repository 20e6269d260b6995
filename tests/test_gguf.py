"""GGUF model files: the reader (simd_ml_kernels.gguf) against the reference's
own reader, the upload to device memory, and the dequantization kernel.

The fixtures (tests/golden/tiny_v3.gguf, tiny_v2_align64.gguf) and what the
reference's reader (examples/llama/gguf_reader.py) returns for them
(ref_gguf.npz) come from tests/golden/make_gguf.py. CPU tests parse the files;
`gpu` tests load them onto the device.
"""

from __future__ import annotations

import hashlib
import json
import os
import shutil

import numpy as np
import pytest

import oracle as O
from simd_ml_kernels import gguf

GOLD = os.path.join(os.path.dirname(__file__), "golden")
FILES = ["tiny_v3.gguf", "tiny_v2_align64.gguf"]


def golden():
    return np.load(os.path.join(GOLD, "ref_gguf.npz"))


def _plain(v):
    if isinstance(v, np.ndarray):
        return {"array": v.tolist(), "dtype": str(v.dtype)}
    if isinstance(v, list):
        return [_plain(x) for x in v]
    return v


@pytest.mark.parametrize("fname", FILES)
def test_reader_matches_reference(fname):
    """Version, metadata (every value kind), tensor names in file order, types,
    shapes and bytes: what the reference's reader returns for the same file."""
    g = golden()
    f = gguf.GGUF(os.path.join(GOLD, fname))
    assert f.version == int(g[f"{fname}:version"])
    assert json.loads(json.dumps({k: _plain(v) for k, v in f.metadata.items()})) == \
        json.loads(str(g[f"{fname}:metadata"]))
    assert list(f.tensors) == [str(n) for n in g[f"{fname}:names"]]
    for n, t in f.tensors.items():
        assert t.type == int(g[f"{fname}:{n}:type"])
        assert t.shape == tuple(int(d) for d in g[f"{fname}:{n}:shape"])
        assert hashlib.sha256(np.ascontiguousarray(t.data).tobytes()).hexdigest() == str(g[f"{fname}:{n}:sha"])


def test_oracle_dequantize_matches_reference():
    """The oracle's dequantize_rows reproduces the reference's bit for bit."""
    g = golden()
    f = gguf.GGUF(os.path.join(GOLD, FILES[0]))
    for n, t in f.tensors.items():
        if t.type_name not in ("Q4_0", "Q8_0"):
            continue
        rows = g[f"{FILES[0]}:{n}:rows"]
        got = O.dequantize_rows(t.type_name.lower(), np.asarray(t.data), t.shape[1], rows)
        np.testing.assert_array_equal(got.view(np.uint32), g[f"{FILES[0]}:{n}:dequant"].view(np.uint32))


def test_reader_errors(tmp_path):
    """The reference's errors: not a GGUF file, an unsupported version or
    tensor type; and a file cut short is caught before any read past its end."""
    src = os.path.join(GOLD, FILES[0])
    bad = tmp_path / "x.gguf"
    bad.write_bytes(b"GGML" + open(src, "rb").read()[4:])
    with pytest.raises(ValueError, match="not a GGUF file"):
        gguf.GGUF(str(bad))
    raw = bytearray(open(src, "rb").read())
    raw[4:8] = (1).to_bytes(4, "little")
    bad.write_bytes(bytes(raw))
    with pytest.raises(ValueError, match="version 1"):
        gguf.GGUF(str(bad))
    f = gguf.GGUF(src)
    cut = tmp_path / "cut.gguf"
    shutil.copyfile(src, cut)
    with open(cut, "r+b") as h:
        h.truncate(f.tensors["output_norm.weight"].offset + 16)
    with pytest.raises(ValueError, match="past the end"):
        gguf.GGUF(str(cut))
    # ggml type 12 (Q4_K) in the first tensor info: located by its name.
    raw = bytearray(open(src, "rb").read())
    key = b"token_embd.weight"
    at = raw.index(key) + len(key)
    ndims = int.from_bytes(raw[at:at + 4], "little")
    t_at = at + 4 + 8 * ndims
    raw[t_at:t_at + 4] = (12).to_bytes(4, "little")
    bad.write_bytes(bytes(raw))
    with pytest.raises(ValueError, match="ggml type 12"):
        gguf.GGUF(str(bad))


# ---- on the device ----------------------------------------------------------------

@pytest.fixture(scope="module")
def torch(cuda_device):
    import torch as t
    return t


@pytest.mark.gpu
@pytest.mark.parametrize("fname", FILES)
def test_load_to_device(torch, fname):
    """Every tensor lands on the device byte for byte, 256-byte aligned, in the
    dtype of the reference's view; the upload also works in chunks smaller
    than one tensor (the double-buffered path)."""
    path = os.path.join(GOLD, fname)
    host = gguf.GGUF(path)
    for chunk in (32 << 20, 1 << 20):
        dev = gguf.load(path, chunk_bytes=chunk)
        assert list(dev) == list(host.tensors)
        for n, t in dev.items():
            h = host.tensors[n]
            assert t.data.is_cuda and t.data.data_ptr() % 256 == 0
            assert t.type == h.type and t.shape == h.shape
            got = t.data.contiguous().view(torch.uint8).cpu().numpy().tobytes()
            assert got == np.ascontiguousarray(h.data).tobytes(), n
            if h.type_name in ("Q4_0", "Q8_0"):
                assert tuple(t.data.shape) == h.data.shape and t.data.dtype == torch.uint8
            else:
                want = {"F32": torch.float32, "F16": torch.float16, "BF16": torch.bfloat16}[h.type_name]
                assert t.data.dtype == want and tuple(t.data.shape) == h.shape
    some = gguf.load(path, names=["blk.0.ffn_down.weight"])
    assert list(some) == ["blk.0.ffn_down.weight"]
    with pytest.raises(KeyError):
        gguf.load(path, names=["nope"])


@pytest.mark.gpu
def test_loaded_weights_feed_the_gemv(torch):
    """The loaded Q4_0 / Q8_0 tensors are the GEMV's Wq as they stand: the same
    bits as the GEMV on the file's host bytes."""
    import simd_ml_kernels as sk
    path = os.path.join(GOLD, FILES[1])
    host = gguf.GGUF(path)
    dev = gguf.load(path)
    rng = np.random.default_rng(3)
    for n in ("token_embd.weight", "blk.0.attn_q.weight", "blk.0.ffn_down.weight"):
        t = dev[n]
        N, K = t.shape
        fn = sk.gemv_q4_0 if t.type_name == "Q4_0" else sk.gemv_q8_0
        x = rng.standard_normal(K).astype(np.float32)
        want = fn(x, np.ascontiguousarray(host.tensors[n].data), N, K)
        got = fn(torch.from_numpy(x).cuda(), t.data.reshape(-1), N, K).cpu().numpy()
        np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32), err_msg=n)


@pytest.mark.gpu
def test_dequantize_rows_kernel(torch):
    """Device dequantize_rows: bitwise the reference's on the fixture's rows
    (all five types), bitwise the oracle on a larger random Q4_0 / Q8_0
    matrix; host indices out of range raise IndexError, device indices out of
    range give NaN rows and a device error."""
    from simd_ml_kernels import _core
    g = golden()
    dev = gguf.load(os.path.join(GOLD, FILES[0]))
    for n, t in dev.items():
        key = f"{FILES[0]}:{n}:rows"
        if key not in g.files:
            continue
        rows = g[key]
        got = gguf.dequantize_rows(t, rows).cpu().numpy()
        np.testing.assert_array_equal(got.view(np.uint32), g[f"{FILES[0]}:{n}:dequant"].view(np.uint32), err_msg=n)
        got_dev_idx = gguf.dequantize_rows(t, torch.tensor(rows, dtype=torch.int32, device="cuda")).cpu().numpy()
        np.testing.assert_array_equal(got_dev_idx.view(np.uint32), got.view(np.uint32))
    rng = np.random.default_rng(8)
    for fmt, ttype in (("q4_0", gguf.GGML_Q4_0), ("q8_0", gguf.GGML_Q8_0)):
        N, K = 1000, 4096 + 32
        Wq = O.quantize(fmt, (rng.standard_normal((N, K)) * 0.1).astype(np.float32))
        t = gguf.GGUFTensor("w", ttype, (N, K), torch.from_numpy(Wq).cuda())
        rows = rng.integers(0, N, 37)
        got = gguf.dequantize_rows(t, rows).cpu().numpy()
        np.testing.assert_array_equal(got.view(np.uint32), O.dequantize_rows(fmt, Wq, K, rows).view(np.uint32))
        np.testing.assert_array_equal(gguf.dequantize_rows(t, -1).cpu().numpy(), O.dequantize_rows(fmt, Wq, K, [N - 1]))
    with pytest.raises(IndexError):
        gguf.dequantize_rows(t, [N])
    stream = torch.cuda.current_stream().cuda_stream
    assert _core._device_error(stream) == 0
    bad = gguf.dequantize_rows(t, torch.tensor([0, N, -5], dtype=torch.int32, device="cuda")).cpu().numpy()
    assert np.isfinite(bad[0]).all() and np.isnan(bad[1:]).all()
    assert _core._device_error(stream) & 2   # kErrBadLaunch, read and cleared
    assert _core._device_error(stream) == 0
