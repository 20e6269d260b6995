"""GGUF model files (llama.cpp's format, versions 2 and 3) into device memory.

The reference reads GGUF files on the host (examples/llama/gguf_reader.py):
metadata, then each tensor as a NumPy view of the memory-mapped file, with
Q4_0 / Q8_0 tensors as their raw ggml blocks, the bytes gemv_q4_0 /
gemv_q8_0 take. `GGUF(path)` here parses the same files into the same
structure (`version`, `metadata`, `tensors[name]` with `type`, `shape`,
`data`), with the reference's error messages.

What the B200 build adds is the way onto the GPU. `load(path)` (or
`GGUF.to_device()`) copies the chosen tensors into one device allocation:

* each tensor starts on a 256-byte boundary, so Q4_0 / Q8_0 rows reach the
  fast GEMV kernels (16-byte aligned blocks) and dense tensors can be viewed
  in their own dtype;
* the file is streamed through two page-locked buffers: while one buffer's
  DMA to the device runs on a side stream, the next stretch of the file is read
  into the other, so the upload runs at the slower of disk and PCIe rather
  than their sum;
* the result maps each name to a `GGUFTensor` whose `data` is a CUDA tensor:
  uint8 [rows, row_bytes] for Q4_0 / Q8_0 (the GEMV's `Wq`), float32, float16
  or bfloat16 shaped like the reference's view for the dense types.

`dequantize_rows(t, rows)` gives float32 rows of a device tensor (the
embedding lookup of a decode step), exactly as the reference's
dequantize_rows (gguf_reader.py:113-129) does on the host.

Layout (the published GGUF format, kept as is so files from llama.cpp load):
"GGUF", u32 version, u64 tensor count, u64 metadata count; metadata entries
(string key, u32 value type, value); tensor infos (string name, u32 n_dims,
u64 dims innermost first, u32 ggml type, u64 offset); tensor data from the
next multiple of general.alignment (default 32) after the infos.
"""

from __future__ import annotations

import sys
from dataclasses import dataclass
from functools import partial

import numpy as np

from . import _core

# ggml tensor type codes of the format (the public constants of this module).
GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q8_0, GGML_BF16 = 0, 1, 2, 8, 30
TYPE_NAMES = {GGML_F32: "F32", GGML_F16: "F16", GGML_Q4_0: "Q4_0", GGML_Q8_0: "Q8_0", GGML_BF16: "BF16"}


@dataclass(frozen=True)
class _TensorKind:
    """How a ggml type is stored: `block_bytes` bytes hold `block_values`
    values along the innermost dimension; `host` is the NumPy dtype of a dense
    type's host view (None: rows of raw blocks)."""

    block_bytes: int
    block_values: int
    host: str | None


_KINDS = {GGML_F32: _TensorKind(4, 1, "<f4"), GGML_F16: _TensorKind(2, 1, "<f2"),
          GGML_BF16: _TensorKind(2, 1, "<u2"), GGML_Q4_0: _TensorKind(18, 32, None),
          GGML_Q8_0: _TensorKind(34, 32, None)}
# (bytes, values) per block of each supported ggml type
BLOCK = {t: (k.block_bytes, k.block_values) for t, k in _KINDS.items()}
_ALIGN = 256   # start of each tensor in the device allocation


@dataclass
class GGUFTensor:
    name: str
    type: int
    shape: tuple[int, ...]   # outermost first: [N, K] for a weight matrix
    data: object             # host: NumPy view of the file; device: CUDA tensor
    offset: int = 0          # absolute byte offset of the data in the file
    nbytes: int = 0

    @property
    def type_name(self) -> str:
        return TYPE_NAMES.get(self.type, str(self.type))

    @property
    def row_bytes(self) -> int:
        bsize, bvals = BLOCK[self.type]
        return self.shape[-1] // bvals * bsize


class _Fields:
    """Little-endian fields of a mapped file, read at a moving offset. Every read
    is checked against the end of the file first."""

    def __init__(self, mm: np.ndarray, path: str):
        self.mm, self.path, self.at = mm, path, 0

    def _span(self, nbytes: int) -> int:
        start = self.at
        if nbytes < 0 or start + nbytes > self.mm.shape[0]:
            raise ValueError(f"{self.path}: the header runs past the end of the file")
        self.at = start + nbytes
        return start

    def number(self, dtype: str):
        dt = np.dtype(dtype)
        return np.frombuffer(self.mm, dt, 1, self._span(dt.itemsize))[0].item()

    def u32(self) -> int:
        return self.number("<u4")

    def u64(self) -> int:
        return self.number("<u8")

    def text(self) -> str:
        n = self.u64()
        start = self._span(n)
        return self.mm[start:start + n].tobytes().decode("utf-8", errors="replace")

    def vector(self, dtype: str, count: int) -> np.ndarray:
        dt = np.dtype(dtype)
        return np.frombuffer(self.mm, dt, count, self._span(dt.itemsize * count))


# Metadata value type codes of the format: numbers (little-endian, by NumPy
# dtype), a string, or an array (element type code, count, elements).
_NUMBER_DTYPES = {0: "u1", 1: "i1", 2: "<u2", 3: "<i2", 4: "<u4", 5: "<i4", 6: "<f4", 7: "?", 10: "<u8",
                  11: "<i8", 12: "<f8"}
_STRING, _ARRAY, _BOOL = 8, 9, 7


def _read_array(f: _Fields):
    """An array value. Numbers come back as one NumPy view of the file (token
    scores and types of a vocabulary stay zero-copy); strings, booleans and
    nested arrays as a list, as the reference's reader gives them."""
    kind, count = f.u32(), f.u64()
    if kind in _NUMBER_DTYPES and kind != _BOOL:
        return f.vector(_NUMBER_DTYPES[kind], count)
    read = _value_reader(kind, f.path)
    return [read(f) for _ in range(count)]


def _value_reader(kind: int, path: str):
    if kind in _NUMBER_DTYPES:
        return partial(_Fields.number, dtype=_NUMBER_DTYPES[kind])
    if kind == _STRING:
        return _Fields.text
    if kind == _ARRAY:
        return _read_array
    raise ValueError(f"{path}: unknown GGUF metadata type {kind}")


@dataclass
class _Info:
    name: str
    dims: list[int]          # innermost first, as stored
    type: int
    rel_offset: int          # from the start of the data section


def _tensor_view(path: str, mm: np.ndarray, base: int, info: _Info) -> GGUFTensor:
    kind = _KINDS.get(info.type)
    if kind is None:
        raise ValueError(f"{path}: tensor {info.name} has ggml type {info.type} (not F32/F16/BF16/Q8_0/Q4_0)")
    row_len = info.dims[0] if info.dims else 1
    if row_len % kind.block_values:
        raise ValueError(f"{path}: tensor {info.name}: row length {row_len} not a multiple of {kind.block_values}")
    rows = 1
    for d in info.dims[1:]:
        rows *= d
    row_bytes = row_len // kind.block_values * kind.block_bytes
    nbytes = rows * row_bytes
    start = base + info.rel_offset
    if start + nbytes > mm.shape[0]:
        raise ValueError(f"{path}: tensor {info.name} runs past the end of the file")
    raw = mm[start:start + nbytes]
    shape = tuple(int(d) for d in info.dims[::-1])
    data = raw.view(kind.host).reshape(shape) if kind.host else raw.reshape(rows, row_bytes)
    return GGUFTensor(info.name, info.type, shape, data, start, nbytes)


class GGUF:
    """A GGUF file: `version`, `metadata` and `tensors` (NumPy views of the
    memory-mapped file, as the reference's reader gives them)."""

    def __init__(self, path: str):
        self.path = path
        self._mm = np.memmap(path, dtype=np.uint8, mode="r")
        if self._mm[:4].tobytes() != b"GGUF":
            raise ValueError(f"{path}: not a GGUF file")
        f = _Fields(self._mm, path)
        f.at = 4
        self.version = f.u32()
        if self.version not in (2, 3):
            raise ValueError(f"{path}: GGUF version {self.version} (2 and 3 are supported)")
        n_tensors, n_values = f.u64(), f.u64()
        self.metadata: dict[str, object] = {}
        for _ in range(n_values):
            key = f.text()
            self.metadata[key] = _value_reader(f.u32(), path)(f)
        infos = []
        for _ in range(n_tensors):
            name = f.text()
            dims = [f.u64() for _ in range(f.u32())]
            infos.append(_Info(name, dims, f.u32(), f.u64()))
        align = int(self.metadata.get("general.alignment", 32))
        self.data_start = -(-f.at // align) * align
        self.tensors: dict[str, GGUFTensor] = {
            i.name: _tensor_view(path, self._mm, self.data_start, i) for i in infos}

    def to_device(self, names=None, device=None, chunk_bytes: int = 32 << 20) -> dict[str, GGUFTensor]:
        """Copy tensors (all, or `names`) into one allocation on a CUDA device
        (default: torch's current one) and return them by name with CUDA
        tensors as `data` (see the module docstring)."""
        return _upload(self, names, device, chunk_bytes)


def load(path: str, names=None, device=None, chunk_bytes: int = 32 << 20) -> dict[str, GGUFTensor]:
    """GGUF(path).to_device(names, device): a model file's tensors on the GPU."""
    return GGUF(path).to_device(names, device, chunk_bytes)


def _torch():
    t = sys.modules.get("torch")
    if t is None:
        import torch as t   # noqa: F811
    return t


def _upload(g: GGUF, names, device, chunk_bytes: int) -> dict[str, GGUFTensor]:
    t = _torch()
    dev = t.device("cuda", t.cuda.current_device()) if device is None else t.device(device)
    if dev.index is None:
        dev = t.device("cuda", t.cuda.current_device())
    chosen = list(g.tensors) if names is None else list(names)
    for n in chosen:
        if n not in g.tensors:
            raise KeyError(f"{g.path}: no tensor named {n!r}")
    # Device layout: file order, each tensor at a 256-byte boundary.
    order = sorted(chosen, key=lambda n: g.tensors[n].offset)
    place, total = {}, 0
    for n in order:
        place[n] = total
        total += (g.tensors[n].nbytes + _ALIGN - 1) // _ALIGN * _ALIGN
    blob = t.empty(max(total, 1), dtype=t.uint8, device=dev)
    chunk = max(1 << 20, min(int(chunk_bytes), max(total, 1)))
    staging = [t.empty(chunk, dtype=t.uint8).pin_memory() for _ in range(2)]
    views = [memoryview(s.numpy()) for s in staging]
    done = [None, None]
    side = t.cuda.Stream(dev)
    side.wait_stream(t.cuda.current_stream(dev))   # the allocation is free for the copies
    k = 0
    with open(g.path, "rb", buffering=0) as f, t.cuda.stream(side):
        for n in order:
            info = g.tensors[n]
            f.seek(info.offset)
            pos = 0
            while pos < info.nbytes:
                m = min(chunk, info.nbytes - pos)
                b = k & 1
                if done[b] is not None:
                    done[b].synchronize()   # that buffer's previous DMA has finished
                got = f.readinto(views[b][:m])
                if got != m:
                    raise ValueError(f"{g.path}: tensor {n} ends early (read {got} of {m} bytes)")
                dst = blob[place[n] + pos: place[n] + pos + m]
                dst.copy_(staging[b][:m], non_blocking=True)
                ev = t.cuda.Event()
                ev.record(side)
                done[b] = ev
                pos += m
                k += 1
    side.synchronize()
    out = {}
    for n in chosen:
        info = g.tensors[n]
        raw = blob[place[n]: place[n] + info.nbytes]
        if info.type == GGML_F32:
            data = raw.view(t.float32).reshape(info.shape)
        elif info.type == GGML_F16:
            data = raw.view(t.float16).reshape(info.shape)
        elif info.type == GGML_BF16:
            data = raw.view(t.bfloat16).reshape(info.shape)
        else:
            data = raw.view(info.nbytes // info.row_bytes, info.row_bytes)
        out[n] = GGUFTensor(n, info.type, info.shape, data, info.offset, info.nbytes)
    return out


def dequantize_rows(t_: GGUFTensor, rows) -> object:
    """float32 values of some rows of a 2-D tensor on the device (the embedding
    lookup): [len(rows), K], bitwise the reference's dequantize_rows.
    `rows`: an int, a sequence or NumPy array (checked against the row count;
    IndexError as NumPy's), or an int32 CUDA tensor (rows outside the tensor
    give NaN rows and a device error, as the kernel cannot raise)."""
    t = _torch()
    w = t_.data
    if not (isinstance(w, t.Tensor) and w.is_cuda):
        raise ValueError("dequantize_rows takes a tensor loaded to the device (GGUF.to_device / load)")
    N, K = (t_.shape[0], t_.shape[-1]) if len(t_.shape) > 1 else (1, t_.shape[0])
    if isinstance(rows, t.Tensor) and rows.is_cuda:
        idx = rows.to(t.int32).reshape(-1).contiguous()
    else:
        r = np.atleast_1d(np.asarray(rows)).astype(np.int64).reshape(-1)
        bad = (r < -N) | (r >= N)
        if bad.any():
            raise IndexError(f"index {int(r[bad][0])} is out of bounds for axis 0 with size {N}")
        r = np.where(r < 0, r + N, r).astype(np.int32)
        idx = t.from_numpy(r).to(w.device, non_blocking=False)
    n = idx.numel()
    if t_.type in (GGML_Q4_0, GGML_Q8_0):
        out = t.empty((n, K), dtype=t.float32, device=w.device)
        dev = w.device.index if w.device.index is not None else t.cuda.current_device()
        stream = t.cuda.current_stream(w.device).cuda_stream
        _core._dequantize_rows(0 if t_.type == GGML_Q4_0 else 1, N, K, w.data_ptr(), idx.data_ptr(), n,
                               out.data_ptr(), K, stream, dev)
        return out
    dense = w.reshape(N, K)
    return dense.index_select(0, idx.long()).to(t.float32)


__all__ = ["GGUF", "GGUFTensor", "load", "dequantize_rows", "TYPE_NAMES", "GGML_F32", "GGML_F16", "GGML_Q4_0",
           "GGML_Q8_0", "GGML_BF16"]
