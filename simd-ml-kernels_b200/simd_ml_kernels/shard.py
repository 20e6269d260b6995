"""shard.py — row-sharded decode GEMV across the GPUs of one node.

W [N, K] is split by output rows into one contiguous slice per rank, whole
8-row groups each, sizes within one group of each other: the reference's
OpenMP split (gemv_slice, src/dispatch/dispatch.cpp:373-379,
kGemvRowGroup = 8) moved from threads to GPUs. Each output row is computed by
one rank with the same arithmetic as unsharded whenever the slice takes the
same kernel as the whole matrix (always at K = 2048), so the gathered y is
then bitwise identical for any rank count. x is replicated (every rank quantizes
it itself, deterministically); y slices are all-gathered over NVLink, either
by the GEMV kernel itself (gather="nvlink": each rank's kernel stores its
slice into every peer's receive buffer through CUDA IPC mappings, each value
paired with the step's tag in one 64-bit store, and a wait kernel polls the
tags and assembles the full y) or by NCCL's all-gather (gather="nccl"). One process per GPU. No reduction: K is never split across
ranks.
"""

from __future__ import annotations

ROW_GROUP = 8


def row_slice(N: int, t: int, parts: int) -> tuple[int, int]:
    """Rows [lo, hi) of part t of `parts`: whole 8-row groups, contiguous."""
    if parts <= 0 or not 0 <= t < parts:
        raise ValueError("need 0 <= t < parts")
    groups = (N + ROW_GROUP - 1) // ROW_GROUP
    lo = min(N, groups * t // parts * ROW_GROUP)
    hi = min(N, groups * (t + 1) // parts * ROW_GROUP)
    return lo, hi


def shard_sizes(N: int, parts: int) -> list[int]:
    return [hi - lo for lo, hi in (row_slice(N, t, parts) for t in range(parts))]


def block_bytes(fmt: str) -> int:
    return {"q4_0": 18, "q8_0": 34}[fmt]


def local_rows(Wq_full, fmt: str, N: int, K: int, rank: int, world: int):
    """This rank's rows of a full weight matrix (flat ggml bytes or [N, row_bytes])."""
    lo, hi = row_slice(N, rank, world)
    rb = K // 32 * block_bytes(fmt)
    return Wq_full.reshape(-1)[lo * rb:hi * rb]


class _Area:
    """__cuda_array_interface__ of one fused-gather output area."""

    __slots__ = ("__cuda_array_interface__",)

    def __init__(self, ptr: int, rows: int, cols: int):
        self.__cuda_array_interface__ = {"data": (ptr, False), "shape": (rows, cols), "typestr": "<f4",
                                         "strides": None, "version": 2}


class ShardedGemv:
    """One rank's share of y = x @ W.T with W row-sharded over a process group.

    Wq_local: this rank's rows (ggml blocks) — rows row_slice(N, rank, world).
    forward(x) runs the local GEMV (on the current CUDA stream for CUDA
    tensors) and gathers the slices: y [N] (or [M, N] for x [M, K]) on every
    rank. gather="nvlink" (CUDA tensors, world > 1) fuses the gather into the
    GEMV kernel; its result is a view into the gather buffer that stays valid
    until this rank's next forward call: queue its readers on the stream (or
    clone it) before that call. gather="nccl" uses NCCL's all-gather. `local_fn(x, Wq_local, n, K,
    out)` replaces the GPU GEMV (tests run the CPU oracle there on gloo ranks).
    Every rank must make the same sequence of forward calls.
    """

    def __init__(self, fmt: str, Wq_local, N: int, K: int, group=None, local_fn=None, gather: str = "nccl",
                 m_max: int = 8):
        import torch
        import torch.distributed as dist

        self.fmt, self.N, self.K, self.group = fmt, N, K, group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.lo, self.hi = row_slice(N, self.rank, self.world)
        self.sizes = shard_sizes(N, self.world)
        self.pad = max(self.sizes) if self.sizes else 0
        if Wq_local.numel() != (self.hi - self.lo) * (K // 32) * block_bytes(fmt):
            raise ValueError("Wq_local does not hold this rank's rows")
        if gather not in ("nccl", "nvlink"):
            raise ValueError("gather must be 'nccl' or 'nvlink'")
        self.Wq = Wq_local
        self.local_fn = local_fn or self._gpu_local
        self._torch, self._dist = torch, dist
        self._gather_list = dist.is_initialized() and dist.get_backend(group) == "gloo"
        self._g = None
        if gather == "nvlink" and self.world > 1:
            self._open_nvlink(m_max)

    # -- fused NVLink gather ---------------------------------------------------------

    def _open_nvlink(self, m_max: int):
        torch, dist = self._torch, self._dist
        from simd_ml_kernels import _core
        if self.local_fn != self._gpu_local:
            raise ValueError("gather='nvlink' runs the GPU kernel; local_fn cannot replace it")
        if self.pad < 1 or self.K % 256 or not self.Wq.is_cuda:
            raise ValueError("gather='nvlink' needs CUDA weights, K % 256 == 0 and rows on every rank")
        self.device = self.Wq.device
        index = self.device.index if self.device.index is not None else torch.cuda.current_device()
        self._index, self.m_max = index, m_max
        handle, ipc = _core._gather_create(self.world, self.rank, self.pad, m_max, index)
        handles = [None] * self.world
        dist.all_gather_object(handles, ipc, group=self.group)
        _core._gather_connect(handle, b"".join(handles))
        self._g = handle
        cols = self.world * self.pad
        self._areas = {}
        dist.barrier(group=self.group)   # every rank's buffer is mapped and zeroed before any step
        self._cols = cols

    def _area_view(self, ptr: int, M: int):
        t = self._areas.get(ptr)
        if t is None:
            t = self._torch.as_tensor(_Area(ptr, self.m_max, self._cols), device=self.device)
            self._areas[ptr] = t
        return t[:M]

    def close(self):
        """Release the fused gather's buffers (before destroying the process group)."""
        if self._g is not None:
            from simd_ml_kernels import _core
            self._torch.cuda.synchronize(self.device)
            _core._gather_destroy(self._g)
            self._g, self._areas = None, {}

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass

    def _forward_nvlink(self, x):
        torch = self._torch
        from simd_ml_kernels import _core, _current_stream
        xx = x.reshape(-1, self.K)
        if x.dtype != torch.float32 or not xx.is_contiguous():
            raise ValueError("x must be a contiguous float32 CUDA tensor")
        M = xx.shape[0]
        ptr = _core._gemv_q_gather(self._g, 0 if self.fmt == "q4_0" else 1, M, self.hi - self.lo, self.K,
                                   xx.data_ptr(), self.K, self.Wq.data_ptr(), _current_stream(self._index),
                                   self._index)
        area = self._area_view(ptr, M)
        if all(s == self.pad for s in self.sizes):
            y = area
        else:
            y = torch.cat([area[:, r * self.pad:r * self.pad + self.sizes[r]] for r in range(self.world)], dim=1)
        return y[0] if x.dim() == 1 else y

    def _gpu_local(self, x, Wq, n, K, out):
        import simd_ml_kernels as sk
        if x.dim() == 1:
            fn = sk.gemv_q4_0 if self.fmt == "q4_0" else sk.gemv_q8_0
            return fn(x, Wq, n, K, out=out.reshape(-1) if out is not None else None)
        fn = sk.gemv_q4_0_batch if self.fmt == "q4_0" else sk.gemv_q8_0_batch
        return fn(x, Wq, n, K, out=out)

    def local(self, x, out=None):
        """This rank's y slice [M, hi - lo] (a 1-D x gives [hi - lo])."""
        return self.local_fn(x, self.Wq, self.hi - self.lo, self.K, out)

    def forward(self, x):
        """y [N] (or [M, N]) on every rank: local slice, then an all-gather."""
        if self._g is not None:
            return self._forward_nvlink(x)
        torch, dist = self._torch, self._dist
        M = 1 if x.dim() == 1 else x.shape[0]
        n = self.hi - self.lo
        send = torch.empty((M, self.pad), dtype=torch.float32, device=x.device)
        if n == self.pad and n > 0:
            self.local(x, out=send)
        else:   # a short slice: pad its rows (the padding is dropped after the gather)
            send.zero_()
            if n:
                send[:, :n].copy_(self.local(x).reshape(M, n))
        if self.world == 1:
            y = send[:, :n]
        else:
            if self._gather_list:
                parts = [torch.empty_like(send) for _ in range(self.world)]
                dist.all_gather(parts, send, group=self.group)
                recv = torch.stack(parts)
            else:
                recv = torch.empty((self.world, M, self.pad), dtype=torch.float32, device=x.device)
                dist.all_gather_into_tensor(recv, send, group=self.group)
            if all(s == self.pad for s in self.sizes):
                y = recv.permute(1, 0, 2).reshape(M, self.world * self.pad)
            else:
                y = torch.cat([recv[r, :, :self.sizes[r]] for r in range(self.world)], dim=1)
        return y[0] if x.dim() == 1 else y
