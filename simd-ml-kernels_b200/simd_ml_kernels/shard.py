"""shard.py — row-sharded decode GEMV across the GPUs of one node.

W [N, K] is split by output rows into one contiguous slice per rank, whole
8-row groups each, sizes within one group of each other: the reference's
OpenMP split (gemv_slice, src/dispatch/dispatch.cpp:373-379,
kGemvRowGroup = 8) moved from threads to GPUs. Each output row is computed by
one rank with the same kernel and order as unsharded, so the gathered y is
bitwise identical for any rank count. x is replicated (every rank quantizes
it itself, deterministically); y slices are all-gathered over NVLink with
NCCL (torch.distributed, one process per GPU). No reduction: K is never
split across ranks.
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


class ShardedGemv:
    """One rank's share of y = x @ W.T with W row-sharded over a process group.

    Wq_local: this rank's rows (ggml blocks, a CUDA uint8 tensor) — rows
    row_slice(N, rank, world). forward(x) runs the local GEMV on the current
    stream, then all-gathers the slices into y [M, N] on every rank.
    """

    def __init__(self, fmt: str, Wq_local, N: int, K: int, group=None):
        import torch
        import torch.distributed as dist

        self.fmt, self.N, self.K, self.group = fmt, N, K, group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.lo, self.hi = row_slice(N, self.rank, self.world)
        self.sizes = shard_sizes(N, self.world)
        self.pad = max(self.sizes) if self.sizes else 0
        bpb = 18 if fmt == "q4_0" else 34
        if Wq_local.numel() != (self.hi - self.lo) * (K // 32) * bpb:
            raise ValueError("Wq_local does not hold this rank's rows")
        self.Wq = Wq_local
        self._torch, self._dist = torch, dist

    def local(self, x, out=None):
        """This rank's y slice [M, hi - lo] (M = rows of x; a 1-D x gives [hi - lo])."""
        import simd_ml_kernels as sk
        n = self.hi - self.lo
        if x.dim() == 1:
            fn = sk.gemv_q4_0 if self.fmt == "q4_0" else sk.gemv_q8_0
        else:
            fn = sk.gemv_q4_0_batch if self.fmt == "q4_0" else sk.gemv_q8_0_batch
        return fn(x, self.Wq, n, self.K, out=out)

    def forward(self, x):
        """y [N] (or [M, N]) on every rank: local slice, then an all-gather."""
        torch, dist = self._torch, self._dist
        M = 1 if x.dim() == 1 else x.shape[0]
        n = self.hi - self.lo
        send = torch.empty((M, self.pad), dtype=torch.float32, device=x.device)
        if n == self.pad:
            self.local(x, out=send)
        else:   # a short last slice: pad its rows (the padding is dropped after the gather)
            send[:, :n].copy_(self.local(x).reshape(M, n))
        if self.world == 1:
            y = send[:, :n]
        else:
            recv = torch.empty((self.world, M, self.pad), dtype=torch.float32, device=x.device)
            dist.all_gather_into_tensor(recv, send, group=self.group)
            if all(s == self.pad for s in self.sizes):
                y = recv.permute(1, 0, 2).reshape(M, self.world * self.pad)
            else:
                y = torch.cat([recv[r, :, :self.sizes[r]] for r in range(self.world)], dim=1)
        return y[0] if x.dim() == 1 else y
