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


def block_bytes(fmt: str) -> int:
    return {"q4_0": 18, "q8_0": 34}[fmt]


def local_rows(Wq_full, fmt: str, N: int, K: int, rank: int, world: int):
    """This rank's rows of a full weight matrix (flat ggml bytes or [N, row_bytes])."""
    lo, hi = row_slice(N, rank, world)
    rb = K // 32 * block_bytes(fmt)
    return Wq_full.reshape(-1)[lo * rb:hi * rb]


class ShardedGemv:
    """One rank's share of y = x @ W.T with W row-sharded over a process group.

    Wq_local: this rank's rows (ggml blocks) — rows row_slice(N, rank, world).
    forward(x) runs the local GEMV (on the current CUDA stream for CUDA
    tensors), then all-gathers the slices: y [N] (or [M, N] for x [M, K]) on
    every rank. `local_fn(x, Wq_local, n, K, out)` replaces the GPU GEMV (tests
    run the CPU oracle there on gloo ranks).
    """

    def __init__(self, fmt: str, Wq_local, N: int, K: int, group=None, local_fn=None):
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
        self.Wq = Wq_local
        self.local_fn = local_fn or self._gpu_local
        self._torch, self._dist = torch, dist
        self._gather_list = dist.is_initialized() and dist.get_backend(group) == "gloo"

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
