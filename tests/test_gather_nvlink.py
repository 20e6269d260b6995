"""Row-sharded GEMV with the all-gather fused into the kernel (gather="nvlink"):
2 GPUs, one spawned process each, NCCL only for the set-up handshake. Every
step's gathered y equals the unsharded GEMV on one GPU (bitwise for one and
two rows of x, which take the same kernel; within the reference's bound of the
float64 sums for four and eight rows, which take the tensor-core kernel with
the gather fused into its stores), a reader queued on the stream before the next
step sees the step's result intact (the contract: y_full is valid until this
rank's next call), and no device error is raised. Needs two GPUs; skipped
otherwise."""

from __future__ import annotations

import os
import socket
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out_dir):
    for p in (os.path.join(REPO, "simd-ml-kernels_b200"), os.path.join(REPO, "oracle"), HERE):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    import simd_ml_kernels as sk
    from simd_ml_kernels import _core, shard

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    status = "ok"
    try:
        N, K = 1003, 2048
        g = torch.Generator(device="cuda").manual_seed(11)
        W = torch.randn((N, K), generator=g, device="cuda") * 0.02
        Wq = sk.quantize_q4_0(W).reshape(-1)
        rb = K // 32 * 18
        lo, hi = shard.row_slice(N, rank, world)
        sg = shard.ShardedGemv("q4_0", Wq[lo * rb:hi * rb].clone(), N, K, gather="nvlink")
        prev = None
        for step in range(8):
            M = (1, 2, 4, 8)[step % 4]
            X = torch.randn((M, K), generator=torch.Generator(device="cuda").manual_seed(100 + step), device="cuda")
            Y = sg.forward(X if M > 1 else X[0]).reshape(M, N)
            copy = Y.clone()   # a reader queued on the stream before the next call
            want = sk.gemv_q4_0_batch(X, Wq, N, K)
            if prev is not None:   # the previous step's reader saw its result whole
                torch.cuda.synchronize()
                assert torch.equal(prev[0].view(torch.int32), prev[1].view(torch.int32)), \
                    f"step {step}: the previous step's copy differs from its own check"
            torch.cuda.synchronize()
            if M <= 2:
                assert torch.equal(copy.view(torch.int32), want.view(torch.int32)), f"step {step}: not bitwise"
            else:
                assert (copy - want).abs().max().item() <= 1e-5 * want.abs().max().item(), f"step {step}"
            prev = (copy, copy.clone())
        torch.cuda.synchronize()
        assert _core._device_error(torch.cuda.current_stream().cuda_stream) == 0
        # Data-free gather steps (a device-side barrier across the ranks) and the
        # NVLink ping-pong diagnostic: both end, in time, without a device error.
        stream = torch.cuda.current_stream().cuda_stream
        for _ in range(50):
            _core._gather_barrier(sg._g, stream)
        ns = _core._gather_pingpong(sg._g, 1000, 0, stream) + _core._gather_pingpong(sg._g, 1000, 1, stream)
        assert (ns > 0) if rank == 0 else (ns == 0)
        Y = sg.forward(X).reshape(M, N)   # the gather still works after them
        torch.cuda.synchronize()
        assert (Y - sk.gemv_q4_0_batch(X, Wq, N, K)).abs().max().item() <= 1e-5 * Y.abs().max().item()
        assert _core._device_error(stream) == 0
        sg.close()
        # Long rows, few tiles per GPU: the kernel that splits K over warps, with
        # the gather fused in; two steps in a row against the unsharded GEMV
        # (split differently, so within the bound).
        N2, K2 = 1002, 16384
        W2 = sk.quantize_q4_0(torch.randn((N2, K2), generator=g, device="cuda") * 0.02).reshape(-1)
        rb2 = K2 // 32 * 18
        lo2, hi2 = shard.row_slice(N2, rank, world)
        sg2 = shard.ShardedGemv("q4_0", W2[lo2 * rb2:hi2 * rb2].clone(), N2, K2, gather="nvlink")
        for step in range(2):
            x2 = torch.randn(K2, generator=torch.Generator(device="cuda").manual_seed(200 + step), device="cuda")
            Y2 = sg2.forward(x2).reshape(N2).clone()
            want2 = sk.gemv_q4_0(x2, W2, N2, K2)
            torch.cuda.synchronize()
            assert (Y2 - want2).abs().max().item() <= 1e-5 * want2.abs().max().item(), f"long rows, step {step}"
        assert _core._device_error(stream) == 0
        sg2.close()
    except Exception as exc:  # noqa: BLE001 - reported to the parent
        status = f"error: {type(exc).__name__}: {exc}"
    with open(os.path.join(out_dir, f"rank{rank}.txt"), "w") as f:
        f.write(status)
    dist.barrier()
    dist.destroy_process_group()


def test_fused_gather_two_gpus(tmp_path):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    mp.start_processes(_rank, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    for r in range(2):
        assert (tmp_path / f"rank{r}.txt").read_text() == "ok", (tmp_path / f"rank{r}.txt").read_text()
