"""Row-sharded GEMV across ranks, on CPU gloo process groups (world size 2
and 3): the planner's slices, the padded all-gather of uneven slices, and
bitwise equality with the unsharded result — with the CPU oracle standing in
for each rank's GPU GEMV. Plus the failure path: a rank that dies before the
gather makes the other rank's collective end with an error, not a hang."""

from __future__ import annotations

import os
import socket
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _setup_paths():
    for p in (os.path.join(REPO, "simd-ml-kernels_b200"), os.path.join(REPO, "oracle")):
        if p not in sys.path:
            sys.path.insert(0, p)


def _rank_main(rank, world, port, fmt, N, K, M, out_dir):
    _setup_paths()
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    import oracle as O
    from simd_ml_kernels import shard

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    rng = np.random.default_rng(N + K)
    W = rng.standard_normal((N, K)).astype(np.float32)
    X = rng.standard_normal((M, K)).astype(np.float32)
    Wq = O.quantize(fmt, W)
    local = shard.local_rows(Wq, fmt, N, K, rank, world)

    def oracle_local(x, Wl, n, k, out):
        xs = x.numpy().reshape(-1, k)
        ys = np.stack([O.gemv_scalar(fmt, xs[m], Wl.numpy(), n, k) for m in range(xs.shape[0])])
        res = torch.from_numpy(ys.reshape(x.shape[:-1] + (n,)))
        if out is not None:
            out.reshape(res.shape).copy_(res)
            return out
        return res

    sg = shard.ShardedGemv(fmt, torch.from_numpy(np.ascontiguousarray(local)), N, K, local_fn=oracle_local)
    y1 = sg.forward(torch.from_numpy(X[0]))
    yM = sg.forward(torch.from_numpy(X))
    np.save(os.path.join(out_dir, f"y1_{rank}.npy"), y1.numpy())
    np.save(os.path.join(out_dir, f"yM_{rank}.npy"), yM.numpy())
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world,N", [(2, 1003), (3, 1003), (2, 64), (3, 8)])
def test_sharded_gather_equals_unsharded(tmp_path, world, N):
    _setup_paths()
    import oracle as O

    fmt, K, M = "q4_0", 256, 3
    mp.start_processes(_rank_main, args=(world, _free_port(), fmt, N, K, M, str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    rng = np.random.default_rng(N + K)
    W = rng.standard_normal((N, K)).astype(np.float32)
    X = rng.standard_normal((M, K)).astype(np.float32)
    Wq = O.quantize(fmt, W)
    want = np.stack([O.gemv_scalar(fmt, X[m], Wq, N, K) for m in range(M)])
    for r in range(world):
        y1 = np.load(tmp_path / f"y1_{r}.npy")
        yM = np.load(tmp_path / f"yM_{r}.npy")
        assert y1.shape == (N,) and yM.shape == (M, N)
        np.testing.assert_array_equal(y1.view(np.uint32), want[0].view(np.uint32))
        np.testing.assert_array_equal(yM.view(np.uint32), want.view(np.uint32))


def _failing_rank_main(rank, world, port, out_dir):
    _setup_paths()
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    if rank == 1:
        os._exit(3)            # dies between steps, before the collective
    status = "no error"
    try:
        parts = [torch.empty(4) for _ in range(world)]
        dist.all_gather(parts, torch.ones(4))
    except Exception as exc:  # noqa: BLE001 - any collective error is the expected outcome
        status = "error: " + type(exc).__name__
    with open(os.path.join(out_dir, "status.txt"), "w") as f:
        f.write(status)
    os._exit(0)


def test_dead_rank_ends_the_collective_with_an_error(tmp_path):
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_failing_rank_main, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    assert (tmp_path / "status.txt").exists(), "rank 0 did not finish"
    assert (tmp_path / "status.txt").read_text().startswith("error"), (tmp_path / "status.txt").read_text()
