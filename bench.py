"""bench.py — decode-GEMV throughput on B200.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--all]

Workload: Q4_0 decode GEMV y = x @ W.T, M = 1, K = 2048,
N = 8192 per GPU; W ~ N(0, 0.02) from seed 0 quantized ggml-style (the
device quantizer, byte-identical to the reference's), x ~ N(0, 1). A step is
one GEMV over the whole matrix. The timed region holds exactly K steps,
launched as CUDA graphs with programmatic dependent launch; consecutive steps
read different weight copies, together more than 2x the L2 cache, so every
step streams its weights from HBM. value = algorithmic bytes (W + x + y per
step, the reference's convention, _cli.py:1198) of all steps of all ranks /
max-over-ranks device time.

N > 1 (torchrun): weak scaling. Each rank holds its 8192-row slice of a
[8192*N, 2048] matrix (the reference's row slicing, gemv_slice), and every
step all-gathers the y slices over NVLink, so every rank ends the step with
all 8192*N outputs: by default inside the GEMV kernel (it stores its slice
into every rank's buffer through CUDA IPC mappings; a one-warp kernel then
waits for the peers' signals), or with NCCL (--gather nccl).

--impl reference: the reference's own CPU kernel (Mattral/simd-ml-kernels
compiled from its sources, oracle/_ref) on the same workload with every host
thread, rank 0 only.

One JSON line on rank 0.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "simd-ml-kernels_b200"))

METRIC = "Q4_0 decode-GEMV HBM GB/s (% of B200 peak); Llama-1B-shape GEMV stack tok/s"
N_ROWS, K_COLS = 8192, 2048
Q4_ROW_BYTES = K_COLS // 32 * 18
W_BYTES = N_ROWS * Q4_ROW_BYTES
STEP_BYTES = W_BYTES + 4 * K_COLS + 4 * N_ROWS          # 9,478,144 (W + x + y)
LLAMA_SHAPES = [(2048, 2048), (512, 2048), (512, 2048), (2048, 2048), (8192, 2048), (8192, 2048), (2048, 8192)]
LLAMA_LAYERS, LLAMA_VOCAB, LLAMA_TOKENS = 16, 128256, 128


def measured_peaks() -> dict:
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


def committed_traffic(name: str):
    """dram__bytes_read.sum + dram__bytes_write.sum per launch from a committed ncu summary."""
    p = os.path.join(REPO, "profiles", name)
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f).get("dram_bytes_per_launch")
    return None


# ---- clocks during the timed region (NVML) --------------------------------------

class ClockSampler:
    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
               "sw_power_cap": 0x4, "hw_power_brake_slowdown": 0x80}

    def __init__(self, device: int, period_s: float = 0.01):
        self.samples, self.reasons, self.period = [], set(), period_s
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(device)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:  # noqa: BLE001
            self.nv = None

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                r = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for name, bit in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:  # noqa: BLE001
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.nv is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread:
            self._thread.join()

    def summary(self) -> dict:
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ---- the reference's CPU kernel -------------------------------------------------------

def llc_bytes() -> int:
    """Total last-level cache of the host: every distinct cache instance of the
    highest level, summed (a multi-die CPU has several L3s)."""
    import glob as _glob

    def size(path):
        s = open(path).read().strip()
        return int(s[:-1]) * {"K": 1 << 10, "M": 1 << 20, "G": 1 << 30}.get(s[-1], 1) if s[-1].isalpha() else int(s)

    seen, best_level, total = set(), 0, 0
    for d in _glob.glob("/sys/devices/system/cpu/cpu[0-9]*/cache/index[0-9]*"):
        try:
            level = int(open(os.path.join(d, "level")).read())
            shared = open(os.path.join(d, "shared_cpu_list")).read().strip()
            sz = size(os.path.join(d, "size"))
        except (OSError, ValueError):
            continue
        if level > best_level:
            seen, best_level, total = set(), level, 0
        if level == best_level and shared not in seen:
            seen.add(shared)
            total += sz
    return total or 64 << 20


def reference_setup(threads: int):
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import oracle as O

    if not O.ref_available():
        return None
    R = O.ref()
    R.smkref_set_num_threads(threads)
    rng = np.random.default_rng(0)
    W = (rng.standard_normal((N_ROWS, K_COLS)) * 0.02).astype(np.float32)
    x = rng.standard_normal(K_COLS).astype(np.float32)
    Wq = O.ref_quantize("q4_0", W)
    copies = max(2, -(-2 * llc_bytes() // W_BYTES))
    ws = [Wq] + [Wq.copy() for _ in range(copies - 1)]
    y = np.empty(N_ROWS, np.float32)
    state = {"i": 0}

    def call():
        state["i"] = (state["i"] + 1) % copies
        R.smkref_gemv_q4_0(-1, N_ROWS, K_COLS, x.ctypes.data, ws[state["i"]].ctypes.data, y.ctypes.data)

    return call, copies, R.smkref_q8_0_path().decode()


def cpu_threads() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count() or 1


def time_reference(steps: int | None, warmup: int, budget_s: float):
    """GB/s of the reference's gemv_q4_0 on the config-0 workload, every host thread."""
    th = cpu_threads()
    setup = reference_setup(th)
    if setup is None:
        return None
    call, copies, path = setup
    for _ in range(max(warmup, 1)):
        call()
    t0 = time.perf_counter()
    n = 0
    while (steps is not None and n < steps) or (steps is None and time.perf_counter() - t0 < budget_s):
        call()
        n += 1
    dt = time.perf_counter() - t0
    return {"value": STEP_BYTES * n / dt / 1e9, "unit": "GB/s", "cores": th, "kind": "reference", "calls": n,
            "seconds": dt, "sample": f"{n} gemv_q4_0 calls, N=8192 K=2048, {copies} weight copies rotated "
                                   f"past the host LLC, path {path}, {th} threads"}


# ---- the GPU arm ---------------------------------------------------------------------------

def gpu_bench(args, rank: int, world: int, local_rank: int) -> dict | None:
    import torch
    import torch.distributed as dist

    import simd_ml_kernels as sk
    from simd_ml_kernels import shard

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    sk.set_pdl(True, local_rank)
    props = torch.cuda.get_device_properties(dev)
    l2 = getattr(props, "L2_cache_size", 126 << 20)

    # Weights: this rank's 8192 rows of the [8192*world, 2048] matrix (seed 0 for rank 0).
    g = torch.Generator(device=dev)
    g.manual_seed(0 + rank)
    W = torch.randn((N_ROWS, K_COLS), generator=g, device=dev) * 0.02
    Wq0 = sk.quantize_q4_0(W).reshape(-1)
    del W
    copies = max(2, -(-2 * l2 // W_BYTES) + 1)
    ws = [Wq0] + [Wq0.clone() for _ in range(copies - 1)]
    x = torch.randn(K_COLS, generator=g, device=dev)
    y = torch.empty(N_ROWS, device=dev)
    Ntot = N_ROWS * world
    nvlink = world > 1 and args.gather == "nvlink"
    gathered = torch.empty((world, N_ROWS), device=dev) if world > 1 and not nvlink else None
    sg = shard.ShardedGemv("q4_0", Wq0, Ntot, K_COLS, gather="nvlink") if nvlink else None

    stream = torch.cuda.Stream(device=dev)
    launches_per_step = 2 if nvlink else 1
    from simd_ml_kernels import _core

    def one_step(i):
        if nvlink:   # GEMV storing its slice into every rank's y over NVLink, then the peers' signals
            _core._gemv_q_gather(sg._g, 0, 1, N_ROWS, K_COLS, x.data_ptr(), K_COLS, ws[i % copies].data_ptr(),
                                 stream.cuda_stream, local_rank)
            return
        sk.gemv_q4_0(x, ws[i % copies], N_ROWS, K_COLS, out=y)
        if world > 1:
            dist.all_gather_into_tensor(gathered, y)

    # CUDA graphs of `chunk` steps, cycling through the weight copies.
    chunk = copies * max(1, 512 // copies)
    steps = args.steps
    full, rem = divmod(steps, chunk)

    def capture(n):
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            one_step(0)   # warm the path (first-use allocations) outside capture
            torch.cuda.synchronize(dev)
            with torch.cuda.graph(gr, stream=stream):
                for i in range(n):
                    one_step(i)
        return gr

    g_full = capture(chunk) if full else None
    g_rem = capture(rem) if rem else None
    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            one_step(i)
    torch.cuda.synchronize(dev)

    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    with ClockSampler(local_rank) as clocks:
        with torch.cuda.stream(stream):
            start.record(stream)
            for _ in range(full):
                g_full.replay()
            if g_rem is not None:
                g_rem.replay()
            end.record(stream)
        torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    ms = start.elapsed_time(end)
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    # Kernel-only time per launch (no all-gather), for the roofline: the
    # same graphs without the collective, on this rank.
    kernel_ms = ms
    if world > 1:
        gk = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            with torch.cuda.graph(gk, stream=stream):
                for i in range(chunk):
                    sk.gemv_q4_0(x, ws[i % copies], N_ROWS, K_COLS, out=y)
            s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s2.record(stream)
            reps = max(1, steps // chunk)
            for _ in range(reps):
                gk.replay()
            e2.record(stream)
        torch.cuda.synchronize(dev)
        kernel_ms = s2.elapsed_time(e2) * steps / (reps * chunk)
        del gk
    del g_full, g_rem

    if args.only_gemv:
        if rank == 0:
            out = {"metric": METRIC, "value": round(STEP_BYTES * world * steps / (ms_max * 1e-3) / 1e9, 2),
                   "unit": "GB/s", "n_gpus": world, "steps": steps, "ms_per_step": ms_max / steps,
                   "only_gemv": True}
            if args.case and world == 1:
                out["configs"] = other_configs(sk, torch, dev, stream, args.case)
            return out
        return None

    # End to end through the public API: x from pinned host memory, y back to
    # host memory, weights resident on the device (uploaded once, as a model's).
    e2e_steps = min(max(steps // 10, 200), 2000)
    xh = torch.randn(K_COLS, generator=torch.Generator().manual_seed(1)).pin_memory()
    xh_np = xh.numpy()
    sk.set_pdl(False, local_rank)
    if world == 1:
        for _ in range(20):
            sk.gemv_q4_0(xh_np, ws[0], N_ROWS, K_COLS)
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        for i in range(e2e_steps):
            yh = sk.gemv_q4_0(xh_np, ws[i % copies], N_ROWS, K_COLS)
        e2e_s = time.perf_counter() - t0
        assert yh.shape == (N_ROWS,)
        e2e_bytes_out = 4 * N_ROWS
    else:
        if sg is None:
            sg = shard.ShardedGemv("q4_0", ws[0], Ntot, K_COLS)
        yfull_h = torch.empty(Ntot).pin_memory()
        for _ in range(20):
            yfull_h.copy_(sg.forward(xh.to(dev, non_blocking=True)))
        torch.cuda.synchronize(dev)
        dist.barrier()
        t0 = time.perf_counter()
        for i in range(e2e_steps):
            yfull_h.copy_(sg.forward(xh.to(dev, non_blocking=True)))
        torch.cuda.synchronize(dev)
        e2e_s = time.perf_counter() - t0
        tt = torch.tensor([e2e_s], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e2e_s = float(tt.item())
        e2e_bytes_out = 4 * Ntot
    sk.set_pdl(True, local_rank)
    if sg is not None:
        sg.close()   # release the gather buffers before the process group goes

    extra = {}
    if not args.only_gemv:
        sharded = sharded_configs(sk, torch, dev, stream, world, rank, local_rank)
        if rank == 0:
            extra["sharded_config4"] = sharded
    if rank == 0 and world == 1:
        extra["llama_stack"] = llama_stack(sk, torch, dev, stream, args)
        extra["llama_decode_swiglu"] = llama_stack(sk, torch, dev, stream, args, swiglu="fused")
        extra["llama_decode_swiglu_unfused"] = llama_stack(sk, torch, dev, stream, args, swiglu="unfused")
        if args.all or args.case:
            extra["configs"] = other_configs(sk, torch, dev, stream, args.case)

    if rank != 0:
        return None
    peaks = measured_peaks()
    achieved = STEP_BYTES / (kernel_ms / steps * 1e-3) / 1e9
    value = STEP_BYTES * world * steps / (ms_max * 1e-3) / 1e9
    out = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": steps,
        "warmup": args.warmup, "ms_per_step": ms_max / steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "q4_0 weights x int8 activations (dp4a int32, fp32 accumulate)",
        "data": "synthetic: W ~ N(0, 0.02) seed 0 quantized ggml Q4_0 on device, x ~ N(0, 1)",
        "config": {"workload": "config 0: Q4_0 decode GEMV M=1 K=2048 N=8192 per GPU"
                               + ((f", rows sharded over {world} GPUs, all-gather of y fused into the GEMV "
                                   "(stores into every rank's y over NVLink, then a wait on the peers' signals)"
                                   if nvlink else f", rows sharded over {world} GPUs + NCCL all-gather of y")
                                  if world > 1 else ""),
                   "M": 1, "K": K_COLS, "N_per_gpu": N_ROWS, "N_total": Ntot,
                   "bytes_per_step_per_gpu": STEP_BYTES,
                   "l2_policy": f"{copies} rotated weight copies ({copies * W_BYTES / 2**20:.0f} MiB > 2x L2 "
                                f"{l2 / 2**20:.0f} MiB): inputs larger than L2",
                   "launch": f"CUDA graphs of {chunk} steps, programmatic dependent launch"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / peaks["hbm_gbs"], 4),
                     "traffic": committed_traffic("gemv_q4_0_cfg0_traffic.json"),
                     "peak_source": peaks["source"] + " (MEASURED_PEAKS.json hbm_gbs, burst copy)",
                     "kernel": "gemv_q_fast2<Q4_0, M=1>", "algorithmic_bytes_per_launch": STEP_BYTES},
        "e2e": {"value": round(STEP_BYTES * world * e2e_steps / e2e_s / 1e9, 2), "unit": "GB/s",
                "h2d_bytes_per_step": 4 * K_COLS, "d2h_bytes_per_step": e2e_bytes_out,
                "us_per_step": e2e_s / e2e_steps * 1e6, "steps": e2e_steps,
                "api": "simd_ml_kernels.gemv_q4_0(numpy x in pinned memory, device weights) -> numpy y"
                       if world == 1 else "ShardedGemv.forward(x host->device) + y device->host"},
        "gpu_launches": steps * launches_per_step,
        "clocks": clocks.summary(),
    }
    if world > 1:
        out["kernel_only_ms_per_step"] = kernel_ms / steps
    out.update(extra)
    return out


def llama_stack(sk, torch, dev, stream, args, swiglu: str = "") -> dict:
    """a Llama-3.2-1B decode step's GEMVs — 16 layers of
    q 2048->2048, k, v 2048->512, o 2048->2048, gate, up 2048->8192, down
    8192->2048, and the tied 2048->128256 LM head — on random-init Q4_0 weights
    (seed 2), fresh activations every step, --llama-tokens (128) steps in one
    CUDA graph.
    q, k and v read the same activation row within a step, as do gate and up,
    so each group runs as one GEMV over its concatenated rows (the same bytes
    and outputs as the separate GEMVs): 4 GEMVs per layer + the LM head.
    swiglu "fused": the down projection reads silu(gate) * up of the layer's
    gate/up GEMV instead of fresh activations, as the decoder does, with the
    SwiGLU product formed inside it (more work than the GEMV-only stack);
    "unfused": the same step with silu_mul as its own kernel before a plain
    down-projection GEMV."""
    g = torch.Generator(device=dev)
    g.manual_seed(2)
    groups = []   # (rows N, K, logical GEMVs)
    for _ in range(LLAMA_LAYERS):
        groups += [(2048 + 512 + 512, 2048, 3), (2048, 2048, 1), (8192 + 8192, 2048, 2), (2048, 8192, 1)]
    groups.append((LLAMA_VOCAB, 2048, 1))
    weights = []
    wbytes = 0
    for n, k, _ in groups:
        wq = torch.empty((n, k // 32 * 18), dtype=torch.uint8, device=dev)
        for r0 in range(0, n, 16384):
            r1 = min(n, r0 + 16384)
            sk.quantize_q4_0(torch.randn((r1 - r0, k), generator=g, device=dev) * 0.02, out=wq[r0:r1])
        weights.append(wq.reshape(-1))
        wbytes += wq.numel()
    xs_per_tok = sum(k for _, k, _ in groups)
    ys_per_tok = sum(n for n, _, _ in groups)
    tokens = args.llama_tokens
    X = torch.randn((tokens, xs_per_tok), generator=g, device=dev)
    Y = torch.empty((ys_per_tok,), device=dev)
    act = torch.empty((8192,), device=dev)
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(gr, stream=stream):
            for t in range(tokens):
                xo = yo = 0
                gate_up = None
                for (n, k, _), wq in zip(groups, weights):
                    if swiglu and gate_up is not None and n == 2048 and k == 8192:
                        # The down projection takes silu(gate) * up of the gate/up GEMV just
                        # before it, formed while its activations are quantized.
                        if swiglu == "fused":
                            sk.gemv_q4_0_silu_mul(gate_up[:8192], gate_up[8192:], wq, n, k, out=Y[yo:yo + n])
                        else:
                            sk.silu_mul(gate_up[:8192], gate_up[8192:], out=act)
                            sk.gemv_q4_0(act, wq, n, k, out=Y[yo:yo + n])
                        gate_up = None
                    else:
                        sk.gemv_q4_0(X[t, xo:xo + k], wq, n, k, out=Y[yo:yo + n])
                        if n == 16384:
                            gate_up = Y[yo:yo + n]
                    xo += k
                    yo += n
        for _ in range(3):
            gr.replay()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        gr.replay()
        e.record(stream)
    torch.cuda.synchronize(dev)
    ms = s.elapsed_time(e)
    per_tok_ms = ms / tokens
    # Algorithmic bytes of the 113 separate GEMVs: weights, x of each, y of each.
    logical_x = sum(k * c for _, k, c in groups)
    tok_bytes = wbytes + 4 * (logical_x + ys_per_tok)
    del gr
    return {"tok_s": round(1e3 / per_tok_ms, 1), "ms_per_token": per_tok_ms,
            "gemvs_per_token": sum(c for _, _, c in groups),
            "launches_per_token": len(groups) + (LLAMA_LAYERS if swiglu == "unfused" else 0),
            "bytes_per_token": tok_bytes, "gb_s": round(tok_bytes / (per_tok_ms * 1e-3) / 1e9, 1),
            "tokens": tokens,
            "launch": f"one CUDA graph of {tokens} decode steps, PDL; q/k/v and gate/up as fused row groups"
                      + {"": "", "fused": "; down projection fed by silu(gate)*up inside its activation quantization",
                         "unfused": "; silu(gate)*up as a separate kernel before the down projection"}[swiglu]}


SHARDED_SHAPES = [(28672, 8192), (8192, 28672), (128256, 8192)]   # config 4: 70B layers, LM head


def sharded_configs(sk, torch, dev, stream, world: int, rank: int, local_rank: int) -> dict:
    """Config 4 (Q4_0, M = 1, W ~ N(0, 0.015) from seed 4) split by rows over
    the ranks: each step is this rank's GEMV plus the all-gather of y fused
    into it (world > 1), timed in CUDA graphs as the max over ranks; aggregate
    GB/s = the whole matrix's algorithmic bytes per step time (strong scaling).
    Every rank calls this with the same shapes (collectives inside)."""
    import torch.distributed as dist
    from simd_ml_kernels import _core, shard
    res = {}
    l2 = getattr(torch.cuda.get_device_properties(dev), "L2_cache_size", 126 << 20)
    for N, K in SHARDED_SHAPES:
        lo, hi = shard.row_slice(N, rank, world)
        n, rb = hi - lo, K // 32 * 18
        g = torch.Generator(device=dev)
        g.manual_seed(4 * 1000 + rank)
        wq = torch.empty(n * rb, dtype=torch.uint8, device=dev)
        for r0 in range(0, n, 8192):
            rows = min(8192, n - r0)
            wq[r0 * rb:(r0 + rows) * rb] = sk.quantize_q4_0(
                torch.randn((rows, K), generator=g, device=dev) * 0.015).reshape(-1)
        copies = max(2, -(-2 * l2 // (n * rb)) + 1)
        ws = [wq] + [wq.clone() for _ in range(copies - 1)]
        x = torch.randn(K, generator=g, device=dev)
        y = torch.empty(n, device=dev)
        sg = shard.ShardedGemv("q4_0", wq, N, K, gather="nvlink") if world > 1 else None

        def step(i):
            if sg is not None:
                _core._gemv_q_gather(sg._g, 0, 1, n, K, x.data_ptr(), K, ws[i % copies].data_ptr(),
                                     stream.cuda_stream, local_rank)
            else:
                sk.gemv_q4_0(x, ws[i % copies], n, K, out=y)

        reps = copies * max(1, 64 // copies)
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            step(0)
            torch.cuda.synchronize(dev)
            with torch.cuda.graph(gr, stream=stream):
                for i in range(reps):
                    step(i)
            gr.replay()
            torch.cuda.synchronize(dev)
            if world > 1:
                dist.barrier()
            s0, e0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record(stream)
            for _ in range(5):
                gr.replay()
            e0.record(stream)
        torch.cuda.synchronize(dev)
        t = torch.tensor([s0.elapsed_time(e0) * 1e3 / (5 * reps)], device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        us = float(t.item())
        del gr
        if sg is not None:
            sg.close()
        nbytes = N * K // 32 * 18 + 4 * K + 4 * N
        res[f"q4_0 M=1 N={N} K={K} over {world} GPU(s)"] = {
            "us_per_step": round(us, 3), "gb_s_aggregate": round(nbytes / (us * 1e-6) / 1e9, 1),
            "rows_per_gpu": n, "gather": "fused NVLink" if world > 1 else None}
        del ws, wq
    return res


def other_configs(sk, torch, dev, stream, only: str | None = None) -> dict:
    """Configs 1 (Q8_0), 3 (dense fp32/bf16/fp16, M in 1,4,8) and 4 (large Q4_0, M 1/8) on one GPU;
    `only`: time just the cases whose label contains it (for profilers)."""
    res = {}
    l2 = getattr(torch.cuda.get_device_properties(dev), "L2_cache_size", 126 << 20)

    def timeit(fn, nbytes, reps=200):
        copies_needed = max(2, -(-2 * l2 // max(1, nbytes)) + 1)
        return copies_needed, fn, reps

    def run(label, make_w, call, nbytes):
        if only is not None and only not in label:
            return
        copies = max(2, -(-2 * l2 // nbytes) + 1)
        ws = [make_w()] + []
        for _ in range(copies - 1):
            ws.append(ws[0].clone())
        gr = torch.cuda.CUDAGraph()
        reps = copies * max(1, 64 // copies)
        with torch.cuda.stream(stream):
            call(ws[0])
            torch.cuda.synchronize(dev)
            with torch.cuda.graph(gr, stream=stream):
                for i in range(reps):
                    call(ws[i % copies])
            gr.replay()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(stream)
            for _ in range(5):
                gr.replay()
            e.record(stream)
        torch.cuda.synchronize(dev)
        us = s.elapsed_time(e) * 1e3 / (5 * reps)
        res[label] = {"us": round(us, 3), "gb_s": round(nbytes / (us * 1e-6) / 1e9, 1)}
        del gr, ws

    g = torch.Generator(device=dev)
    g.manual_seed(1)
    for n, k in ((512, 2048), (2048, 2048), (8192, 2048), (2048, 8192)):
        x = torch.randn(k, generator=g, device=dev)
        y = torch.empty(n, device=dev)
        nb = n * k // 32 * 34
        run(f"q8_0 N={n} K={k}", lambda: sk.quantize_q8_0(torch.randn((n, k), generator=g, device=dev) * 0.02).reshape(-1),
            lambda w: sk.gemv_q8_0(x, w, n, k, out=y), nb + 4 * k + 4 * n)
    g.manual_seed(3)
    for wt in (torch.float32, torch.bfloat16, torch.float16):
        for m in (1, 4, 8):
            for n in (4096, 14336):
                k = 4096
                x = torch.randn((m, k), generator=g, device=dev)
                y = torch.empty((m, n), device=dev)
                es = 4 if wt == torch.float32 else 2
                run(f"dense {str(wt).split('.')[-1]} M={m} N={n} K={k}",
                    lambda: (torch.randn((n, k), generator=g, device=dev) * 0.02).to(wt),
                    lambda w: sk.gemv_dense(x, w, out=y), n * k * es + 4 * m * k + 4 * m * n)
    g.manual_seed(5)
    for m in (1, 4, 8):   # INT8 sgemm_u8s8 with trans_b: uint8 A, int8 W [N, K], per-row scales
        for n in (4096, 14336):
            k = 4096
            a = torch.randint(0, 256, (m, k), generator=g, device=dev, dtype=torch.uint8)
            sc = torch.rand(n, generator=g, device=dev) * 0.01
            y = torch.empty((m, n), device=dev)
            run(f"u8s8 M={m} N={n} K={k}",
                lambda n=n, k=k: torch.randint(-128, 128, (n, k), generator=g, device=dev, dtype=torch.int8),
                lambda w, a=a, sc=sc, y=y: sk.sgemm_u8s8(a, w, 0.02, 128, sc, y, trans_b=True),
                n * k + m * k + 4 * n + 4 * m * n)
    g.manual_seed(4)
    for n, k in ((28672, 8192), (8192, 28672), (128256, 8192)):
        for m in (1, 8):
            x = torch.randn((m, k), generator=g, device=dev)
            y = torch.empty((m, n), device=dev)
            nb = n * k // 32 * 18

            def mk(n=n, k=k):
                wq = torch.empty((n, k // 32 * 18), dtype=torch.uint8, device=dev)
                for r0 in range(0, n, 8192):
                    r1 = min(n, r0 + 8192)
                    sk.quantize_q4_0(torch.randn((r1 - r0, k), generator=g, device=dev) * 0.015, out=wq[r0:r1])
                return wq.reshape(-1)
            run(f"q4_0 M={m} N={n} K={k}", mk, lambda w, x=x, y=y, n=n, k=k: sk.gemv_q4_0_batch(x, w, n, k, out=y),
                nb + 4 * m * (k + n))
    return res


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100000)
    ap.add_argument("--warmup", type=int, default=2000)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--all", action="store_true", help="also time configs 1, 3 and 4 (one GPU)")
    ap.add_argument("--cpu-baseline-seconds", type=float, default=8.0)
    ap.add_argument("--gather", choices=["nvlink", "nccl"], default="nvlink",
                    help="N > 1: all-gather of y fused into the GEMV over NVLink, or NCCL's all-gather")
    ap.add_argument("--case", default=None,
                    help="time only the config 1/3/4 cases whose label contains this text (after the config-0 line)")
    ap.add_argument("--llama-tokens", type=int, default=LLAMA_TOKENS,
                    help="decode steps per Llama-stack CUDA graph (fewer: shorter profiler launch lists)")
    ap.add_argument("--only-gemv", action="store_true",
                    help="time the config-0 GEMV only (no e2e, Llama stack or CPU baseline): for profilers")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank != 0:
            return
        r = time_reference(args.steps, args.warmup, 0.0)
        if r is None:
            print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libsmk_ref.so was not built"}))
            return
        print(json.dumps({"impl": "reference", "metric": METRIC, "value": round(r["value"], 3), "unit": "GB/s",
                          "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                          "ms_per_step": r["seconds"] / r["calls"] * 1e3, "higher_is_better": True,
                          "scaling": "weak", "vs_baseline": None, "dtype": "q4_0 x int8 (vpdpbusd), fp32 accumulate",
                          "data": "synthetic: W ~ N(0, 0.02) seed 0 quantized ggml Q4_0, x ~ N(0, 1)",
                          "config": {"workload": "config 0: Q4_0 decode GEMV M=1 K=2048 N=8192", "M": 1,
                                     "K": K_COLS, "N": N_ROWS},
                          "cpu_baseline": {"value": round(r["value"], 3), "unit": "GB/s", "cores": r["cores"],
                                           "kind": "reference", "sample": r["sample"]},
                          "e2e": {"value": round(r["value"], 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                                  "d2h_bytes_per_step": 0}}))
        return

    import torch
    import torch.distributed as dist
    from datetime import timedelta

    if world > 1:
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local_rank))
    try:
        out = gpu_bench(args, rank, world, local_rank)
        if rank == 0 and out is not None:
            if world == 1 and not args.only_gemv:
                cb = time_reference(None, 2, args.cpu_baseline_seconds)
                out["cpu_baseline"] = None if cb is None else {
                    "value": round(cb["value"], 3), "unit": "GB/s", "cores": cb["cores"], "kind": "reference",
                    "sample": cb["sample"] + f", {cb['seconds']:.1f} s"}
            print(json.dumps(out))
    finally:
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
