"""bench.py — decode-GEMV throughput on B200.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline workload: Q4_0 decode GEMV y = x @ W.T, M = 1,
K = 2048, N = 8192 per GPU; W ~ N(0, 0.02) drawn by numpy's default_rng(0)
in 8192-row chunks (then x ~ N(0, 1) from the same generator), quantized
ggml-style on the device (byte-identical to the reference's quantize_q4_0).
A step is one GEMV over the whole matrix. value = algorithmic bytes (W + x +
y per step, the reference's convention, _cli.py:1198) of all steps of all
ranks / max-over-ranks device time of exactly K steps.

Timing. The steps are CUDA-graph launches chained with programmatic dependent
launch; consecutive steps read different weight copies, together more than
2x the L2 cache, so every step streams its weights from HBM. The start and
end events are recorded inside the graphs (the start one on a forked stream,
after a full rotation of untimed steps), so the K timed steps are the steady
state of a decode chain and no graph-launch latency falls inside them.

The same line carries every BASELINE config on one GPU (config 1 Q8_0,
config 2 Llama-3.2-1B GEMV stack, config 3 dense, config 4 large Q4_0 at
M = 1 and 8), each with its roofline fraction and the reference's CPU
kernel timed on this host with all threads and with one pinned thread.

N > 1 (torchrun): weak scaling for the headline. Every rank runs config-0
steps on its own 8192-row slice of a [8192*N, 2048] matrix, with no
collective: the north star row-shards only config 4's large matrices. Timed
after it, in the same line (`config0_row_sharded`), the same slices as one
row-sharded GEMV whose y is all-gathered over NVLink inside the GEMV every
step; and config 4 split by rows over the ranks (strong scaling, the
reference's row slicing) with the gather.

--impl reference: the reference's own CPU kernel (Mattral/simd-ml-kernels
compiled from its sources, oracle/_ref) on the same workload and config with
every host thread, rank 0 only; a step is one rotation over its weight copies.

The workload generators (Workload, LLAMA_MATRICES, ...) are shared with the
parity tests, which pin the quantized bytes by SHA-256.

One JSON line on rank 0.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import json
import os
import queue
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
ROW_CHUNK = 8192
BLOCK_BYTES = {"q4_0": 18, "q8_0": 34}

# ---- the BASELINE workloads ------------------------------------------------------------

CFG1_SHAPES = [(512, 2048), (2048, 2048), (8192, 2048), (2048, 8192)]     # (N, K), Q8_0, seed 1
CFG3_SHAPES = [(4096, 4096), (14336, 4096)]                               # (N, K), dense, seed 3
CFG3_ROWS = (1, 4, 8)
CFG4_SHAPES = [(28672, 8192), (8192, 28672), (128256, 8192)]              # (N, K), Q4_0, seed 4
CFG4_ROWS = (1, 8)
# Llama-3.2-1B: per layer q, k, v, o, gate, up, down (N, K), then the tied LM head.
LLAMA_LAYER = [(2048, 2048), (512, 2048), (512, 2048), (2048, 2048), (8192, 2048), (8192, 2048), (2048, 8192)]
LLAMA_LAYERS, LLAMA_VOCAB, LLAMA_TOKENS = 16, 128256, 128
LLAMA_MATRICES = LLAMA_LAYER * LLAMA_LAYERS + [(LLAMA_VOCAB, 2048)]       # 113 GEMVs per token


class Workload:
    """W ~ N(0, sigma) [N, K] and then x ~ N(0, 1) [M, K], both from one numpy
    generator: W in 8192-row chunks (float64 normals times sigma, rounded to
    float32), the order of the reference's bench (_cli.py:948-966), so a
    128256-row matrix is never held whole in float32. `entropy` is the seed (an
    int) or a sequence of ints for numpy's SeedSequence. x exists only after
    every chunk has been drawn."""

    def __init__(self, entropy, N: int, K: int, sigma: float, M: int = 1):
        self.entropy, self.N, self.K, self.sigma, self.M = entropy, N, K, sigma, M
        self.x = None

    def chunks(self):
        rng = np.random.default_rng(self.entropy)
        for r0 in range(0, self.N, ROW_CHUNK):
            rows = min(ROW_CHUNK, self.N - r0)
            yield r0, (rng.standard_normal((rows, self.K)) * self.sigma).astype(np.float32)
        self.x = rng.standard_normal((self.M, self.K)).astype(np.float32)

    def full(self):
        """(W [N, K] float32, x [M, K] float32)."""
        W = np.concatenate([c for _, c in self.chunks()]) if self.N else np.empty((0, self.K), np.float32)
        return W, self.x


def config0(world: int = 1) -> Workload:
    """Config 0; for N GPUs the [8192*N, 2048] matrix whose first 8192 rows are config 0's."""
    return Workload(0, N_ROWS * world, K_COLS, 0.02)


def config1(N: int, K: int) -> Workload:
    return Workload(1, N, K, 0.02)


def config3(N: int, K: int) -> Workload:
    return Workload(3, N, K, 0.02, M=max(CFG3_ROWS))


def config4(N: int, K: int) -> Workload:
    return Workload(4, N, K, 0.015, M=max(CFG4_ROWS))


def config2(i: int) -> Workload:
    """Matrix i of the Llama stack (LLAMA_MATRICES order), its own generator
    seeded (2, i) so the 113 matrices can be drawn in parallel."""
    N, K = LLAMA_MATRICES[i]
    return Workload([2, i], N, K, 0.02, M=0)


def q_bytes(fmt: str, N: int, K: int) -> int:
    return N * (K // 32) * BLOCK_BYTES[fmt]


def gemv_bytes(wbytes: int, M: int, N: int, K: int, xsize: int = 4) -> int:
    """Algorithmic bytes of one call: W + x + y, each once (_cli.py:1198)."""
    return wbytes + xsize * M * K + 4 * M * N


# ---- host-side helpers -------------------------------------------------------------------

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


def quantiles(ts: list[float]) -> dict:
    q = statistics.quantiles(ts, n=4) if len(ts) >= 4 else [min(ts), statistics.median(ts), max(ts)]
    return {"p25": q[0], "median": statistics.median(ts), "p75": q[2], "mean": sum(ts) / len(ts)}


class ClockSampler:
    """SM clock and throttle reasons through NVML, sampled while the GPU is under load."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
               "sw_power_cap": 0x4, "hw_power_brake_slowdown": 0x80}

    def __init__(self, device: int, period_s: float = 0.005):
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


def cpu_threads() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count() or 1


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


# ---- the reference's CPU kernels ----------------------------------------------------------

class RefCPU:
    """The reference library compiled from its sources (oracle/_ref), timed on
    this host: all host threads, or one thread pinned to one core. Each case
    rotates weight copies past the host's last-level caches (the reference's
    _Rotor rule, _cli.py:569-581) and is warmed over at least one rotation
    before it is timed."""

    def __init__(self):
        sys.path.insert(0, os.path.join(REPO, "oracle"))
        import oracle as O
        self.O = O
        self.ok = O.ref_available()
        if self.ok:
            self.R = O.ref()
            self.path = self.R.smkref_q8_0_path().decode()
        self.threads = cpu_threads()
        self.llc = llc_bytes()

    def copies(self, nbytes: int) -> int:
        return max(2, -(-2 * self.llc // max(1, nbytes)))

    def time(self, calls, nbytes_per_call: int, seconds: float, threads: int | None = None,
             pin: bool = False) -> dict:
        """calls: one callable per weight copy (a rotation). GB/s from the median call."""
        R = self.R
        th = threads or self.threads
        old = os.sched_getaffinity(0) if pin else None
        try:
            if pin:
                os.sched_setaffinity(0, {min(old)})
            R.smkref_set_num_threads(th)
            n = len(calls)
            t0 = time.perf_counter()
            i = 0
            while i < n or time.perf_counter() - t0 < min(0.2, seconds / 3):   # warm: >= one rotation
                calls[i % n]()
                i += 1
            ts = []
            t0 = time.perf_counter()
            while len(ts) < max(n, 3) or time.perf_counter() - t0 < seconds:
                a = time.perf_counter()
                calls[len(ts) % n]()
                ts.append(time.perf_counter() - a)
        finally:
            if pin:
                os.sched_setaffinity(0, old)
        q = quantiles(ts)
        return {"gb_s": round(nbytes_per_call / q["median"] / 1e9, 3), "us_median": round(q["median"] * 1e6, 3),
                "us_p25": round(q["p25"] * 1e6, 3), "us_p75": round(q["p75"] * 1e6, 3), "calls": len(ts),
                "threads": 1 if pin else th, "pinned": pin, "weight_copies": n}

    def both(self, calls, nbytes: int, seconds: float = 0.3) -> dict:
        return {"all_threads": self.time(calls, nbytes, seconds), "one_thread": self.time(calls, nbytes, seconds,
                                                                                           threads=1, pin=True)}

    # Calls of the reference's table entries on host arrays.
    def gemv_q(self, fmt, ws, x, N, K):
        fn = self.R.smkref_gemv_q4_0 if fmt == "q4_0" else self.R.smkref_gemv_q8_0
        X = np.ascontiguousarray(x, np.float32).reshape(-1, K)
        y = np.empty((X.shape[0], N), np.float32)

        def mk(w):
            def call():   # the reference has no batched quantized GEMV: one call per row of x
                for m in range(X.shape[0]):
                    fn(-1, N, K, X[m].ctypes.data, w.ctypes.data, y[m].ctypes.data)
            return call
        return [mk(w) for w in ws]

    def dense(self, kind, ws, X, N, K):
        M = X.shape[0]
        C = np.empty((M, N), np.float32)
        if kind == "float32":
            A = np.ascontiguousarray(X, np.float32)
            fn = self.R.smkref_sgemm_tb
        else:   # the reference's 16-bit GEMV takes x in the same 16-bit type (_cli.py:1189-1194)
            import torch
            t = torch.from_numpy(np.ascontiguousarray(X)).to(getattr(torch, kind))
            A = t.view(torch.int16).numpy().view(np.uint16)
            fn = self.R.smkref_sgemm_f16_tb if kind == "float16" else self.R.smkref_sgemm_bf16_tb
        return [lambda w=w: fn(-1, M, N, K, 1.0, A.ctypes.data, w.ctypes.data, 0.0, C.ctypes.data) for w in ws]


def time_reference_arm(steps: int, warmup: int, world: int) -> dict | None:
    """The reference's gemv_q4_0 on the headline workload (the GPU arm's config at
    this world size), every host thread. A step is a bounded sample: whole
    rotations over the weight copies, as many as take about 20 ms; exactly
    `steps` steps are timed after `warmup` untimed ones and at least half a
    second of untimed calls (the thread team and the core clocks settle)."""
    ref = RefCPU()
    if not ref.ok:
        return None
    wl = config0(world)
    W, x = wl.full()
    Wq = ref.O.ref_quantize("q4_0", W)
    del W
    N = wl.N
    wb = q_bytes("q4_0", N, K_COLS)
    copies = ref.copies(wb)
    ws = [Wq] + [Wq.copy() for _ in range(copies - 1)]
    calls = ref.gemv_q("q4_0", ws, x[0], N, K_COLS)
    ref.R.smkref_set_num_threads(ref.threads)
    t0 = time.perf_counter()
    rot = 0
    while rot < 1 or time.perf_counter() - t0 < 0.5:
        for c in calls:
            c()
        rot += 1
    rots = max(1, round(0.02 / ((time.perf_counter() - t0) / rot)))   # rotations per step
    for _ in range(warmup * rots):
        for c in calls:
            c()
    t0 = time.perf_counter()
    for _ in range(steps * rots):
        for c in calls:
            c()
    dt = time.perf_counter() - t0
    per_call = STEP_BYTES * world
    n = steps * rots * copies
    return {"value": per_call * n / dt / 1e9, "seconds": dt, "calls": n,
            "ms_per_step": dt / steps * 1e3, "cores": ref.threads, "path": ref.path, "copies": copies,
            "sample": f"{steps} steps of {rots * copies} gemv_q4_0 calls ({rots} rotations over {copies} weight "
                      f"copies, past the host LLC of {ref.llc >> 20} MiB), N={N} K={K_COLS}, path {ref.path}, "
                      f"{ref.threads} threads, {cpu_model()}"}


def headline_config(world: int) -> dict:
    """The `config` of the headline line, identical in both arms."""
    return {"workload": "config 0: Q4_0 decode GEMV M=1 K=2048 N=8192" +
                        (f" on each of {world} GPUs, independent steps, no collective (rank r: rows "
                         f"8192r..8192r+8191 of the seed-0 [{N_ROWS * world}, 2048] matrix)" if world > 1 else ""),
            "M": 1, "K": K_COLS, "N": N_ROWS, "gpus": world, "seed": 0, "weights": "N(0, 0.02) -> ggml Q4_0",
            "bytes_per_step": STEP_BYTES * world}


# ---- GPU timing -------------------------------------------------------------------------------

def chained_ms(torch, dev, stream, step, n: int, period: int, pre: int | None = None, chunk: int = 512,
               barrier=None, load_s: float = 0.0, sampler=None) -> float:
    """Device milliseconds of exactly n consecutive calls step(i) on `stream`.

    The calls are captured into CUDA graphs, so consecutive kernels keep their
    programmatic-dependent-launch edges. The first graph runs `pre` untimed
    calls (one rotation of the weight copies by default), then records the
    start event on a forked stream (the next call keeps its edge to the
    previous one), then timed calls; the last graph ends with the end event.
    step(i) must use weight copy i % period; graphs hold multiples of `period`
    calls, so their replays continue the rotation. Every graph is replayed
    once before the timed replays; `load_s` seconds of untimed replays (with
    `sampler` running) precede the timed ones. `barrier` (multi-rank) is
    called with the device synchronised right before and after the timed
    replays; every rank must pass the same n, period and load count."""
    pre = period if pre is None else pre
    chunk = max(period, chunk // period * period)
    side = torch.cuda.Stream(device=dev)
    ev0 = torch.cuda.Event(enable_timing=True, external=True)
    ev1 = torch.cuda.Event(enable_timing=True, external=True)
    first = min(n, chunk)
    rest = n - first
    mids, last = divmod(rest, chunk)
    if last == 0 and mids > 0:
        mids, last = mids - 1, chunk

    def capture(base: int, count: int, start: bool, end: bool, lead: int = 0):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            with torch.cuda.graph(g, stream=stream):
                for i in range(lead):
                    step(i)
                if start:
                    side.wait_stream(stream)
                    ev0.record(side)
                for i in range(count):
                    step(base + i)
                if end:
                    ev1.record(stream)
                if start:
                    stream.wait_stream(side)
        return g

    with torch.cuda.stream(stream):
        step(0)   # first-use set-up (scratch, launch caches) outside any capture
    torch.cuda.synchronize(dev)
    g_first = capture(pre, first, True, last == 0, lead=pre)
    g_mid = capture(pre + first, chunk, False, False) if mids else None
    g_last = capture(pre + first, last, False, True) if last else None
    g_load = g_mid or capture(0, chunk, False, False)
    with torch.cuda.stream(stream):
        for g in (g_first, g_mid, g_last, g_load):
            if g is not None:
                g.replay()
    torch.cuda.synchronize(dev)

    def run_load():
        if load_s <= 0:
            return
        t0 = time.perf_counter()
        with torch.cuda.stream(stream):
            g_load.replay()
        torch.cuda.synchronize(dev)
        one = max(time.perf_counter() - t0, 1e-5)
        reps = int(min(2000, max(1, load_s / one)))
        if barrier is not None:   # the same count on every rank
            t = torch.tensor([reps], device=dev)
            barrier(t)
            reps = int(t.item())
        with torch.cuda.stream(stream):
            for _ in range(reps):
                g_load.replay()

    outer = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
    if sampler is not None:
        with sampler:
            run_load()
            _timed(torch, dev, stream, g_first, g_mid, mids, g_last, barrier, outer)
    else:
        run_load()
        _timed(torch, dev, stream, g_first, g_mid, mids, g_last, barrier, outer)
    try:
        ms = ev0.elapsed_time(ev1)
    except RuntimeError:   # events recorded by graph nodes not readable: time the replays instead
        ms = outer[0].elapsed_time(outer[1])
        CHAINED_FALLBACKS.append(n)
    del g_first, g_mid, g_last, g_load
    return ms


CHAINED_FALLBACKS: list[int] = []   # chained_ms calls that had to time whole graph replays


def _timed(torch, dev, stream, g_first, g_mid, mids, g_last, barrier, outer):
    torch.cuda.synchronize(dev)
    if barrier is not None:
        barrier(None)
    torch.cuda.synchronize(dev)
    with torch.cuda.stream(stream):
        outer[0].record(stream)
        g_first.replay()
        for _ in range(mids):
            g_mid.replay()
        if g_last is not None:
            g_last.replay()
        outer[1].record(stream)
    torch.cuda.synchronize(dev)
    if barrier is not None:
        barrier(None)


class Producer:
    """Draws Workload chunks on worker threads (numpy releases the GIL while it
    fills arrays), in submission order, at most `ahead` chunks per workload
    waiting. Consume workloads in the order they were submitted."""

    def __init__(self, workers: int = 6, ahead: int = 2):
        self.pool = cf.ThreadPoolExecutor(max_workers=workers)
        self.ahead = ahead

    def submit(self, wl: Workload, lo: int = 0, hi: int | None = None):
        """Rows [lo, hi) of wl's chunks (the whole stream is still drawn, for x)."""
        q = queue.Queue(maxsize=self.ahead)
        hi = wl.N if hi is None else hi

        def run():
            try:
                for r0, c in wl.chunks():
                    r1 = r0 + c.shape[0]
                    if r1 > lo and r0 < hi:
                        q.put((max(r0, lo), c[max(r0, lo) - r0:min(r1, hi) - r0]))
                q.put(None)
            except BaseException as e:  # noqa: BLE001
                q.put(e)
        self.pool.submit(run)
        return wl, q

    def close(self):
        self.pool.shutdown(wait=True)


def device_weights(torch, sk, dev, job, fmt: str | None, dtype=None):
    """The rows a Producer job delivers, on the device: quantized to `fmt` by the
    device quantizer, or rounded (round to nearest even) to `dtype`."""
    wl, q = job
    out = []
    while True:
        item = q.get()
        if item is None:
            break
        if isinstance(item, BaseException):
            raise item
        _, c = item
        t = torch.from_numpy(c).to(dev)
        if fmt == "q4_0":
            out.append(sk.quantize_q4_0(t))
        elif fmt == "q8_0":
            out.append(sk.quantize_q8_0(t))
        else:
            out.append(t.to(dtype))
        del t
    w = torch.cat(out) if len(out) > 1 else out[0]
    return w, wl.x


def roofline(nbytes: int, us: float, peak: dict) -> dict:
    achieved = nbytes / (us * 1e-6) / 1e9
    return {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak["hbm_gbs"], "unit": "GB/s",
            "frac": round(achieved / peak["hbm_gbs"], 4), "of": peak["source"]}


def gpu_bench(args, rank: int, world: int, local_rank: int) -> dict | None:
    import torch
    import torch.distributed as dist

    import simd_ml_kernels as sk
    from simd_ml_kernels import _core, shard

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    sk.set_pdl(True, local_rank)
    props = torch.cuda.get_device_properties(dev)
    l2 = getattr(props, "L2_cache_size", 126 << 20)
    peak = measured_peaks()
    stream = torch.cuda.Stream(device=dev)

    def barrier(t):
        if world > 1:
            if t is None:
                dist.barrier()
            else:
                dist.all_reduce(t, op=dist.ReduceOp.MAX)

    full_run = not args.only_gemv
    prod = Producer()
    # Headline weights first; the other configs' generators run on worker
    # threads while the headline is timed.
    # Jobs are submitted in the order they are consumed below (the producer's
    # bounded queues need that).
    lo, hi = rank * N_ROWS, (rank + 1) * N_ROWS
    j0 = prod.submit(config0(world), lo, hi)
    jobs = {}
    if full_run:
        for N, K in CFG4_SHAPES:
            slo, shi = shard.row_slice(N, rank, world)
            jobs[("c4", N, K)] = prod.submit(config4(N, K), slo, shi)
    if full_run and world == 1:
        for N, K in CFG1_SHAPES:
            jobs[("c1", N, K)] = prod.submit(config1(N, K))
        for N, K in CFG3_SHAPES:
            jobs[("c3", N, K)] = prod.submit(config3(N, K))
        for i in range(len(LLAMA_MATRICES)):
            jobs[("c2", i)] = prod.submit(config2(i))

    Wq0, x0 = device_weights(torch, sk, dev, j0, "q4_0")
    Wq0 = Wq0.reshape(-1)
    copies = max(2, -(-2 * l2 // W_BYTES) + 1)
    ws = [Wq0] + [Wq0.clone() for _ in range(copies - 1)]
    x = torch.from_numpy(x0[0]).to(dev)
    y = torch.empty(N_ROWS, device=dev)
    # N > 1: every GPU runs its own config-0 steps (its slice of the seed-0
    # [8192·N, 2048] matrix; rank 0's rows are config 0's), no collective: the
    # north star row-shards only config 4's large matrices. The same slices as
    # one row-sharded GEMV with y all-gathered are timed after the headline.
    nvlink = world > 1 and args.gather == "nvlink"
    gathered = torch.empty((world, N_ROWS), device=dev) if world > 1 and not nvlink else None
    sg = shard.ShardedGemv("q4_0", Wq0, N_ROWS * world, K_COLS, gather="nvlink") if nvlink else None
    launches_per_step = 1

    def one_step(i):
        sk.gemv_q4_0(x, ws[i % copies], N_ROWS, K_COLS, out=y)

    def sharded_step(i):
        if nvlink:   # GEMV storing its slice into every rank's y over NVLink, then the peers' signals
            _core._gemv_q_gather(sg._g, 0, 1, N_ROWS, K_COLS, x.data_ptr(), K_COLS, ws[i % copies].data_ptr(),
                                 stream.cuda_stream, local_rank)
            return
        sk.gemv_q4_0(x, ws[i % copies], N_ROWS, K_COLS, out=y)
        dist.all_gather_into_tensor(gathered, y)

    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            one_step(i)
            if world > 1:
                sharded_step(i)
    torch.cuda.synchronize(dev)
    signal = None
    if nvlink:   # the fused gather's fixed cost: NVLink flag round trips, and data-free gather steps
        iters = 20000
        ns = _core._gather_pingpong(sg._g, iters, 0, stream.cuda_stream)
        ns_relaxed = _core._gather_pingpong(sg._g, iters, 1, stream.cuda_stream)
        bar_ms = chained_ms(torch, dev, stream, lambda i: _core._gather_barrier(sg._g, stream.cuda_stream), 2000, 1,
                            chunk=500, barrier=barrier)
        t = torch.tensor([bar_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        signal = {"pingpong_round_trip_us": round(ns / (iters - iters // 8) / 1e3, 3) if rank == 0 else None,
                  "pingpong_relaxed_round_trip_us": round(ns_relaxed / (iters - iters // 8) / 1e3, 3)
                  if rank == 0 else None,
                  "gather_barrier_step_us": round(float(t.item()) * 1e3 / 2000, 3),
                  "note": "round trip of a flag between ranks 0 and 1 inside one kernel each; a chain of data-free "
                          "gather steps (signal every peer, wait for every peer), one launch per step"}
    clocks = ClockSampler(local_rank)
    steps = args.steps
    ms = chained_ms(torch, dev, stream, one_step, steps, copies, barrier=barrier if world > 1 else None,
                    load_s=0.3, sampler=clocks)
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    kernel_ms = ms   # this rank's GEMV alone, for the roofline
    # Ranks that ran the timed steps, each on its own GPU (a sum over the group).
    active = torch.tensor([1.0], device=dev)
    if world > 1:
        dist.all_reduce(active)
    gpus_active = int(active.item())
    value = STEP_BYTES * world * steps / (ms_max * 1e-3) / 1e9
    cfg = headline_config(world)
    row_sharded = None
    if world > 1:
        sms = chained_ms(torch, dev, stream, sharded_step, steps, copies, barrier=barrier)
        t = torch.tensor([sms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        us = float(t.item()) * 1e3 / steps
        row_sharded = {
            "workload": f"config 0's rows sharded: one [{N_ROWS * world}, {K_COLS}] Q4_0 GEMV, {N_ROWS} rows per GPU, "
                        "every step's y all-gathered to every GPU before the next step starts",
            "gather": "fused NVLink stores (tagged words) + wait kernel" if nvlink else "NCCL all-gather",
            "us_per_step": round(us, 3), "gb_s_aggregate": round(STEP_BYTES * world / (us * 1e-6) / 1e9, 1),
            "gemv_alone_us_per_step": round(ms_max * 1e3 / steps, 3),
            "gpu_launches_per_step": 2 if nvlink else 1, "nvlink_signal": signal}

    if args.only_gemv:
        prod.close()
        if rank == 0:
            out = {"metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": steps,
                   "ms_per_step": ms_max / steps, "only_gemv": True, "config": cfg,
                   "roofline": roofline(STEP_BYTES, kernel_ms / steps * 1e3, peak)}
            return out
        return None

    extra = {}
    host = {"c0": (Wq0.cpu().numpy(), x0)}   # host copies of the device-quantized weights, for the CPU arms
    # Config 4 (all ranks: row-sharded over the world at N > 1).
    c4 = {}
    for N, K in CFG4_SHAPES:
        wq, X = device_weights(torch, sk, dev, jobs[("c4", N, K)], "q4_0")
        c4.update(sharded_case(torch, sk, _core, shard, dev, stream, N, K, wq.reshape(-1), X, rank, world,
                               local_rank, l2, peak, barrier))
        if world == 1:
            host[("c4", N, K)] = (wq.reshape(-1).cpu().numpy(), X)
        del wq
    if rank == 0:
        extra["config4"] = c4

    if world == 1:
        extra["config1_q8_0"] = {}
        for N, K in CFG1_SHAPES:
            wq, X = device_weights(torch, sk, dev, jobs[("c1", N, K)], "q8_0")
            wq = wq.reshape(-1)
            xd = torch.from_numpy(X[0]).to(dev)
            yd = torch.empty(N, device=dev)
            nb = gemv_bytes(q_bytes("q8_0", N, K), 1, N, K)
            extra["config1_q8_0"][f"q8_0 M=1 N={N} K={K}"] = rotated_case(
                torch, dev, stream, wq, lambda w, xd=xd, yd=yd, N=N, K=K: sk.gemv_q8_0(xd, w, N, K, out=yd), nb,
                l2, peak)
            host[("c1", N, K)] = (wq.cpu().numpy(), X)
        extra["config3_dense"] = {}
        for N, K in CFG3_SHAPES:
            W32, X = device_weights(torch, sk, dev, jobs[("c3", N, K)], None, torch.float32)
            for wt, es in ((torch.float32, 4), (torch.bfloat16, 2), (torch.float16, 2)):
                w = W32.to(wt)
                kind = str(wt).split(".")[-1]
                host[("c3", kind, N, K)] = w.view(torch.int32 if es == 4 else torch.int16).cpu().numpy()
                for M in CFG3_ROWS:
                    xd = torch.from_numpy(X[:M]).to(dev)
                    yd = torch.empty((M, N), device=dev)
                    extra["config3_dense"][f"dense {kind} M={M} N={N} K={K}"] = rotated_case(
                        torch, dev, stream, w, lambda w_, xd=xd, yd=yd: sk.gemv_dense(xd, w_, out=yd),
                        N * K * es + 4 * M * K + 4 * M * N, l2, peak)
                del w
            host[("c3x", N, K)] = X
            del W32
        extra["config2_llama_stack"] = llama_stack(torch, sk, dev, stream, args, jobs, peak, host)
    prod.close()

    # End to end through the public API: x from page-locked host memory, y back to host memory,
    # weights resident on the device (uploaded once, as a model's).
    e2e = e2e_headline(torch, sk, shard, dev, local_rank, world, ws, copies, None, x0[0])
    e2e_sharded = e2e_headline(torch, sk, shard, dev, local_rank, world, ws, copies, sg, x0[0], sharded=True) \
        if world > 1 else None
    if sg is not None:
        sg.close()   # release the gather buffers before the process group goes

    if rank != 0:
        return None
    if world == 1:
        extra["cpu_arms"] = cpu_arms(host, extra)
    us = kernel_ms / steps * 1e3
    rl = roofline(STEP_BYTES, us, peak)
    rl.update({"traffic": committed_traffic("gemv_q4_0_cfg0_traffic.json"), "kernel": "gemv_q4_r4<x in shared memory>",
               "algorithmic_bytes_per_launch": STEP_BYTES,
               "peak_source": peak["source"] + " (MEASURED_PEAKS.json hbm_gbs, burst copy)"})
    out = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": steps,
        "warmup": args.warmup, "ms_per_step": ms_max / steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "q4_0 weights x int8 activations (dp4a int32, fp32 accumulate)",
        "data": "synthetic: numpy default_rng(0), W ~ N(0, 0.02) quantized ggml Q4_0 on device, x ~ N(0, 1)",
        "config": cfg,
        "timing": {"l2_policy": f"{copies} rotated weight copies ({copies * W_BYTES / 2**20:.0f} MiB > 2x L2 "
                                f"{l2 / 2**20:.0f} MiB): inputs larger than L2",
                   "launch": "CUDA graphs, programmatic dependent launch; start/end events recorded inside the "
                             f"graphs after {copies} untimed steps (steady state)"},
        "roofline": rl,
        "e2e": e2e,
        "gpu_launches": steps * launches_per_step,
        "gpus_active": gpus_active,
        "clocks": clocks.summary(),
    }
    if CHAINED_FALLBACKS:
        out["timing"]["in_graph_events"] = f"unreadable; {len(CHAINED_FALLBACKS)} cases timed over whole replays"

    if row_sharded is not None:
        out["config0_row_sharded"] = row_sharded
    if e2e_sharded is not None:
        out["e2e_row_sharded"] = e2e_sharded
    out.update(extra)
    if world == 1:
        cb = extra["cpu_arms"].get("config0")
        if cb:
            a = cb["all_threads"]
            out["cpu_baseline"] = {"value": a["gb_s"], "unit": "GB/s", "cores": a["threads"], "kind": "reference",
                                   "one_thread_value": cb["one_thread"]["gb_s"],
                                   "sample": f"{a['calls']} gemv_q4_0 calls (median {a['us_median']} us), "
                                             f"{a['weight_copies']} weight copies rotated past the host LLC, "
                                             f"path {cb['path']}, {a['threads']} threads, {cpu_model()}; one "
                                             f"thread pinned: {cb['one_thread']['gb_s']} GB/s"}
    return out


def rotated_case(torch, dev, stream, w, call, nbytes: int, l2: int, peak: dict, n: int = 200) -> dict:
    """One GPU case: `n` chained calls over weight copies totalling more than 2x L2."""
    wb = w.numel() * w.element_size()
    copies = max(2, -(-2 * l2 // wb) + 1)
    ws = [w] + [w.clone() for _ in range(copies - 1)]
    ms = chained_ms(torch, dev, stream, lambda i: call(ws[i % copies]), n, copies, chunk=max(64, copies))
    us = ms * 1e3 / n
    del ws
    return {"us": round(us, 3), "gb_s": round(nbytes / (us * 1e-6) / 1e9, 1), "bytes": nbytes,
            "roofline": roofline(nbytes, us, peak), "weight_copies": copies}


def sharded_case(torch, sk, _core, shard, dev, stream, N, K, wq, X, rank, world, local_rank, l2, peak,
                 barrier) -> dict:
    """Config 4 shape (N, K): this rank's row slice at M = 1 and M = 8. N = 1: the
    GEMV; N > 1: the GEMV with the all-gather of y fused into its stores over
    NVLink (the one-row kernels at M = 1, the tensor-core kernel at M = 8),
    strong scaling, max over ranks."""
    lo, hi = shard.row_slice(N, rank, world)
    n = hi - lo
    copies = max(2, -(-2 * l2 // max(1, wq.numel())) + 1)
    ws = [wq] + [wq.clone() for _ in range(copies - 1)]
    res = {}
    for M in CFG4_ROWS:
        xd = torch.from_numpy(np.ascontiguousarray(X[:M])).to(dev)
        yd = torch.empty((M, n), device=dev)
        sg = None
        if world > 1:
            sg = shard.ShardedGemv("q4_0", wq, N, K, gather="nvlink")

            def step(i, sg=sg, xd=xd, M=M):
                _core._gemv_q_gather(sg._g, 0, M, n, K, xd.data_ptr(), K, ws[i % copies].data_ptr(),
                                     stream.cuda_stream, local_rank)
        elif M == 1:
            def step(i, xd=xd, yd=yd):
                sk.gemv_q4_0(xd[0], ws[i % copies], n, K, out=yd[0])
        else:
            def step(i, xd=xd, yd=yd):
                sk.gemv_q4_0_batch(xd, ws[i % copies], n, K, out=yd)
        reps = 64 if N < 100000 else 32
        ms = chained_ms(torch, dev, stream, step, reps, copies, chunk=max(reps, copies),
                        barrier=barrier if world > 1 else None)
        t = torch.tensor([ms * 1e3 / reps], device=dev)
        if world > 1:
            dist_all_max(t)
        us = float(t.item())
        if sg is not None:
            sg.close()
        nbytes = gemv_bytes(q_bytes("q4_0", N, K), M, N, K)
        key = f"q4_0 M={M} N={N} K={K}" + (f" over {world} GPUs" if world > 1 else "")
        res[key] = {"us": round(us, 3), "gb_s_aggregate": round(nbytes / (us * 1e-6) / 1e9, 1),
                    "rows_per_gpu": n, "bytes": nbytes, "roofline": roofline(nbytes, us, peak),
                    "roofline_per_gpu": roofline(nbytes // world, us, peak),
                    "gather": None if world == 1 else "fused NVLink stores"}
        del xd, yd
    del ws
    return res


def dist_all_max(t):
    import torch.distributed as dist
    dist.all_reduce(t, op=dist.ReduceOp.MAX)


def llama_stack(torch, sk, dev, stream, args, jobs, peak, host) -> dict:
    """a Llama-3.2-1B decode step's GEMVs, 16 layers of
    q 2048->2048, k, v 2048->512, o 2048->2048, gate, up 2048->8192, down
    8192->2048, and the tied 2048->128256 LM head, on random-init Q4_0 weights
    (seed 2), fresh activations every token, LLAMA_TOKENS tokens in one CUDA
    graph. q, k and v read the same activation row within a token, as do gate
    and up, so each group runs as one GEMV over its concatenated rows (the same
    bytes and outputs as the separate GEMVs): 4 GEMVs per layer + the LM head.
    Also the decode step with SwiGLU: the down projection reads silu(gate) * up
    of the layer's gate/up GEMV, formed inside its activation quantization."""
    mats = []
    for i in range(len(LLAMA_MATRICES)):
        w, _ = device_weights(torch, sk, dev, jobs[("c2", i)], "q4_0")
        mats.append(w)
    groups, weights = [], []   # (rows N, K, logical GEMVs), concatenated rows
    for layer in range(LLAMA_LAYERS):
        m = mats[7 * layer:7 * layer + 7]
        groups += [(3072, 2048, 3), (2048, 2048, 1), (16384, 2048, 2), (2048, 8192, 1)]
        weights += [torch.cat(m[0:3]).reshape(-1), m[3].reshape(-1), torch.cat(m[4:6]).reshape(-1),
                    m[6].reshape(-1)]
    groups.append((LLAMA_VOCAB, 2048, 1))
    weights.append(mats[-1].reshape(-1))
    host["c2"] = [w.cpu().numpy() for w in weights]
    del mats
    wbytes = sum(w.numel() for w in weights)
    xs_per_tok = sum(k for _, k, _ in groups)
    ys_per_tok = sum(n for n, _, _ in groups)
    tokens = args.llama_tokens
    g = torch.Generator(device=dev)
    g.manual_seed(2)
    X = torch.randn((tokens, xs_per_tok), generator=g, device=dev)
    Y = torch.empty((ys_per_tok,), device=dev)
    act = torch.empty((8192,), device=dev)
    logical_x = sum(k * c for _, k, c in groups)
    tok_bytes = wbytes + 4 * (logical_x + ys_per_tok)
    res = {}
    for swiglu in ("", "fused", "unfused"):
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            with torch.cuda.graph(gr, stream=stream):
                for t in range(tokens):
                    xo = yo = 0
                    gate_up = None
                    for (n, k, _), wq in zip(groups, weights):
                        if swiglu and gate_up is not None and n == 2048 and k == 8192:
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
        per_tok_ms = s.elapsed_time(e) / tokens
        del gr
        name = {"": "gemv_stack", "fused": "decode_swiglu_fused", "unfused": "decode_swiglu_unfused"}[swiglu]
        res[name] = {"tok_s": round(1e3 / per_tok_ms, 1), "ms_per_token": per_tok_ms,
                     "gb_s": round(tok_bytes / (per_tok_ms * 1e-3) / 1e9, 1),
                     "roofline": roofline(tok_bytes, per_tok_ms * 1e3, peak),
                     "launches_per_token": len(groups) + (LLAMA_LAYERS if swiglu == "unfused" else 0)}
    res["decode_full"] = llama_full_decode(torch, sk, dev, stream, weights, tokens, peak, wbytes)
    res.update({"gemvs_per_token": len(LLAMA_MATRICES), "bytes_per_token": tok_bytes, "tokens": tokens,
                "weights": "per matrix i numpy default_rng((2, i)), N(0, 0.02) -> Q4_0 on device",
                "launch": f"one CUDA graph of {tokens} decode steps, PDL; q/k/v and gate/up as fused row groups"})
    return res


def llama_full_decode(torch, sk, dev, stream, weights, tokens: int, peak, wbytes: int) -> dict:
    """Whole decode tokens of config 2's architecture on the GPU (LlamaDecoder):
    embedding row, per layer RMSNorm, q/k/v GEMV, RoPE (Llama-3 scaling) and
    KV-cache write, GQA attention over the positions so far, o GEMV, residual
    RMSNorm, gate/up GEMV, down GEMV on silu(gate)*up; final norm and the tied
    LM head. The config-2 Q4_0 weights; norm weights 1 + N(0, 0.1^2) from seed 2;
    `tokens` tokens from position 0 in one CUDA graph."""
    from simd_ml_kernels import decode as D
    shape = D.LlamaShape(hidden=2048, layers=LLAMA_LAYERS, heads=32, kv_heads=8, head_dim=64, ffn=8192,
                         vocab=LLAMA_VOCAB, eps=1e-5)
    rng = np.random.default_rng([2, 2000])
    norm = lambda: torch.from_numpy((1 + 0.1 * rng.standard_normal(2048)).astype(np.float32)).to(dev)  # noqa: E731
    layers = [D.LlamaLayerWeights(attn_norm=norm(), qkv=weights[4 * i], o=weights[4 * i + 1], mlp_norm=norm(),
                                  gate_up=weights[4 * i + 2], down=weights[4 * i + 3]) for i in range(LLAMA_LAYERS)]
    w = D.LlamaWeights(layers=layers, norm=norm(), embed=weights[-1], lm_head=weights[-1], fmt="q4_0")
    inv = D.rope_inv_freq(64, 500000.0, {"factor": 32.0, "high_freq_factor": 4.0, "low_freq_factor": 1.0,
                                         "original_max_position_embeddings": 8192, "rope_type": "llama3"})
    cap = max(256, tokens)
    dec = D.LlamaDecoder(shape, w, inv, capacity=cap)
    toks = [(7919 * t + 13) % LLAMA_VOCAB for t in range(tokens)]
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        dec.step(toks[0])   # first-use set-up outside the capture
        dec.reset()
        with torch.cuda.graph(gr, stream=stream):
            for t in toks:
                dec.step(t)
        for _ in range(2):
            dec.reset()
            gr.replay()
        dec.reset()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        gr.replay()
        e.record(stream)
    torch.cuda.synchronize(dev)
    per_tok_ms = s.elapsed_time(e) / tokens
    del gr
    # Bytes a token reads: the weights once, the KV cache rows so far (average position), x/y of the GEMVs.
    kv = 2 * LLAMA_LAYERS * 8 * 64 * 4 * (tokens + 1) / 2
    nbytes = wbytes + kv
    return {"tok_s": round(1e3 / per_tok_ms, 1), "ms_per_token": per_tok_ms,
            "roofline": roofline(nbytes, per_tok_ms * 1e3, peak), "bytes_per_token": int(nbytes),
            "launches_per_token": dec.launches_per_token(), "tokens": tokens,
            "launch": f"one CUDA graph of {tokens} whole decode steps from position 0, PDL"}


def e2e_headline(torch, sk, shard, dev, local_rank, world, ws, copies, sg, x_np, sharded: bool = False) -> dict:
    """The headline metric through the public API with host buffers: every call
    copies x (page-locked host memory) to the device and returns y in host memory.
    At least 2,000 timed calls after 200 warm-up calls; per-call times. N > 1:
    every rank's own calls, the median of the slowest rank; `sharded`: calls of
    the row-sharded GEMV that return the all-gathered y."""
    import torch.distributed as dist
    xh = torch.from_numpy(np.ascontiguousarray(x_np)).pin_memory()
    xh_np = xh.numpy()
    sk.set_pdl(False, local_rank)
    calls = 2000
    ts = []
    if not sharded:
        if world > 1:
            dist.barrier()
        for i in range(200):
            sk.gemv_q4_0(xh_np, ws[i % copies], N_ROWS, K_COLS)
        for i in range(calls):
            t0 = time.perf_counter()
            yh = sk.gemv_q4_0(xh_np, ws[i % copies], N_ROWS, K_COLS)
            ts.append(time.perf_counter() - t0)
        assert yh.shape == (N_ROWS,)
        if world > 1:
            t = torch.tensor([statistics.median(ts)], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        d2h = 4 * N_ROWS
        api = "simd_ml_kernels.gemv_q4_0(numpy x in page-locked memory, device-resident weights) -> numpy y" + \
            (", on every GPU" if world > 1 else "")
    else:
        if sg is None:
            sg = shard.ShardedGemv("q4_0", ws[0], N_ROWS * world, K_COLS)
        yfull_h = torch.empty(N_ROWS * world).pin_memory()
        for _ in range(200):
            yfull_h.copy_(sg.forward(xh.to(dev, non_blocking=True)))
        torch.cuda.synchronize(dev)
        dist.barrier()
        for _ in range(calls):
            t0 = time.perf_counter()
            yfull_h.copy_(sg.forward(xh.to(dev, non_blocking=True)))   # the copy to host synchronises
            ts.append(time.perf_counter() - t0)
        t = torch.tensor([statistics.median(ts)], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        d2h = 4 * N_ROWS * world * world   # every rank reads the whole gathered y
        api = "ShardedGemv.forward(x host->device, fused NVLink gather) + y device->host"
    sk.set_pdl(True, local_rank)
    q = quantiles(ts)
    nb = STEP_BYTES * world
    med = float(t.item()) if world > 1 else q["median"]   # the slowest rank's median
    return {"value": round(nb / med / 1e9, 2), "unit": "GB/s", "h2d_bytes_per_step": 4 * K_COLS * world,
            "d2h_bytes_per_step": d2h if sharded else d2h * world, "us_median": round(med * 1e6, 3),
            "us_p25": round(q["p25"] * 1e6, 3), "us_p75": round(q["p75"] * 1e6, 3),
            "us_mean": round(q["mean"] * 1e6, 3), "steps": calls, "api": api}


def cpu_arms(host: dict, extra: dict) -> dict:
    """The reference's CPU kernels on the same bytes as the GPU cases, all host
    threads and one pinned thread (after every GPU case and every generator
    thread has finished)."""
    ref = RefCPU()
    if not ref.ok:
        return {"unavailable": "oracle/_ref/libsmk_ref.so was not built"}
    out = {"threads": ref.threads, "cpu": cpu_model(), "path": ref.path, "llc_bytes": ref.llc}
    # Config 0.
    Wq, x = host["c0"]
    ws = [Wq] + [Wq.copy() for _ in range(ref.copies(W_BYTES) - 1)]
    out["config0"] = ref.both(ref.gemv_q("q4_0", ws, x[0], N_ROWS, K_COLS), STEP_BYTES, seconds=2.0)
    out["config0"]["path"] = ref.path
    # Config 1.
    out["config1_q8_0"] = {}
    for N, K in CFG1_SHAPES:
        wq, X = host[("c1", N, K)]
        nb = gemv_bytes(wq.nbytes, 1, N, K)
        ws = [wq] + [wq.copy() for _ in range(ref.copies(wq.nbytes) - 1)]
        out["config1_q8_0"][f"q8_0 M=1 N={N} K={K}"] = ref.both(ref.gemv_q("q8_0", ws, X[0], N, K), nb)
    # Config 3.
    out["config3_dense"] = {}
    for N, K in CFG3_SHAPES:
        X = host[("c3x", N, K)]
        for kind, es in (("float32", 4), ("bfloat16", 2), ("float16", 2)):
            w = host[("c3", kind, N, K)]
            ws = [w] + [w.copy() for _ in range(ref.copies(w.nbytes) - 1)]
            for M in CFG3_ROWS:
                nb = N * K * es + es * M * K + 4 * M * N
                out["config3_dense"][f"dense {kind} M={M} N={N} K={K}"] = ref.both(
                    ref.dense(kind, ws, X[:M], N, K), nb, seconds=0.25)
    # Config 4 (the bytes of this GPU, rank 0 = the whole matrix at N = 1).
    out["config4"] = {}
    for N, K in CFG4_SHAPES:
        wq, X = host[("c4", N, K)]
        ws = [wq] + [wq.copy() for _ in range(ref.copies(wq.nbytes) - 1)]
        one = None
        for M in CFG4_ROWS:
            nb = gemv_bytes(wq.nbytes, M, N, K)
            calls = ref.gemv_q("q4_0", ws, X[:M], N, K)
            if M == 1:
                one = ref.both(calls, nb, seconds=0.5)
                out["config4"][f"q4_0 M=1 N={N} K={K}"] = one
                continue
            # M rows are M separate calls in the reference (no batched quantized GEMV);
            # on one thread their time is M times the one-row call's, not re-timed.
            a = ref.time(calls, nb, 0.5)
            o = dict(one["one_thread"])
            o.update(us_median=round(M * o["us_median"], 3), us_p25=round(M * o["us_p25"], 3),
                     us_p75=round(M * o["us_p75"], 3), gb_s=round(nb / (M * o["us_median"] * 1e-6) / 1e9, 3),
                     derived=f"{M} x the one-row call on one pinned thread")
            out["config4"][f"q4_0 M={M} N={N} K={K}"] = {"all_threads": a, "one_thread": o}
        del ws, wq
    # Config 2: the 113 GEMVs of a token (the fused row groups called as the reference's separate GEMVs).
    ws = host["c2"]
    rng = np.random.default_rng(2)
    calls = []
    rb = lambda k: k // 32 * 18  # noqa: E731
    for layer in range(LLAMA_LAYERS):
        qkv, o, gu, down = ws[4 * layer:4 * layer + 4]
        for w, n, k, r0 in ((qkv, 2048, 2048, 0), (qkv, 512, 2048, 2048), (qkv, 512, 2048, 2560), (o, 2048, 2048, 0),
                            (gu, 8192, 2048, 0), (gu, 8192, 2048, 8192), (down, 2048, 8192, 0)):
            calls.append((w[r0 * rb(k):(r0 + n) * rb(k)], n, k))
    calls.append((ws[-1], LLAMA_VOCAB, 2048))
    xs = [rng.standard_normal(k).astype(np.float32) for _, _, k in calls]
    ys = [np.empty(n, np.float32) for _, n, _ in calls]
    R = ref.R

    def token():
        for (w, n, k), xv, yv in zip(calls, xs, ys):
            R.smkref_gemv_q4_0(-1, n, k, xv.ctypes.data, w.ctypes.data, yv.ctypes.data)
    tok_bytes = extra["config2_llama_stack"]["bytes_per_token"]
    c2 = ref.both([token], tok_bytes, seconds=1.0)
    for v in c2.values():
        v["tok_s"] = round(1e6 / v["us_median"], 2)
        v["ms_per_token"] = v["us_median"] / 1e3
    out["config2_llama_stack"] = c2
    return out


def profile_case(torch, args) -> dict:
    """One GEMV shape on one GPU (--case KIND:M:N:K): weights N(0, 0.02) and x
    N(0, 1) from torch's generator (seed 7) on the device, rotated copies past
    2x L2, `--steps` chained calls after `--warmup`; what profilers capture."""
    import simd_ml_kernels as sk
    if args.case.startswith("llama-decode:"):
        return profile_decode(torch, sk, int(args.case.split(":")[1]))
    kind, M, N, K = args.case.split(":")
    M, N, K = int(M), int(N), int(K)
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(7)
    W = torch.randn((N, K), generator=g, device=dev) * 0.02
    X = torch.randn((M, K), generator=g, device=dev)
    Y = torch.empty((M, N), device=dev)
    if kind in ("q4_0", "q8_0"):
        w = (sk.quantize_q4_0 if kind == "q4_0" else sk.quantize_q8_0)(W).reshape(-1)
        batch = sk.gemv_q4_0_batch if kind == "q4_0" else sk.gemv_q8_0_batch
        call = lambda w_: batch(X, w_, N, K, out=Y)   # noqa: E731
        nbytes = gemv_bytes(q_bytes(kind, N, K), M, N, K)
    else:
        w = W.to(getattr(torch, kind))
        call = lambda w_: sk.gemv_dense(X, w_, out=Y)   # noqa: E731
        nbytes = N * K * w.element_size() + 4 * M * K + 4 * M * N
    del W
    l2 = torch.cuda.get_device_properties(dev).L2_cache_size
    stream = torch.cuda.Stream(device=dev)
    r = rotated_case(torch, dev, stream, w, call, nbytes, l2, measured_peaks(), n=args.steps)
    return {"case": args.case, **r}


def profile_decode(torch, sk, tokens: int) -> dict:
    """--case llama-decode:T: T whole decode tokens of config 2's architecture
    (LlamaDecoder) in one CUDA graph, on weights drawn on the device (torch,
    seed 7, N(0, 0.02) -> Q4_0; norms 1 + N(0, 0.01)): a short launch list of
    the decode step for profilers."""
    from simd_ml_kernels import decode as D
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(7)

    def q(n, k):
        return sk.quantize_q4_0(torch.randn((n, k), generator=g, device=dev) * 0.02).reshape(-1)

    def norm():
        return 1 + 0.1 * torch.randn(2048, generator=g, device=dev)

    layers = [D.LlamaLayerWeights(attn_norm=norm(), qkv=q(3072, 2048), o=q(2048, 2048), mlp_norm=norm(),
                                  gate_up=q(16384, 2048), down=q(2048, 8192)) for _ in range(LLAMA_LAYERS)]
    emb = q(LLAMA_VOCAB, 2048)
    shape = D.LlamaShape(hidden=2048, layers=LLAMA_LAYERS, heads=32, kv_heads=8, head_dim=64, ffn=8192,
                         vocab=LLAMA_VOCAB, eps=1e-5)
    inv = D.rope_inv_freq(64, 500000.0, {"factor": 32.0, "high_freq_factor": 4.0, "low_freq_factor": 1.0,
                                         "original_max_position_embeddings": 8192, "rope_type": "llama3"})
    dec = D.LlamaDecoder(shape, D.LlamaWeights(layers=layers, norm=norm(), embed=emb, lm_head=emb), inv,
                         capacity=max(256, tokens))
    stream = torch.cuda.Stream(device=dev)
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        dec.step(1)
        dec.reset()
        with torch.cuda.graph(gr, stream=stream):
            for t in range(tokens):
                dec.step((7919 * t + 13) % LLAMA_VOCAB)
        dec.reset()
        gr.replay()
        dec.reset()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        gr.replay()
        e.record(stream)
    torch.cuda.synchronize(dev)
    ms = s.elapsed_time(e) / tokens
    return {"case": f"llama-decode:{tokens}", "tok_s": round(1e3 / ms, 1), "ms_per_token": ms,
            "launches_per_token": dec.launches_per_token()}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20000)
    ap.add_argument("--warmup", type=int, default=100)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--gather", choices=["nvlink", "nccl"], default="nvlink",
                    help="N > 1: all-gather of y fused into the GEMV over NVLink, or NCCL's all-gather")
    ap.add_argument("--llama-tokens", type=int, default=LLAMA_TOKENS,
                    help="decode steps per Llama-stack CUDA graph (fewer: shorter profiler launch lists)")
    ap.add_argument("--only-gemv", action="store_true",
                    help="time the headline GEMV only (no other configs, e2e or CPU arms): for profilers")
    ap.add_argument("--case", default=None,
                    help="KIND:M:N:K (KIND q4_0, q8_0, float32, bfloat16 or float16): time that one GEMV on "
                         "seeded device data instead of the bench, one GPU (for profilers)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank != 0:
            return
        r = time_reference_arm(args.steps, args.warmup, world)
        if r is None:
            print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libsmk_ref.so was not built"}))
            return
        print(json.dumps({"impl": "reference", "metric": METRIC, "value": round(r["value"], 3), "unit": "GB/s",
                          "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                          "ms_per_step": r["ms_per_step"], "higher_is_better": True, "scaling": "weak",
                          "vs_baseline": None, "dtype": "q4_0 weights x int8 activations (vpdpbusd), fp32 accumulate",
                          "data": "synthetic: numpy default_rng(0), W ~ N(0, 0.02) quantized ggml Q4_0, x ~ N(0, 1)",
                          "config": headline_config(world),
                          "cpu_baseline": {"value": round(r["value"], 3), "unit": "GB/s", "cores": r["cores"],
                                           "kind": "reference", "sample": r["sample"]},
                          "e2e": {"value": round(r["value"], 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                                  "d2h_bytes_per_step": 0}}))
        return

    import torch
    import torch.distributed as dist
    from datetime import timedelta

    if args.case:
        print(json.dumps(profile_case(torch, args)))
        return
    if world > 1:
        os.environ.setdefault("NCCL_DEBUG", "WARN")   # stdout carries only the JSON line
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local_rank))
    try:
        out = gpu_bench(args, rank, world, local_rank)
        if rank == 0 and out is not None:
            print(json.dumps(out))
    finally:
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
