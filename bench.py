"""Benchmark of the W4A16 GEMV hot path on B200 (one JSON line on rank 0).

Workload (the metric's own config): M = 1, N = K = 8192, RTN 4-bit group
128, fp16 scale and zero, weights N(0, 0.02), activations N(0, 1), seeded synthetic data. One
step = one call of the operator (int4gemv.ops.w4a16) on one batch.

Measurement:
  value       effective HBM bandwidth, algorithmic bytes (N K/2 + N K/32 + 2 M K + 2 M N, the
              reference's int4_bytes) per call / device time per call, summed over ranks;
              exactly K (--steps) back-to-back calls captured in one CUDA graph and replayed
              once after W (--warmup) eager calls, each call on a different weight set from a
              rotation whose total size is > 2x the L2, so every call reads its weights from HBM
              (no flush kernel in the timed region; one 1 GiB write just before it)
  eager / host  the same calls launched one by one from the host (eager_us_per_call, device
              time) and the host's own time per ops.w4a16 call (host_us_per_call)
  sweep       the BASELINE shapes (M sweep at 8192 x 8192, the MLP shapes) against cuBLAS FP16
  e2e         the same metric through the public API with host buffers: per step, copy x from
              pinned host memory, call ops.w4a16, copy y back to pinned host memory and wait
  roofline    achieved bytes/s of the GEMV kernel (algorithmic bytes / its average launch
              duration over the timed region) vs the measured HBM copy peak (MEASURED_PEAKS.json),
              DRAM traffic per launch from the committed ncu summary; the isolated call (L2 flush,
              events around one call) beside it
  cuBLAS FP16 F.linear(x, W16) on the same box, same rotation rule: the speedup of the metric
  cpu_baseline the reference's own CPU path (csrc/sequential.cpp built from its sources into
              oracle/_ref; else the C oracle port), single-threaded, a bounded sample of rows

--impl reference times the reference's CPU implementation (all host threads) on a bounded row
sample of the same workload, in the same unit.
Multi-GPU (torchrun): every rank runs the same workload on its own weights (independent weight
matrices, e.g. different layers); no collective in the data path; value = sum over ranks of bytes
/ the slowest rank's time ("scaling": "weak"). With more than one rank the line also carries
"sharded": the multi-GPU configs (up 28672 x 8192 rows split, down 8192 x 28672 K split, M = 1
and 8) timed with the exchange fused into the GEMV (int4gemv.exchange) and with the NCCL stack
(int4gemv.sharded), device time max over ranks (--no-sharded skips it).
"""

from __future__ import annotations

import argparse
import importlib.util
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "int4-gemv-cuda_b200"))
sys.path.insert(0, str(REPO / "oracle"))

import numpy as np  # noqa: E402
import torch  # noqa: E402

M, N, K, GROUP = 1, 8192, 8192, 128
METRIC = "µs/call and HBM GB/s (% of B200 peak) at M=1, 8192×8192 W4A16; × vs cuBLAS FP16"
FALLBACK_HBM_GBS = 6650.0
L2_BYTES = 126 * 1024 * 1024


def int4_bytes(m, n, k, g):
    """Bytes one W4A16 call must move (the reference's bench/timing.py int4_bytes)."""
    return n * k // 2 + 2 * n * (k // g) * 2 + m * k * 2 + m * n * 2


def fp16_bytes(m, n, k):
    return n * k * 2 + m * k * 2 + m * n * 2


def measured_peak():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


def ncu_traffic():
    p = REPO / "profiles" / "ncu_traffic.json"
    if not p.exists():
        return None
    try:
        return json.loads(p.read_text())
    except Exception:
        return None


# ---------------------------------------------------------------- clocks during the timed region
class ClockSampler:
    """Samples SM clock, max clock and throttle reasons with NVML in a thread."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
        0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
    }

    def __init__(self, index: int):
        self.samples = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._ok = False
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self._ok = True
        except Exception:
            self._ok = False

    def _read(self):
        nv = self._nv
        sm = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
        try:
            reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
        except Exception:
            reasons = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self._h)
        return time.perf_counter(), sm, reasons

    def _loop(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self._read())
            except Exception:
                return
            time.sleep(0.002)

    def start(self):
        if self._ok:
            self._t = threading.Thread(target=self._loop, daemon=True)
            self._t.start()
        return self

    def stop(self):
        self._stop.set()
        if self._ok:
            self._t.join()
        return self

    def summary(self, t0: float, t1: float) -> dict:
        if not self._ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0,
                    "note": "NVML unavailable"}
        inside = [s for s in self.samples if t0 <= s[0] <= t1]
        if not inside and self.samples:  # region shorter than the sampling period: nearest sample
            inside = [min(self.samples, key=lambda s: abs(s[0] - 0.5 * (t0 + t1)))]
        reasons = set()
        for _, _, r in inside:
            for bit, name in self.REASONS.items():
                if r & bit and name != "gpu_idle":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(s[1] for s in inside) if inside else None,
                "sm_max_mhz": self.max_mhz, "reasons": sorted(reasons), "samples": len(inside)}


# ---------------------------------------------------------------- distributed plumbing
def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(value: float, world: int) -> float:
    if world == 1:
        return value
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------- data
def make_sets(n_sets: int, seed: int):
    from int4gemv import quant

    gen = torch.Generator(device="cuda").manual_seed(seed)
    sets = []
    for _ in range(n_sets):
        w = torch.randn(N, K, generator=gen, device="cuda") * 0.02
        sets.append(quant.quantize(w, GROUP))
        del w
    x = torch.randn(M, K, generator=gen, device="cuda").half()
    return sets, x


def reference_module():
    so = sorted((REPO / "oracle" / "_ref").glob("int4gemv_ref*.so"))
    if not so:
        return None
    spec = importlib.util.spec_from_file_location("int4gemv_ref", so[0])
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


# ---------------------------------------------------------------- timing helpers
def graph_of(calls):
    """Capture a list of zero-argument callables into one CUDA graph."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for c in calls:  # warm: lazy init, shared-memory attributes
            c()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for c in calls:
            c()
    return g


def time_graph_calls(calls, total_calls: int, warmup_calls: int):
    """Replay `calls` (one graph) until total_calls calls ran; returns seconds per call."""
    per = len(calls)
    g = graph_of(calls)
    reps_w = max(1, math.ceil(warmup_calls / per))
    for _ in range(reps_w):
        g.replay()
    torch.cuda.synchronize()
    reps = max(1, math.ceil(total_calls / per))
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(reps):
        g.replay()
    end.record()
    end.synchronize()
    return start.elapsed_time(end) / 1e3 / (reps * per)


_flush_buf = None


def time_isolated(fn, iters: int = 100, warmup: int = 10) -> float:
    """Seconds per call the reference's way (bench/timing.py time_cuda): before every call, read a
    buffer far larger than the L2 (1 GiB; the 126 MB L2 is the reason for the size), then time the
    one call with CUDA events. The flush also keeps the host ahead of the GPU, so the events
    bracket the kernel and not the host's launch latency. Median of `iters` calls."""
    global _flush_buf
    if _flush_buf is None:
        _flush_buf = torch.ones(256 * 1024 * 1024, device="cuda")  # 1 GiB of fp32
    for _ in range(warmup):
        fn()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(iters)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(iters)]
    for a, b in zip(starts, ends):
        _flush_buf.sum()
        a.record()
        fn()
        b.record()
    torch.cuda.synchronize()
    return statistics.median(a.elapsed_time(b) for a, b in zip(starts, ends)) / 1e3


def time_steps_graph(calls, steps: int, warmup: int, world: int = 1):
    """Seconds per call of exactly `steps` calls (calls[i % len(calls)]) captured in one CUDA graph
    and replayed once, timed with CUDA events on the replaying stream; `warmup` untimed eager calls
    first. A 1 GiB write is queued right before the start event, so the GPU is busy while the host
    launches the graph and the first timed call starts from a flushed L2. Returns (seconds per
    call, wall-clock start, wall-clock end) of the timed region."""
    global _flush_buf
    if _flush_buf is None:
        _flush_buf = torch.ones(256 * 1024 * 1024, device="cuda")
    for i in range(warmup):
        calls[i % len(calls)]()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(steps):
            calls[i % len(calls)]()
    barrier(world)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    _flush_buf.fill_(1.0)
    start.record()
    g.replay()
    end.record()
    end.synchronize()
    t1 = time.perf_counter()
    barrier(world)
    del g
    return start.elapsed_time(end) / 1e3 / steps, t0, t1


def time_eager_calls(calls, n: int) -> float:
    """Seconds per call of `n` calls launched one by one from the host (no graph), CUDA events."""
    for i in range(8):
        calls[i % len(calls)]()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for i in range(n):
        calls[i % len(calls)]()
    end.record()
    end.synchronize()
    return start.elapsed_time(end) / 1e3 / n


def host_time_per_call(calls, n: int) -> float:
    """Host seconds per call (argument checks, allocation of y, launch) with the GPU queue kept
    non-empty, so no call waits for the device: wall clock over `n` calls, before any sync."""
    torch.cuda.synchronize()
    global _flush_buf
    if _flush_buf is None:
        _flush_buf = torch.ones(256 * 1024 * 1024, device="cuda")
    _flush_buf.fill_(1.0)  # a few hundred microseconds of device work ahead of the calls
    t0 = time.perf_counter()
    for i in range(n):
        calls[i % len(calls)]()
    t1 = time.perf_counter()
    torch.cuda.synchronize()
    return (t1 - t0) / n


def cpu_sample(ref, x_cpu, q_cpu, s_cpu, z_cpu, budget_s: float, threads: int):
    """Time the reference's CPU path on growing row samples until budget_s is spent."""
    if ref is not None:
        def run(rows):
            if threads > 1:
                return ref.sequential_threads(x_cpu, q_cpu[:rows], s_cpu[:rows], z_cpu[:rows],
                                              GROUP, threads)
            return ref.sequential(x_cpu, q_cpu[:rows].contiguous(), s_cpu[:rows].contiguous(),
                                  z_cpu[:rows].contiguous(), GROUP)
        kind = "reference"
    else:
        import oracle

        xn, qn, sn, zn = (t.numpy() for t in (x_cpu, q_cpu, s_cpu, z_cpu))

        def run(rows):
            return oracle.sequential(xn, qn[:rows], sn[:rows], zn[:rows], GROUP)
        kind = "port"
        threads = 1
    rows = 256
    run(rows)  # warm
    t0 = time.perf_counter()
    done_rows, calls = 0, 0
    while time.perf_counter() - t0 < budget_s:
        run(rows)
        done_rows += rows
        calls += 1
        elapsed = time.perf_counter() - t0
        if elapsed < budget_s / 8 and rows < N:
            rows = min(N, rows * 2)
    elapsed = time.perf_counter() - t0
    bytes_done = done_rows / N * int4_bytes(M, N, K, GROUP)
    return {"value": bytes_done / elapsed / 1e9, "unit": "GB/s", "cores": threads, "kind": kind,
            "sample": f"{calls} calls over {done_rows} rows of the {N}x{K} M=1 workload "
                      f"({done_rows / N:.2f} full GEMVs) in {elapsed:.1f} s",
            "us_per_call": elapsed / (done_rows / N) * 1e6}


# ---------------------------------------------------------------- arms
def time_quantize(n: int = 28672, k: int = 8192, calls: int = 20) -> dict:
    """Device quantize (ops.quantize) of an fp16 [n, k] matrix (the sharded up projection, 470 MB,
    larger than L2): read 2 B and write 0.5 + 4 / GROUP B per weight."""
    from int4gemv import ops

    gen = torch.Generator(device="cuda").manual_seed(7)
    w = torch.randn(n, k, generator=gen, device="cuda", dtype=torch.float16) * 0.02
    for _ in range(3):
        ops.quantize(w, GROUP)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(calls):
        ops.quantize(w, GROUP)
    end.record()
    end.synchronize()
    sec = start.elapsed_time(end) / 1e3 / calls
    moved = n * k * 2 + n * k // 2 + 2 * n * (k // GROUP) * 2
    peak = measured_peak()
    del w
    return {"shape": [n, k], "dtype_in": "fp16", "us": round(sec * 1e6, 2),
            "gb_s": round(moved / sec / 1e9, 1), "frac_of_hbm": round(moved / sec / 1e9 / peak[0], 4)}


def time_grouped(k: int = 4096, sizes=(4096, 1024, 1024)) -> dict:
    """q / k / v of a Llama-3-8B attention block at M = 1 (shared x, K = 4096): one grouped launch
    (ops.w4a16_grouped on stacked weights) against three ops.w4a16 launches, CUDA-graph replays
    over enough weight sets that every call streams from HBM."""
    from int4gemv import ops, quant

    n_total = sum(sizes)
    set_bytes = n_total * k // 2 + 2 * n_total * (k // GROUP) * 2
    n_sets = math.ceil(2 * L2_BYTES / set_bytes) + 1
    gen = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(1, k, generator=gen, device="cuda", dtype=torch.float16)
    sets = []
    for _ in range(n_sets):
        mats = [ops.quantize(torch.randn(n, k, generator=gen, device="cuda",
                                         dtype=torch.float16) * 0.02, GROUP) for n in sizes]
        sets.append((mats, [quant.stack_rows(*(mt[j] for mt in mats)) for j in range(3)]))
    separate = [lambda mats=mats, i=i: ops.w4a16(x, *mats[i], GROUP)
                for mats, _ in sets for i in range(len(sizes))]
    grouped = [lambda st=st: ops.w4a16_grouped(x, *st, GROUP, list(sizes)) for _, st in sets]
    sep_s = time_graph_calls(separate, 300 * len(separate), 3 * len(separate)) * len(sizes)
    grp_s = time_graph_calls(grouped, 300 * len(grouped), 3 * len(grouped))
    del sets
    return {"shape": {"k": k, "n": list(sizes), "m": 1},
            "separate_launches_us": round(sep_s * 1e6, 2), "grouped_us": round(grp_s * 1e6, 2),
            "speedup": round(sep_s / grp_s, 3)}


def time_sharded(world: int, rank: int, reps: int = 5) -> dict:
    """The sharded configs of the multi-GPU rows (up 28672 x 8192 rows split, down 8192 x 28672 K
    split, M = 1 and 8) on this job's ranks: the fused exchange (int4gemv.exchange) against the
    NCCL stack (int4gemv.sharded), both replayed from CUDA graphs, device time max over ranks.
    Enough layers with distinct weights rotate through each graph that every call streams its
    shard from HBM (more than 2x L2 per rank)."""
    from int4gemv import capi, ops
    from int4gemv.exchange import FusedShardedW4A16
    from int4gemv.sharded import ShardedW4A16

    out = {}
    for name, (n, k, mode) in (("up_28672x8192_rows_split", (28672, 8192, "n")),
                               ("down_8192x28672_k_split", (8192, 28672, "k"))):
        shard_bytes = n * k // 2 // world
        layers = max(2, math.ceil(2 * L2_BYTES / shard_bytes) + 1)
        gen = torch.Generator(device="cuda").manual_seed(11)
        fused, nccl = [], []
        for _ in range(layers):
            w = torch.randn(n, k, generator=gen, device="cuda", dtype=torch.float16) * 0.02
            q, s, z = ops.quantize(w, GROUP)
            del w
            fused.append(FusedShardedW4A16(q, s, z, GROUP, mode))
            nccl.append(ShardedW4A16(q, s, z, GROUP, mode))
            del q, s, z
        res = {"layers_rotated": layers}
        for m in (1, 8):
            x = torch.randn(m, k, generator=gen, device="cuda", dtype=torch.float16)
            row = {}
            for label, stack in (("fused_us", fused), ("nccl_us", nccl)):
                for layer in stack:
                    layer(x)
                torch.cuda.synchronize()
                if label == "fused_us":
                    # every rank learns whether any rank's bounded peer wait ran out
                    bad = max_over_ranks(float(capi.device_status()), world)
                    if bad:
                        row[label] = None
                        row["fused_error"] = f"device status {int(bad)} (peer wait ran out)"
                        continue
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph):
                    for layer in stack:
                        layer(x)
                graph.replay()
                torch.cuda.synchronize()
                barrier(world)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(reps):
                    graph.replay()
                e1.record()
                e1.synchronize()
                sec = max_over_ranks(e0.elapsed_time(e1) / 1e3, world) / (reps * layers)
                row[label] = round(sec * 1e6, 2)
                del graph
            if row["fused_us"]:
                row["speedup_fused_vs_nccl"] = round(row["nccl_us"] / row["fused_us"], 3)
                row["fused_gb_s_total"] = round(int4_bytes(m, n, k, GROUP)
                                                / (row["fused_us"] / 1e6) / 1e9, 1)
            res[f"m{m}"] = row
        torch.cuda.synchronize()
        barrier(world)
        for layer in fused:
            layer.close()
        out[name] = res
    return out


def run_reference_arm(args, world, rank):
    if rank != 0:
        return
    ref = reference_module()
    threads = os.cpu_count() or 1
    gen = torch.Generator().manual_seed(0)
    from int4gemv import quant

    w = torch.randn(N, K, generator=gen) * 0.02
    q, s, z = quant.quantize(w, GROUP)
    x = torch.randn(M, K, generator=gen).half()
    # Each step is a bounded row sample, sized from a calibration call so that warmup + steps
    # take about a minute and a half whatever K is.
    kind = "reference" if ref is not None else "port"

    def run(rows):
        if ref is not None:
            return ref.sequential_threads(x, q[:rows], s[:rows], z[:rows], GROUP, threads)
        import oracle

        return oracle.sequential(x.numpy(), q[:rows].numpy(), s[:rows].numpy(), z[:rows].numpy())

    cal_rows = min(N, 1024)
    run(cal_rows)
    t_cal = time.perf_counter()
    run(cal_rows)
    per_row = (time.perf_counter() - t_cal) / cal_rows
    budget = 90.0
    rows = int(budget / max(1, args.steps + args.warmup) / per_row)
    rows = max(min(N, 8 * threads), min(N, rows))

    def step():
        return run(rows)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = (time.perf_counter() - t0) / max(1, args.steps)
    full_us = dt * N / rows * 1e6
    value = int4_bytes(M, N, K, GROUP) / (full_us * 1e-6) / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dt * 1e3, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp32 accumulate, fp16 in/out", "data": "synthetic",
        "us_per_call": round(full_us, 1),
        "config": {"workload": f"W4A16 GEMV M={M} N={N} K={K} group={GROUP}",
                   "m": M, "n": N, "k": K, "group_size": GROUP,
                   "sample_rows_per_step": rows},
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": threads,
                         "kind": kind,
                         "sample": f"{rows} of {N} rows per step, {args.steps} steps"},
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def time_stream_ceiling(sets, n_sets: int, bytes_call: int) -> dict:
    """int4gemv_stripe_load_only back to back over the weight rotation: how fast the stripe stream
    alone moves the call's bytes (what the GEMV on top of it could reach)."""
    from int4gemv import capi

    lib = capi.lib()
    out = torch.empty(N, dtype=torch.int32, device="cuda")

    def lo(i):
        q, s, z = sets[i]
        return lambda: capi.check(lib.int4gemv_stripe_load_only(
            out.data_ptr(), q.data_ptr(), s.data_ptr(), z.data_ptr(), N, K, GROUP,
            torch.cuda.current_stream().cuda_stream))

    fns = [lo(i) for i in range(n_sets)]
    t = time_graph_calls(fns * max(1, 32 // n_sets), 2000, 100)
    peak = measured_peak()[0]
    return {"kernel": "stripe_mma loads only (int4gemv_stripe_load_only)",
            "us": round(t * 1e6, 3), "gb_s": round(bytes_call / t / 1e9, 1),
            "frac_of_hbm": round(bytes_call / t / 1e9 / peak, 4)}


def run_ours(args, world, rank, local):
    from int4gemv import ops
    import torch.nn.functional as F

    set_bytes = N * K // 2 + 2 * N * (K // GROUP) * 2
    n_sets = max(2, math.ceil(2 * L2_BYTES / set_bytes) + 1)
    sets, x = make_sets(n_sets, seed=1234 + rank)

    # Parity gate before timing (as the reference's benchmarks do): set 0 against the oracle.
    import oracle

    q0, s0, z0 = (t.cpu().numpy() for t in sets[0])
    ref = oracle.reference(x.cpu().numpy(), q0, s0, z0, GROUP)
    y0 = ops.w4a16(x, *sets[0], GROUP)
    ok, msg = oracle.check_close(y0.float().cpu().numpy(), ref)
    if not ok:
        raise SystemExit(f"bench: parity gate failed: {msg}")
    kernel = ops.w4a16_kernel(x, *sets[0], GROUP)

    def call(i):
        return lambda: ops.w4a16(x, *sets[i], GROUP)

    calls = [call(i) for i in range(n_sets)]
    # ---- timed region: exactly `steps` back-to-back calls, captured in one CUDA graph (each call
    # on the next weight set of the rotation) and replayed once; `warmup` eager calls before it
    sampler = ClockSampler(torch.cuda.current_device()).start()
    per_call_s, t0, t1 = time_steps_graph(calls, args.steps, args.warmup, world)
    sampler.stop()
    total_s = max_over_ranks(per_call_s * args.steps, world)
    per_call_s = total_s / args.steps
    bytes_call = int4_bytes(M, N, K, GROUP)
    value = world * bytes_call * args.steps / total_s / 1e9
    clocks = sampler.summary(t0, t1)
    # the same calls launched one by one from the host (no graph), and the host's own time per call
    eager_s = time_eager_calls(calls, 200)
    host_s = host_time_per_call(calls, 200)

    # ---- one isolated call, the reference's way (L2 read-flush before each call, events around
    # the call): the per-launch duration the roofline fraction uses
    rot = iter(range(10**9))
    launch_s = time_isolated(lambda: calls[next(rot) % n_sets]())

    extra = {}
    if rank == 0:
        # ---- cuBLAS FP16 on the same box (F.linear, rotation > 2x L2)
        w16 = [torch.randn(N, K, device="cuda", dtype=torch.float16) * 0.02
               for _ in range(max(2, math.ceil(2 * L2_BYTES / (N * K * 2)) + 1))]
        cub = [(lambda w=w: F.linear(x, w)) for w in w16]
        cublas_s = time_graph_calls(cub * max(1, 16 // len(cub)), 2000, 50)
        cublas_iso_s = time_isolated(cub[0])
        del w16, cub
        extra["cublas_fp16_us"] = round(cublas_s * 1e6, 3)
        extra["speedup_vs_cublas_fp16"] = round(cublas_s / per_call_s, 3)
        extra["isolated"] = {"method": "1 GiB L2 read-flush, then CUDA events around one call "
                                       "(the reference's bench/timing.py), median of 100",
                             "w4a16_us": round(launch_s * 1e6, 3),
                             "cublas_fp16_us": round(cublas_iso_s * 1e6, 3),
                             "speedup_vs_cublas_fp16": round(cublas_iso_s / launch_s, 3)}
        # ---- the reference's own vectorized kernel, built for sm_100a, same rotation
        refm = reference_module()
        if refm is not None:
            rv = [(lambda i=i: refm.vectorized(x, *sets[i], GROUP)) for i in range(n_sets)]
            ref_s = time_graph_calls(rv * max(1, 64 // n_sets), 5000, 100)
            extra["reference_vectorized_us"] = round(ref_s * 1e6, 3)
            extra["speedup_vs_reference_vectorized"] = round(ref_s / per_call_s, 3)
            extra["isolated"]["reference_vectorized_us"] = round(time_isolated(rv[0]) * 1e6, 3)
        # ---- our vectorized (the reference-shaped API kernel)
        vv = [(lambda i=i: ops.vectorized(x, *sets[i], GROUP)) for i in range(n_sets)]
        extra["vectorized_us"] = round(time_graph_calls(vv * max(1, 64 // n_sets), 5000, 100) * 1e6, 3)
        # ---- the loads-only ceiling of the fast path's stream (same tiles, ring, grid and
        # launch; the arithmetic replaced by an XOR fold, no x), same rotation
        if kernel == "stripe_mma":
            extra["stream_ceiling"] = time_stream_ceiling(sets, n_sets, bytes_call)
        extra["quantize"] = time_quantize()
        extra["grouped_qkv"] = time_grouped()
        if not args.no_sweep:
            peak_gbs = measured_peak()[0]
            extra["sweep"] = [sweep_one(m, n, k, peak_gbs) for m, n, k in SWEEP_DEFAULT]

    # ---- end to end through the public API with host buffers
    x_host = x.cpu().pin_memory()
    y_host = torch.empty(M, N, dtype=torch.float16).pin_memory()
    x_dev = torch.empty_like(x)
    stream = torch.cuda.current_stream()
    e2e_steps = min(max(args.steps, 50), 2000)
    for i in range(20):
        x_dev.copy_(x_host, non_blocking=True)
        y_host.copy_(ops.w4a16(x_dev, *sets[i % n_sets], GROUP), non_blocking=True)
        stream.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(e2e_steps):
        x_dev.copy_(x_host, non_blocking=True)
        y_host.copy_(ops.w4a16(x_dev, *sets[i % n_sets], GROUP), non_blocking=True)
        stream.synchronize()  # the host reads this step's result
    e1.record()
    e1.synchronize()
    e2e_s = max_over_ranks(e0.elapsed_time(e1) / 1e3, world) / e2e_steps
    e2e = {"value": round(world * bytes_call / e2e_s / 1e9, 3), "unit": "GB/s",
           "us_per_call": round(e2e_s * 1e6, 3),
           "h2d_bytes_per_step": M * K * 2, "d2h_bytes_per_step": M * N * 2}

    sharded = None
    if world > 1 and not args.no_sharded:
        try:
            sharded = time_sharded(world, rank)
        except Exception as e:  # the headline line is printed either way
            sharded = {"error": f"{type(e).__name__}: {e}"[:300]}

    peak, peak_kind = measured_peak()
    # achieved: algorithmic bytes per launch / the kernel's average launch duration over the timed
    # region (CUDA events on the launching stream around the K timed launches, every one of which
    # is this kernel). The isolated single call after an L2 flush is reported beside it.
    achieved = bytes_call / per_call_s / 1e9
    traffic = ncu_traffic()
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                "traffic": traffic.get("bytes_per_launch") if traffic else None,
                "algorithmic_bytes": bytes_call,
                "kernel": kernel, "launch_us": round(per_call_s * 1e6, 3),
                "launch_timing": "the timed region's average: exactly `steps` back-to-back "
                                 "launches replayed from one CUDA graph, CUDA events on the "
                                 "replaying stream",
                "isolated_launch_us": round(launch_s * 1e6, 3),
                "isolated_frac": round(bytes_call / launch_s / 1e9 / peak, 4)}

    if rank != 0:
        return
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        x_cpu = x.cpu()
        q_cpu, s_cpu, z_cpu = (t.cpu() for t in sets[0])
        cpu = cpu_sample(reference_module(), x_cpu, q_cpu, s_cpu, z_cpu, args.cpu_seconds, 1)
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per_call_s * 1e3, 6),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "fp16 in/out, int4 weights, fp32 accumulate", "data": "synthetic",
        "us_per_call": round(per_call_s * 1e6, 3),
        "pct_of_peak": round(100 * bytes_call / per_call_s / 1e9 / peak, 2),
        "config": {"workload": f"W4A16 GEMV M={M} N={N} K={K} group={GROUP} (BASELINE config 1)",
                   "m": M, "n": N, "k": K, "group_size": GROUP, "kernel": kernel,
                   "l2": f"no flush; {n_sets} rotating weight sets of {set_bytes / 2**20:.1f} MiB "
                         f"(> 2x the 126 MB L2) so every call reads its weights from HBM",
                   "timing": f"one CUDA graph of exactly {args.steps} back-to-back calls, replayed "
                             f"once after {args.warmup} eager warm-up calls, CUDA events",
                   "parallelism": f"independent weights per GPU x{world}"},
        "roofline": roofline, "clocks": clocks, "e2e": e2e, "gpu_launches": args.steps,
        "eager_us_per_call": round(eager_s * 1e6, 3),
        "host_us_per_call": round(host_s * 1e6, 3),
        **extra, "parity": msg,
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    if sharded is not None:
        line["sharded"] = sharded
    print(json.dumps(line), flush=True)


SWEEP = ([(m, 8192, 8192) for m in (1, 2, 4, 8, 16, 32, 64)]
         + [(1, 4096, 4096), (1, 14336, 4096), (1, 4096, 14336), (16, 14336, 4096),
            (16, 4096, 14336), (1, 28672, 8192), (1, 8192, 28672), (8, 28672, 8192),
            (8, 8192, 28672), (16, 28672, 8192)])


# The shapes of the default line's "sweep" key: BASELINE's M sweep at 8192 x 8192 (plus M = 64),
# the M = 1 shapes of the other single-GPU configs and M = 16 at the two MLP shapes.
SWEEP_DEFAULT = ([(m, 8192, 8192) for m in (1, 2, 4, 8, 16, 32, 64)]
                 + [(1, 4096, 4096), (1, 14336, 4096), (1, 4096, 14336), (16, 14336, 4096),
                    (16, 4096, 14336)])


def sweep_one(m: int, n: int, k: int, peak: float, calls_timed: int = 1000) -> dict:
    """One BASELINE shape: ops.w4a16 and cuBLAS FP16 (F.linear on fp16 weights) back to back from
    CUDA graphs over weight rotations larger than 2x L2, plus one isolated call after an L2 flush."""
    from int4gemv import ops
    import torch.nn.functional as F

    gen = torch.Generator(device="cuda").manual_seed(m * 7 + n + k)
    set_bytes = n * k // 2 + 2 * n * (k // GROUP) * 2
    n_sets = max(2, math.ceil(2 * L2_BYTES / set_bytes) + 1)
    sets = [ops.quantize(torch.randn(n, k, generator=gen, device="cuda",
                                     dtype=torch.float16) * 0.02, GROUP)
            for _ in range(n_sets)]
    x = torch.randn(m, k, generator=gen, device="cuda", dtype=torch.float16)
    calls = [(lambda st=st: ops.w4a16(x, *st, GROUP)) for st in sets]
    ours = time_graph_calls(calls * max(1, 32 // n_sets), calls_timed, 100)
    rot = iter(range(10**9))
    iso = time_isolated(lambda: calls[next(rot) % n_sets](), iters=50)
    kernel = ops.w4a16_kernel(x, *sets[0], GROUP)
    del sets, calls
    w16 = [torch.randn(n, k, generator=gen, device="cuda", dtype=torch.float16) * 0.02
           for _ in range(max(2, math.ceil(2 * L2_BYTES / (n * k * 2)) + 1))]
    cub = [(lambda w=w: F.linear(x, w)) for w in w16]
    cublas = time_graph_calls(cub * max(1, 16 // len(cub)), calls_timed, 50)
    del w16, cub
    b = int4_bytes(m, n, k, GROUP)
    return {"m": m, "n": n, "k": k, "kernel": kernel,
            "us": round(ours * 1e6, 2), "gb_s": round(b / ours / 1e9, 1),
            "frac_of_hbm": round(b / ours / 1e9 / peak, 3),
            "isolated_us": round(iso * 1e6, 2),
            "cublas_fp16_us": round(cublas * 1e6, 2),
            "speedup_vs_cublas": round(cublas / ours, 2)}


def run_sweep(args):
    """--sweep: the BASELINE shapes (M sweep at 8192 x 8192, the MLP shapes, the unsharded
    multi-GPU shapes), one JSON line each (sweep_one)."""
    torch.cuda.set_device(0)
    peak, _ = measured_peak()
    for m, n, k in SWEEP:
        if m < args.sweep_min_m:
            continue
        print(json.dumps(sweep_one(m, n, k, peak, 2000)), flush=True)


def run_profile_case(args):
    """A few launches of one kernel for ncu (no timing, no JSON): --profile KERNEL."""
    from int4gemv import ops
    import torch.nn.functional as F

    global M, N, K
    M, N, K = args.m, args.n, args.k
    torch.cuda.set_device(0)
    if args.profile == "quantize":  # device quantize of an fp16 [N, K] matrix
        gen = torch.Generator(device="cuda").manual_seed(7)
        w = torch.randn(N, K, generator=gen, device="cuda", dtype=torch.float16) * 0.02
        for _ in range(args.calls):
            ops.quantize(w, GROUP)
        torch.cuda.synchronize()
        print(f"profile case quantize N={N} K={K}: {args.calls} calls")
        return
    set_bytes = N * K // 2 + 2 * N * (K // GROUP) * 2
    n_sets = max(2, math.ceil(L2_BYTES / set_bytes) + 1)
    sets, x = make_sets(n_sets, seed=7)
    if args.profile == "cublas":
        w16 = [torch.randn(N, K, device="cuda", dtype=torch.float16) for _ in range(2)]
        fns = [lambda w=w: F.linear(x, w) for w in w16]
    elif args.profile == "reference_vectorized":
        ref = reference_module()
        fns = [lambda i=i: ref.vectorized(x, *sets[i], GROUP) for i in range(n_sets)]
    elif args.profile.startswith("kernel:"):  # one named kernel, e.g. kernel:tc_wide
        name = args.profile.split(":", 1)[1]
        fns = [lambda i=i: ops.w4a16_with(x, *sets[i], GROUP, name) for i in range(n_sets)]
    else:
        fn = getattr(ops, args.profile)
        fns = [lambda i=i: fn(x, *sets[i], GROUP) for i in range(n_sets)]
    for i in range(args.calls):
        fns[i % len(fns)]()
    torch.cuda.synchronize()
    print(f"profile case {args.profile} M={M} N={N} K={K}: {args.calls} calls, "
          f"{n_sets} weight sets")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--profile", default=None,
                    help="run --calls launches of one kernel (w4a16, vectorized, naive, coalesced, "
                         "load_only, quantize, cublas, reference_vectorized, or kernel:NAME for "
                         "a named kernel) for ncu, then exit")
    ap.add_argument("--m", type=int, default=M)
    ap.add_argument("--n", type=int, default=N)
    ap.add_argument("--k", type=int, default=K)
    ap.add_argument("--calls", type=int, default=6)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20000)
    ap.add_argument("--warmup", type=int, default=200)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--sweep", action="store_true",
                    help="time the BASELINE shapes (one JSON line each) instead of the headline")
    ap.add_argument("--sweep-min-m", type=int, default=1, help="--sweep: only shapes with M >= this")
    ap.add_argument("--no-sweep", action="store_true",
                    help="skip the 'sweep' key (the BASELINE shapes against cuBLAS) of the line")
    ap.add_argument("--no-sharded", action="store_true",
                    help="with more than one GPU, skip the sharded-layer timing")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    if args.profile:
        run_profile_case(args)
        return
    if args.sweep:
        run_sweep(args)
        return
    world, rank, local = (int(os.environ.get("WORLD_SIZE", "1")),
                          int(os.environ.get("RANK", "0")),
                          int(os.environ.get("LOCAL_RANK", "0")))
    if args.impl == "reference":
        if rank == 0:
            run_reference_arm(args, world, rank)
        return
    if not torch.cuda.is_available():
        raise SystemExit("bench: no CUDA device")
    world, rank, local = dist_setup()
    try:
        run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
