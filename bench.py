#!/usr/bin/env python
"""Benchmark of the B200 sampling op on NanoServe's decode-batch configuration.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One *step* is one ``Sampler.sample`` over a batch of B=256 rows of fp32
logits with V=128256 (mixed greedy / top-k / top-p /
full-filter rows, repetition-penalty histories of U[128,2048] ids).  Inputs
are resident in HBM when the timed region starts; four rotating copies of
the logits (4 x 131 MB > the 126 MB L2) keep every step's reads coming from
HBM.  The K timed steps run as CUDA-graph replays, bracketed by a barrier and
``cuda.synchronize()``, timed with CUDA events on the launching stream; for
N > 1 each rank samples its own 256 rows and the step ends with one NCCL
all-gather of the int32 ids (weak scaling), and the max over ranks is taken.

The JSON line also carries: ``roofline`` (achieved HBM GB/s of the sampling
kernel against MEASURED_PEAKS.json), ``e2e`` (the same metric through
``Sampler.sample`` from host buffers: logits H2D, Python histories packed and
uploaded, token ids read back, every step), ``cpu_baseline`` (the numpy
restatement of the reference algorithm timed on this host), ``clocks``
(nvidia-smi samples taken during the timed region) and ``gpu_launches``.

``--impl reference`` times the CPU restatement of the reference sampler
(oracle/, the reference itself is Python and cannot travel) on all host
cores, on the same configuration, metric and unit.
"""
from __future__ import annotations

import argparse
import datetime
import importlib
import json
import os
import re
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))
PKG = "nanoserve---custom-llm-inference-engine_b200"
ROWS = 256
VOCAB = 128256
COPIES = 4
GRAPH_STEPS = 50
METRIC = "sampler rows/s (B=256, V=128256 fp32, mixed params)"
WORKLOAD = ("config2 decode batch: fp32 [256,128256] N(0,2^2) + 20 ids/row boosted by +8; "
            "rows cycle greedy / top_k=50 / top_p=0.9 / (t=0.7,k=50,p=0.9,rp=1.1); histories U[128,2048]")


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-graph", action="store_true", help="launch every step from Python")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=10)
    return ap.parse_args()


def trace(rank: int, what: str) -> None:
    """Stage marks on stderr when NS_BENCH_TRACE=1 (for locating a stuck rank)."""
    if os.environ.get("NS_BENCH_TRACE") == "1":
        print(f"[rank {rank}] {what}", file=sys.stderr, flush=True)


def dist_env():
    return int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("LOCAL_RANK", "0"))


def measured_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def profiled_traffic():
    """DRAM bytes of one sampling step (pre-pass + row kernel) from the committed ncu summary."""
    f = REPO / "profiles" / "pre_and_row_kernels_config2.md"
    if not f.exists():
        return None
    m = re.search(r"dram_bytes_per_launch:\s*([0-9]+)", f.read_text())
    return int(m.group(1)) if m else None


def cpu_model():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


# ---------------------------------------------------------------- workload
def make_host_workload(rank: int):
    W = importlib.import_module(PKG + ".workloads")
    rng = np.random.default_rng(1000 + rank)
    params = W.mixed_params(ROWS)
    hist = W.histories(rng, ROWS, 128, 2048, VOCAB)
    return params, hist


def make_device_logits(torch, dev, copies: int, seed: int):
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    x = torch.randn(copies, ROWS, VOCAB, generator=g, device=dev, dtype=torch.float32).mul_(2.0)
    ids = torch.randint(0, VOCAB, (copies, ROWS, 20), generator=g, device=dev)
    x.scatter_add_(2, ids, torch.full(ids.shape, 8.0, device=dev))
    return x


# ---------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, bus_id: str):
        self.bus_id = bus_id
        self.lines = []
        self.proc = None
        self.t = None
        self.marks = {}

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "20",
                 "-i", self.bus_id], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.t = threading.Thread(target=self._read, daemon=True)
        self.t.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.time(), line.strip()))

    def mark(self, name):
        self.marks[name] = time.time()

    def stop(self):
        if self.proc is None:
            return
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.t:
            self.t.join(timeout=2)

    def summary(self):
        lo, hi = self.marks.get("t0", 0), self.marks.get("t1", time.time())
        rows = [l for (ts, l) in self.lines if lo - 0.05 <= ts <= hi + 0.05]
        if len(rows) < 2:
            rows = [l for (_, l) in self.lines]
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            parts = [p.strip() for p in r.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------- CPU legs (oracle)
def _oracle_rows(args):
    """Worker: run the CPU restatement on rows [lo, hi) of the host workload."""
    lo, hi, seed = args
    sys.path.insert(0, str(REPO))
    from oracle import sampler_oracle as O

    W = importlib.import_module(PKG + ".workloads")
    rng = np.random.default_rng(seed)
    x = W.peaked_logits(rng, hi - lo, VOCAB)
    params, hist = make_host_workload(0)
    t0 = time.perf_counter()
    for j, i in enumerate(range(lo, hi)):
        O.sample_row(x[j], params[i % ROWS], hist[i % ROWS], 0.5)
    return time.perf_counter() - t0


def cpu_baseline_single(budget_s: float = 12.0):
    """The oracle on one core over a bounded sample of the workload (rows/s)."""
    t_probe = _oracle_rows((0, 4, 7))
    per_row = t_probe / 4
    n = int(max(4, min(ROWS, budget_s / max(per_row, 1e-6))))
    n -= n % 4
    t = _oracle_rows((0, n, 8))
    return {"value": n / t, "unit": "rows/s", "cores": 1, "kind": "port",
            "sample": f"{n} of the 256 config-2 rows (every parameter kind), numpy restatement in "
                      f"oracle/, one thread, {cpu_model()}"}


# ---------------------------------------------------------------- our arm
def run_ours(args):
    import torch
    import torch.distributed as dist

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    NS = importlib.import_module(PKG)
    packing = importlib.import_module(PKG + ".packing")
    sampler_mod = importlib.import_module(PKG + ".sampler")

    # CPU baseline first (no GPU work yet)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_single()

    params, hist = make_host_workload(rank)
    pk = packing.pack(params, hist, VOCAB, sms=torch.cuda.get_device_properties(dev).multi_processor_count)
    rp, off, ids, order = sampler_mod.upload_packed(pk, dev)
    logits = make_device_logits(torch, dev, COPIES, 1234 + rank)
    hist_bytes = int(pk.ids.nbytes)
    algo_bytes = ROWS * VOCAB * 4 + hist_bytes

    s = NS.Sampler(dev)
    out = torch.empty(ROWS, dtype=torch.int32, device=dev)
    gathered = torch.empty(ROWS * world, dtype=torch.int32, device=dev) if world > 1 else None
    seed = 2024

    def step(k: int, with_comm: bool = True):
        s.sample_packed(logits[k % COPIES], rp, off, ids, out=out, seed=seed, offset=k, row_offset=rank * ROWS,
                        row_order=order)
        if world > 1 and with_comm:
            dist.all_gather_into_tensor(gathered, out)

    K, Wm = args.steps, max(3, args.warmup)
    trace(rank, "warm-up")
    for k in range(Wm):
        step(k)
    torch.cuda.synchronize()
    trace(rank, "capturing")

    stream = torch.cuda.Stream()
    graphs = []

    def capture(n, with_comm=True):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            with torch.cuda.graph(g, stream=stream):
                for k in range(n):
                    step(k, with_comm)
        return g

    use_graph = not args.no_graph
    G = min(GRAPH_STEPS, K)
    if use_graph:
        stream.wait_stream(torch.cuda.current_stream())
        g_main = capture(G)
        g_rem = capture(K % G) if K % G else None
        graphs += [g_main] + ([g_rem] if g_rem else [])
        torch.cuda.synchronize()
        for _ in range(2):
            g_main.replay()
        torch.cuda.synchronize()

    props = torch.cuda.get_device_properties(dev)
    try:
        bus = f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"
    except AttributeError:
        bus = str(local)
    trace(rank, "timing")
    clocks = ClockSampler(bus)
    clocks.start()
    time.sleep(0.1)

    run_stream = stream if use_graph else torch.cuda.current_stream()
    chunk_events = []
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.mark("t0")
    with torch.cuda.stream(run_stream):
        ev0 = torch.cuda.Event(enable_timing=True)
        ev1 = torch.cuda.Event(enable_timing=True)
        ev0.record(run_stream)
        if use_graph:
            for c in range(K // G):
                e = torch.cuda.Event(enable_timing=True)
                e.record(run_stream)
                chunk_events.append(e)
                g_main.replay()
            if K % G:
                graphs[1].replay()
        else:
            for k in range(K):
                step(k)
        ev1.record(run_stream)
    torch.cuda.synchronize()
    clocks.mark("t1")
    if world > 1:
        dist.barrier()
    elapsed_ms = ev0.elapsed_time(ev1)
    t_max = torch.tensor([elapsed_ms], device=dev)
    if world > 1:
        dist.all_reduce(t_max, op=dist.ReduceOp.MAX)
    elapsed_ms = float(t_max.item())
    clocks.stop()
    ms_per_step = elapsed_ms / K
    per_chunk_us = []
    if use_graph and chunk_events:
        marks = chunk_events + [ev1]
        for a, b in zip(marks[:-1], marks[1:]):
            per_chunk_us.append(a.elapsed_time(b) * 1000.0 / G)

    # kernel-only timing for the roofline (at N=1 identical to the main loop)
    if world > 1 and use_graph:
        gk = capture(G, with_comm=False)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(max(1, K // G)):
                gk.replay()
            e1.record(stream)
        torch.cuda.synchronize()
        kern_ms = e0.elapsed_time(e1) / (max(1, K // G) * G)
        del gk
    else:
        kern_ms = ms_per_step
    peak, peak_kind = measured_peaks()
    achieved = algo_bytes / (kern_ms * 1e-3) / 1e9

    trace(rank, "end to end")
    # ---- end to end through the public API from host buffers
    host_logits = logits[0].cpu().pin_memory()
    lg_dev = torch.empty_like(logits[0])
    E = max(3, min(args.e2e_steps, K))
    for k in range(2):
        lg_dev.copy_(host_logits, non_blocking=True)
        o = s.sample(lg_dev, params, hist, out_dtype=torch.int32)
        o.cpu()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for k in range(E):
        lg_dev.copy_(host_logits, non_blocking=True)
        o = s.sample(lg_dev, params, hist, out_dtype=torch.int32)
        if world > 1:
            dist.all_gather_into_tensor(gathered, o)
            toks = gathered.cpu()
        else:
            toks = o.cpu()
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / E
    t_e = torch.tensor([e2e_ms], device=dev)
    if world > 1:
        dist.all_reduce(t_e, op=dist.ReduceOp.MAX)
    e2e_ms = float(t_e.item())
    del toks
    packed_bytes = packing.layout(pk)[-1]

    # every CUDA graph holding NCCL calls must be gone before the process
    # group is destroyed, or the teardown waits for them forever
    trace(rank, "releasing graphs")
    g_main = g_rem = None
    graphs.clear()
    torch.cuda.synchronize()
    import gc

    gc.collect()
    if world > 1:
        trace(rank, "final barrier")
        dist.barrier()
        dist.destroy_process_group()
    trace(rank, "done")
    if rank != 0:
        return
    rows_total = ROWS * world
    line = {
        "metric": METRIC,
        "value": rows_total / (ms_per_step * 1e-3),
        "unit": "rows/s",
        "n_gpus": world,
        "steps": K,
        "warmup": Wm,
        "ms_per_step": ms_per_step,
        "us_per_step_p50": statistics.median(per_chunk_us) if per_chunk_us else ms_per_step * 1000.0,
        "hbm_gbs": achieved,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": {
            "workload": WORKLOAD,
            "rows_per_gpu": ROWS,
            "vocab": VOCAB,
            "global_batch": rows_total,
            "l2": f"{COPIES} rotating input copies ({COPIES * ROWS * VOCAB * 4 / 1e6:.0f} MB > 126 MB L2)",
            "parallelism": f"row-sharded x{world}" + (" + NCCL all-gather of int32 ids" if world > 1 else ""),
            "timing": f"CUDA-graph replays of {G} steps" if use_graph else "eager launches",
        },
        "roofline": {
            "bound": "hbm",
            "achieved": achieved,
            "peak": peak,
            "unit": "GB/s",
            "frac": achieved / peak,
            "peak_kind": peak_kind,
            "algorithmic_bytes_per_launch": algo_bytes,
            "kernel_us": kern_ms * 1000.0,
            "traffic": profiled_traffic(),
        },
        "e2e": {
            "value": rows_total / (e2e_ms * 1e-3),
            "unit": "rows/s",
            "ms_per_step": e2e_ms,
            "h2d_bytes_per_step": ROWS * VOCAB * 4 + packed_bytes,
            "d2h_bytes_per_step": rows_total * 4,
            "path": "Sampler.sample(host-pinned logits copied in, Python params/histories packed) + ids .cpu()",
        },
        # the library launches the top-p pre-pass before the row kernel when a
        # call has at most 256 rows and no debug outputs (NS_PREPASS=0: never)
        "gpu_launches": K * (2 if ROWS <= 256 and os.environ.get("NS_PREPASS") != "0" else 1),
        "clocks": clocks.summary(),
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- reference arm
def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    import multiprocessing as mp

    cores = os.cpu_count() or 1
    ctx = mp.get_context("spawn")
    K, Wm = args.steps, max(3, args.warmup)
    with ctx.Pool(cores) as pool:
        t_probe = max(pool.map(_oracle_rows, [(0, 2, 3)] * min(cores, 4)))
        per_row = t_probe / 2
        budget = 150.0 / (K + Wm)  # whole run within a few minutes
        rows_per_step = int(max(1, min(ROWS, budget / per_row * cores)))
        chunks = max(1, min(cores, rows_per_step))

        def one_step(k):
            base = (k * rows_per_step) % ROWS
            bounds = np.linspace(0, rows_per_step, chunks + 1).astype(int)
            jobs = [(base + int(a), base + int(b), 100 + k) for a, b in zip(bounds[:-1], bounds[1:]) if b > a]
            pool.map(_oracle_rows, jobs)

        for k in range(Wm):
            one_step(k)
        t0 = time.perf_counter()
        for k in range(K):
            one_step(k)
        el = time.perf_counter() - t0
    val = rows_per_step * K / el
    line = {
        "metric": METRIC, "value": val, "unit": "rows/s", "n_gpus": world, "steps": K, "warmup": Wm,
        "ms_per_step": el / K * 1000.0, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic", "impl": "reference",
        "config": {"workload": WORKLOAD, "rows_per_step": rows_per_step, "vocab": VOCAB},
        "cpu_baseline": {"value": val, "unit": "rows/s", "cores": cores, "kind": "port",
                         "sample": f"{rows_per_step} config-2 rows per step over {cores} processes; numpy "
                                   f"restatement of nanoserve/scheduler/sampler.py (the reference is Python "
                                   f"and is not present on this host); {cpu_model()}"},
        "e2e": {"value": val, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
