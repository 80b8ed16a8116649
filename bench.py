#!/usr/bin/env python
"""Benchmark of the B200 sampling op on NanoServe's decode-batch configuration.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One *step* is one sampling call over a batch of B=256 rows of fp32 logits
with V=128256 (mixed greedy / top-k / top-p / full-filter
rows, repetition-penalty histories of U[128,2048] ids).  Inputs are resident
in HBM when the timed region starts; four rotating copies of the logits
(4 x 131 MB > the 126 MB L2) keep every step's reads coming from HBM.  The K
timed steps run as CUDA-graph replays, bracketed by a barrier and
``cuda.synchronize()``, timed with CUDA events on the launching stream; for
N > 1 each rank samples its own 256 rows and the step ends with one NCCL
all-gather of the int32 ids (weak scaling), and the max over ranks is taken.

The JSON line also carries:

* ``roofline``: achieved HBM GB/s of the row kernel (algorithmic bytes
  over its CUDA-event time) against MEASURED_PEAKS.json; ``traffic`` is the
  DRAM bytes per launch of the ncu capture named in ``traffic_source``;
* ``us_per_step_p50``: the median of per-step times (one-step graph replays,
  an event between consecutive steps);
* ``config5_strong``: BASELINE config 5 at the same N -- 16384 rows split
  into contiguous blocks, one per rank, each block generated in place, one
  NCCL all-gather of the int32 ids per step, max over ranks;
* ``e2e``: the same metric through ``Sampler.sample`` from host buffers
  (logits copied in from pinned memory, Python params and histories packed
  and uploaded, ids read back), every step; ``e2e_store`` the same through
  ``HistoryStore.sample`` with the logits resident (as an engine's lm_head
  leaves them) and the histories kept on the device;
* ``cpu_baseline``: the reference ``Sampler.sample`` itself (copied unmodified
  by oracle/build_ref.py) on CPU torch with every host thread, on a bounded
  sample of the rows; the numpy port in oracle/ when that copy is absent;
* ``clocks`` (nvidia-smi samples taken during the timed region) and
  ``gpu_launches``.

``--impl reference`` times the reference ``Sampler.sample`` the same way on
the same configuration, metric and unit (rank 0 only under torchrun).
"""
from __future__ import annotations

import argparse
import datetime
import gc
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
C5_ROWS = 16384
METRIC = "sampler rows/s (B=256, V=128256 fp32, mixed params)"
WORKLOAD = ("config2 decode batch: fp32 [256,128256] N(0,2^2) + 20 ids/row boosted by +8; "
            "rows cycle greedy / top_k=50 / top_p=0.9 / (t=0.7,k=50,p=0.9,rp=1.1); histories U[128,2048]")
PROFILE = REPO / "profiles" / "split_kernel_config2.md"


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-graph", action="store_true", help="launch every step from Python")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-config5", action="store_true")
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
    """DRAM bytes per launch of the row kernel in the committed ncu summary."""
    if not PROFILE.exists():
        return None
    m = re.search(r"dram_bytes_per_launch:\s*([0-9]+)", PROFILE.read_text())
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
def make_host_workload(rank: int, rows: int = ROWS, lo: int = 128, hi: int = 2048):
    W = importlib.import_module(PKG + ".workloads")
    rng = np.random.default_rng(1000 + rank)
    params = W.mixed_params(rows)
    hist = W.histories(rng, rows, lo, hi, VOCAB)
    return params, hist


def make_device_logits(torch, dev, copies: int, rows: int, seed: int):
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    x = torch.randn(copies, rows, VOCAB, generator=g, device=dev, dtype=torch.float32).mul_(2.0)
    ids = torch.randint(0, VOCAB, (copies, rows, 20), generator=g, device=dev)
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


# ---------------------------------------------------------------- CPU legs
def _port_rows(args):
    """Worker: the numpy port (oracle/) on rows [lo, hi) of the workload."""
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


class ReferenceCPU:
    """The reference ``Sampler.sample`` on CPU torch (oracle/_ref, every host
    thread), on ``rows`` config-2 rows per call: a multiple of 4, so every
    parameter kind is in each call.  The input is cloned outside the timed
    call (the reference writes its penalised logits into it)."""

    def __init__(self, rows: int):
        import torch

        from oracle import build_ref

        loaded = build_ref.load_sampler()
        if loaded is None:
            raise FileNotFoundError("oracle/_ref is absent")
        Sampler, SP = loaded
        self.torch = torch
        self.threads = os.cpu_count() or 1
        torch.set_num_threads(self.threads)
        W = importlib.import_module(PKG + ".workloads")
        rows = max(4, rows - rows % 4)
        self.rows = rows
        params, hist = make_host_workload(0)
        self.params = [SP(temperature=p.temperature, top_p=p.top_p, top_k=p.top_k,
                          repetition_penalty=p.repetition_penalty) for p in params[:rows]]
        self.hist = hist[:rows]
        self.x = torch.from_numpy(W.peaked_logits(np.random.default_rng(7), rows, VOCAB))
        self.sampler = Sampler(torch.device("cpu"))
        self.source = build_ref.source_note()

    def step(self) -> float:
        x = self.x.clone()
        t0 = time.perf_counter()
        self.sampler.sample(x, self.params, self.hist)
        return time.perf_counter() - t0


def reference_rows_per_step(budget_s: float) -> int:
    """Rows per reference call so that one call takes about budget_s."""
    probe = ReferenceCPU(4)
    probe.step()
    per_row = min(probe.step(), probe.step()) / 4
    return int(max(4, min(ROWS, budget_s / max(per_row, 1e-6))))


def cpu_baseline(budget_s: float = 12.0) -> dict:
    """The reference on this host over a bounded sample of the workload (rows/s)."""
    try:
        n = reference_rows_per_step(budget_s / 4)
        ref = ReferenceCPU(n)
        ref.step()
        times = [ref.step() for _ in range(3)]
        return {"value": ref.rows / statistics.median(times), "unit": "rows/s", "cores": ref.threads,
                "kind": "reference",
                "sample": f"{ref.rows} of the 256 config-2 rows per call (every parameter kind), median of 3 calls; "
                          f"the reference Sampler.sample on CPU torch {importlib.import_module('torch').__version__} "
                          f"with {ref.threads} threads ({ref.source}); {cpu_model()}"}
    except FileNotFoundError:
        t_probe = _port_rows((0, 4, 7))
        n = int(max(4, min(ROWS, budget_s / max(t_probe / 4, 1e-6))))
        n -= n % 4
        t = _port_rows((0, n, 8))
        return {"value": n / t, "unit": "rows/s", "cores": 1, "kind": "port",
                "sample": f"{n} of the 256 config-2 rows, numpy restatement in oracle/ (oracle/_ref absent), "
                          f"one thread, {cpu_model()}"}


# ---------------------------------------------------------------- timing helpers
def graph_time(torch, stream, graphs_to_replay, dist=None, world=1, dev=None):
    """Replay the given graphs back to back; max over ranks of the event time (ms)."""
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for g in graphs_to_replay:
            g.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms


def capture(torch, stream, fn, n):
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(g, stream=stream):
            for k in range(n):
                fn(k)
    return g


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
    sharded = importlib.import_module(PKG + ".sharded")

    # CPU baseline first (no GPU work yet)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline()

    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    params, hist = make_host_workload(rank)
    pk = packing.pack(params, hist, VOCAB, sms=sms)
    rp, off, ids, order = sampler_mod.upload_packed(pk, dev)
    logits = make_device_logits(torch, dev, COPIES, ROWS, 1234 + rank)
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
    stream = torch.cuda.Stream()
    graphs = []
    use_graph = not args.no_graph
    run_stream = stream if use_graph else torch.cuda.current_stream()
    trace(rank, "warm-up")
    # warm up on the stream that is captured, so that its workspace exists
    # (and is zero) before the graph is made
    run_stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(run_stream):
        for k in range(Wm):
            step(k)
    torch.cuda.synchronize()
    trace(rank, "capturing")

    G = min(GRAPH_STEPS, K)
    g_main = g_rem = g_one = None
    if use_graph:
        g_main = capture(torch, stream, step, G)
        g_rem = capture(torch, stream, step, K % G) if K % G else None
        g_one = capture(torch, stream, step, 1)
        graphs += [g_main, g_one] + ([g_rem] if g_rem else [])
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
                g_main.replay()
            if g_rem is not None:
                g_rem.replay()
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

    # per-step times: one-step graph replays with an event between steps
    per_step_us = []
    if use_graph:
        P = min(K, 200)
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(P + 1)]
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            evs[0].record(stream)
            for i in range(P):
                g_one.replay()
                evs[i + 1].record(stream)
        torch.cuda.synchronize()
        per_step_us = [evs[i].elapsed_time(evs[i + 1]) * 1000.0 for i in range(P)]

    # kernel-only timing for the roofline (at N=1 the main loop is kernel-only)
    if world > 1 and use_graph:
        gk = capture(torch, stream, lambda k: step(k, with_comm=False), G)
        torch.cuda.synchronize()
        kern_ms = graph_time(torch, stream, [gk] * max(1, K // G)) / (max(1, K // G) * G)
        del gk
    else:
        kern_ms = ms_per_step
    peak, peak_kind = measured_peaks()
    achieved = algo_bytes / (kern_ms * 1e-3) / 1e9

    # ---- config 5, strong scaling: 16384 rows split over the ranks
    c5 = None
    if not args.no_config5:
        trace(rank, "config 5")
        c5 = run_config5(torch, dist, world, rank, dev, NS, packing, sampler_mod, sharded, stream, sms)

    trace(rank, "end to end")
    # ---- end to end through the public API from host buffers
    host_logits = logits[0].cpu().pin_memory()
    lg_dev = torch.empty_like(logits[0])
    E = max(3, min(args.e2e_steps, K))

    def e2e_step():
        lg_dev.copy_(host_logits, non_blocking=True)
        o = s.sample(lg_dev, params, hist, out_dtype=torch.int32)
        if world > 1:
            dist.all_gather_into_tensor(gathered, o)
            return gathered.cpu()
        return o.cpu()

    def timed(fn, n):
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            fn()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / n
        t_e = torch.tensor([ms], device=dev)
        if world > 1:
            dist.all_reduce(t_e, op=dist.ReduceOp.MAX)
        return float(t_e.item())

    e2e_ms = timed(e2e_step, E)
    packed_bytes = packing.layout(pk)[-1]

    # ---- the engine-side path: histories on the device, logits resident
    store = NS.HistoryStore(dev, capacity=int(sum(len(h) for h in hist)) + ROWS * (E + 8), vocab=VOCAB)
    handles = [store.add(h, max_new_tokens=E + 8) for h in hist]
    s_store = NS.Sampler(dev)

    def store_step():
        o = store.sample(s_store, logits[0], params, handles, out_dtype=torch.int32, append=False)
        if world > 1:
            dist.all_gather_into_tensor(gathered, o)
            return gathered.cpu()
        return o.cpu()

    store_ms = timed(store_step, E)
    store_h2d = int(packing.derive_rows(params, VOCAB, [len(h) for h in hist]).nbytes) + 16 * (ROWS + 1) + 4 * ROWS
    del store

    # every CUDA graph holding NCCL calls must be gone before the process
    # group is destroyed, or the teardown waits for them forever
    trace(rank, "releasing graphs")
    g_main = g_rem = g_one = None
    graphs.clear()
    torch.cuda.synchronize()
    gc.collect()
    if world > 1:
        trace(rank, "final barrier")
        dist.barrier()
        dist.destroy_process_group()
    trace(rank, "done")
    if rank != 0:
        return
    rows_total = ROWS * world
    traffic = profiled_traffic()
    line = {
        "metric": METRIC,
        "value": rows_total / (ms_per_step * 1e-3),
        "unit": "rows/s",
        "n_gpus": world,
        "steps": K,
        "warmup": Wm,
        "ms_per_step": ms_per_step,
        "us_per_step_p50": statistics.median(per_step_us) if per_step_us else None,
        "us_per_step_p90": float(np.percentile(per_step_us, 90)) if per_step_us else None,
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
            "traffic": traffic,
            "traffic_source": (f"{PROFILE.relative_to(REPO)} (ncu capture of this kernel on this workload; "
                               "not measured in this run)") if traffic else None,
        },
        "config5_strong": c5,
        "e2e": {
            "value": rows_total / (e2e_ms * 1e-3),
            "unit": "rows/s",
            "ms_per_step": e2e_ms,
            "h2d_bytes_per_step": ROWS * VOCAB * 4 + packed_bytes,
            "d2h_bytes_per_step": rows_total * 4,
            "path": "Sampler.sample(host-pinned logits copied in, Python params/histories packed) + ids .cpu()",
        },
        "e2e_store": {
            "value": rows_total / (store_ms * 1e-3),
            "unit": "rows/s",
            "ms_per_step": store_ms,
            "h2d_bytes_per_step": store_h2d,
            "d2h_bytes_per_step": rows_total * 4,
            "path": ("HistoryStore.sample(logits resident in HBM, histories on the device, row params packed and "
                     "uploaded) + ids .cpu(): the engine-side path"),
        },
        # one row-kernel launch per step
        "gpu_launches": K,
        "clocks": clocks.summary(),
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)


def run_config5(torch, dist, world, rank, dev, NS, packing, sampler_mod, sharded, stream, sms, steps: int = 20):
    """BASELINE config 5 at this N: 16384 rows in contiguous blocks, one per
    rank (generated in place), one all-gather of int32 ids per step.  Returns
    the max-over-ranks step time and rows/s (strong scaling: total rows fixed)."""
    lo, hi = sharded.shard_bounds(C5_ROWS, world, rank)
    n = hi - lo
    blk = sharded.block_rows(C5_ROWS, world)
    params, hist = make_host_workload(10_000 + rank, rows=n, lo=128, hi=1024)
    pk = packing.pack(params, hist, VOCAB, sms=sms)
    rp, off, ids, order = sampler_mod.upload_packed(pk, dev)
    x = make_device_logits(torch, dev, 1, n, 777 + rank)[0]
    s = NS.Sampler(dev)
    buf = torch.zeros(blk, dtype=torch.int32, device=dev)
    gath = torch.empty(blk * world, dtype=torch.int32, device=dev) if world > 1 else None

    def step(k):
        s.sample_packed(x, rp, off, ids, out=buf[:n], seed=99, offset=k, row_offset=lo, row_order=order)
        if world > 1:
            dist.all_gather_into_tensor(gath, buf)

    with torch.cuda.stream(stream):
        for k in range(3):
            step(k)
    torch.cuda.synchronize()
    g = capture(torch, stream, step, steps)
    torch.cuda.synchronize()
    g.replay()
    ms = graph_time(torch, stream, [g], dist, world, dev) / steps
    algo = C5_ROWS * VOCAB * 4 + int(pk.ids.nbytes) * world
    del g
    torch.cuda.synchronize()
    gc.collect()
    return {"rows": C5_ROWS, "rows_per_gpu": n, "ms_per_step": ms, "rows_per_s": C5_ROWS / (ms * 1e-3),
            "hbm_gbs_per_gpu": algo / world / (ms * 1e-3) / 1e9,
            "timing": f"{steps} CUDA-graph-captured steps incl. the all-gather, max over ranks",
            "scaling": "strong"}


# ---------------------------------------------------------------- reference arm
def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    K, Wm = args.steps, max(3, args.warmup)
    budget = 150.0 / (K + Wm)  # the whole run within a few minutes
    try:
        n = reference_rows_per_step(budget)
        ref = ReferenceCPU(n)
        for _ in range(Wm):
            ref.step()
        el = sum(ref.step() for _ in range(K))
        val = ref.rows * K / el
        base = {"value": val, "unit": "rows/s", "cores": ref.threads, "kind": "reference",
                "sample": f"{ref.rows} config-2 rows per step (every parameter kind); the reference "
                          f"Sampler.sample on CPU torch with {ref.threads} threads ({ref.source}); {cpu_model()}"}
        rows_per_step = ref.rows
    except FileNotFoundError:
        import multiprocessing as mp

        cores = os.cpu_count() or 1
        with mp.get_context("spawn").Pool(cores) as pool:
            per_row = max(pool.map(_port_rows, [(0, 2, 3)] * min(cores, 4))) / 2
            rows_per_step = int(max(1, min(ROWS, budget / per_row * cores)))
            chunks = max(1, min(cores, rows_per_step))

            def one_step(k):
                base_row = (k * rows_per_step) % ROWS
                bounds = np.linspace(0, rows_per_step, chunks + 1).astype(int)
                jobs = [(base_row + int(a), base_row + int(b), 100 + k) for a, b in zip(bounds[:-1], bounds[1:])
                        if b > a]
                pool.map(_port_rows, jobs)

            for k in range(Wm):
                one_step(k)
            t0 = time.perf_counter()
            for k in range(K):
                one_step(k)
            el = time.perf_counter() - t0
        val = rows_per_step * K / el
        base = {"value": val, "unit": "rows/s", "cores": cores, "kind": "port",
                "sample": f"{rows_per_step} config-2 rows per step over {cores} processes; numpy restatement "
                          f"(oracle/_ref absent); {cpu_model()}"}
    line = {
        "metric": METRIC, "value": val, "unit": "rows/s", "n_gpus": world, "steps": K, "warmup": Wm,
        "ms_per_step": el / K * 1000.0, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic", "impl": "reference",
        "config": {"workload": WORKLOAD, "rows_per_step": rows_per_step, "vocab": VOCAB},
        "cpu_baseline": base,
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
