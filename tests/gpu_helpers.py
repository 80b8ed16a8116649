"""Shared helpers for the GPU parity tests (test infrastructure).

``run_cabi`` drives the library through the C ABI (ctypes, raw device
pointers); ``compare`` checks its outputs against the numpy oracle with the
tolerances the tests state.
"""
from __future__ import annotations

import importlib
from dataclasses import dataclass, field
from typing import List, Optional

import numpy as np
import torch

from oracle import sampler_oracle as O

PKG = "nanoserve---custom-llm-inference-engine_b200"
cabi = importlib.import_module(PKG + "._cabi")
packing = importlib.import_module(PKG + ".packing")

PROB_TOL = 1e-6       # |p_gpu - p_oracle| in fp32
DRAW_BAND = 1e-6      # uniforms this close to a CDF step may pick a neighbour
# A top-p decision whose deciding cumulative mass lies within TOPP_BAND of the
# float32 boundary may differ between two correct implementations (the GPU
# sums 2^-44 fixed-point masses of fp32 exponentials, the oracle float64).
TOPP_BAND = 2e-7

# The kernel run_cabi asks for ("auto", "cluster" or "split"); the parity
# modules' fixtures run every case through both kernels.
KERNEL = {"name": "auto"}
_WS = {}


def workspace(device, rows: int) -> torch.Tensor:
    """A zeroed workspace for ns_sample (kept per device; every call leaves it zero)."""
    need = cabi.ns_workspace_bytes(rows)
    t = _WS.get(str(device))
    if t is None or t.numel() < need:
        t = torch.zeros(need, dtype=torch.uint8, device=device)
        _WS[str(device)] = t
    return t


def make_sampler(device):
    """The drop-in Sampler on the kernel the current test asks for."""
    ns = importlib.import_module(PKG)
    return ns.Sampler(device, kernel=KERNEL["name"])


def to_bf16_tensor(x: np.ndarray, device) -> torch.Tensor:
    return torch.from_numpy(x).to(device).to(torch.bfloat16)


def prepare_cabi(logits: torch.Tensor, params, histories, uniforms: Optional[np.ndarray] = None,
                 sample_indices: Optional[np.ndarray] = None, debug: bool = True, out_i32: bool = False,
                 seed: int = 1234, offset: int = 0, row_offset: int = 0,
                 row_order: Optional[torch.Tensor] = None, kernel: Optional[str] = None) -> dict:
    """The NsSampleArgs of one call (``"a"``) with the device tensors it points to."""
    dev = logits.device
    V = logits.shape[1]
    S = len(params)
    pk = packing.pack(params, histories, V)
    t = {}
    t["rp"] = torch.from_numpy(pk.row_params.view(np.uint8).copy()).to(dev)
    t["off"] = torch.from_numpy(pk.offsets.copy()).to(dev)
    t["ids"] = torch.from_numpy(pk.ids.copy() if pk.ids.size else np.zeros(1, np.int32)).to(dev)
    t["uni"] = torch.from_numpy(np.asarray(uniforms, dtype=np.float32)).to(dev) if uniforms is not None else None
    t["si"] = (torch.from_numpy(np.asarray(sample_indices, dtype=np.int64)).to(dev)
               if sample_indices is not None else None)
    t["out"] = torch.full((S,), -7, dtype=torch.int32 if out_i32 else torch.int64, device=dev)
    for key in ("pen", "filt", "probs"):
        t[key] = torch.full((S, V), np.nan, dtype=torch.float32, device=dev) if debug else None
    t["status"] = torch.zeros(1, dtype=torch.int32, device=dev)
    ws = workspace(dev, S)
    a = cabi.NsSampleArgs()
    a.logits = logits.data_ptr()
    a.logits_dtype = cabi.NS_DTYPE_BF16 if logits.dtype == torch.bfloat16 else cabi.NS_DTYPE_F32
    a.vocab_size = V
    a.num_logit_rows = logits.shape[0]
    a.logits_row_stride = V if logits.shape[0] == 1 else logits.stride(0)
    a.num_rows = S
    a.out_dtype = cabi.NS_OUT_I32 if out_i32 else cabi.NS_OUT_I64
    a.sample_indices = t["si"].data_ptr() if t["si"] is not None else None
    a.row_params = t["rp"].data_ptr()
    a.history_offsets = t["off"].data_ptr()
    a.history_ids = t["ids"].data_ptr()
    a.uniforms = t["uni"].data_ptr() if t["uni"] is not None else None
    a.philox_seed = seed
    a.philox_offset = offset
    a.row_offset = row_offset
    a.out_tokens = t["out"].data_ptr()
    a.out_penalized = t["pen"].data_ptr() if debug else None
    a.out_filtered = t["filt"].data_ptr() if debug else None
    a.out_probs = t["probs"].data_ptr() if debug else None
    a.status = t["status"].data_ptr()
    a.row_order = row_order.data_ptr() if row_order is not None else None
    a.kernel = {"auto": cabi.NS_KERNEL_AUTO, "cluster": cabi.NS_KERNEL_CLUSTER,
                "split": cabi.NS_KERNEL_SPLIT}[kernel or KERNEL["name"]]
    a.workspace = ws.data_ptr()
    a.workspace_bytes = ws.numel()
    t["a"] = a
    t["ws"] = ws
    t["row_order"] = row_order
    return t


def run_cabi(logits: torch.Tensor, params, histories, uniforms: Optional[np.ndarray] = None,
             sample_indices: Optional[np.ndarray] = None, debug: bool = True, out_i32: bool = False,
             seed: int = 1234, offset: int = 0, row_offset: int = 0,
             row_order: Optional[torch.Tensor] = None, entry: str = "ns_sample", kernel: Optional[str] = None):
    """One ns_sample (or ``entry``) call through ctypes; returns numpy outputs."""
    dev = logits.device
    t = prepare_cabi(logits, params, histories, uniforms, sample_indices, debug, out_i32, seed, offset, row_offset,
                     row_order, kernel)
    getattr(cabi, entry)(t["a"], torch.cuda.current_stream(dev).cuda_stream)
    torch.cuda.synchronize(dev)
    res = dict(tokens=t["out"].cpu().numpy().astype(np.int64), status=int(t["status"].item()))
    if debug:
        res.update(penalized=t["pen"].cpu().numpy(), filtered=t["filt"].cpu().numpy(),
                   probs=t["probs"].cpu().numpy())
    return res


@dataclass
class Report:
    rows: int = 0
    topp_band_rows: int = 0
    draw_band_rows: int = 0
    failures: List[str] = field(default_factory=list)

    def fail(self, msg: str) -> None:
        if len(self.failures) < 20:
            self.failures.append(msg)


def oracle_rows(rows_fp32: np.ndarray, params, histories, uniforms) -> list:
    """The oracle's result for every row (reusable across comparisons)."""
    return [O.sample_row(rows_fp32[i], params[i], histories[i], float(uniforms[i])) for i in range(len(params))]


def compare(gpu: dict, rows_fp32: np.ndarray, params, histories, uniforms, check_tokens: bool = True,
            expected: Optional[list] = None) -> Report:
    """Row-by-row comparison of GPU outputs with the oracle (``expected``:
    precomputed ``oracle_rows`` of the same inputs)."""
    rep = Report()
    for i in range(len(params)):
        rep.rows += 1
        res = expected[i] if expected is not None else O.sample_row(rows_fp32[i], params[i], histories[i],
                                                                    float(uniforms[i]))
        V = rows_fp32.shape[1]
        # penalty: bit-exact (sampler.py:31-38)
        if "penalized" in gpu:
            g = gpu["penalized"][i]
            if not np.array_equal(g.view(np.uint32), res.penalized.view(np.uint32)):
                bad = np.nonzero(g.view(np.uint32) != res.penalized.view(np.uint32))[0]
                rep.fail(f"row {i}: penalized differs at {bad[:5]} (gpu {g[bad[:3]]}, oracle {res.penalized[bad[:3]]})")
        if res.degenerate:
            if "probs" in gpu and np.max(np.abs(gpu["probs"][i] - 1.0 / V)) > PROB_TOL:
                rep.fail(f"row {i}: degenerate row probs not uniform")
            if check_tokens and res.greedy and gpu["tokens"][i] != res.token:
                rep.fail(f"row {i}: degenerate greedy token {gpu['tokens'][i]} != {res.token}")
            if check_tokens and not res.greedy:
                want = min(V - 1, int(float(uniforms[i]) * V))
                if gpu["tokens"][i] != want:
                    rep.fail(f"row {i}: degenerate sampled token {gpu['tokens'][i]} != {want}")
            continue
        in_band = res.topp_margin < TOPP_BAND
        rep.topp_band_rows += int(in_band)
        same_set = True
        if "filtered" in gpu:
            gf = gpu["filtered"][i]
            gk = gf > -np.inf
            ok = res.filtered > -np.inf
            same_set = np.array_equal(gk, ok)
            if not same_set and not in_band:
                rep.fail(f"row {i}: kept set differs (gpu {gk.sum()}, oracle {ok.sum()}, margin {res.topp_margin:.2e})")
            if same_set and not np.array_equal(gf.view(np.uint32), res.filtered.view(np.uint32)):
                bad = np.nonzero(gf.view(np.uint32) != res.filtered.view(np.uint32))[0]
                rep.fail(f"row {i}: filtered values differ at {bad[:5]}")
            if not same_set and in_band and abs(int(gk.sum()) - int(ok.sum())) > 2:
                rep.fail(f"row {i}: in-band kept sizes too far apart ({gk.sum()} vs {ok.sum()})")
        if "probs" in gpu and same_set:
            d = np.max(np.abs(gpu["probs"][i] - res.probs))
            if d > PROB_TOL:
                rep.fail(f"row {i}: probs differ by {d:.3e}")
        if check_tokens:
            if res.greedy:
                if gpu["tokens"][i] != res.token:
                    rep.fail(f"row {i}: greedy token {gpu['tokens'][i]} != {res.token}")
            elif same_set and not ("filtered" not in gpu and in_band):
                if res.draw_margin > DRAW_BAND:
                    if gpu["tokens"][i] != res.token:
                        rep.fail(f"row {i}: sampled token {gpu['tokens'][i]} != {res.token} (u={uniforms[i]})")
                else:
                    rep.draw_band_rows += 1
    return rep
