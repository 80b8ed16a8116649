"""Deterministic sampling cases shared by the golden-vector script and the tests.

Every case is rebuilt from seeds, so fixtures only store the reference's
outputs (plus a hash of the inputs to catch generator drift).
"""
from __future__ import annotations

import hashlib
import importlib
import sys
from dataclasses import dataclass
from pathlib import Path
from typing import List

import numpy as np

REPO = Path(__file__).resolve().parents[2]
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))
PKG = importlib.import_module("nanoserve---custom-llm-inference-engine_b200")
workloads = importlib.import_module("nanoserve---custom-llm-inference-engine_b200.workloads")
SamplingParams = PKG.SamplingParams


@dataclass
class Case:
    name: str
    logits: np.ndarray          # fp32 [R, V] rows as the reference sampler sees them
    params: list
    histories: List[List[int]]
    uniforms: np.ndarray        # fp32 [R]
    draw_uniforms: np.ndarray   # fp32 [R, 8] extra uniforms for inverse-CDF checks


def row_hash(x: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(x).tobytes()).hexdigest()[:16]


def _extra_uniforms(rows: int, seed: int) -> np.ndarray:
    return np.random.default_rng(1000 + seed).random((rows, 8)).astype(np.float32)


def edge_case(V: int = 4096) -> Case:
    """Hand-built rows that exercise the reference's special cases."""
    rng = np.random.default_rng(7)
    rows, params, hists = [], [], []

    def add(x, p, h=()):
        rows.append(np.asarray(x, dtype=np.float32))
        params.append(p)
        hists.append(list(h))

    base = lambda: (rng.standard_normal(V) * 2.0).astype(np.float32)  # noqa: E731
    # 0: NaN row, greedy -> first NaN index
    x = base(); x[[77, 901]] = np.nan; add(x, SamplingParams(temperature=0.0))
    # 1: NaN row, sampled -> uniform
    x = base(); x[5] = np.nan; add(x, SamplingParams(temperature=1.0, top_k=20))
    # 2: +inf present, greedy -> first +inf
    x = base(); x[[300, 12]] = np.inf; add(x, SamplingParams(temperature=0.0))
    # 3: +inf present, sampled -> uniform
    x = base(); x[1000] = np.inf; add(x, SamplingParams(temperature=0.8, top_p=0.5))
    # 4: all -inf, greedy -> 0
    add(np.full(V, -np.inf), SamplingParams(temperature=0.0))
    # 5: all -inf, sampled -> uniform
    add(np.full(V, -np.inf), SamplingParams(temperature=1.0))
    # 6: some -inf entries, top-p
    x = base(); x[::3] = -np.inf; add(x, SamplingParams(temperature=1.0, top_p=0.8))
    # 7: ties at the top-k threshold are all kept
    x = base(); x[[10, 20, 30, 40]] = 9.0; x[[11, 21]] = 9.5; add(x, SamplingParams(temperature=1.0, top_k=4))
    # 8: top_k >= V (off) and top_k = 0 (off)
    add(base(), SamplingParams(temperature=1.0, top_k=V))
    add(base(), SamplingParams(temperature=1.0, top_k=0))
    # 10: top_p = 1.0 (off), top_p = 0.0 (top-1 only), top_p tiny
    add(base(), SamplingParams(temperature=1.0, top_p=1.0))
    add(base(), SamplingParams(temperature=1.0, top_p=0.0))
    add(base(), SamplingParams(temperature=1.0, top_p=1e-5))
    # 13: negative temperature -> divisor 1, not greedy; tiny t -> 1e-6
    add(base(), SamplingParams(temperature=-0.5, top_k=10))
    add(base() * np.float32(1e-6), SamplingParams(temperature=1e-9, top_k=10))
    # 15: repetition penalty < 1 (boost), with duplicate ids
    x = base(); add(x, SamplingParams(temperature=1.0, top_k=30, repetition_penalty=0.8),
                    [3, 3, 3, 50, 51, 4095, 0, 0])
    # 16: penalty with an empty history -> off
    add(base(), SamplingParams(temperature=1.0, top_p=0.9, repetition_penalty=1.3), [])
    # 17: greedy with top-k and penalty
    x = base(); add(x, SamplingParams(temperature=0.0, top_k=5, repetition_penalty=1.5),
                    list(np.argsort(-x)[:3]))
    # 18: greedy with a tie at the maximum -> first index
    x = base(); x[[17, 2000]] = 20.0; add(x, SamplingParams(temperature=0.0))
    # 19: large top-k with top-p and a low temperature
    add(base(), SamplingParams(temperature=0.3, top_k=1500, top_p=0.97))
    # 20: plain sampling at t=2
    add(base(), SamplingParams(temperature=2.0))
    # 21: penalty hitting zero and negative zero
    x = base(); x[[8, 9]] = [0.0, -0.0]; add(x, SamplingParams(temperature=1.0, top_k=100, repetition_penalty=1.2),
                                             [8, 9, 10])
    R = len(rows)
    u = np.random.default_rng(11).random(R).astype(np.float32)
    return Case("edge", np.stack(rows), params, hists, u, _extra_uniforms(R, 99))


def build_cases() -> List[Case]:
    out = []
    w = workloads.make(1)
    out.append(Case("config1", w.gathered().copy(), w.params, w.histories, w.uniforms, _extra_uniforms(w.num_rows, 1)))
    w = workloads.make(2, rows=16, seed=2)
    out.append(Case("config2_16", w.gathered().copy(), w.params, w.histories, w.uniforms, _extra_uniforms(16, 2)))
    w = workloads.make(3, rows=8, seed=3)
    out.append(Case("config3_8", w.gathered().copy(), w.params, w.histories, w.uniforms,
                    _extra_uniforms(w.num_rows, 3)))
    w = workloads.make(4, rows=8, seed=4)
    out.append(Case("config4_8", w.gathered().copy(), w.params, w.histories, w.uniforms, _extra_uniforms(8, 4)))
    out.append(edge_case())
    return out
