"""Seeded synthetic sampling workloads shaped like the benchmark configurations.

No dataset is involved: logits are Gaussian, optionally with a few boosted
ids per row so that the distribution is peaked, as an LLM head's logits are.

==========  ===============================================================
config 1    fp32 [16, V], N(0, 2^2) + 20 ids boosted by +8 per row; rows
            8..15 sampled; t=0.7, top_k=50, top_p=0.9, rp=1.1; histories of
            U[32,256] ids
config 2    fp32 [256, V], same generator, every row sampled; parameters
            cycle greedy / top_k=50 / top_p=0.9 / (t=0.7,k=50,p=0.9,rp=1.1);
            histories U[128,2048]
config 3    bf16 [4096, V] (16 prefill chunks of 253 rows, then 48 decode
            rows); 64 rows sampled (last row of each chunk + the decode
            rows); t=1.0, top_p=0.95, rp=1.2; histories U[512,4096]
config 4    fp32 [1024, V], N(0, 0.5^2), no peaks; t=1.3, top_p=0.99
config 5    fp32 [16384, V], peaked; config-2 parameters; histories
            U[128,1024]
==========  ===============================================================
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional

import numpy as np

from .config import SamplingParams

VOCAB = 128256


@dataclass
class Workload:
    name: str
    logits: np.ndarray              # fp32 [T, V] (bf16 configs: values already bf16-rounded)
    dtype: str                      # "f32" or "bf16"
    sample_indices: Optional[np.ndarray]  # int64 [S] or None
    params: List[SamplingParams]
    histories: List[List[int]]
    uniforms: np.ndarray            # fp32 [S]

    @property
    def num_rows(self) -> int:
        return len(self.params)

    def gathered(self) -> np.ndarray:
        """The fp32 rows the reference sampler sees (after the gather)."""
        if self.sample_indices is None:
            return self.logits
        return self.logits[self.sample_indices]


def peaked_logits(rng: np.random.Generator, rows: int, vocab: int = VOCAB, sigma: float = 2.0,
                  n_peaks: int = 20, peak: float = 8.0) -> np.ndarray:
    x = rng.standard_normal((rows, vocab), dtype=np.float32)
    x *= np.float32(sigma)
    if n_peaks:
        for r in range(rows):
            ids = rng.choice(vocab, size=n_peaks, replace=False)
            x[r, ids] += np.float32(peak)
    return x


def flat_logits(rng: np.random.Generator, rows: int, vocab: int = VOCAB, sigma: float = 0.5) -> np.ndarray:
    x = rng.standard_normal((rows, vocab), dtype=np.float32)
    x *= np.float32(sigma)
    return x


def to_bf16_values(x: np.ndarray) -> np.ndarray:
    """Round fp32 values to bf16 (nearest-even) and return them as fp32."""
    u = x.view(np.uint32).astype(np.uint64)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return rounded.astype(np.uint32).view(np.float32)


def histories(rng: np.random.Generator, rows: int, lo: int, hi: int, vocab: int = VOCAB) -> List[List[int]]:
    lens = rng.integers(lo, hi + 1, size=rows)
    return [rng.integers(0, vocab, size=int(n)).tolist() for n in lens]


def mixed_params(rows: int) -> List[SamplingParams]:
    out = []
    for i in range(rows):
        kind = i % 4
        if kind == 0:
            out.append(SamplingParams(temperature=0.0))
        elif kind == 1:
            out.append(SamplingParams(temperature=1.0, top_k=50))
        elif kind == 2:
            out.append(SamplingParams(temperature=1.0, top_p=0.9))
        else:
            out.append(SamplingParams(temperature=0.7, top_k=50, top_p=0.9, repetition_penalty=1.1))
    return out


def make(config: int, rows: Optional[int] = None, seed: int = 0, vocab: int = VOCAB) -> Workload:
    """Build BASELINE configuration ``config`` (1..5), optionally with fewer rows."""
    rng = np.random.default_rng(seed)
    if config == 1:
        T = 16 if rows is None else 2 * rows
        x = peaked_logits(rng, T, vocab)
        idx = np.arange(T // 2, T, dtype=np.int64)
        S = len(idx)
        params = [SamplingParams(temperature=0.7, top_k=50, top_p=0.9, repetition_penalty=1.1) for _ in range(S)]
        hist = histories(rng, S, 32, 256, vocab)
        u = np.random.default_rng(0).random(S).astype(np.float32)
        return Workload("config1", x, "f32", idx, params, hist, u)
    if config == 2:
        S = 256 if rows is None else rows
        x = peaked_logits(rng, S, vocab)
        params = mixed_params(S)
        hist = histories(rng, S, 128, 2048, vocab)
        u = rng.random(S).astype(np.float32)
        return Workload("config2", x, "f32", None, params, hist, u)
    if config == 3:
        chunks, chunk_rows, decode = 16, 253, 48
        if rows is not None:
            chunks, decode = max(1, rows // 4), max(1, rows - max(1, rows // 4))
            chunk_rows = 8
        T = chunks * chunk_rows + decode
        x = to_bf16_values(peaked_logits(rng, T, vocab))
        idx = np.concatenate([np.arange(chunks) * chunk_rows + chunk_rows - 1,
                              np.arange(chunks * chunk_rows, T)]).astype(np.int64)
        S = len(idx)
        params = [SamplingParams(temperature=1.0, top_p=0.95, repetition_penalty=1.2) for _ in range(S)]
        hist = histories(rng, S, 512, 4096, vocab)
        u = rng.random(S).astype(np.float32)
        return Workload("config3", x, "bf16", idx, params, hist, u)
    if config == 4:
        S = 1024 if rows is None else rows
        x = flat_logits(rng, S, vocab)
        params = [SamplingParams(temperature=1.3, top_p=0.99) for _ in range(S)]
        hist = [[] for _ in range(S)]
        u = rng.random(S).astype(np.float32)
        return Workload("config4", x, "f32", None, params, hist, u)
    if config == 5:
        S = 16384 if rows is None else rows
        x = peaked_logits(rng, S, vocab)
        params = mixed_params(S)
        hist = histories(rng, S, 128, 1024, vocab)
        u = rng.random(S).astype(np.float32)
        return Workload("config5", x, "f32", None, params, hist, u)
    raise ValueError(f"unknown config {config}")
