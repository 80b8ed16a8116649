"""Host-side packing of per-request sampling inputs for the C ABI.

Turns ``List[SamplingParams]`` and ``List[List[int]]`` histories into the
``NsRowParams`` byte array and the int32 CSR history arrays of
``include/nanoserve_sampler.h``.  The Python-double comparisons that decide
which filters run are made here exactly as the reference makes them:

* temperature divisor ``max(t, 1e-6) if t > 0 else 1.0`` and greedy flag
  ``t == 0.0`` (nanoserve/scheduler/sampler.py:41-50);
* top-k on iff ``0 < top_k < vocab`` (sampler.py:55);
* top-p on iff ``top_p < 1.0`` (sampler.py:63);
* repetition penalty on iff ``rp != 1.0`` and the history is non-empty
  (sampler.py:33).  Only those rows' histories are shipped, and their ids
  must lie in ``[0, vocab)``; otherwise ``IndexError`` is raised, as the
  reference's ``index_select`` does (sampler.py:35).
"""
from __future__ import annotations

import itertools
from dataclasses import dataclass
from typing import Optional, Sequence

import numpy as np

from . import _cabi

ROW_DTYPE = np.dtype(
    [
        ("temperature", "<f4"),
        ("top_p", "<f4"),
        ("repetition_penalty", "<f4"),
        ("top_k", "<i4"),
        ("flags", "<u4"),
        ("reserved", "<u4"),
        ("seed", "<u8"),
    ]
)
assert ROW_DTYPE.itemsize == 32


def derive_row(p, vocab: int, hist_len: int) -> tuple:
    """One NsRowParams record from one SamplingParams-like object."""
    t = p.temperature
    temp = max(t, 1e-6) if t > 0 else 1.0
    flags = 0
    if t == 0.0:
        flags |= _cabi.NS_ROW_GREEDY
    k = p.top_k
    k_eff = int(k) if (k > 0 and k < vocab) else 0
    if p.top_p < 1.0:
        flags |= _cabi.NS_ROW_TOP_P
    rp = p.repetition_penalty
    if rp != 1.0 and hist_len > 0:
        flags |= _cabi.NS_ROW_PENALTY
    seed = getattr(p, "seed", None)
    seed_u64 = 0
    if seed is not None:
        flags |= _cabi.NS_ROW_SEED
        seed_u64 = int(seed) & 0xFFFFFFFFFFFFFFFF
    top_p32 = np.float32(p.top_p) if p.top_p < 1.0 else np.float32(1.0)
    return (np.float32(temp), top_p32, np.float32(rp), k_eff, flags, 0, seed_u64)


@dataclass
class Packed:
    """Packed host arrays, all little-endian numpy."""

    row_params: np.ndarray  # ROW_DTYPE [S]
    offsets: np.ndarray     # int64 [S+1]
    ids: np.ndarray         # int32 [N]

    @property
    def num_rows(self) -> int:
        return int(self.row_params.shape[0])


def pack(params: Sequence, histories: Sequence[Sequence[int]], vocab: int) -> Packed:
    S = len(params)
    if len(histories) < S:
        raise IndexError("history_token_ids has fewer entries than sampling_params_list")
    rows = np.empty(S, dtype=ROW_DTYPE)
    active = []
    lens = np.zeros(S, dtype=np.int64)
    for i, p in enumerate(params):
        h = histories[i]
        rec = derive_row(p, vocab, len(h))
        rows[i] = rec
        if rec[4] & _cabi.NS_ROW_PENALTY:
            active.append(h)
            lens[i] = len(h)
    offsets = np.zeros(S + 1, dtype=np.int64)
    np.cumsum(lens, out=offsets[1:])
    total = int(offsets[-1])
    if total:
        ids64 = np.fromiter(itertools.chain.from_iterable(active), dtype=np.int64, count=total)
        lo, hi = int(ids64.min()), int(ids64.max())
        if lo < 0 or hi >= vocab:
            bad = lo if lo < 0 else hi
            raise IndexError(f"history token id {bad} is out of range for vocab size {vocab}")
        ids = ids64.astype(np.int32)
    else:
        ids = np.zeros(0, dtype=np.int32)
    return Packed(rows, offsets, ids)


def layout(packed: Packed) -> tuple[int, int, int, int]:
    """Byte offsets of (row_params, offsets, ids) in one staging buffer, and its size."""
    a = 0
    b = (a + packed.row_params.nbytes + 15) & ~15
    c = (b + packed.offsets.nbytes + 15) & ~15
    end = (c + packed.ids.nbytes + 15) & ~15
    return a, b, c, max(end, 16)


def to_bytes(packed: Packed, out: Optional[np.ndarray] = None) -> np.ndarray:
    """Serialise into one uint8 buffer (row_params | offsets | ids)."""
    a, b, c, end = layout(packed)
    if out is None:
        out = np.zeros(end, dtype=np.uint8)
    out[a : a + packed.row_params.nbytes] = packed.row_params.view(np.uint8)
    out[b : b + packed.offsets.nbytes] = packed.offsets.view(np.uint8)
    out[c : c + packed.ids.nbytes] = packed.ids.view(np.uint8)
    return out
