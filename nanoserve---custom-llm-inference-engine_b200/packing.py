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

A request with a ``seed`` (nanoserve/config.py:79, which the reference
ignores) gets its own Philox key and, as the counter, the length of its
history (prompt plus tokens so far): the same request in the same state
draws the same number whatever batch it is in.

It also builds the optional row order (``NsSampleArgs.row_order``), a
scheduling hint that starts the rows with the longest finishing work first.
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
        ("seed_step", "<u4"),
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
    step = 0
    if seed is not None:
        flags |= _cabi.NS_ROW_SEED
        seed_u64 = int(seed) & 0xFFFFFFFFFFFFFFFF
        step = int(hist_len) & 0xFFFFFFFF
    top_p32 = np.float32(p.top_p) if p.top_p < 1.0 else np.float32(1.0)
    return (np.float32(temp), top_p32, np.float32(rp), k_eff, flags, step, seed_u64)


def derive_rows(params: Sequence, vocab: int, hist_lens) -> np.ndarray:
    """``derive_row`` for every row at once (ROW_DTYPE [S]), bit for bit the
    same records: the comparisons run on float64 arrays, as Python compares
    floats, and each value is rounded to float32 once."""
    S = len(params)
    rows = np.zeros(S, dtype=ROW_DTYPE)
    if S == 0:
        return rows
    t = np.array([p.temperature for p in params], dtype=np.float64)
    tp = np.array([p.top_p for p in params], dtype=np.float64)
    rp = np.array([p.repetition_penalty for p in params], dtype=np.float64)
    lens = np.asarray(hist_lens, dtype=np.int64)
    with np.errstate(invalid="ignore"):
        rows["temperature"] = np.where(t > 0, np.maximum(t, 1e-6), 1.0).astype(np.float32)
        rows["top_p"] = np.where(tp < 1.0, tp, 1.0).astype(np.float32)
        rows["repetition_penalty"] = rp.astype(np.float32)
        flags = np.where(t == 0.0, _cabi.NS_ROW_GREEDY, 0) | np.where(tp < 1.0, _cabi.NS_ROW_TOP_P, 0)
        flags |= np.where((rp != 1.0) & (lens > 0), _cabi.NS_ROW_PENALTY, 0)
    rows["top_k"] = [int(k) if (k > 0 and k < vocab) else 0 for k in (p.top_k for p in params)]
    seeds = [getattr(p, "seed", None) for p in params]
    if any(sd is not None for sd in seeds):
        seeded = np.array([sd is not None for sd in seeds])
        flags |= np.where(seeded, _cabi.NS_ROW_SEED, 0)
        rows["seed"] = [int(sd) & 0xFFFFFFFFFFFFFFFF if sd is not None else 0 for sd in seeds]
        rows["seed_step"] = np.where(seeded, lens & 0xFFFFFFFF, 0).astype(np.uint32)
    rows["flags"] = flags
    return rows


# Relative cost of a row on the row kernel: greedy rows stream once and only
# track the maximum, top-k <= 128 rows also keep a candidate list and sort it,
# plain sampling re-reads the row for its draw, top-p rows stream twice (the
# boundary window is collected on a second pass) and rank the window's
# members, large top-k rows re-read the row several times.
TOPK_LIST_MAX = 128
COST_GREEDY, COST_TOPK, COST_PLAIN, COST_TOPP, COST_LARGE_K = 1, 3, 5, 7, 8


def row_costs(row_params: np.ndarray) -> np.ndarray:
    """Cost class of every packed row (larger = longer finishing work)."""
    flags = row_params["flags"]
    k = row_params["top_k"]
    greedy = (flags & _cabi.NS_ROW_GREEDY) != 0
    topp = (flags & _cabi.NS_ROW_TOP_P) != 0
    cost = np.full(row_params.shape[0], COST_PLAIN, dtype=np.int32)
    cost[topp] = COST_TOPP
    cost[k > TOPK_LIST_MAX] = COST_LARGE_K
    cost[(k > 0) & (k <= TOPK_LIST_MAX)] = COST_TOPK
    cost[greedy] = COST_GREEDY
    return cost


def schedule(row_params: np.ndarray, sms: int) -> np.ndarray:
    """Row order for ``NsSampleArgs.row_order``: the most expensive rows first.

    The row kernel's persistent blocks claim rows in this order, one at a
    time, as they finish the previous one (longest-processing-time-first
    list scheduling): the costly rows start at once and the cheap rows fill
    the gaps at the end of the step.  (``sms`` only says that the caller has
    a GPU to schedule for; the order does not depend on its size.)
    """
    S = row_params.shape[0]
    if S == 0 or sms <= 0:
        return np.arange(S, dtype=np.int32)
    return np.argsort(-row_costs(row_params), kind="stable").astype(np.int32)


@dataclass
class Packed:
    """Packed host arrays, all little-endian numpy."""

    row_params: np.ndarray  # ROW_DTYPE [S]
    offsets: np.ndarray     # int64 [S+1]
    ids: np.ndarray         # int32 [N]
    order: Optional[np.ndarray] = None  # int32 [S] row order, or None

    @property
    def num_rows(self) -> int:
        return int(self.row_params.shape[0])


def pack(params: Sequence, histories: Sequence[Sequence[int]], vocab: int, sms: Optional[int] = None) -> Packed:
    """Pack one step's rows; with ``sms`` (the GPU's SM count) also their row order."""
    S = len(params)
    if len(histories) < S:
        raise IndexError("history_token_ids has fewer entries than sampling_params_list")
    hl = np.fromiter((len(histories[i]) for i in range(S)), dtype=np.int64, count=S)
    rows = derive_rows(params, vocab, hl)
    pen = (rows["flags"] & _cabi.NS_ROW_PENALTY) != 0
    lens = np.where(pen, hl, 0)
    active = [histories[i] for i in np.flatnonzero(pen)]
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
    order = schedule(rows, sms) if sms else None
    return Packed(rows, offsets, ids, order)


def layout(packed: Packed) -> tuple[int, int, int, int, int]:
    """Byte offsets of (row_params, offsets, ids, order) in one staging buffer, and its size."""
    a = 0
    b = (a + packed.row_params.nbytes + 15) & ~15
    c = (b + packed.offsets.nbytes + 15) & ~15
    d = (c + packed.ids.nbytes + 15) & ~15
    end = (d + (packed.order.nbytes if packed.order is not None else 0) + 15) & ~15
    return a, b, c, d, max(end, 16)


def to_bytes(packed: Packed, out: Optional[np.ndarray] = None) -> np.ndarray:
    """Serialise into one uint8 buffer (row_params | offsets | ids | order)."""
    a, b, c, d, end = layout(packed)
    if out is None:
        out = np.zeros(end, dtype=np.uint8)
    out[a : a + packed.row_params.nbytes] = packed.row_params.view(np.uint8)
    out[b : b + packed.offsets.nbytes] = packed.offsets.view(np.uint8)
    out[c : c + packed.ids.nbytes] = packed.ids.view(np.uint8)
    if packed.order is not None:
        out[d : d + packed.order.nbytes] = packed.order.view(np.uint8)
    return out
