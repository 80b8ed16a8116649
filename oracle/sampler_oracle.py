"""Numpy restatement of NanoServe's ``Sampler.sample`` -- TEST INFRASTRUCTURE ONLY.

Reference: nanoserve/scheduler/sampler.py:21-89 (reference tree, not copied).
This module is the checker for the CUDA path and the timed CPU baseline; the
product never imports it.

Pinning: the reference has no tests or golden vectors of its own, so this
restatement is pinned against fixtures produced by running the reference
``Sampler.sample`` itself (``tests/golden/make_golden.py`` imports it from
the reference tree and records its outputs; ``tests/test_oracle_golden.py``
checks this module against them).

Arithmetic follows the reference step by step:

* penalty (sampler.py:31-38): on the unique history ids, ``x*rp`` where
  ``x < 0`` else ``x/rp``, IEEE fp32 with ``rp`` rounded to fp32;
* temperature (sampler.py:40-51): ``x / float32(max(t,1e-6))`` for ``t > 0``,
  divisor 1 otherwise; greedy iff ``t == 0.0``;
* top-k (sampler.py:53-58): the k-th largest scaled value is the threshold,
  values strictly below it become ``-inf`` (ties at it are kept);
* top-p (sampler.py:60-73): descending order, softmax, cumulative sum, keep
  rank ``j`` iff ``j == 0`` or ``float32(cum[j-1]) <= float32(top_p)``.  The
  reference sums fp32 softmax terms whose own rounding moves ``cum`` by up to
  a few 1e-7; this oracle sums exact float64 terms and reports, per row, the
  distance (``margin``) of the deciding cumulative masses from the float32
  decision boundary, so that a test can tell decisions that any faithful
  implementation must share from those inside the noise band;
* final softmax and NaN guard (sampler.py:75-80): rows containing NaN, +inf
  or only -inf become uniform ``1/V``;
* greedy (sampler.py:82-83): first index of the maximum (NaN counts as the
  maximum, as in ``torch.argmax``);
* draw (sampler.py:84-89): ``torch.multinomial`` is replaced by an inverse
  CDF over the final probabilities in vocabulary order, driven by a caller
  uniform ``u``: the token is the first index whose cumulative probability
  exceeds ``u`` times the total.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Sequence

import numpy as np

F32 = np.float32


@dataclass
class RowResult:
    penalized: np.ndarray      # fp32 [V]   logits after the penalty (sampler.py:38)
    scaled: np.ndarray         # fp32 [V]   penalized / temperature (sampler.py:51)
    filtered: np.ndarray       # fp32 [V]   after top-k / top-p masks (sampler.py:58,73)
    probs: np.ndarray          # fp32 [V]   final probabilities (sampler.py:76-80)
    argmax: int                # sampler.py:83
    token: int                 # greedy ? argmax : inverse-CDF(u)
    greedy: bool
    degenerate: bool           # NaN/+inf/all -inf row -> uniform
    kept: int                  # number of non-masked entries
    topk_thr: Optional[float]  # k-th largest scaled value (if top-k on)
    topp_margin: float         # distance of the deciding masses from the boundary (inf if off)
    draw_margin: float         # distance of u from the nearest CDF step (normalised)


def derive(p, vocab: int, hist_len: int) -> dict:
    """Per-row derived parameters, with the reference's Python-double tests."""
    t = p.temperature
    return dict(
        temp=F32(max(t, 1e-6) if t > 0 else 1.0),                      # sampler.py:41-46
        greedy=(t == 0.0),                                              # sampler.py:47-50
        topk=(int(p.top_k) if (p.top_k > 0 and p.top_k < vocab) else 0),  # sampler.py:55
        topp_on=(p.top_p < 1.0),                                        # sampler.py:63
        p32=F32(p.top_p) if p.top_p < 1.0 else F32(1.0),
        pen_on=(p.repetition_penalty != 1.0 and hist_len > 0),          # sampler.py:33
        rp32=F32(p.repetition_penalty),
    )


def penalize(x: np.ndarray, hist: Sequence[int], rp32: np.float32) -> np.ndarray:
    """sampler.py:31-38 -- HF repetition penalty on the unique history ids."""
    out = x.copy()
    ids = np.unique(np.asarray(hist, dtype=np.int64))
    if ids.size and (ids[0] < 0 or ids[-1] >= x.shape[0]):
        raise IndexError("history id out of range")
    score = out[ids]
    out[ids] = np.where(score < 0, score * rp32, score / rp32).astype(F32)
    return out


def scale(x: np.ndarray, temp32: np.float32) -> np.ndarray:
    """sampler.py:51 -- fp32 IEEE division by the row's temperature."""
    return (x / temp32).astype(F32)


def topk_mask(s: np.ndarray, k: int) -> tuple[np.ndarray, float]:
    """sampler.py:53-58 -- keep values >= the k-th largest (ties kept)."""
    V = s.shape[0]
    thr = np.partition(s, V - k)[V - k]
    return np.where(s < thr, F32(-np.inf), s).astype(F32), float(thr)


def topp_mask(s: np.ndarray, p32: np.float32) -> tuple[np.ndarray, float]:
    """sampler.py:60-73 -- nucleus filter; returns (masked row, decision margin)."""
    order = np.argsort(-s.astype(np.float64), kind="stable")
    ss = s[order].astype(np.float64)
    e = np.exp(ss - ss[0])
    cum = np.cumsum(e) / e.sum()
    cum32 = cum.astype(F32)
    over = cum32 > p32
    j0 = int(np.argmax(over)) if over.any() else len(s) - 1
    # float32 rounding boundary: fp32(c) > p32  <=>  c > mid
    mid = (float(p32) + float(np.nextafter(p32, F32(np.inf)))) / 2.0
    margin = abs(cum[j0] - mid)
    if j0 >= 1:
        margin = min(margin, abs(cum[j0 - 1] - mid))
    if not over.any():
        margin = abs(cum[-1] - mid)
    keep_sorted = np.zeros(len(s), dtype=bool)
    keep_sorted[: j0 + 1] = True
    keep = np.zeros(len(s), dtype=bool)
    keep[order] = keep_sorted
    return np.where(keep, s, F32(-np.inf)).astype(F32), float(margin)


def is_degenerate(s: np.ndarray) -> bool:
    """sampler.py:76-80: the softmax is NaN for rows with NaN, +inf or only -inf."""
    return bool(np.isnan(s).any() or np.isposinf(s).any() or not (s > -np.inf).any())


def final_probs(s: np.ndarray) -> np.ndarray:
    """sampler.py:76-80 -- softmax over the filtered row; NaN rows -> 1/V."""
    V = s.shape[0]
    if is_degenerate(s):
        return np.full(V, 1.0 / V, dtype=F32)
    d = s.astype(np.float64)
    e = np.exp(d - d.max())
    return (e / e.sum()).astype(F32)


def argmax_first(s: np.ndarray) -> int:
    """sampler.py:83 -- torch.argmax: first maximum, NaN counts as largest."""
    nan = np.isnan(s)
    if nan.any():
        return int(np.argmax(nan))
    return int(np.argmax(s))


def inverse_cdf(probs: np.ndarray, u: float) -> tuple[int, float]:
    """Stands in for sampler.py:87: first index with cdf > u * total."""
    cdf = np.cumsum(probs.astype(np.float64))
    tot = cdf[-1]
    t = float(u) * tot
    tok = int(np.searchsorted(cdf, t, side="right"))
    nz = np.nonzero(probs > 0)[0]
    if tok >= len(probs):
        tok = int(nz[-1])
    hi = cdf[tok]
    lo = cdf[tok - 1] if tok > 0 else 0.0
    return tok, float(min(hi - t, t - lo) / tot)


def filtered_row(x: np.ndarray, p, hist: Sequence[int]) -> tuple:
    """Penalty, temperature, top-k and top-p for one row (sampler.py:31-73)."""
    V = x.shape[0]
    d = derive(p, V, len(hist))
    xp = penalize(x, hist, d["rp32"]) if d["pen_on"] else x.astype(F32).copy()
    s = scale(xp, d["temp"])
    f = s
    thr = None
    if d["topk"]:
        f, thr = topk_mask(f, d["topk"])
    margin = float("inf")
    if d["topp_on"] and not is_degenerate(f):
        f, margin = topp_mask(f, d["p32"])
    return d, xp, s, f, thr, margin


def sample_row(x: np.ndarray, p, hist: Sequence[int], u: float) -> RowResult:
    d, xp, s, f, thr, margin = filtered_row(x, p, hist)
    probs = final_probs(f)
    am = argmax_first(f)
    deg = is_degenerate(f)
    tok, dm = inverse_cdf(probs, u)
    token = am if d["greedy"] else tok
    kept = int((f > -np.inf).sum()) if not deg else x.shape[0]
    return RowResult(xp, s, f, probs, am, token, d["greedy"], deg, kept, thr, margin,
                     float("inf") if d["greedy"] else dm)


def sample_batch(logits: np.ndarray, params: Sequence, histories: Sequence[Sequence[int]],
                 uniforms: Sequence[float]) -> List[RowResult]:
    """The whole of sampler.py:21-89 for fp32 rows, with caller uniforms."""
    return [sample_row(logits[i], params[i], histories[i], float(uniforms[i])) for i in range(len(params))]
