"""Golden vectors from the REFERENCE sampler (run in the build container only).

Imports ``nanoserve.scheduler.sampler.Sampler`` from a reference checkout
(``--ref PATH``, else ``$NANOSERVE_REF``; one of them is required), runs it
on CPU torch on
every case of ``cases.py`` and stores, per row, what the reference leaves
observable:

* the penalised logits it writes back into its input (sampler.py:38),
* the filtered logits handed to the final softmax (sampler.py:76),
* the final probabilities handed to ``torch.multinomial`` (sampler.py:87),
* the returned token, with ``torch.multinomial`` replaced by an inverse CDF
  over those probabilities driven by the case's uniforms (greedy rows return
  the reference's own argmax, sampler.py:88),
* inverse-CDF tokens for 8 more uniforms per row.

Large arrays are stored as hashes plus values at probe indices, so the
fixture stays small.  Usage: ``python tests/golden/make_golden.py --ref PATH``.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import cases as C  # noqa: E402

REF = None  # the reference checkout, set by main()


def load_reference():
    sys.path.insert(0, str(REF))
    from nanoserve.scheduler.sampler import Sampler  # type: ignore

    return Sampler


def inverse_cdf(probs: np.ndarray, u: float) -> tuple[int, float]:
    cdf = np.cumsum(probs.astype(np.float64))
    tot = cdf[-1]
    t = float(u) * tot
    tok = int(np.searchsorted(cdf, t, side="right"))
    if tok >= len(probs):
        tok = int(np.nonzero(probs > 0)[0][-1])
    lo = cdf[tok - 1] if tok > 0 else 0.0
    return tok, float(min(cdf[tok] - t, t - lo) / tot)


def run_reference(Sampler, case: C.Case):
    cap = {}
    orig_mult, orig_softmax = torch.multinomial, torch.softmax

    def fake_multinomial(probs, num_samples=1, **kw):
        cap["probs"] = probs.detach().clone()
        toks = [inverse_cdf(probs[i].numpy(), case.uniforms[i])[0] for i in range(probs.shape[0])]
        return torch.tensor(toks, dtype=torch.long).unsqueeze(1)

    def rec_softmax(x, dim=None, **kw):
        if x.dim() == 2:
            cap["filtered"] = x.detach().clone()
        return orig_softmax(x, dim=dim, **kw)

    logits = torch.from_numpy(case.logits.copy())
    torch.multinomial, torch.softmax = fake_multinomial, rec_softmax
    try:
        out = Sampler(torch.device("cpu")).sample(logits, case.params, case.histories)
    finally:
        torch.multinomial, torch.softmax = orig_mult, orig_softmax
    return logits.numpy(), cap["filtered"].numpy(), cap["probs"].numpy(), out.numpy()


def main() -> None:
    Sampler = load_reference()
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    store = {}
    for case in C.build_cases():
        pen, filt, probs, toks = run_reference(Sampler, case)
        R, V = case.logits.shape
        g = f"{case.name}/"
        store[g + "input_hash"] = np.array([C.row_hash(case.logits[i]) for i in range(R)])
        store[g + "pen_hash"] = np.array([C.row_hash(pen[i]) for i in range(R)])
        store[g + "filt_hash"] = np.array([C.row_hash(filt[i]) for i in range(R)])
        store[g + "tokens"] = toks.astype(np.int64)
        kept = (filt > -np.inf).sum(1)
        store[g + "kept"] = kept.astype(np.int64)
        # torch.sort is unstable on CPU, so which members of a group of equal
        # values survive at the top-p boundary is implementation-defined.
        # Record the boundary value, how many of its copies were kept, and a
        # hash of the filtered row with that value's positions blanked.
        thr = np.zeros(R, dtype=np.float32)
        n_at = np.zeros(R, dtype=np.int64)
        blank_hash = []
        for i in range(R):
            f = filt[i]
            fin = f[f > -np.inf]
            t = np.float32(fin.min()) if fin.size and not np.isnan(fin).any() else np.float32(np.nan)
            thr[i] = t
            temp = np.float32(max(case.params[i].temperature, 1e-6) if case.params[i].temperature > 0 else 1.0)
            s_ref = (pen[i] / temp).astype(np.float32)
            n_at[i] = int((f == t).sum())
            b = f.copy()
            b[(s_ref == t) | (f == t)] = 0.0
            blank_hash.append(C.row_hash(b))
        store[g + "thr"] = thr
        store[g + "n_at_thr"] = n_at
        store[g + "blank_hash"] = np.array(blank_hash)
        # penalised values that changed (sparse)
        ch_rows, ch_ids, ch_vals = [], [], []
        for i in range(R):
            diff = np.nonzero(pen[i].view(np.uint32) != case.logits[i].view(np.uint32))[0]
            ch_rows += [i] * len(diff)
            ch_ids += diff.tolist()
            ch_vals += pen[i, diff].tolist()
        store[g + "pen_rows"] = np.array(ch_rows, dtype=np.int64)
        store[g + "pen_ids"] = np.array(ch_ids, dtype=np.int64)
        store[g + "pen_vals"] = np.array(ch_vals, dtype=np.float32)
        # probabilities at probe indices: top 64 by filtered value, 64 random
        rng = np.random.default_rng(5)
        probe = np.zeros((R, 128), dtype=np.int64)
        for i in range(R):
            f = np.where(np.isnan(filt[i]), np.inf, filt[i])
            top = np.argsort(-f, kind="stable")[:64]
            probe[i, :64] = top
            probe[i, 64:] = rng.integers(0, V, 64)
        store[g + "probe_idx"] = probe
        store[g + "probe_probs"] = np.take_along_axis(probs, probe, axis=1).astype(np.float32)
        store[g + "probe_filt"] = np.take_along_axis(filt, probe, axis=1).astype(np.float32)
        store[g + "prob_sum"] = probs.astype(np.float64).sum(1)
        # inverse-CDF tokens for extra uniforms and the distance to the nearest step
        dt = np.zeros((R, 8), dtype=np.int64)
        dm = np.zeros((R, 8), dtype=np.float64)
        for i in range(R):
            for j in range(8):
                dt[i, j], dm[i, j] = inverse_cdf(probs[i], case.draw_uniforms[i, j])
        store[g + "draw_tokens"] = dt
        store[g + "draw_margin"] = dm
        print(f"{case.name}: {R} rows, kept {kept.tolist()}")
    meta = dict(torch=torch.__version__, cpu_capability=torch.backends.cpu.get_cpu_capability(),
                threads=torch.get_num_threads())
    store["meta"] = np.array([f"{k}={v}" for k, v in meta.items()])
    np.savez_compressed(HERE / "reference_sampler.npz", **store)
    print("wrote", HERE / "reference_sampler.npz", meta)


if __name__ == "__main__":
    import argparse

    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("NANOSERVE_REF"),
                    help="reference checkout (default: $NANOSERVE_REF)")
    ref = ap.parse_args().ref
    if not ref:
        ap.error("give the reference checkout with --ref or $NANOSERVE_REF")
    REF = Path(ref)
    main()
