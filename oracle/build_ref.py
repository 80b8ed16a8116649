"""Makes the REFERENCE sampler runnable where the reference tree is absent --
TEST INFRASTRUCTURE ONLY: it feeds the CPU baseline of ``bench.py`` and its
``--impl reference`` arm, nothing else.

The reference is Python on torch, so there is nothing to compile.  This
recipe copies, unmodified, the only two reference files its sampler needs --
``nanoserve/config.py`` (SamplingParams) and ``nanoserve/scheduler/sampler.py``
(``Sampler.sample``, the path this repository rebuilds) -- from a reference
checkout into ``oracle/_ref/``, which git ignores (it travels with the built
libraries, it is never committed).  The package ``__init__.py`` files are
written here as empty stand-ins: the reference's own package inits import the
whole engine (scheduler, KV cache, model), which the sampler does not use.
``oracle/_ref/SOURCE.txt`` records where the copies came from and their
SHA-256, so a run can show which reference it timed.

    python oracle/build_ref.py [--ref REFERENCE_CHECKOUT]

The checkout is ``--ref``, else ``$NANOSERVE_REF``, else the
``reference_path`` recorded in ``BASELINE.json``.  Nothing in the product
imports ``oracle/``.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import shutil
from pathlib import Path
from typing import Optional

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
FILES = ("nanoserve/config.py", "nanoserve/scheduler/sampler.py")


def reference_checkout(explicit: Optional[str] = None) -> Optional[Path]:
    """The reference checkout to copy from, or None when none is available."""
    cand = explicit or os.environ.get("NANOSERVE_REF")
    if not cand:
        bj = HERE.parent / "BASELINE.json"
        if bj.exists():
            cand = json.loads(bj.read_text()).get("reference_path")
    if not cand:
        return None
    p = Path(cand)
    return p if all((p / f).is_file() for f in FILES) else None


def build(ref: Optional[str] = None) -> Optional[Path]:
    """Refresh ``oracle/_ref`` from the reference checkout; returns it, or
    None (and leaves any earlier copy alone) when no checkout is present."""
    src = reference_checkout(ref)
    if src is None:
        return None
    tmp = OUT.with_name("_ref.tmp")
    if tmp.exists():
        shutil.rmtree(tmp)
    lines = [f"copied from {src}"]
    for f in FILES:
        dst = tmp / f
        dst.parent.mkdir(parents=True, exist_ok=True)
        shutil.copyfile(src / f, dst)
        lines.append(f"{f} sha256 {hashlib.sha256(dst.read_bytes()).hexdigest()}")
    for pkg in ("nanoserve", "nanoserve/scheduler"):
        (tmp / pkg / "__init__.py").write_text("")
    (tmp / "SOURCE.txt").write_text("\n".join(lines) + "\n")
    if OUT.exists():
        shutil.rmtree(OUT)
    tmp.rename(OUT)
    return OUT


def load_sampler():
    """(Sampler, SamplingParams) of the copied reference, or None if absent."""
    import importlib
    import sys

    if not (OUT / FILES[1]).is_file():
        return None
    if str(OUT) not in sys.path:
        sys.path.insert(0, str(OUT))
    sampler = importlib.import_module("nanoserve.scheduler.sampler")
    config = importlib.import_module("nanoserve.config")
    return sampler.Sampler, config.SamplingParams


def source_note() -> str:
    f = OUT / "SOURCE.txt"
    return f.read_text().strip().replace("\n", "; ") if f.exists() else "absent"


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=None, help="reference checkout (default: $NANOSERVE_REF, BASELINE.json)")
    out = build(ap.parse_args().ref)
    print("built", out if out else "nothing: no reference checkout found")
