"""Per-request sampling knobs, field for field the schema of
nanoserve/config.py:68-79 (``SamplingParams``).

The sampler reads ``temperature`` (:72), ``top_p`` (:73), ``top_k`` (:74),
``repetition_penalty`` (:75) and, unlike the reference, ``seed`` (:79): a
non-None seed gives the row its own Philox key.  Any object with these
attributes is accepted by :class:`Sampler`, including the reference's own
class, so callers do not have to switch types.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional


@dataclass
class SamplingParams:
    """Per-request sampling configuration (same fields and defaults as the reference)."""

    max_tokens: int = 128
    temperature: float = 1.0
    top_p: float = 1.0
    top_k: int = -1
    repetition_penalty: float = 1.0
    stop_token_ids: list = field(default_factory=list)
    stop: list = field(default_factory=list)
    ignore_eos: bool = False
    seed: Optional[int] = None
