"""CPU oracle for the sampling hot path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline legs of
``bench.py`` may import this package, and only as a checker or as the timed
CPU baseline.  The product path (the ``Sampler`` / C ABI) never calls it.
"""
from .sampler_oracle import (  # noqa: F401
    RowResult,
    argmax_first,
    filtered_row,
    final_probs,
    inverse_cdf,
    penalize,
    sample_batch,
    sample_row,
    scale,
    topk_mask,
    topp_mask,
)
