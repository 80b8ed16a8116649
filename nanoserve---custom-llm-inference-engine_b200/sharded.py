"""Row-sharded sampling across the GPUs of one node.

Rows of one sampling step are independent (nanoserve/scheduler/sampler.py has
no cross-row dependency), so a large batch is split into contiguous row
blocks, one per rank (one process per GPU).  Each rank samples its block
with the single-GPU op -- Philox streams are keyed by the *global* row
index, so results do not depend on the number of ranks -- and one
``all_gather_into_tensor`` of int32 ids (NCCL over NVLink on GPUs) gives
every rank the whole step's tokens.  No logits cross the interconnect.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist


def shard_bounds(total_rows: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous block [lo, hi) of rows for ``rank``; the first ranks take the remainder."""
    if world <= 0 or not (0 <= rank < world):
        raise ValueError("bad world/rank")
    base, rem = divmod(total_rows, world)
    lo = rank * base + min(rank, rem)
    hi = lo + base + (1 if rank < rem else 0)
    return lo, hi


def block_rows(total_rows: int, world: int) -> int:
    """Rows per rank after padding every block to the largest one."""
    return -(-total_rows // world)


class ShardedSampler:
    """Samples this rank's rows and all-gathers everybody's int32 tokens.

    ``local_fn(lo, hi, out)`` must fill ``out`` (int32 [hi-lo], on
    ``device``) with the tokens of global rows [lo, hi); by default it is the
    caller's job to wrap :meth:`Sampler.sample_packed` with
    ``row_offset=lo``.  The collective is the only cross-rank step.
    """

    def __init__(self, device, group: Optional[dist.ProcessGroup] = None):
        self.device = torch.device(device)
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self._buf = None
        self._gather = None

    def bounds(self, total_rows: int) -> tuple[int, int]:
        return shard_bounds(total_rows, self.world, self.rank)

    def step(self, total_rows: int, local_fn: Callable[[int, int, torch.Tensor], None]) -> torch.Tensor:
        blk = block_rows(total_rows, self.world)
        if self._buf is None or self._buf.numel() != blk:
            self._buf = torch.zeros(blk, dtype=torch.int32, device=self.device)
            self._gather = torch.empty(blk * self.world, dtype=torch.int32, device=self.device)
        lo, hi = self.bounds(total_rows)
        if hi > lo:
            local_fn(lo, hi, self._buf[: hi - lo])
        dist.all_gather_into_tensor(self._gather, self._buf, group=self.group)
        # drop the padding of ranks whose block is shorter
        parts = []
        for r in range(self.world):
            rlo, rhi = shard_bounds(total_rows, self.world, r)
            parts.append(self._gather[r * blk : r * blk + (rhi - rlo)])
        return torch.cat(parts)
