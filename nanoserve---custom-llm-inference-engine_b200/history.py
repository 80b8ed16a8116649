"""Device-resident prior-token histories for the repetition penalty.

The reference's caller rebuilds every running request's history as a Python
list each step -- ``history_token_ids = [req.prompt_token_ids +
req.output_token_ids ...]`` (nanoserve/engine.py:242-246) -- and
``Sampler.sample`` turns each list into an index tensor
(nanoserve/scheduler/sampler.py:34).  That is O(total history tokens) of
Python work per step.  ``HistoryStore`` keeps the ids on the GPU instead:

* ``add(prompt_ids, max_new_tokens)`` reserves a region of one int32 device
  pool for a request and copies its prompt in once;
* ``sample(sampler, logits, params, handles)`` packs the step's row
  parameters on the host (O(rows)), gathers the penalty rows' histories
  into CSR form on the device (``ns_history_gather``), samples, and appends
  each row's sampled id to its request's region (``ns_history_append``) --
  three launches after one small host-to-device copy, no host sync;
* ``release(handle)`` returns the region when the request finishes.

The tokens are identical to ``Sampler.sample`` given the same histories as
lists (same row parameters, same CSR histories, same row order).  No
counterpart in the reference.
"""
from __future__ import annotations

import bisect
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np
import torch

from . import _cabi, packing
from .sampler import Sampler, _Staging, _sm_count


class RegionAllocator:
    """First-fit allocator of [start, start + size) regions in a pool of
    ``capacity`` slots, with holes merged on release (host bookkeeping only)."""

    def __init__(self, capacity: int):
        if capacity < 0:
            raise ValueError("capacity must be >= 0")
        self.capacity = capacity
        self._holes: List[Tuple[int, int]] = [(0, capacity)] if capacity else []  # sorted (start, size)

    def alloc(self, size: int) -> int:
        if size < 0:
            raise ValueError("size must be >= 0")
        for i, (s, n) in enumerate(self._holes):
            if n >= size:
                if n == size:
                    del self._holes[i]
                else:
                    self._holes[i] = (s + size, n - size)
                return s
        raise MemoryError(f"history pool full: no free region of {size} ids (capacity {self.capacity})")

    def free(self, start: int, size: int) -> None:
        if size == 0:
            return
        i = bisect.bisect_left(self._holes, (start, 0))
        self._holes.insert(i, (start, size))
        # merge with the right neighbour, then the left one
        if i + 1 < len(self._holes) and self._holes[i][0] + self._holes[i][1] == self._holes[i + 1][0]:
            self._holes[i] = (self._holes[i][0], self._holes[i][1] + self._holes[i + 1][1])
            del self._holes[i + 1]
        if i > 0 and self._holes[i - 1][0] + self._holes[i - 1][1] == self._holes[i][0]:
            self._holes[i - 1] = (self._holes[i - 1][0], self._holes[i - 1][1] + self._holes[i][1])
            del self._holes[i]

    def free_total(self) -> int:
        return sum(n for _, n in self._holes)


def plan_step(params: Sequence, starts: np.ndarray, lengths: np.ndarray, vocab: int):
    """Row parameters, CSR offsets and per-row pool starts of one step.

    Row i's history is ``lengths[i]`` ids at pool position ``starts[i]``.  As in
    ``packing.pack``, only rows with the penalty on carry ids (the others get
    an empty range).  Returns (rows, offsets int64 [S+1], src int64 [S])."""
    S = len(params)
    lengths = np.asarray(lengths, dtype=np.int64)
    rows = packing.derive_rows(params, vocab, lengths)
    lens = np.where((rows["flags"] & _cabi.NS_ROW_PENALTY) != 0, lengths, 0)
    offsets = np.zeros(S + 1, dtype=np.int64)
    np.cumsum(lens, out=offsets[1:])
    src = np.asarray(starts, dtype=np.int64).copy()
    return rows, offsets, src


class HistoryStore:
    """Append-only prior-token histories in one int32 device pool."""

    def __init__(self, device, capacity: int, vocab: int):
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise RuntimeError("HistoryStore keeps its pool on a CUDA device (no CPU fallback)")
        _cabi.load_library()
        self.vocab = int(vocab)
        self.capacity = int(capacity)
        self.pool = torch.empty(max(self.capacity, 1), dtype=torch.int32, device=self.device)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._alloc = RegionAllocator(self.capacity)
        self._regions: Dict[int, List[int]] = {}  # handle -> [start, length, reserved]
        self._next = 0
        self._staging = _Staging()
        self._append_staging = _Staging()
        self._ids: Optional[torch.Tensor] = None  # CSR ids of the last step (grown on demand)

    # -- requests -----------------------------------------------------------
    def add(self, prompt_ids: Sequence[int], max_new_tokens: int) -> int:
        """Reserve room for ``len(prompt_ids) + max_new_tokens`` ids and copy the prompt in."""
        ids = np.asarray(prompt_ids, dtype=np.int64).reshape(-1)
        if ids.size and (int(ids.min()) < 0 or int(ids.max()) >= self.vocab):
            bad = int(ids.min()) if int(ids.min()) < 0 else int(ids.max())
            raise IndexError(f"history token id {bad} is out of range for vocab size {self.vocab}")
        if max_new_tokens < 0:
            raise ValueError("max_new_tokens must be >= 0")
        reserved = int(ids.size) + int(max_new_tokens)
        start = self._alloc.alloc(reserved)
        if ids.size:
            host = torch.from_numpy(ids.astype(np.int32)).pin_memory()
            self.pool[start : start + ids.size].copy_(host, non_blocking=True)
        h = self._next
        self._next += 1
        self._regions[h] = [start, int(ids.size), reserved]
        return h

    def release(self, handle: int) -> None:
        start, _, reserved = self._regions.pop(handle)
        self._alloc.free(start, reserved)

    def length(self, handle: int) -> int:
        return self._regions[handle][1]

    def tokens(self, handle: int) -> List[int]:
        """The request's ids as a list (synchronises; for tests and debugging)."""
        start, n, _ = self._regions[handle]
        return self.pool[start : start + n].tolist()

    # -- one step -----------------------------------------------------------
    def pack(self, params: Sequence, handles: Sequence[int], sms: Optional[int] = None):
        """Device (row_params, offsets, ids, order) for ``Sampler.sample_packed``."""
        S = len(params)
        if len(handles) != S:
            raise ValueError(f"{len(handles)} handles for {S} sampling params")
        reg = [self._regions[h] for h in handles]
        starts = np.fromiter((r[0] for r in reg), dtype=np.int64, count=S)
        lengths = np.fromiter((r[1] for r in reg), dtype=np.int64, count=S)
        rows, offsets, src = plan_step(params, starts, lengths, self.vocab)
        order = packing.schedule(rows, sms) if sms else None
        # one staging buffer: rows | offsets | src | order (16-byte aligned parts)
        parts = [rows.view(np.uint8), offsets.view(np.uint8), src.view(np.uint8)]
        if order is not None:
            parts.append(order.view(np.uint8))
        pos, at = [], 0
        for p in parts:
            pos.append(at)
            at = (at + p.nbytes + 15) & ~15
        host = self._staging.get(max(at, 16))
        hb = host.numpy()
        for p, o in zip(parts, pos):
            hb[o : o + p.nbytes] = p
        dev = host.to(self.device, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.device))
        self._staging.event = ev
        row_params = dev[pos[0] : pos[0] + rows.nbytes]
        off_d = dev[pos[1] : pos[1] + offsets.nbytes].view(torch.int64)
        src_d = dev[pos[2] : pos[2] + src.nbytes].view(torch.int64)
        order_d = dev[pos[3] : pos[3] + order.nbytes].view(torch.int32) if order is not None else None
        total = int(offsets[-1])
        if total == 0:
            return row_params, None, None, order_d
        if self._ids is None or self._ids.numel() < total:
            self._ids = torch.empty(max(total, 1 << 16), dtype=torch.int32, device=self.device)
        ids = self._ids[:total]
        _cabi.ns_history_gather(self.pool.data_ptr(), self.capacity, src_d.data_ptr(), off_d.data_ptr(), S,
                                ids.data_ptr(), self.status.data_ptr(), torch.cuda.current_stream(self.device).cuda_stream)
        return row_params, off_d, ids, order_d

    def append(self, handles: Sequence[int], tokens: torch.Tensor) -> None:
        """Append ``tokens[i]`` (device int64 or int32 [S]) to request ``handles[i]``."""
        S = len(handles)
        if tokens.numel() != S or tokens.device != self.device:
            raise ValueError("tokens must be a device tensor with one id per handle")
        if tokens.dtype not in (torch.int64, torch.int32):
            raise ValueError("tokens must be int64 or int32")
        reg = [self._regions[h] for h in handles]
        for h, r in zip(handles, reg):
            if r[1] >= r[2]:
                raise OverflowError(f"request {h} has used all {r[2]} reserved history slots")
        dst = np.fromiter((r[0] + r[1] for r in reg), dtype=np.int64, count=S)
        host = self._append_staging.get(max(dst.nbytes, 16))
        host.numpy()[: dst.nbytes] = dst.view(np.uint8)
        dev = host[: dst.nbytes].to(self.device, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.device))
        self._append_staging.event = ev
        tokens = tokens.contiguous()
        _cabi.ns_history_append(self.pool.data_ptr(), self.capacity, dev.data_ptr(), tokens.data_ptr(),
                                _cabi.NS_OUT_I32 if tokens.dtype == torch.int32 else _cabi.NS_OUT_I64, S,
                                self.status.data_ptr(), torch.cuda.current_stream(self.device).cuda_stream)
        for r in reg:
            r[1] += 1

    def sample(self, sampler: Sampler, logits: torch.Tensor, sampling_params_list: Sequence, handles: Sequence[int],
               *, append: bool = True, **kw):
        """``Sampler.sample`` with the histories taken from this store; the
        sampled ids are appended to the requests' histories (``append``).
        Runs on the store's device (whatever device is current) inside an NVTX
        range named ``logits+sample`` (nanoserve/engine/engine.py:234)."""
        torch.cuda.nvtx.range_push("logits+sample")
        try:
            with torch.cuda.device(self.device):
                rp, off, ids, order = self.pack(sampling_params_list, handles, sms=_sm_count(logits.device))
                out = sampler.sample_packed(logits, rp, off, ids, row_order=order, **kw)
                if append:
                    self.append(handles, out[0] if isinstance(out, tuple) else out)
                return out
        finally:
            torch.cuda.nvtx.range_pop()
