"""Drop-in replacement for nanoserve/scheduler/sampler.py (``Sampler``).

``Sampler(device).sample(logits, sampling_params_list, history_token_ids,
generators=None)`` keeps the reference signature (sampler.py:17-27) and
returns int64 token ids on ``logits.device``, so ``engine.py:247-250`` and
``Scheduler.update_with_sampled`` work unchanged.  The work is one call of
the sm_100a library behind ``torch.ops.nanoserve_b200.sample``: one kernel
launch, enqueued on the current stream of ``logits.device``.  The call is
wrapped in an NVTX range named ``logits+sample``, the range the reference's
engine opens around the same step (nanoserve/engine/engine.py:234).

Differences from the reference, all additive:

* the input ``logits`` is never modified (the reference writes the penalised
  logits back into it, sampler.py:38; ``return_debug=True`` returns them);
* keyword-only extensions: ``sample_indices`` (fused row gather from a flat
  ``[T, V]`` fp32/bf16 tensor), ``uniforms`` (one caller uniform per row),
  ``seed`` (Philox key), ``out_dtype`` (int64 or int32);
* randomness comes from per-row Philox4x32-10 streams keyed by
  ``(seed, step, row)`` instead of the global generator that
  ``torch.multinomial`` uses (sampler.py:87); ``SamplingParams.seed``, which
  the reference ignores, gives a request its own stream, keyed by the seed
  and the length of its history, so it draws the same tokens whatever batch
  it is in;
* ``generators`` is accepted and ignored, as in the reference (sampler.py:26);
* ``sample_async`` returns int32 ids through a non-blocking copy to pinned
  host memory (``PendingTokens.wait()``), in place of the caller's blocking
  ``.tolist()`` (engine.py:250).

There is no CPU path: the op raises if the CUDA library is not built or the
tensors are not on a CUDA device.
"""
from __future__ import annotations

from pathlib import Path
from typing import List, Optional, Sequence

import numpy as np
import torch

from . import packing

_PKG_DIR = Path(__file__).resolve().parent
_OPS_PATH = _PKG_DIR / "_nanoserve_ops.so"
_ops_loaded = False


def load_ops() -> None:
    """Register torch.ops.nanoserve_b200.* (raises if the library was not built)."""
    global _ops_loaded
    if _ops_loaded:
        return
    if not _OPS_PATH.exists():
        raise RuntimeError(
            f"{_OPS_PATH} is missing: build it with __graft_entry__.build() "
            "(there is no CPU fallback for the sampling op)"
        )
    torch.ops.load_library(str(_OPS_PATH))
    _ops_loaded = True


class _Staging:
    """A reusable pinned host buffer plus the event of its last H2D copy."""

    def __init__(self) -> None:
        self.host: Optional[torch.Tensor] = None
        self.event: Optional[torch.cuda.Event] = None

    def get(self, nbytes: int) -> torch.Tensor:
        if self.event is not None:
            self.event.synchronize()
        if self.host is None or self.host.numel() < nbytes:
            cap = max(nbytes, 1 << 16)
            self.host = torch.empty(cap, dtype=torch.uint8, pin_memory=True)
        return self.host[:nbytes]


class PendingTokens:
    """Sampled ids on their way to the host: an int32 copy into pinned memory,
    enqueued behind the sampling kernel, and the event that marks its end.
    ``wait()`` blocks until then and returns the ids as a list (what
    ``engine.py:250`` gets from ``.tolist()``)."""

    def __init__(self, host: torch.Tensor, event: torch.cuda.Event, n: int):
        self._host = host
        self._event = event
        self._n = n
        self._ids: Optional[List[int]] = None

    def ready(self) -> bool:
        return self._ids is not None or self._event.query()

    def wait(self) -> List[int]:
        if self._ids is None:
            self._event.synchronize()
            self._ids = self._host[: self._n].numpy().tolist()
        return self._ids


class _HostRing:
    """A few pinned int32 buffers reused round robin for PendingTokens; a
    buffer is handed out again only after its previous copy has finished."""

    def __init__(self, slots: int = 4):
        self._bufs: List[Optional[torch.Tensor]] = [None] * slots
        self._pending: List[Optional[PendingTokens]] = [None] * slots
        self._next = 0

    def copy(self, tokens: torch.Tensor) -> PendingTokens:
        i = self._next
        self._next = (i + 1) % len(self._bufs)
        prev = self._pending[i]
        if prev is not None:
            prev.wait()  # its list is taken before the buffer is reused
        n = tokens.numel()
        if self._bufs[i] is None or self._bufs[i].numel() < n:
            self._bufs[i] = torch.empty(max(n, 1024), dtype=torch.int32, pin_memory=True)
        host = self._bufs[i]
        src = tokens if tokens.dtype == torch.int32 else tokens.to(torch.int32)
        with torch.cuda.device(tokens.device):
            host[:n].copy_(src, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(torch.cuda.current_stream(tokens.device))
        pt = PendingTokens(host, ev, n)
        self._pending[i] = pt
        return pt


KERNELS = {"auto": 0, "cluster": 1, "split": 2}


class Sampler:
    """B200 sampling op with the reference ``Sampler`` interface.

    ``kernel`` picks the CUDA kernel: ``"auto"`` (the row kernel, whose
    persistent blocks split the batch's rows among the SMs, for
    batches of at least 32 aligned rows, the cluster kernel otherwise),
    ``"cluster"`` or ``"split"`` (where its layout conditions hold)."""

    def __init__(self, device, kernel: str = "auto"):
        if kernel not in KERNELS:
            raise ValueError(f"kernel must be one of {sorted(KERNELS)}")
        self.device = torch.device(device)
        self.kernel = kernel
        self._step = 0
        self._staging = _Staging()
        self._ring = _HostRing()
        load_ops()

    def sample_async(self, logits: torch.Tensor, sampling_params_list: List,
                     history_token_ids: List[List[int]], generators=None, **kw) -> PendingTokens:
        """``sample`` with int32 ids and a non-blocking copy to pinned host
        memory in place of the caller's blocking ``.tolist()`` (engine.py:250):
        the host can prepare the next step while this one samples, then
        ``wait()``.  Up to four results may be outstanding at once; a fifth
        call first waits for the oldest."""
        if kw.get("return_debug"):
            raise ValueError("sample_async returns ids only; use sample(return_debug=True) for debug outputs")
        kw["out_dtype"] = torch.int32
        out = self.sample(logits, sampling_params_list, history_token_ids, generators, **kw)
        return self._ring.copy(out)

    def to_host_async(self, tokens: torch.Tensor) -> PendingTokens:
        """Non-blocking int32 copy of device ids (e.g. from ``sample_packed`` or
        ``HistoryStore.sample``) to pinned host memory."""
        return self._ring.copy(tokens)

    # -- the reference entry point (sampler.py:21-27) ---------------------
    def sample(
        self,
        logits: torch.Tensor,
        sampling_params_list: List,
        history_token_ids: List[List[int]],
        generators: Optional[List[Optional[torch.Generator]]] = None,
        *,
        sample_indices: Optional[torch.Tensor] = None,
        uniforms: Optional[torch.Tensor] = None,
        seed: Optional[int] = None,
        out_dtype: torch.dtype = torch.int64,
        return_debug: bool = False,
    ):
        if logits.dim() != 2:
            raise ValueError("logits must be [num_seqs, vocab]")
        if not logits.is_cuda:
            raise RuntimeError("Sampler.sample needs CUDA logits (no CPU fallback)")
        vocab = logits.shape[1]
        S = len(sampling_params_list)
        if sample_indices is None and logits.shape[0] != S:
            raise ValueError(f"logits has {logits.shape[0]} rows but {S} sampling params were given")
        torch.cuda.nvtx.range_push("logits+sample")
        try:
            # every copy, event and launch below goes to the logits' device,
            # whatever device is current for the caller
            with torch.cuda.device(logits.device):
                packed = packing.pack(sampling_params_list, history_token_ids, vocab,
                                      sms=_sm_count(logits.device))
                row_params, offsets, ids, order = self._upload(packed, logits.device)
                return self.sample_packed(
                    logits, row_params, offsets, ids,
                    sample_indices=sample_indices, uniforms=uniforms, seed=seed,
                    out_dtype=out_dtype, return_debug=return_debug, row_order=order,
                )
        finally:
            torch.cuda.nvtx.range_pop()

    # -- pre-packed device inputs (graph-capturable) ------------------------
    def sample_packed(
        self,
        logits: torch.Tensor,
        row_params: torch.Tensor,
        history_offsets: Optional[torch.Tensor],
        history_ids: Optional[torch.Tensor],
        *,
        sample_indices: Optional[torch.Tensor] = None,
        uniforms: Optional[torch.Tensor] = None,
        seed: Optional[int] = None,
        offset: Optional[int] = None,
        row_offset: int = 0,
        out: Optional[torch.Tensor] = None,
        out_dtype: torch.dtype = torch.int64,
        return_debug: bool = False,
        row_order: Optional[torch.Tensor] = None,
    ):
        """One step over pre-packed device inputs (``packing.pack`` + ``upload_packed``).

        ``row_order`` (int32 [S], a permutation) only changes the order in
        which the kernel takes rows, never the result."""
        S = row_params.numel() // packing.ROW_DTYPE.itemsize
        dev = logits.device
        if logits.stride(1) != 1:
            logits = logits.contiguous()
        if out is None:
            out = torch.empty(S, dtype=out_dtype, device=dev)
        if seed is None:
            seed = torch.initial_seed()
        if offset is None:
            offset = self._step
            self._step += 1
        dbg = None
        if return_debug:
            V = logits.shape[1]
            dbg = {
                "penalized": torch.empty(S, V, dtype=torch.float32, device=dev),
                "filtered": torch.empty(S, V, dtype=torch.float32, device=dev),
                "probs": torch.empty(S, V, dtype=torch.float32, device=dev),
                "status": torch.zeros(1, dtype=torch.int32, device=dev),
            }
        torch.ops.nanoserve_b200.sample(
            logits, sample_indices, row_params, history_offsets, history_ids, uniforms,
            int(seed) & 0x7FFFFFFFFFFFFFFF, int(offset), int(row_offset), out,
            dbg["penalized"] if dbg else None, dbg["filtered"] if dbg else None,
            dbg["probs"] if dbg else None, dbg["status"] if dbg else None, row_order, KERNELS[self.kernel],
        )
        if return_debug:
            return out, dbg
        return out

    def _upload(self, packed: packing.Packed, device: torch.device):
        a, b, c, d, end = packing.layout(packed)
        host = self._staging.get(end)
        packing.to_bytes(packed, host.numpy())
        dev = host.to(device, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(device))
        self._staging.event = ev
        row_params = dev[a : a + packed.row_params.nbytes]
        offsets = dev[b : b + packed.offsets.nbytes].view(torch.int64)
        ids = dev[c : c + packed.ids.nbytes].view(torch.int32) if packed.ids.size else None
        if ids is None:
            offsets = None
        order = dev[d : d + packed.order.nbytes].view(torch.int32) if packed.order is not None else None
        return row_params, offsets, ids, order


def upload_packed(packed: packing.Packed, device) -> tuple:
    """Device tensors (row_params uint8, offsets int64 or None, ids int32 or
    None, row order int32 or None) for :meth:`Sampler.sample_packed`."""
    device = torch.device(device)
    rp = torch.from_numpy(packed.row_params.view(np.uint8).copy()).to(device)
    if packed.ids.size:
        off = torch.from_numpy(packed.offsets.copy()).to(device)
        ids = torch.from_numpy(packed.ids.copy()).to(device)
    else:
        off, ids = None, None
    order = torch.from_numpy(packed.order.copy()).to(device) if packed.order is not None else None
    return rp, off, ids, order


_SMS: dict = {}


def _sm_count(device) -> int:
    """SM count of a CUDA device (cached)."""
    device = torch.device(device)
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _SMS:
        _SMS[idx] = torch.cuda.get_device_properties(idx).multi_processor_count
    return _SMS[idx]
