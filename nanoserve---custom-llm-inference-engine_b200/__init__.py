"""B200-native (sm_100a) replacement for NanoServe's token-sampling hot path.

Public surface:

* :class:`Sampler` -- drop-in for ``nanoserve.scheduler.sampler.Sampler``
  (nanoserve/scheduler/sampler.py:17-89), backed by
  ``torch.ops.nanoserve_b200.sample``;
* :class:`SamplingParams` -- same fields as nanoserve/config.py:68-79;
* :mod:`._cabi` -- ctypes binding of ``include/nanoserve_sampler.h``;
* :class:`HistoryStore` -- device-resident, append-only prior-token
  histories (replaces the per-step lists of nanoserve/engine.py:242-246);
* :mod:`.sharded` -- row-sharded sampling over several GPUs (one process per
  GPU, one NCCL all-gather of the sampled ids);
* :mod:`.workloads` -- seeded synthetic inputs shaped like the benchmark
  configurations.
"""
from .config import SamplingParams
from .sampler import Sampler, load_ops
from .history import HistoryStore

__all__ = ["HistoryStore", "Sampler", "SamplingParams", "load_ops"]
