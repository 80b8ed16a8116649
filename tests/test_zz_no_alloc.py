"""ns_sample_noalloc, the entry point for callers that may not allocate
device memory (an engine that hands all of the GPU's memory to its own pool at
start-up, or a host embedding the library under a fixed memory budget).  It
must give exactly what ns_sample gives.  GPU tests; this file is collected
last, so a run that stops at its first failure has run every other test."""
import importlib

import numpy as np
import pytest
import torch

import gpu_helpers as H

pytestmark = pytest.mark.gpu

W = importlib.import_module(H.PKG + ".workloads")


def _dev():
    assert torch.cuda.is_available(), "GPU test run without a CUDA device"
    return torch.device("cuda:0")


@pytest.mark.parametrize("debug", [False, True])
def test_noalloc_matches_ns_sample_on_two_calls_in_a_row(debug):
    """Two consecutive calls on different batches, so the second runs on the
    scratch the first left behind: tokens, status and debug outputs equal
    ns_sample's bit for bit (the same kernels compute them)."""
    dev = _dev()
    for call, seed in enumerate((0, 1)):
        w = W.make(2, rows=256, seed=seed)  # config 2: its top-p rows go through the static scratch
        lg = torch.from_numpy(w.logits).to(dev)
        kw = dict(sample_indices=w.sample_indices, debug=debug, offset=call)
        want = H.run_cabi(lg, w.params, w.histories, None, **kw)
        got = H.run_cabi(lg, w.params, w.histories, None, entry="ns_sample_noalloc", **kw)
        assert got["status"] == want["status"] == 0
        assert np.array_equal(got["tokens"], want["tokens"]), f"call {call}"
        for key in ("penalized", "filtered", "probs"):
            if key in want:
                assert np.array_equal(got[key].view(np.uint32), want[key].view(np.uint32)), (call, key)


def test_noalloc_rejects_batches_beyond_its_scratch():
    dev = _dev()
    rows = H.cabi.NS_NOALLOC_MAX_ROWS + 1
    w = W.make(2, rows=rows)
    lg = torch.from_numpy(w.logits).to(dev)
    with pytest.raises(H.cabi.NsError, match="NS_NOALLOC_MAX_ROWS") as e:
        H.run_cabi(lg, w.params, w.histories, None, sample_indices=w.sample_indices, debug=False,
                   entry="ns_sample_noalloc")
    assert e.value.code == H.cabi.NS_ERR_UNSUPPORTED
