"""ns_sample_noalloc, the entry point for callers that may not allocate
device memory: an engine that hands all of the GPU's memory to its own pool at
start-up, or a host embedding the library under a fixed memory budget.  It
runs on a static workspace inside the library instead of the caller's, and
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


def _same(got, want, what):
    assert got["status"] == want["status"] == 0, what
    assert np.array_equal(got["tokens"], want["tokens"]), what
    for key in ("penalized", "filtered", "probs"):
        if key in want:
            assert np.array_equal(got[key].view(np.uint32), want[key].view(np.uint32)), (what, key)


@pytest.mark.parametrize("debug", [False, True])
def test_noalloc_matches_ns_sample_on_two_calls_in_a_row(debug):
    """Two consecutive calls on different batches, so the second runs on the
    static workspace the first left behind: tokens, status and debug outputs
    equal ns_sample's bit for bit (the same kernel computes them)."""
    dev = _dev()
    for call, seed in enumerate((0, 1)):
        w = W.make(2, rows=256, seed=seed)  # config 2: every row kind uses the workspace
        lg = torch.from_numpy(w.logits).to(dev)
        kw = dict(sample_indices=w.sample_indices, debug=debug, offset=call)
        want = H.run_cabi(lg, w.params, w.histories, None, **kw)
        got = H.run_cabi(lg, w.params, w.histories, None, entry="ns_sample_noalloc", **kw)
        _same(got, want, f"call {call}")


@pytest.mark.parametrize("rows", [8, 32, 600])
def test_noalloc_small_and_large_batches(rows):
    """Below 32 rows (the cluster kernel, which needs no scratch), exactly 32
    (the row kernel's smallest automatic batch) and more rows than the GPU has
    SMs (every block takes several rows from the static counter)."""
    dev = _dev()
    w = W.make(2, rows=rows, seed=rows)
    lg = torch.from_numpy(w.logits).to(dev)
    want = H.run_cabi(lg, w.params, w.histories, None, debug=False, offset=5)
    for call in range(2):
        got = H.run_cabi(lg, w.params, w.histories, None, debug=False, offset=5, entry="ns_sample_noalloc")
        _same(got, want, f"{rows} rows, call {call}")


def test_noalloc_allocates_nothing():
    """A warm call changes the device's free memory by nothing: no cudaMalloc
    behind the caller's back (the static workspace was loaded with the library)."""
    dev = _dev()
    w = W.make(2, rows=256, seed=3)
    lg = torch.from_numpy(w.logits).to(dev)
    args = H.prepare_cabi(lg, w.params, w.histories, None, debug=False)
    H.cabi.ns_sample_noalloc(args["a"], torch.cuda.current_stream(dev).cuda_stream)  # first call: module loaded
    torch.cuda.synchronize(dev)
    free0, _ = torch.cuda.mem_get_info(dev)
    for _ in range(3):
        H.cabi.ns_sample_noalloc(args["a"], torch.cuda.current_stream(dev).cuda_stream)
    torch.cuda.synchronize(dev)
    free1, _ = torch.cuda.mem_get_info(dev)
    assert free1 == free0


def test_noalloc_rejects_what_it_cannot_serve():
    """A vocabulary beyond ns_max_vocab fails with a clear error, before any work."""
    dev = _dev()
    V = int(H.cabi.load_library().ns_max_vocab(H.cabi.NS_DTYPE_F32)) + 16
    lg = torch.zeros(1, V, device=dev)
    SP = importlib.import_module(H.PKG + ".config").SamplingParams
    with pytest.raises(H.cabi.NsError, match="exceeds the supported maximum") as e:
        H.run_cabi(lg, [SP(temperature=1.0)], [[]], None, debug=False, entry="ns_sample_noalloc")
    assert e.value.code == H.cabi.NS_ERR_UNSUPPORTED
