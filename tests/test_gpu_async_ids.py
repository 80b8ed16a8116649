"""Asynchronous int32 ids: Sampler.sample_async and to_host_async give the
lists that the blocking ``.tolist()`` of engine.py:250 gives, with several
results outstanding at once."""
import importlib

import numpy as np
import pytest
import torch

import gpu_helpers as H

pytestmark = pytest.mark.gpu

NS = importlib.import_module(H.PKG)
W = importlib.import_module(H.PKG + ".workloads")
history = importlib.import_module(H.PKG + ".history")


def _dev():
    assert torch.cuda.is_available(), "GPU test run without a CUDA device"
    return torch.device("cuda:0")


@pytest.mark.parametrize("S", [8, 256])
def test_async_ids_equal_blocking_ids(S):
    dev = _dev()
    V = 128256
    rng = np.random.default_rng(31)
    params = W.mixed_params(S)
    hists = W.histories(rng, S, 0, 500, V)
    logits = [torch.from_numpy((rng.standard_normal((S, V)) * 2).astype(np.float32)).to(dev) for _ in range(6)]
    a, b = NS.Sampler(dev), NS.Sampler(dev)
    want = [a.sample(lg, params, hists, seed=5).tolist() for lg in logits]
    # six calls before any wait: the ring of four pinned buffers makes the
    # fifth and sixth calls wait for the first two, whose lists are kept
    pend = [b.sample_async(lg, params, hists, seed=5) for lg in logits]
    got = [p.wait() for p in pend]
    assert got == want
    assert all(p.ready() for p in pend)


def test_to_host_async_after_the_history_store():
    dev = _dev()
    V = 50000
    rng = np.random.default_rng(32)
    S = 40
    params = W.mixed_params(S)
    hists = W.histories(rng, S, 1, 300, V)
    st = history.HistoryStore(dev, capacity=S * 400, vocab=V)
    handles = [st.add(h, 10) for h in hists]
    s = NS.Sampler(dev)
    lg = torch.from_numpy((rng.standard_normal((S, V)) * 2).astype(np.float32)).to(dev)
    out = st.sample(s, lg, params, handles, seed=9, offset=0)
    pt = s.to_host_async(out)
    assert pt.wait() == out.tolist()


def test_sample_async_rejects_debug_outputs():
    s = NS.Sampler(_dev())
    with pytest.raises(ValueError, match="ids only"):
        s.sample_async(torch.zeros(1, 8, device="cuda"), [], [], return_debug=True)
