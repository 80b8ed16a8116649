"""Device-resident histories on the GPU: the gathered CSR histories equal
packing.pack's bit for bit, appends land where the host expects, and sampling
through the store gives the same tokens as Sampler.sample over Python lists,
step after step."""
import importlib

import numpy as np
import pytest
import torch

import gpu_helpers as H

pytestmark = pytest.mark.gpu

PKG = H.PKG
history = importlib.import_module(PKG + ".history")
packing = importlib.import_module(PKG + ".packing")
cabi = importlib.import_module(PKG + "._cabi")
W = importlib.import_module(PKG + ".workloads")
NS = importlib.import_module(PKG)
SP = importlib.import_module(PKG + ".config").SamplingParams


def _dev():
    assert torch.cuda.is_available(), "GPU test run without a CUDA device"
    return torch.device("cuda:0")


def _fragmented_store(dev, V, hists, extra=64):
    """A store whose regions are scattered: dummies are added between the
    requests and released again."""
    st = history.HistoryStore(dev, capacity=sum(len(h) + extra for h in hists) * 3 + 4096, vocab=V)
    rng = np.random.default_rng(9)
    handles, dummies = [], []
    for h in hists:
        dummies.append(st.add(rng.integers(0, V, size=int(rng.integers(0, 50))).tolist(), 5))
        handles.append(st.add(h, extra))
    for d in dummies:
        st.release(d)
    return st, handles


def test_gather_equals_host_packing():
    dev = _dev()
    V = 128256
    rng = np.random.default_rng(21)
    params = W.mixed_params(96) + [SP(temperature=0.8, repetition_penalty=1.25)] * 8
    hists = W.histories(rng, len(params), 0, 3000, V)
    hists[3] = []
    st, handles = _fragmented_store(dev, V, hists)
    rp, off, ids, order = st.pack(params, handles, sms=148)
    ref = packing.pack(params, hists, V, sms=148)
    torch.cuda.synchronize()
    assert rp.cpu().numpy().tobytes() == ref.row_params.tobytes()
    assert np.array_equal(off.cpu().numpy(), ref.offsets)
    assert np.array_equal(ids.cpu().numpy(), ref.ids)
    assert np.array_equal(order.cpu().numpy(), ref.order)
    assert int(st.status.item()) == 0


def test_append_extends_each_history():
    dev = _dev()
    V = 50000
    rng = np.random.default_rng(22)
    hists = W.histories(rng, 40, 1, 200, V)
    st, handles = _fragmented_store(dev, V, hists, extra=3)
    for step in range(3):
        tok = torch.from_numpy(rng.integers(0, V, size=len(handles))).to(dev)
        tok = tok.to(torch.int32) if step == 1 else tok
        st.append(handles, tok)
        for h, t in zip(hists, tok.tolist()):
            h.append(int(t))
    for h, handle in zip(hists, handles):
        assert st.tokens(handle) == h
    with pytest.raises(OverflowError):
        st.append(handles, torch.zeros(len(handles), dtype=torch.int64, device=dev))
    assert int(st.status.item()) == 0


@pytest.mark.parametrize("path", ["split", "cluster"])
def test_sampling_through_the_store_matches_lists(path):
    """Three decode steps: Sampler.sample over Python lists (the reference's
    calling convention, engine.py:242-249) against HistoryStore.sample; the
    lists grow by the sampled ids, the store by its own appends."""
    dev = _dev()
    V = 128256
    rng = np.random.default_rng(23)
    S = 64 if path == "split" else 12
    params = W.mixed_params(S)
    params = [SP(temperature=p.temperature, top_k=p.top_k, top_p=p.top_p,
                 repetition_penalty=1.3 if i % 3 == 0 else p.repetition_penalty) for i, p in enumerate(params)]
    hists = W.histories(rng, S, 0, 600, V)
    st, handles = _fragmented_store(dev, V, [list(h) for h in hists], extra=8)
    s_list, s_store = NS.Sampler(dev, kernel=path), NS.Sampler(dev, kernel=path)
    for step in range(3):
        x = (rng.standard_normal((S, V)) * 2.0).astype(np.float32)
        for r in range(S):  # make the penalty decide: boost a few prior ids
            if hists[r]:
                x[r, rng.choice(hists[r], size=min(4, len(hists[r])))] += 9.0
        lg = torch.from_numpy(x).to(dev)
        a = s_list.sample(lg, params, hists, seed=77, out_dtype=torch.int64)
        b = st.sample(s_store, lg, params, handles, seed=77, offset=step, out_dtype=torch.int64)
        a_l = a.tolist()
        assert a_l == b.tolist(), f"step {step}"
        for h, t in zip(hists, a_l):
            h.append(int(t))
    for h, handle in zip(hists, handles):
        assert st.tokens(handle) == h
    assert int(st.status.item()) == 0


def test_ranges_outside_the_pool_are_reported():
    dev = _dev()
    pool = torch.arange(100, dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    src = torch.tensor([10, 95, -3, 0], dtype=torch.int64, device=dev)
    off = torch.tensor([0, 4, 14, 16, 16], dtype=torch.int64, device=dev)
    ids = torch.full((16,), 7, dtype=torch.int32, device=dev)
    cabi.ns_history_gather(pool.data_ptr(), 100, src.data_ptr(), off.data_ptr(), 4, ids.data_ptr(), status.data_ptr())
    torch.cuda.synchronize()
    got = ids.cpu().tolist()
    assert got[:4] == [10, 11, 12, 13]
    assert got[4:16] == [-1] * 12  # 95 + 10 leaves the pool; -3 is before it
    assert int(status.item()) == cabi.NS_STATUS_BAD_POOL_RANGE
    status.zero_()
    dst = torch.tensor([5, 100, -1], dtype=torch.int64, device=dev)
    tok = torch.tensor([555, 666, 777], dtype=torch.int64, device=dev)
    cabi.ns_history_append(pool.data_ptr(), 100, dst.data_ptr(), tok.data_ptr(), cabi.NS_OUT_I64, 3, status.data_ptr())
    torch.cuda.synchronize()
    p = pool.cpu().tolist()
    assert p[5] == 555 and p[:5] == [0, 1, 2, 3, 4] and p[6:] == list(range(6, 100))
    assert int(status.item()) == cabi.NS_STATUS_BAD_POOL_RANGE
