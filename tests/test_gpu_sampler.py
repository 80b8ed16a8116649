"""The drop-in ``Sampler`` (torch.ops path) on the GPU, and the draw distribution."""
import importlib

import numpy as np
import pytest
import torch

import gpu_helpers as H
from oracle import sampler_oracle as O

pytestmark = pytest.mark.gpu

NS = importlib.import_module(H.PKG)
W = importlib.import_module(H.PKG + ".workloads")


@pytest.fixture(params=["cluster", "split"], autouse=True)
def sample_path(request, monkeypatch):
    """Run every test through both kernels (split only where its layout holds)."""
    monkeypatch.setitem(H.KERNEL, "name", request.param)
    return request.param


def _dev():
    assert torch.cuda.is_available(), "GPU test run without a CUDA device"
    return torch.device("cuda:0")


def test_sampler_drop_in_signature_and_results():
    dev = _dev()
    w = W.make(2, rows=32, seed=21)
    lg = torch.from_numpy(w.logits).to(dev)
    s = H.make_sampler(dev)
    out = s.sample(lg, w.params, w.histories)  # the reference call, engine.py:247-249
    assert out.dtype == torch.int64 and out.shape == (32,) and out.device == lg.device
    toks = out.tolist()  # engine.py:250
    for i, p in enumerate(w.params):
        if p.temperature == 0.0:
            res = O.sample_row(w.logits[i], p, w.histories[i], 0.5)
            assert toks[i] == res.argmax
    # uniforms + debug outputs through the torch op agree with the C ABI
    uni = torch.from_numpy(w.uniforms).to(dev)
    out2, dbg = s.sample(lg, w.params, w.histories, uniforms=uni, return_debug=True)
    ref = H.run_cabi(lg, w.params, w.histories, w.uniforms)
    assert np.array_equal(out2.cpu().numpy(), ref["tokens"])
    assert np.array_equal(dbg["probs"].cpu().numpy(), ref["probs"])
    assert dbg["status"].item() == 0


def test_sampler_accepts_reference_sampling_params_objects():
    dev = _dev()

    class Ref:  # any object with the reference's attribute names
        temperature, top_p, top_k, repetition_penalty, seed = 0.0, 1.0, -1, 1.0, None

    lg = torch.randn(2, 1000, device=dev)
    out = H.make_sampler(dev).sample(lg, [Ref(), Ref()], [[], []])
    assert out.tolist() == torch.argmax(lg, dim=-1).tolist()


def test_sampler_gather_and_bf16():
    dev = _dev()
    w = W.make(3, rows=8, seed=31)
    lg = H.to_bf16_tensor(w.logits, dev)
    idx = torch.from_numpy(w.sample_indices).to(dev)
    uni = torch.from_numpy(w.uniforms).to(dev)
    out, dbg = H.make_sampler(dev).sample(lg, w.params, w.histories, sample_indices=idx, uniforms=uni,
                                      return_debug=True)
    gpu = dict(tokens=out.cpu().numpy(), penalized=dbg["penalized"].cpu().numpy(),
               filtered=dbg["filtered"].cpu().numpy(), probs=dbg["probs"].cpu().numpy())
    rep = H.compare(gpu, w.gathered(), w.params, w.histories, w.uniforms)
    assert not rep.failures, "\n".join(rep.failures)


def test_sampler_rejects_bad_history_like_the_reference():
    dev = _dev()
    lg = torch.randn(1, 100, device=dev)
    p = NS.SamplingParams(temperature=1.0, repetition_penalty=1.2)
    with pytest.raises(IndexError):
        H.make_sampler(dev).sample(lg, [p], [[5, 100]])


def test_sampler_graph_capture():
    """Pre-packed inputs: the op records into a CUDA graph and replays."""
    dev = _dev()
    w = W.make(2, rows=16, seed=41)
    lg = torch.from_numpy(w.logits).to(dev)
    s = H.make_sampler(dev)
    pk = H.packing.pack(w.params, w.histories, lg.shape[1])
    rp, off, ids, _ = importlib.import_module(H.PKG + ".sampler").upload_packed(pk, dev)
    out = torch.empty(16, dtype=torch.int64, device=dev)
    uni = torch.from_numpy(w.uniforms).to(dev)
    s.sample_packed(lg, rp, off, ids, uniforms=uni, out=out, offset=0)
    torch.cuda.synchronize()
    want = out.clone()
    g = torch.cuda.CUDAGraph()
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(g, stream=stream):
            s.sample_packed(lg, rp, off, ids, uniforms=uni, out=out, offset=0)
    out.fill_(-1)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, want)


@pytest.mark.parametrize("kind", ["topk", "topp"])
def test_draw_distribution_chi_square(kind):
    """10^6 Philox draws from one row against the oracle's probabilities."""
    from scipy.stats import chi2

    dev = _dev()
    rng = np.random.default_rng(77)
    V = 128256
    x = W.peaked_logits(rng, 1, V)[0]
    if kind == "topk":
        p = NS.SamplingParams(temperature=0.7, top_k=50)
    else:
        p = NS.SamplingParams(temperature=1.0, top_p=0.2)
    ref = O.sample_row(x, p, [], 0.5)
    probs = ref.probs.astype(np.float64)
    lg = torch.from_numpy(x[None, :]).to(dev)
    R = 2048
    reps = 489  # 2048 * 489 = 1,001,472 draws
    idx = torch.zeros(R, dtype=torch.int64, device=dev)
    pk = H.packing.pack([p] * R, [[]] * R, V)
    rp = torch.from_numpy(pk.row_params.view(np.uint8).copy()).to(dev)
    s = H.make_sampler(dev)
    counts = torch.zeros(V, dtype=torch.int64, device=dev)
    out = torch.empty(R, dtype=torch.int64, device=dev)
    for k in range(reps):
        s.sample_packed(lg, rp, None, None, sample_indices=idx, out=out, seed=2024, offset=k)
        counts += torch.bincount(out, minlength=V)
    counts = counts.cpu().numpy().astype(np.float64)
    n = counts.sum()
    assert counts[probs == 0].sum() == 0, "drew a token the filters removed"
    exp = probs * n
    order = np.argsort(-exp)
    # pool categories with expected count < 5 into one bin
    big = order[exp[order] >= 5]
    small = order[exp[order] < 5]
    obs = np.concatenate([counts[big], [counts[small].sum()]]) if small.size else counts[big]
    ex = np.concatenate([exp[big], [exp[small].sum()]]) if small.size else exp[big]
    keep = ex > 0
    stat = float(((obs[keep] - ex[keep]) ** 2 / ex[keep]).sum())
    dof = int(keep.sum()) - 1
    pval = chi2.sf(stat, dof)
    print(f"{kind}: {int(n)} draws, {dof} dof, chi2 {stat:.1f}, p {pval:.3g}")
    assert pval > 1e-3


def test_seeded_requests_are_reproducible():
    """A request with a seed (nanoserve/config.py:79) draws the same token in
    the same state whatever batch it is in, wherever it sits in it and however
    many calls the sampler has made; other seeds draw other tokens."""
    dev = _dev()
    V = 32768
    rng = np.random.default_rng(91)
    x = W.peaked_logits(rng, 1, V)[0]
    hist = rng.integers(0, V, 300).tolist()

    def req(seed):
        return NS.SamplingParams(temperature=1.0, top_p=0.95, repetition_penalty=1.1, seed=seed)

    def batch(n_other, pos, seed, warm_calls):
        others = W.peaked_logits(rng, n_other, V)
        rows = np.insert(others, pos, x, axis=0)
        params = W.mixed_params(n_other)
        params.insert(pos, req(seed))
        hists = W.histories(rng, n_other, 0, 200, V)
        hists.insert(pos, hist)
        s = H.make_sampler(dev)
        lg = torch.from_numpy(rows).to(dev)
        for _ in range(warm_calls):
            s.sample(lg, params, hists)
        return int(s.sample(lg, params, hists)[pos].item())

    a = batch(7, 0, 1234, 0)
    b = batch(40, 23, 1234, 3)
    c = batch(63, 63, 1234, 1)
    assert a == b == c
    others = {batch(7, 0, sd, 0) for sd in range(16)}
    assert len(others) > 1
