"""GPU parity: the sm_100a kernel (through the C ABI) against the numpy oracle.

Tolerances (see tests/gpu_helpers.py): bit-exact penalised and filtered
logits, greedy and top-k decisions; |dprob| <= 1e-6; sampled tokens equal the
oracle's inverse CDF except when the uniform lies within 1e-6 of a CDF step;
top-p sets equal except when the deciding mass lies within 2e-7 of the
float32 boundary.
"""
import importlib

import numpy as np
import pytest
import torch

import cases as C
import gpu_helpers as H

pytestmark = pytest.mark.gpu

W = importlib.import_module(H.PKG + ".workloads")


@pytest.fixture(params=["cluster", "split"], autouse=True)
def sample_path(request, monkeypatch):
    """Run every test through both kernels (split only where its layout holds)."""
    monkeypatch.setitem(H.KERNEL, "name", request.param)
    return request.param


def _check(rep: H.Report):
    assert not rep.failures, "\n".join(rep.failures)


def _dev():
    assert torch.cuda.is_available(), "GPU test run without a CUDA device"
    return torch.device("cuda:0")


@pytest.mark.parametrize("config,rows", [(1, None), (2, 64), (4, 32), (5, 32)])
def test_config_parity(config, rows):
    dev = _dev()
    w = W.make(config, rows=rows, seed=10 + config)
    lg = torch.from_numpy(w.logits).to(dev)
    gpu = H.run_cabi(lg, w.params, w.histories, w.uniforms, sample_indices=w.sample_indices)
    assert gpu["status"] == 0
    rep = H.compare(gpu, w.gathered(), w.params, w.histories, w.uniforms)
    print(f"config {config}: rows {rep.rows}, top-p band {rep.topp_band_rows}, draw band {rep.draw_band_rows}")
    _check(rep)


_FULL = {}


def _full_size(config: int):
    """Config 4 at its 1024 rows, or a 1024-row slice of config 5 (every
    parameter kind, histories U[128,1024]), with the oracle's results."""
    if config not in _FULL:
        w = W.make(config, rows=1024, seed=50 + config)
        _FULL[config] = (w, H.oracle_rows(w.gathered(), w.params, w.histories, w.uniforms))
    return _FULL[config]


@pytest.mark.parametrize("debug", [False, True])
@pytest.mark.parametrize("config", [4, 5])
def test_full_size_batches(config, debug):
    """More than twice as many rows as the GPU has SMs in one call, so every
    persistent block of either kernel takes many rows (and the row
    kernel reuses its workspace slots): bit-exact penalised and filtered
    logits, |dp| <= 1e-6 and the oracle's tokens (debug on), the oracle's
    tokens (debug off)."""
    dev = _dev()
    w, expected = _full_size(config)
    lg = torch.from_numpy(w.logits).to(dev)
    gpu = H.run_cabi(lg, w.params, w.histories, w.uniforms, sample_indices=w.sample_indices, debug=debug)
    assert gpu["status"] == 0
    rep = H.compare(gpu, w.gathered(), w.params, w.histories, w.uniforms, expected=expected)
    print(f"config {config}: rows {rep.rows}, top-p band {rep.topp_band_rows}, draw band {rep.draw_band_rows}")
    _check(rep)


def test_config3_bf16_gather():
    dev = _dev()
    w = W.make(3, rows=16, seed=33)
    lg = H.to_bf16_tensor(w.logits, dev)
    assert torch.equal(lg.float().cpu(), torch.from_numpy(w.logits))  # values are exactly bf16
    gpu = H.run_cabi(lg, w.params, w.histories, w.uniforms, sample_indices=w.sample_indices)
    assert gpu["status"] == 0
    _check(H.compare(gpu, w.gathered(), w.params, w.histories, w.uniforms))


def test_full_decode_batch_tokens():
    """Config 2 at its full 256 rows: tokens only (no debug outputs)."""
    dev = _dev()
    w = W.make(2, seed=2)
    lg = torch.from_numpy(w.logits).to(dev)
    gpu = H.run_cabi(lg, w.params, w.histories, w.uniforms, debug=False)
    dbg = H.run_cabi(lg, w.params, w.histories, w.uniforms, debug=True)
    # debug outputs must not change the drawn tokens
    assert np.array_equal(gpu["tokens"], dbg["tokens"])
    _check(H.compare(dbg, w.logits, w.params, w.histories, w.uniforms))


@pytest.mark.parametrize("V", [4096, 32768])
def test_edge_cases(V):
    dev = _dev()
    case = C.edge_case(V)
    lg = torch.from_numpy(case.logits).to(dev)
    gpu = H.run_cabi(lg, case.params, case.histories, case.uniforms)
    _check(H.compare(gpu, case.logits, case.params, case.histories, case.uniforms))


@pytest.mark.parametrize("V", [1000, 32000, 151936, 50])
def test_other_vocab_sizes(V):
    dev = _dev()
    w = W.make(2, rows=16, seed=V, vocab=V)
    lg = torch.from_numpy(w.logits).to(dev)
    gpu = H.run_cabi(lg, w.params, w.histories, w.uniforms)
    _check(H.compare(gpu, w.logits, w.params, w.histories, w.uniforms))


def test_unaligned_rows_take_the_scalar_path():
    dev = _dev()
    w = W.make(2, rows=8, seed=5)
    V = w.logits.shape[1]
    big = torch.zeros(8, V + 3, device=dev)
    big[:, 1:V + 1] = torch.from_numpy(w.logits).to(dev)
    view = big[:, 1:V + 1]  # row stride V+3, base offset 4 bytes: no bulk copies
    gpu = H.run_cabi(view, w.params, w.histories, w.uniforms)
    _check(H.compare(gpu, w.logits, w.params, w.histories, w.uniforms))


def test_int32_output_and_determinism():
    dev = _dev()
    w = W.make(2, rows=32, seed=6)
    lg = torch.from_numpy(w.logits).to(dev)
    a = H.run_cabi(lg, w.params, w.histories, None, debug=False, out_i32=True, seed=99, offset=3)
    b = H.run_cabi(lg, w.params, w.histories, None, debug=False, seed=99, offset=3)
    assert np.array_equal(a["tokens"], b["tokens"])
    c = H.run_cabi(lg, w.params, w.histories, None, debug=False, seed=99, offset=4)
    greedy = np.array([p.temperature == 0.0 for p in w.params])
    assert np.array_equal(a["tokens"][greedy], c["tokens"][greedy])
    assert not np.array_equal(a["tokens"][~greedy], c["tokens"][~greedy])


def test_row_offset_makes_shards_match_the_whole_batch():
    dev = _dev()
    w = W.make(2, rows=32, seed=8)
    lg = torch.from_numpy(w.logits).to(dev)
    whole = H.run_cabi(lg, w.params, w.histories, None, debug=False, seed=5, offset=1)["tokens"]
    parts = []
    for lo in (0, 16):
        parts.append(H.run_cabi(lg[lo:lo + 16], w.params[lo:lo + 16], w.histories[lo:lo + 16], None,
                                debug=False, seed=5, offset=1, row_offset=lo)["tokens"])
    assert np.array_equal(whole, np.concatenate(parts))


def test_input_not_modified():
    dev = _dev()
    w = W.make(1, seed=1)
    lg = torch.from_numpy(w.logits).to(dev)
    before = lg.clone()
    H.run_cabi(lg, w.params, w.histories, w.uniforms, sample_indices=w.sample_indices)
    assert torch.equal(lg, before)


def test_bad_inputs_set_status_without_faulting():
    dev = _dev()
    w = W.make(2, rows=4, seed=9)
    lg = torch.from_numpy(w.logits).to(dev)
    # sample_indices out of range -> status bit, no out-of-bounds access
    gpu = H.run_cabi(lg, w.params, w.histories, w.uniforms, sample_indices=np.array([0, 1, 2, 99]),
                     debug=False)
    assert gpu["status"] & H.cabi.NS_STATUS_BAD_SAMPLE_INDEX
    # a history id outside the vocabulary (bypassing the host check) -> status bit
    pk = H.packing.pack(w.params, w.histories, lg.shape[1])
    ids = pk.ids.copy()
    if ids.size:
        ids[0] = lg.shape[1] + 5
    import ctypes  # noqa: F401

    rp = torch.from_numpy(pk.row_params.view(np.uint8).copy()).to(dev)
    off = torch.from_numpy(pk.offsets.copy()).to(dev)
    idt = torch.from_numpy(ids).to(dev)
    out = torch.empty(4, dtype=torch.int64, device=dev)
    st = torch.zeros(1, dtype=torch.int32, device=dev)
    a = H.cabi.NsSampleArgs()
    a.logits, a.logits_dtype, a.vocab_size = lg.data_ptr(), 0, lg.shape[1]
    a.num_logit_rows, a.logits_row_stride, a.num_rows = 4, lg.stride(0), 4
    a.row_params, a.history_offsets, a.history_ids = rp.data_ptr(), off.data_ptr(), idt.data_ptr()
    a.out_tokens, a.status = out.data_ptr(), st.data_ptr()
    H.cabi.ns_sample(a, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    if ids.size:
        assert st.item() & H.cabi.NS_STATUS_BAD_HISTORY_ID


def test_host_side_errors_are_reported():
    a = H.cabi.NsSampleArgs()
    a.num_rows = 3
    with pytest.raises(H.cabi.NsError, match="required"):
        H.cabi.ns_sample(a, 0)


def test_fallback_paths():
    """Rows that leave the single-pass fast paths: candidate overflow on ties,
    a maximum far above the first chunk's, wide and deep top-p windows."""
    dev = _dev()
    V = 32768
    rng = np.random.default_rng(21)
    SP = importlib.import_module(H.PKG + ".config").SamplingParams
    rows, params, hists = [], [], []

    def add(x, p, h=()):
        rows.append(np.asarray(x, dtype=np.float32))
        params.append(p)
        hists.append(list(h))

    base = lambda: (rng.standard_normal(V) * 2.0).astype(np.float32)  # noqa: E731
    add(np.full(V, 1.5), SP(temperature=1.0, top_k=50))                       # all tied: top-k overflow
    add(np.linspace(-5, 5, V), SP(temperature=1.0, top_k=64))                 # ascending: bound rises late
    x = base(); x[V - 3] = 200.0; add(x, SP(temperature=1.0, top_p=0.9))      # max far above chunk 0
    x = base(); x[V - 3] = 200.0; add(x, SP(temperature=1.0))                 # same, plain sampling
    add(base() * np.float32(0.1), SP(temperature=1.0, top_p=0.999))          # flat: big window
    add(base(), SP(temperature=1.0, top_p=0.9999))                            # boundary deep in the tail
    add(np.round(base() * 4) / 4, SP(temperature=1.0, top_p=0.7))            # many exact ties
    add(base(), SP(temperature=0.25, top_k=300, top_p=0.95, repetition_penalty=1.3),
        rng.integers(0, V, 500).tolist())                                     # large top-k + penalty
    add(base(), SP(temperature=0.0, top_k=40, top_p=0.5))                     # greedy with filters
    x = base(); x[:8192] = -np.inf; add(x, SP(temperature=1.0, top_p=0.8))    # first chunks all -inf
    x = base() * np.float32(30.0); add(x, SP(temperature=1.0, top_p=0.95))    # masses below 2^-32
    lg = torch.from_numpy(np.stack(rows)).to(dev)
    u = np.random.default_rng(5).random(len(rows)).astype(np.float32)
    gpu = H.run_cabi(lg, params, hists, u)
    assert gpu["status"] == 0  # every fallback here is exact
    _check(H.compare(gpu, np.stack(rows), params, hists, u))


@pytest.mark.parametrize("V", [32768, 128256])
def test_tie_groups_at_the_top_p_boundary(V):
    """Tie groups larger than any candidate list straddle the top-p boundary:
    exactly the first ranks (value descending, index ascending) are kept."""
    dev = _dev()
    rng = np.random.default_rng(33)
    SP = importlib.import_module(H.PKG + ".config").SamplingParams
    rows, params, hists = [], [], []

    def add(x, p, h=()):
        rows.append(np.asarray(x, dtype=np.float32))
        params.append(p)
        hists.append(list(h))

    base = lambda: (rng.standard_normal(V) * 2.0).astype(np.float32)  # noqa: E731
    add(np.full(V, 1.5), SP(temperature=1.0, top_p=0.9))                       # one group: the whole row
    add(np.full(V, -3.25), SP(temperature=0.7, top_p=0.37))                    # same, tempered
    x = np.full(V, 1.0); x[rng.permutation(V)[: V // 2]] = 2.0
    add(x, SP(temperature=1.0, top_p=0.5))                                     # boundary inside the top group
    add(x, SP(temperature=1.0, top_p=0.95))                                    # boundary inside the lower group
    add(np.round(base()), SP(temperature=1.0, top_p=0.6))                      # integer logits: big groups
    add(np.round(base()), SP(temperature=0.8, top_p=0.8, repetition_penalty=1.2),
        rng.integers(0, V, 300).tolist())                                      # with penalty
    add(np.full(V, 0.5), SP(temperature=1.0, top_k=5000, top_p=0.5))          # top-k ties, then top-p
    lg = torch.from_numpy(np.stack(rows)).to(dev)
    u = np.random.default_rng(6).random(len(rows)).astype(np.float32)
    gpu = H.run_cabi(lg, params, hists, u)
    assert gpu["status"] == 0
    _check(H.compare(gpu, np.stack(rows), params, hists, u))


def test_row_order_changes_nothing_but_the_schedule():
    """NsSampleArgs.row_order is a scheduling hint: any permutation gives the
    same tokens and debug outputs; an out-of-range entry is flagged and that
    slot takes its own row."""
    dev = _dev()
    w = W.make(2, rows=256)
    lg = torch.from_numpy(w.logits).to(dev)
    u, si = w.uniforms, w.sample_indices
    perm = np.random.default_rng(3).permutation(256).astype(np.int32)
    sched = H.packing.pack(w.params, w.histories, lg.shape[1], sms=148).order
    for debug in (False, True):
        base = H.run_cabi(lg, w.params, w.histories, u, sample_indices=si, debug=debug)
        for order in (perm, sched):
            got = H.run_cabi(lg, w.params, w.histories, u, sample_indices=si, debug=debug,
                             row_order=torch.from_numpy(order).to(dev))
            assert got["status"] == base["status"] == 0
            assert np.array_equal(got["tokens"], base["tokens"])
            for key in ("penalized", "filtered", "probs"):
                if key in base:
                    assert np.array_equal(got[key].view(np.uint32), base[key].view(np.uint32)), key
    bad = np.arange(256, dtype=np.int32)
    bad[5] = -1
    bad[9] = 256
    base = H.run_cabi(lg, w.params, w.histories, u, sample_indices=si, debug=False)
    got = H.run_cabi(lg, w.params, w.histories, u, sample_indices=si, debug=False,
                     row_order=torch.from_numpy(bad).to(dev))
    assert got["status"] == H.cabi.NS_STATUS_BAD_ROW_ORDER
    assert np.array_equal(got["tokens"], base["tokens"])


@pytest.mark.parametrize("V", [32768, 128256])
def test_top_p_rows_without_debug_outputs(V):
    """The production path (no debug outputs): top-p rows are finished from
    their parts' histograms and give the oracle's tokens."""
    dev = _dev()
    rng = np.random.default_rng(44)
    SP = importlib.import_module(H.PKG + ".config").SamplingParams
    rows, params, hists = [], [], []
    kinds = [SP(temperature=1.0, top_p=0.9), SP(temperature=0.7, top_p=0.9, repetition_penalty=1.2),
             SP(temperature=1.3, top_p=0.99), SP(temperature=0.0), SP(temperature=1.0, top_k=50),
             SP(temperature=1.0, top_p=0.5), SP(temperature=0.9, top_p=0.95, repetition_penalty=0.8)]
    for r in range(48):
        p = kinds[r % len(kinds)]
        flat = r % len(kinds) == 2
        x = (rng.standard_normal(V) * (0.5 if flat else 2.0)).astype(np.float32)
        if not flat:
            x[rng.integers(0, V, 20)] += 8.0
        rows.append(x)
        params.append(p)
        hists.append(rng.integers(0, V, 700).tolist() if p.repetition_penalty != 1.0 else [])
    lg = torch.from_numpy(np.stack(rows)).to(dev)
    u = rng.random(len(rows)).astype(np.float32)
    gpu = H.run_cabi(lg, params, hists, u, debug=False)
    assert gpu["status"] == 0
    _check(H.compare(gpu, np.stack(rows), params, hists, u))


def test_config3_bf16_gather_without_debug_outputs():
    """Config 3 as served (64 gathered bf16 rows, top-p 0.95, penalty 1.2, no
    debug outputs) gives the oracle's tokens."""
    dev = _dev()
    w = W.make(3, seed=34)
    lg = H.to_bf16_tensor(w.logits, dev)
    gpu = H.run_cabi(lg, w.params, w.histories, w.uniforms, sample_indices=w.sample_indices, debug=False)
    assert gpu["status"] == 0
    _check(H.compare(gpu, w.gathered(), w.params, w.histories, w.uniforms))


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("V", [32768, 128256])
def test_top_k_rows_without_debug_outputs(V, dtype):
    """Top-k rows as served (no debug outputs), mixed with top-p rows that take
    the second ring pass: ties at the k-th value, k = 1, k = 128 and k = 129 (past the
    candidate-list path), top-k with top-p, the penalty, NaN / +inf / all -inf
    rows, a flat row and a mostly -inf row (candidate lists that overflow into
    the general path) all give the oracle's tokens."""
    dev = _dev()
    rng = np.random.default_rng(45)
    SP = importlib.import_module(H.PKG + ".config").SamplingParams
    kinds = [
        ("normal", SP(temperature=1.0, top_k=50)),
        ("normal", SP(temperature=0.7, top_k=5, repetition_penalty=1.2)),
        ("normal", SP(temperature=1.0, top_k=1)),
        ("normal", SP(temperature=1.3, top_k=128, top_p=0.9)),
        ("normal", SP(temperature=0.9, top_k=20, top_p=0.5, repetition_penalty=0.8)),
        ("normal", SP(temperature=1.0, top_k=129)),
        ("flat", SP(temperature=1.0, top_k=40)),
        ("ties", SP(temperature=1.0, top_k=10)),
        ("nan", SP(temperature=1.0, top_k=16)),
        ("pinf", SP(temperature=1.0, top_k=16)),
        ("ninf", SP(temperature=1.0, top_k=16)),
        ("normal", SP(temperature=1.0, top_p=0.9)),
        ("sparse", SP(temperature=1.0, top_k=64)),
    ]
    rows, params, hists = [], [], []
    for r in range(52):
        kind, p = kinds[r % len(kinds)]
        x = (rng.standard_normal(V) * 2.0).astype(np.float32)
        x[rng.integers(0, V, 20)] += 8.0
        if kind == "flat":
            x[:] = 0.25
        elif kind == "ties":
            x[rng.choice(V, 30, replace=False)] = 20.0
        elif kind == "nan":
            x[rng.integers(0, V)] = np.nan
        elif kind == "pinf":
            x[rng.integers(0, V)] = np.inf
        elif kind == "ninf":
            x[:] = -np.inf
        elif kind == "sparse":
            x[rng.random(V) < 0.9] = -np.inf
        rows.append(x)
        params.append(p)
        hists.append(rng.integers(0, V, 700).tolist() if p.repetition_penalty != 1.0 else [])
    lg = torch.from_numpy(np.stack(rows)).to(dev)
    if dtype == "bf16":
        lg = lg.to(torch.bfloat16)
    ref = lg.float().cpu().numpy()
    u = rng.random(len(rows)).astype(np.float32)
    gpu = H.run_cabi(lg, params, hists, u, debug=False)
    assert gpu["status"] == 0
    _check(H.compare(gpu, ref, params, hists, u))
