"""Host packing follows the reference's Python-double rules (sampler.py:33-63)."""
import importlib

import numpy as np
import pytest

from conftest import PKG_NAME

packing = importlib.import_module(PKG_NAME + ".packing")
cabi = importlib.import_module(PKG_NAME + "._cabi")
SP = importlib.import_module(PKG_NAME).SamplingParams
V = 128256


def rec(p, hist_len=0):
    return packing.derive_row(p, V, hist_len)


def test_temperature_rules():
    # sampler.py:41-50: divisor max(t,1e-6) for t>0 else 1; greedy iff t == 0.0
    assert rec(SP(temperature=0.0))[0] == np.float32(1.0) and rec(SP(temperature=0.0))[4] & cabi.NS_ROW_GREEDY
    t, p, rp, k, fl, _, _ = rec(SP(temperature=-0.5))
    assert t == np.float32(1.0) and not fl & cabi.NS_ROW_GREEDY
    assert rec(SP(temperature=1e-9))[0] == np.float32(1e-6)
    assert rec(SP(temperature=1e-50))[0] == np.float32(1e-6)  # positive in double, not greedy
    assert not rec(SP(temperature=1e-50))[4] & cabi.NS_ROW_GREEDY
    assert rec(SP(temperature=0.7))[0] == np.float32(0.7)
    nan = rec(SP(temperature=float("nan")))
    assert nan[0] == np.float32(1.0) and not nan[4] & cabi.NS_ROW_GREEDY


def test_topk_rules():
    # sampler.py:55: on iff 0 < k < vocab
    assert rec(SP(top_k=-1))[3] == 0
    assert rec(SP(top_k=0))[3] == 0
    assert rec(SP(top_k=V))[3] == 0
    assert rec(SP(top_k=V + 10**12))[3] == 0
    assert rec(SP(top_k=V - 1))[3] == V - 1
    assert rec(SP(top_k=50))[3] == 50


def test_topp_rules():
    # sampler.py:63: on iff top_p < 1.0 (Python double), compared in float32
    assert not rec(SP(top_p=1.0))[4] & cabi.NS_ROW_TOP_P
    assert not rec(SP(top_p=1.5))[4] & cabi.NS_ROW_TOP_P
    r = rec(SP(top_p=0.99999999))
    assert r[4] & cabi.NS_ROW_TOP_P and r[1] == np.float32(1.0)
    assert rec(SP(top_p=0.9))[1] == np.float32(0.9)


def test_penalty_rules():
    # sampler.py:33: on iff rp != 1.0 and the history is non-empty
    assert not rec(SP(repetition_penalty=1.2), 0)[4] & cabi.NS_ROW_PENALTY
    assert rec(SP(repetition_penalty=1.2), 3)[4] & cabi.NS_ROW_PENALTY
    assert not rec(SP(repetition_penalty=1.0), 3)[4] & cabi.NS_ROW_PENALTY


def test_seed_flag():
    assert not rec(SP())[4] & cabi.NS_ROW_SEED
    r = rec(SP(seed=-1))
    assert r[4] & cabi.NS_ROW_SEED and r[6] == 0xFFFFFFFFFFFFFFFF


def test_csr_only_ships_penalised_rows():
    params = [SP(repetition_penalty=1.1), SP(), SP(repetition_penalty=0.9), SP(repetition_penalty=2.0)]
    hists = [[1, 2, 2], [5, 6], [7], []]
    pk = packing.pack(params, hists, V)
    assert pk.offsets.tolist() == [0, 3, 3, 4, 4]
    assert pk.ids.tolist() == [1, 2, 2, 7]
    assert pk.ids.dtype == np.int32
    buf = packing.to_bytes(pk)
    a, b, c, d, end = packing.layout(pk)
    assert buf.size == end and end % 16 == 0
    assert np.array_equal(buf[c:c + 16].view(np.int32), pk.ids)


def test_out_of_range_history_raises_like_index_select():
    with pytest.raises(IndexError):
        packing.pack([SP(repetition_penalty=1.2)], [[0, V]], V)
    with pytest.raises(IndexError):
        packing.pack([SP(repetition_penalty=1.2)], [[-1]], V)
    # rows without the penalty never look at their history (sampler.py:33)
    packing.pack([SP()], [[-5, V + 3]], V)


def test_row_params_byte_layout():
    pk = packing.pack([SP(temperature=0.5, top_k=7, top_p=0.8, repetition_penalty=1.3, seed=9)], [[4]], V)
    raw = pk.row_params.view(np.uint8)
    assert raw.size == 32
    assert raw[0:4].view(np.float32)[0] == np.float32(0.5)
    assert raw[12:16].view(np.int32)[0] == 7
    assert raw[24:32].view(np.uint64)[0] == 9


def test_schedule_puts_the_longest_finishing_work_first():
    W = importlib.import_module(PKG_NAME + ".workloads")
    sms = 148
    for S in (1, 7, 148, 256, 296, 1000):
        pk = packing.pack(W.mixed_params(S), [[]] * S, V, sms=sms)
        order = pk.order
        assert order.dtype == np.int32 and sorted(order.tolist()) == list(range(S))
        cost = packing.row_costs(pk.row_params)[order]
        assert (np.diff(cost) <= 0).all()  # non-increasing cost along the order
    # config 2: the 64 top-p rows first, the 64 greedy rows last, ties in row order
    pk = packing.pack(W.mixed_params(256), [[]] * 256, V, sms=sms)
    cost = packing.row_costs(pk.row_params)[pk.order]
    assert (cost[:64] == packing.COST_TOPP).all() and (cost[-64:] == packing.COST_GREEDY).all()
    assert pk.order[:64].tolist() == list(range(2, 256, 4))
    # without an SM count there is no order; layout then has an empty order region
    pk = packing.pack(W.mixed_params(8), [[]] * 8, V)
    a, b, c, d, end = packing.layout(pk)
    assert pk.order is None and end >= d


def test_seeded_rows_carry_their_history_length_as_the_counter():
    """NS_ROW_SEED rows: key = the request's seed, counter = its history length
    (prompt + tokens so far), so the stream does not depend on the batch."""
    ps = [SP(temperature=1.0, seed=5), SP(temperature=1.0), SP(temperature=0.5, seed=2**64 + 3)]
    hs = [[1, 2, 3], [4] * 9, list(range(70000))]
    pk = packing.pack(ps, hs, 100000)
    r = pk.row_params
    assert (r["flags"][[0, 2]] & cabi.NS_ROW_SEED).all() and not (r["flags"][1] & cabi.NS_ROW_SEED)
    assert r["seed_step"].tolist() == [3, 0, 70000]
    assert r["seed"].tolist() == [5, 0, 3]
    for i in range(3):
        one = packing.derive_row(ps[i], 100000, len(hs[i]))
        assert one[5] == r["seed_step"][i] and one[6] == r["seed"][i]


def test_order_travels_in_the_staging_buffer():
    W = importlib.import_module(PKG_NAME + ".workloads")
    pk = packing.pack(W.mixed_params(300), [[]] * 300, V, sms=148)
    buf = packing.to_bytes(pk)
    a, b, c, d, end = packing.layout(pk)
    assert d % 16 == 0 and np.array_equal(buf[d : d + 4 * 300].view(np.int32), pk.order)


def test_derive_rows_equals_derive_row_on_edge_values():
    """The vectorised row packing gives derive_row's records bit for bit,
    across the comparisons' edge values (zero, negative and NaN temperatures,
    top_p at and past 1, NaN top_p and penalty, top_k at the vocabulary size,
    seeds beyond 64 bits)."""
    import itertools
    import numpy as np
    from conftest import pkg

    packing = pkg("packing")
    SP = pkg("config").SamplingParams
    V = 1000
    temps = [0.0, -0.0, -1.0, 1e-9, 1e-6, 0.7, 1.0, 2.5, float("nan"), float("inf")]
    tps = [1.0, 0.9, 0.0, 1.5, float("nan"), 0.999999999]
    tks = [-1, 0, 1, 50, V - 1, V, V + 5]
    rps = [1.0, 1.1, 0.8, float("nan"), 0.0]
    lens = [0, 3]
    params, hl = [], []
    for i, (t, tp, k, rp, n) in enumerate(itertools.product(temps, tps, tks, rps, lens)):
        p = SP(temperature=t, top_p=tp, top_k=k, repetition_penalty=rp)
        if i % 7 == 0:
            p.seed = [5, -1, 2**70 + 3][i % 3]
        params.append(p)
        hl.append(n)
    got = packing.derive_rows(params, V, hl)
    want = np.array([packing.derive_row(p, V, n) for p, n in zip(params, hl)], dtype=packing.ROW_DTYPE)
    assert got.tobytes() == want.tobytes()
