"""Host side of the device-resident histories: the region allocator, the
per-step plan (which must equal packing.pack's CSR layout), and the C ABI's
host-side validation (no GPU needed)."""
import random

import numpy as np
import pytest

from conftest import pkg

history = pkg("history")
packing = pkg("packing")
cabi = pkg("_cabi")
W = pkg("workloads")
SP = pkg("config").SamplingParams


def test_allocator_first_fit_merge_and_full():
    a = history.RegionAllocator(100)
    s0 = a.alloc(30)
    s1 = a.alloc(30)
    s2 = a.alloc(40)
    assert (s0, s1, s2) == (0, 30, 60)
    with pytest.raises(MemoryError):
        a.alloc(1)
    a.free(s1, 30)
    assert a.alloc(10) == 30  # first fit into the hole
    a.free(s0, 30)
    a.free(30, 10)  # merges with [0, 30) into [0, 60)
    assert a.alloc(60) == 0
    a.free(0, 60)
    a.free(s2, 40)
    assert a.free_total() == 100
    assert a.alloc(100) == 0


def test_allocator_random_ops_keep_regions_disjoint():
    rng = random.Random(5)
    a = history.RegionAllocator(5000)
    live = []
    for _ in range(3000):
        if live and rng.random() < 0.45:
            s, n = live.pop(rng.randrange(len(live)))
            a.free(s, n)
        else:
            n = rng.randint(0, 200)
            try:
                s = a.alloc(n)
            except MemoryError:
                continue
            live.append((s, n))
        used = sum(n for _, n in live)
        assert used + a.free_total() == 5000
        spans = sorted((s, s + n) for s, n in live if n)
        for (_, e0), (s1, _) in zip(spans, spans[1:]):
            assert e0 <= s1
        assert all(0 <= s and s + n <= 5000 for s, n in live)


def test_plan_step_matches_packing():
    rng = np.random.default_rng(3)
    V = 32000
    params = W.mixed_params(37) + [SP(temperature=1.0, repetition_penalty=1.3), SP(temperature=0.5, repetition_penalty=0.7)]
    hists = W.histories(rng, len(params), 0, 300, V)
    hists[1] = []
    ref = packing.pack(params, hists, V)
    starts = rng.integers(0, 10_000, size=len(params))
    lengths = np.array([len(h) for h in hists])
    rows, offsets, src = history.plan_step(params, starts, lengths, V)
    assert rows.tobytes() == ref.row_params.tobytes()
    assert np.array_equal(offsets, ref.offsets)
    assert np.array_equal(src, starts)


@pytest.mark.parametrize(
    "call,match",
    [
        (lambda: cabi.ns_history_gather(16, 10, 16, 16, -1, 16), "num_rows"),
        (lambda: cabi.ns_history_gather(16, -1, 16, 16, 1, 16), "pool_size"),
        (lambda: cabi.ns_history_gather(16, 10, 0, 16, 1, 16), "null"),
        (lambda: cabi.ns_history_append(16, 10, 16, 16, 7, 1), "tokens_dtype"),
        (lambda: cabi.ns_history_append(0, 10, 16, 16, cabi.NS_OUT_I64, 1), "null"),
        (lambda: cabi.ns_history_append(16, 10, 16, 16, cabi.NS_OUT_I32, -2), "num_rows"),
    ],
)
def test_history_abi_validates_on_the_host(call, match):
    with pytest.raises(cabi.NsError, match=match):
        call()


def test_history_abi_zero_rows_is_a_no_op():
    cabi.ns_history_gather(0, 0, 0, 0, 0, 0)
    cabi.ns_history_append(0, 0, 0, 0, cabi.NS_OUT_I64, 0)
