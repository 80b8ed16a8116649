"""Row sharding + the single all-gather, on CPU ranks over gloo (world size 2 and 3).

The per-rank compute is a deterministic stand-in (token = f(global row)) so
that the partition, padding, all-gather and reassembly logic is checked
without a GPU; a dead rank must surface as an error, not a hang.
"""
import importlib
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import PKG_NAME

sharded = importlib.import_module(PKG_NAME + ".sharded")


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_shard_bounds_cover_rows_exactly():
    for total in (0, 1, 7, 256, 16384, 16385):
        for world in (1, 2, 3, 8):
            seen = []
            for r in range(world):
                lo, hi = sharded.shard_bounds(total, world, r)
                assert hi - lo <= sharded.block_rows(total, world)
                seen.extend(range(lo, hi))
            assert seen == list(range(total))


def _worker(rank, world, port, total, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        s = sharded.ShardedSampler("cpu")

        def local(lo, hi, out):
            out.copy_((torch.arange(lo, hi, dtype=torch.int32) * 7 + 3) % 128256)

        got = s.step(total, local)
        q.put((rank, got.tolist()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,total", [(2, 16384), (2, 7), (3, 10)])
def test_all_gather_reassembles_the_batch(world, total):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, total, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    want = [(i * 7 + 3) % 128256 for i in range(total)]
    for r in range(world):
        assert results[r] == want


def _dying_worker(rank, world, port, q):
    import datetime

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(0)  # leaves between steps, before the collective
    s = sharded.ShardedSampler("cpu")
    try:
        s.step(8, lambda lo, hi, out: out.zero_())
        q.put("no error")
    except Exception as e:  # noqa: BLE001
        q.put(type(e).__name__)


def test_dead_rank_surfaces_as_an_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dying_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert res != "no error"
