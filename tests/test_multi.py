"""world_size-2 gloo test of the multi-GPU plumbing on CPU: sharding of independent
streams, the start barrier and the max/sum reductions bench.py times with."""
import os
import socket

import pytest

import fa_multi


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(RANK=str(rank), LOCAL_RANK=str(rank), WORLD_SIZE=str(world), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    try:
        r, local, w = fa_multi.init("gloo", timeout_s=60)
        streams = list(range(13))
        mine = fa_multi.shard(streams, r, w)
        fa_multi.barrier()
        mx = fa_multi.reduce(1.5 + r, "max")
        sm = fa_multi.reduce(len(mine), "sum")
        allshards = fa_multi.gather(mine)
        fa_multi.shutdown()
        q.put((r, mine, mx, sm, allshards))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, "error", repr(e), None, None))


def test_shard_is_a_balanced_partition():
    items = list(range(10))
    parts = [fa_multi.shard(items, r, 3) for r in range(3)]
    assert sum(parts, []) == items
    assert max(map(len, parts)) - min(map(len, parts)) <= 1


def test_two_rank_gloo_barrier_reduce_and_shards():
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r, mine, mx, sm, allshards in res:
        assert mine != "error", mx
        assert mx == 2.5 and sm == 13
        assert sum(allshards, []) == list(range(13))
        assert mine == allshards[r]
