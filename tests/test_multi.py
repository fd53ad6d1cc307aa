"""world_size-2 gloo test of the multi-GPU plumbing on CPU: sharding of independent
streams, the page-aware stream dispatcher, the start barrier and the max/sum
reductions bench.py times with."""
import os
import socket

import pytest

import fa_multi


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _skewed_streams(n=400, seed=7):
    """Arrivals at 100/s; the first half of the streams are long (prompts ~5000, outputs
    ~400 tokens), the second half short, so a contiguous split is badly unbalanced."""
    import numpy as np
    rng = np.random.default_rng(seed)
    arrive = np.cumsum(rng.exponential(0.01, n))
    plen = np.where(np.arange(n) < n // 2, rng.integers(4000, 6000, n), rng.integers(200, 400, n))
    olen = np.where(np.arange(n) < n // 2, rng.integers(300, 512, n), rng.integers(16, 40, n))
    return arrive, plen, olen


def _pages(plen, olen):
    return (plen + olen + 15) // 16


def _dispatch_worker(rank, world, port, q):
    os.environ.update(RANK=str(rank), LOCAL_RANK=str(rank), WORLD_SIZE=str(world), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    try:
        import numpy as np
        r, local, w = fa_multi.init("gloo", timeout_s=60)
        arrive, plen, olen = _skewed_streams()
        owner = fa_multi.dispatch_by_pages(arrive, plen, olen, w)
        mine = [int(i) for i in np.flatnonzero(owner == r)]
        my_pages = int(_pages(plen, olen)[mine].sum())
        total = fa_multi.reduce(my_pages, "sum")
        hi = fa_multi.reduce(my_pages, "max")
        allmine = fa_multi.gather(mine)
        fa_multi.shutdown()
        q.put((r, mine, total, hi, allmine))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, "error", repr(e), None, None))


def _run_ranks(target, world=2):
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return res


def test_page_dispatcher_balances_skewed_streams_over_two_gloo_ranks():
    """Each rank computes the assignment on its own; together the ranks hold every stream
    once, and their KV page totals are within 10 % of each other where the contiguous
    split gives one rank several times the other's pages."""
    import numpy as np
    arrive, plen, olen = _skewed_streams()
    pages = _pages(plen, olen)
    res = _run_ranks(_dispatch_worker)
    for r, mine, total, hi, allmine in res:
        assert mine != "error", total
        assert sorted(sum(allmine, [])) == list(range(len(arrive)))
        assert mine == allmine[r]
        assert total == pages.sum()
        lo = total - hi
        assert hi <= 1.10 * lo, (hi, lo)
    split = [pages[fa_multi.shard(list(range(len(arrive))), r, 2)].sum() for r in range(2)]
    assert max(split) > 3 * min(split)


def test_page_dispatcher_follows_outstanding_pages():
    """A stream that has finished no longer counts: after the first rank's long stream
    ends, the next arrival may go to it again."""
    owner = fa_multi.dispatch_by_pages([0.0, 0.1, 0.2, 10.0], [5000, 100, 100, 100], [100, 10, 10, 10], 2,
                                       token_s=0.02)
    # stream 0 (320 pages) on rank 0 until t = 2.0; 1 and 2 go to rank 1; at t = 10 both are empty
    assert owner.tolist() == [0, 1, 1, 0]


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
