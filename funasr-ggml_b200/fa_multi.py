"""Multi-GPU plumbing for independent utterance streams (no data-path collectives).

Streams never interact, so the GPUs of one box each hold a weight replica and their
own page pool, and a host dispatcher gives each rank its share of the streams: a
contiguous split for equal streams (the decode benchmark), and the least-outstanding-
KV-pages rule for streams of mixed lengths (continuous batching).
torch.distributed (NCCL on GPUs, gloo in CPU tests) is used only for the start
barrier and for max/sum reductions of the timing numbers.
"""
from __future__ import annotations

import os
from datetime import timedelta
from typing import List, Sequence


def env_rank():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)),
            int(os.environ.get("WORLD_SIZE", 1)))


def init(backend: str = "nccl", timeout_s: int = 120):
    """Initialise the process group when launched with WORLD_SIZE > 1."""
    rank, local, world = env_rank()
    if world <= 1:
        return rank, local, world
    import torch
    import torch.distributed as dist
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    if backend == "nccl":
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=timeout_s), device_id=torch.device("cuda", local))
    else:
        dist.init_process_group(backend, timeout=timedelta(seconds=timeout_s))
    return rank, local, world


def _dev():
    import torch
    import torch.distributed as dist
    if dist.get_backend() == "nccl":
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device("cpu")


def barrier():
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized():
        if dist.get_backend() == "nccl":
            import torch
            dist.barrier(device_ids=[torch.cuda.current_device()])
        else:
            dist.barrier()


def reduce(value: float, op: str = "max") -> float:
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()):
        return float(value)
    import torch
    t = torch.tensor([float(value)], dtype=torch.float64, device=_dev())
    dist.all_reduce(t, op={"max": dist.ReduceOp.MAX, "sum": dist.ReduceOp.SUM, "min": dist.ReduceOp.MIN}[op])
    return float(t.item())


def gather(obj) -> List:
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()):
        return [obj]
    out = [None] * dist.get_world_size()
    dist.all_gather_object(out, obj)
    return out


def shard(items: Sequence, rank: int, world: int) -> list:
    """Contiguous, balanced share of `items` for `rank` (sizes differ by at most one)."""
    n = len(items)
    lo = rank * n // world
    hi = (rank + 1) * n // world
    return list(items[lo:hi])


def dispatch_by_pages(arrive, prompt_len, out_len, world: int, token_s: float = 0.02, page_tokens: int = 16):
    """Host dispatcher of independent streams: each stream, in arrival order, goes to the
    rank with the fewest outstanding KV pages at its arrival (ties to the lowest rank).
    A stream holds ceil((prompt + output) / page_tokens) pages from its arrival until its
    estimated finish, arrival + output * token_s (one token per decode step). Every rank
    computes the same assignment from the same seeded stream list, so nothing crosses
    between ranks. Returns the owning rank of each stream."""
    import heapq

    import numpy as np
    arrive = np.asarray(arrive, np.float64)
    plen = np.asarray(prompt_len, np.int64)
    olen = np.asarray(out_len, np.int64)
    n = len(arrive)
    owner = np.empty(n, np.int64)
    load = [0] * world
    live = [[] for _ in range(world)]          # per rank: heap of (finish time, pages)
    for i in np.argsort(arrive, kind="stable"):
        t = arrive[i]
        for r in range(world):
            h = live[r]
            while h and h[0][0] <= t:
                load[r] -= heapq.heappop(h)[1]
        r = min(range(world), key=lambda k: (load[k], k))
        pages = int((plen[i] + olen[i] + page_tokens - 1) // page_tokens)
        load[r] += pages
        heapq.heappush(live[r], (t + float(olen[i]) * token_s, pages))
        owner[i] = r
    return owner


def shutdown():
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized():
        dist.destroy_process_group()
