"""Sequence sharding across the GPUs of one node.

Requests are independent: each has its own GDN state, anchor bank and
sampler stream, so the hot path shards by request with no collective on the
data path (the reference runs one model replica per GPU the same way,
``evaluate.py:131-146``).  This module holds the host side of that:

* ``shard_requests(lengths, world)`` — which requests each rank serves:
  prompts are dealt longest first to the rank with the fewest prompt tokens
  so far (ties to the lower rank), so per-rank prefill work stays balanced
  while the assignment is the same on every rank;
* ``gather_by_request(local, owned, total, group)`` — put per-request
  results back in request order on every rank (one ``all_gather_object``
  after the work, never inside it);
* ``max_over_ranks(value, group)`` — the slowest rank's time, which is the
  job's time.

Everything here works with any ``torch.distributed`` backend: ``nccl`` on
the GPUs, ``gloo`` in the CPU tests.
"""
from __future__ import annotations

import heapq
from typing import Sequence


def shard_requests(lengths: Sequence[int], world: int) -> list[list[int]]:
    """Request indices per rank, each list in ascending request order."""
    if world <= 0:
        raise ValueError('world must be positive')
    heap = [(0, r) for r in range(world)]
    owned: list[list[int]] = [[] for _ in range(world)]
    for i in sorted(range(len(lengths)), key=lambda i: (-int(lengths[i]), i)):
        load, r = heapq.heappop(heap)
        owned[r].append(i)
        heapq.heappush(heap, (load + int(lengths[i]), r))
    return [sorted(o) for o in owned]


def gather_by_request(local: Sequence, owned: Sequence[int], total: int, group=None) -> list:
    """Every rank's ``local`` results (one per request in ``owned``) in global
    request order, on every rank."""
    import torch.distributed as dist
    if len(local) != len(owned):
        raise ValueError('one local result per owned request')
    world = dist.get_world_size(group)
    parts: list = [None] * world
    dist.all_gather_object(parts, (list(owned), list(local)), group=group)
    out: list = [None] * total
    for idx, res in parts:
        for i, x in zip(idx, res):
            if out[i] is not None:
                raise RuntimeError(f'request {i} served by two ranks')
            out[i] = x
    missing = [i for i, x in enumerate(out) if x is None]
    if missing:
        raise RuntimeError(f'requests {missing[:8]} were served by no rank')
    return out


def max_over_ranks(value: float, group=None, device=None) -> float:
    """The largest ``value`` over the ranks of ``group`` (one all-reduce)."""
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
