"""Request sharding across GPUs for the attention hot path.

Sequences are independent, so a batch is partitioned by request: each GPU owns its
requests' pages, block tables and pool and runs the same kernels; nothing crosses GPUs on
the attention path.  Decode attention time is proportional to the KV bytes a GPU reads, so
the partition balances total context length (longest-processing-time-first greedy), not the
request count.

TP2 splits heads instead, exactly as the reference engine does (docs/implementation.md:15,
weights.py:56-58): rank r of a pair holds query heads [r*H/2, (r+1)*H/2) and KV heads
[r*KVH/2, (r+1)*KVH/2) of every sequence of the pair.
"""
from __future__ import annotations

import heapq


def shard_requests(lengths, world: int) -> list[list[int]]:
    """Partitions request indices over `world` ranks, balancing sum(lengths) per rank.

    Longest request first, each to the currently lightest rank (ties: lower rank, then fewer
    requests).  Deterministic; every index appears in exactly one shard, each shard sorted.
    """
    if world < 1:
        raise ValueError("world must be >= 1")
    order = sorted(range(len(lengths)), key=lambda i: (-int(lengths[i]), i))
    heap = [(0, 0, r) for r in range(world)]
    shards: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        load, count, r = heapq.heappop(heap)
        shards[r].append(i)
        heapq.heappush(heap, (load + int(lengths[i]), count + 1, r))
    return [sorted(s) for s in shards]


def tp_head_slice(rank: int, world: int, heads: int, kv_heads: int) -> tuple[slice, slice]:
    """(query-head slice, KV-head slice) of `rank` in a tensor-parallel group of `world`."""
    if heads % world or kv_heads % world:
        raise ValueError("heads and kv_heads must divide by the TP degree")
    qh, kvh = heads // world, kv_heads // world
    return slice(rank * qh, (rank + 1) * qh), slice(rank * kvh, (rank + 1) * kvh)
