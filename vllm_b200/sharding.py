"""Multi-GPU partitioning of the decode path (one process per GPU).

Request sharding: decode rows are independent, so each GPU owns a disjoint set
of requests, its own page pool and block tables, and no data-path collective
is needed.  Rows are assigned longest-first to the GPU with the least attended
tokens so far (greedy LPT), which bounds the slowest GPU to within one row of
the mean.  KV-head sharding splits the 8 KV heads (and their 4 query heads
each) evenly over 1, 2, 4 or 8 GPUs.
"""
from __future__ import annotations

import heapq

import numpy as np


def shard_by_request(lens, world: int) -> list[np.ndarray]:
    """Row indices per rank (each sorted ascending), balanced by sum of L."""
    lens = np.asarray(lens, dtype=np.int64)
    if world <= 0:
        raise ValueError("world must be positive")
    heap = [(0, r) for r in range(world)]
    owned: list[list[int]] = [[] for _ in range(world)]
    for i in sorted(range(lens.size), key=lambda j: (-int(lens[j]), j)):
        load, r = heapq.heappop(heap)
        owned[r].append(i)
        heapq.heappush(heap, (load + int(lens[i]), r))
    return [np.array(sorted(o), dtype=np.int64) for o in owned]


def shard_by_kv_head(world: int, kv_heads: int = 8) -> list[range]:
    """KV heads per rank: contiguous ranges of kv_heads / world."""
    if world <= 0 or kv_heads % world:
        raise ValueError("world must divide the number of KV heads")
    per = kv_heads // world
    return [range(r * per, (r + 1) * per) for r in range(world)]


def imbalance(lens, shards) -> float:
    """max over ranks of sum L divided by the mean (1.0 = perfect)."""
    lens = np.asarray(lens, dtype=np.int64)
    loads = [int(lens[s].sum()) for s in shards]
    mean = sum(loads) / len(loads)
    return max(loads) / mean if mean else 1.0
