"""Length-balanced assignment of decode sequences to GPUs.

Sequences are independent units of the decode step, so a batch shards across
the GPUs of one box by sequence, each GPU with its own block pool, block
tables, slot mapping and context lengths, and no collective on the attention
path. The assignment is LPT (longest processing time first): sort by cost
``context_len + kappa`` descending and give each sequence to the GPU with the
least cost so far. LPT's makespan is within 4/3 of optimal, and no assignment
can beat ``max(max_len, total / n_gpus)`` — the bound reported beside the
measured per-GPU times.
"""

from __future__ import annotations

import heapq

import numpy as np


def lpt_assign(lengths, n_ranks: int, kappa: float = 0.0) -> list[list[int]]:
    """Indices of the sequences each rank gets (each list in ascending order)."""
    if n_ranks < 1:
        raise ValueError("n_ranks must be >= 1")
    cost = np.asarray(lengths, dtype=np.float64) + kappa
    order = np.argsort(-cost, kind="stable")
    heap = [(0.0, r) for r in range(n_ranks)]
    heapq.heapify(heap)
    shards: list[list[int]] = [[] for _ in range(n_ranks)]
    for i in order:
        load, r = heapq.heappop(heap)
        shards[r].append(int(i))
        heapq.heappush(heap, (load + float(cost[i]), r))
    return [sorted(s) for s in shards]


def shard_loads(lengths, shards) -> list[int]:
    L = np.asarray(lengths, dtype=np.int64)
    return [int(L[s].sum()) if len(s) else 0 for s in shards]


def makespan_bound(lengths, n_ranks: int) -> float:
    """Lower bound on the largest per-rank load: max(max_len, total / n)."""
    L = np.asarray(lengths, dtype=np.float64)
    if L.size == 0:
        return 0.0
    return float(max(L.max(), L.sum() / n_ranks))
