"""Sequence sharding for batched decode across the GPUs of one box.

Independent sequences need no exchange during decode, so each rank owns a
subset and runs its own engine; there is no collective on the hot path. The
per-step cost of a sequence is dominated by reading its KV cache, which grows
with its context, so shards are balanced by total KV positions (prompt length
+ steps), not by count: longest-processing-time-first greedy assignment.
"""
from __future__ import annotations

import heapq


def plan_shards(contexts: list[int], world: int) -> list[list[int]]:
    """Partition sequence indices into `world` shards with near-equal total
    context. Deterministic: ties go to the lower rank / lower index."""
    if world < 1:
        raise ValueError("world must be >= 1")
    order = sorted(range(len(contexts)), key=lambda i: (-contexts[i], i))
    heap = [(0, r) for r in range(world)]
    shards: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        load, r = heapq.heappop(heap)
        shards[r].append(i)
        heapq.heappush(heap, (load + contexts[i], r))
    return [sorted(s) for s in shards]


def shard_imbalance(contexts: list[int], shards: list[list[int]]) -> float:
    """max shard load / mean shard load (1.0 = perfect)."""
    loads = [sum(contexts[i] for i in s) for s in shards]
    mean = sum(loads) / len(loads)
    return max(loads) / mean if mean else 1.0
