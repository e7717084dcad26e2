"""Sequence sharding for multi-GPU decode (one process per GPU, no collective).

Configs with independent sequences (C2, C3, C5) split the batch across ranks:
each rank owns whole sequences, their pools and their outputs, so the decode
step needs no exchange.  Sequences go to ranks longest-processing-time first by
the bytes a decode step streams for them (cold tokens x 400 B + hot and new
tokens x 1152 B), which keeps the per-rank HBM traffic within one sequence of
the mean.
"""
from __future__ import annotations

import heapq

COLD_TOKEN_BYTES = 256 + 16 + 128
HOT_TOKEN_BYTES = 1024 + 128


def step_bytes(length: int, hot: int, q_len: int = 1) -> int:
    """Cache bytes one decode step reads for a sequence of `length` cached tokens, `hot` of them BF16."""
    hot = min(hot, length)
    return (length - hot) * COLD_TOKEN_BYTES + (hot + q_len) * HOT_TOKEN_BYTES


def lpt_shard(costs: list[int], world: int) -> list[list[int]]:
    """Indices of `costs` per rank: largest first, each to the currently lightest rank.

    Deterministic (ties go to the lower rank / lower index), so every rank
    computes the same assignment without communicating.
    """
    if world <= 0:
        raise ValueError("world must be positive")
    heap = [(0, r) for r in range(world)]
    out: list[list[int]] = [[] for _ in range(world)]
    for i in sorted(range(len(costs)), key=lambda i: (-costs[i], i)):
        load, r = heapq.heappop(heap)
        out[r].append(i)
        heapq.heappush(heap, (load + costs[i], r))
    for r in range(world):
        out[r].sort()
    return out


def shard_sequences(lengths: list[int], hot: list[int], world: int, q_len: int = 1) -> list[list[int]]:
    return lpt_shard([step_bytes(n, h, q_len) for n, h in zip(lengths, hot)], world)
