"""Partition of a ragged batch of eviction work across ranks (one process per GPU).

The eviction path is independent per (sequence, KV head, layer): selection works
on one head's row (dropkv_cache.py:474), the GQA sum stays inside one KV head's
query group (dropkv_triton.py:541, 603-606), keep_len is a per-sequence host
constant and layers never interact.  So a batch shards with no communication on
the data path: every rank derives the same plan from the same inputs (sequence
lengths, layer count, world size) and runs its own units.

A unit here is one (sequence, layer) pair: all KV heads of that layer of that
sequence, i.e. one ``dropkv_compress`` call of B = 1.  Its cost is proportional to
its key count Lk (K and V are streamed once), so units are balanced by
longest-processing-time-first: the heaviest unit goes to the least loaded rank.
That spreads every sequence over all ranks, though, and a rank makes one call
per sequence it holds; ``contiguous_partition`` instead cuts the units, in
(sequence, layer) order, into runs of nearly equal work, so a rank holds whole
layer ranges of a few sequences and makes a few large calls.
"""

from __future__ import annotations

import heapq
from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True, order=True)
class Unit:
    seq: int
    layer: int
    lk: int


def ragged_lengths(n_seq: int = 16, lo: int = 4096, hi: int = 65536, seed: int = 5) -> list[int]:
    """Seeded sequence lengths drawn uniformly from [lo, hi] (the ragged batch)."""
    rng = np.random.default_rng(seed)
    return [int(x) for x in rng.integers(lo, hi + 1, size=n_seq)]


def make_units(lengths: list[int], layers: int) -> list[Unit]:
    return [Unit(s, l, int(lk)) for s, lk in enumerate(lengths) for l in range(layers)]


def lpt_partition(units: list[Unit], n_ranks: int) -> list[list[Unit]]:
    """Assign units to ranks, heaviest first, each to the currently least loaded
    rank (ties to the lower rank).  Deterministic; every unit is placed once."""
    if n_ranks < 1:
        raise ValueError("n_ranks must be >= 1")
    parts: list[list[Unit]] = [[] for _ in range(n_ranks)]
    heap = [(0, r) for r in range(n_ranks)]
    for u in sorted(units, key=lambda u: (-u.lk, u.seq, u.layer)):
        load, r = heapq.heappop(heap)
        parts[r].append(u)
        heapq.heappush(heap, (load + u.lk, r))
    for p in parts:
        p.sort()
    return parts


def contiguous_partition(units: list[Unit], n_ranks: int) -> list[list[Unit]]:
    """Units in (sequence, layer) order cut into ``n_ranks`` consecutive runs: a
    unit goes to the next rank once the work before its midpoint passes that
    rank's share, so each rank's load is within half a unit of an equal split at
    both of its ends. Deterministic; every unit is placed once."""
    if n_ranks < 1:
        raise ValueError("n_ranks must be >= 1")
    order = sorted(units, key=lambda u: (u.seq, u.layer))
    total = sum(u.lk for u in order)
    parts: list[list[Unit]] = [[] for _ in range(n_ranks)]
    acc, r = 0, 0
    for u in order:
        while r < n_ranks - 1 and 2 * acc + u.lk > 2 * (r + 1) * total / n_ranks:
            r += 1
        parts[r].append(u)
        acc += u.lk
    return parts


PARTITIONS = {"lpt": lpt_partition, "contiguous": contiguous_partition}


def rank_plan(rank: int, n_ranks: int, lengths: list[int], layers: int, method: str = "lpt") -> list[Unit]:
    """The units rank ``rank`` of ``n_ranks`` runs."""
    if not 0 <= rank < n_ranks:
        raise ValueError(f"rank {rank} outside [0, {n_ranks})")
    return PARTITIONS[method](make_units(lengths, layers), n_ranks)[rank]


def head_range(rank: int, n_ranks: int, n_heads: int) -> tuple[int, int]:
    """KV heads [h0, h1) of one layer that rank ``rank`` of ``n_ranks`` scores when a
    single layer is split by KV head (contiguous runs, sizes differing by at most
    one; ranks beyond the head count get an empty range)."""
    if not 0 <= rank < n_ranks:
        raise ValueError(f"rank {rank} outside [0, {n_ranks})")
    return (rank * n_heads) // n_ranks, ((rank + 1) * n_heads) // n_ranks


def load_imbalance(parts: list[list[Unit]]) -> float:
    """Largest rank load over the mean load (1.0 = perfect balance)."""
    loads = [sum(u.lk for u in p) for p in parts]
    mean = sum(loads) / len(loads)
    return max(loads) / mean if mean > 0 else 1.0
