"""Whole-sequence partitioning over GPUs (data-parallel replicas).

The paged-attention path shards by whole sequences: a sequence's KV pages
live in one GPU's pool and its attention reads nothing else, so N GPUs are N
independent replicas — the reference's own plan for data parallelism
(docs/requirements/v2-distributed.md:93-105 in the reference project: each
replica owns its engine, scheduler, model and KV cache, with no step-level
synchronisation).  There is no collective on the data path.

``partition_sequences`` assigns sequences to ranks by longest-processing-time
first: heaviest sequence to the currently lightest rank.  Work of a sequence
is its KV length (what paged attention streams) plus, for prefill, its new
tokens.  The assignment is deterministic (ties broken by index), so every
rank computes the same partition without communicating.
"""

from __future__ import annotations

import heapq
from dataclasses import dataclass
from typing import Sequence


@dataclass(frozen=True)
class Shard:
    rank: int
    indices: tuple[int, ...]  # positions in the global request list, ascending
    work: int


def sequence_work(context_length: int, new_tokens: int = 1) -> int:
    """Cost model: KV tokens streamed + query tokens computed."""

    return int(context_length) + int(new_tokens)


def partition_sequences(
    work: Sequence[int], num_ranks: int
) -> list[Shard]:
    """LPT-greedy partition of sequences (given their work) over ranks."""

    if num_ranks <= 0:
        raise ValueError("num_ranks must be positive")
    order = sorted(range(len(work)), key=lambda i: (-int(work[i]), i))
    heap = [(0, r) for r in range(num_ranks)]
    assigned: list[list[int]] = [[] for _ in range(num_ranks)]
    loads = [0] * num_ranks
    for i in order:
        load, r = heapq.heappop(heap)
        assigned[r].append(i)
        loads[r] = load + int(work[i])
        heapq.heappush(heap, (loads[r], r))
    return [Shard(rank=r, indices=tuple(sorted(assigned[r])), work=loads[r]) for r in range(num_ranks)]


def imbalance(shards: Sequence[Shard]) -> float:
    """max / mean work over ranks (1.0 = perfect balance)."""

    works = [s.work for s in shards]
    mean = sum(works) / max(len(works), 1)
    return max(works) / mean if mean > 0 else 1.0
