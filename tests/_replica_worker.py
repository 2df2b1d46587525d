"""Rank bodies for the multi-process (gloo, CPU) tests of the sequence
partitioner and the replica launcher.  The oracle stands in for each rank's
GPU kernel: these tests cover the host-side logic only."""

from __future__ import annotations

import time
from datetime import timedelta

import numpy as np


def global_batch(seed: int = 0, n: int = 24):
    """A seeded decode batch over one shared logical pool description."""

    from oracle import build_metadata

    rng = np.random.default_rng(seed)
    ctx = rng.integers(1, 300, size=n).tolist()
    bs, hq, hkv, d = 16, 4, 2, 32
    tables, cursor = [], 0
    for c in ctx:
        nb = -(-c // bs)
        tables.append(list(range(cursor, cursor + nb)))
        cursor += nb
    cache = rng.standard_normal((2, cursor, bs, hkv, d)).astype(np.float32)
    q = rng.standard_normal((n, hq, d)).astype(np.float32)
    k = rng.standard_normal((n, hkv, d)).astype(np.float32)
    v = rng.standard_normal((n, hkv, d)).astype(np.float32)
    md = build_metadata([[c - 1] for c in ctx], tables, block_size=bs)
    return ctx, tables, cache, q, k, v, md


def shard_and_attend(rank: int, world_size: int, result_path: str) -> None:
    """Each rank takes its LPT shard of the global batch, rebuilds a local
    pool holding only its sequences' pages (as a per-GPU pool would), runs
    attention on it, and rank 0 gathers everything over gloo."""

    import torch.distributed as dist

    from micro_vllm_b200.partition import partition_sequences, sequence_work
    from oracle import build_metadata, paged_attention

    dist.init_process_group("gloo", timeout=timedelta(seconds=30))
    ctx, tables, cache, q, k, v, _ = global_batch()
    shards = partition_sequences([sequence_work(c) for c in ctx], world_size)
    mine = shards[rank].indices
    local_tables, pages, cursor = [], [], 0
    for i in mine:
        local_tables.append(list(range(cursor, cursor + len(tables[i]))))
        pages.extend(tables[i])
        cursor += len(tables[i])
    local_cache = cache[:, pages].copy()
    md = build_metadata([[ctx[i] - 1] for i in mine], local_tables, block_size=16)
    idx = list(mine)
    out = paged_attention(q[idx], k[idx], v[idx], local_cache, md)
    gathered = [None] * world_size
    dist.all_gather_object(gathered, (list(mine), out))
    if rank == 0:
        full = np.zeros_like(q)
        for ids, o in gathered:
            full[ids] = o
        np.save(result_path, full)
    dist.barrier()
    dist.destroy_process_group()


def fail_on_rank_one(rank: int, world_size: int) -> None:
    if rank == 1:
        raise RuntimeError("injected failure on rank 1")


def hang_on_rank_one(rank: int, world_size: int) -> None:
    """Rank 1 never joins; rank 0's collective times out and errors."""

    import torch.distributed as dist

    dist.init_process_group("gloo", timeout=timedelta(seconds=3))
    if rank == 1:
        time.sleep(600)
    dist.barrier()


def fail_fast_while_rank_zero_waits(rank: int, world_size: int) -> None:
    """Rank 1 fails at once; rank 0 blocks in a barrier with a long timeout."""

    import torch.distributed as dist

    if rank == 1:
        raise RuntimeError("injected failure on rank 1")
    dist.init_process_group("gloo", timeout=timedelta(seconds=300))
    dist.barrier()


def sleep_on_rank_one(rank: int, world_size: int) -> None:
    """Rank 1 never returns and takes no collective; rank 0 finishes."""

    if rank == 1:
        time.sleep(600)
