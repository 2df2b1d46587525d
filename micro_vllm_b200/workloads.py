"""Seeded synthetic batches with the shapes of the benchmark configurations.

All inputs are synthetic (there are no checkpoints or datasets here):
N(0,1) query/key/value values, KV pages scattered at random over a physical
pool, context lengths drawn uniformly.  A batch is built on the host with a
CPU generator, so the same seed gives the same batch on any device.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from micro_vllm_b200.attention import AttentionMetadata


@dataclass
class PagedBatch:
    query: torch.Tensor  # [T, Hq, D]
    key: torch.Tensor  # [T, Hkv, D]
    value: torch.Tensor
    cache: torch.Tensor  # [2, NB, bs, Hkv, D]
    metadata: AttentionMetadata
    context_lengths: list[int]
    query_lengths: list[int]

    @property
    def num_requests(self) -> int:
        return len(self.context_lengths)


def pool_blocks_for_fraction(fraction: float, block_size: int, num_kv_heads: int, head_dim: int,
                             dtype: torch.dtype, device: torch.device) -> int:
    """Physical pool size (blocks) holding `fraction` of the device's memory
    for ONE layer's [2, NB, bs, Hkv, D] cache."""

    total = torch.cuda.get_device_properties(device).total_memory
    per_block = 2 * block_size * num_kv_heads * head_dim * torch.finfo(dtype).bits // 8
    return int(total * fraction) // per_block


def fill_normal_(t: torch.Tensor, seed: int, chunk_elems: int = 1 << 30) -> torch.Tensor:
    """N(0,1) fill in chunks, so pools of ~150 GB need no temporary."""

    flat = t.view(-1)
    gen = torch.Generator(device=t.device).manual_seed(seed)
    for start in range(0, flat.numel(), chunk_elems):
        flat[start : start + chunk_elems].normal_(generator=gen)
    return t


def paged_batch(
    *,
    context_lengths: list[int],
    query_lengths: list[int],
    num_q_heads: int,
    num_kv_heads: int,
    head_dim: int,
    block_size: int,
    num_blocks: int,
    dtype: torch.dtype,
    device: torch.device | str,
    seed: int,
    cache: torch.Tensor | None = None,
    fill_cache: bool = True,
    window: int | None = None,
) -> PagedBatch:
    """Requests whose last `query_lengths[r]` positions are this step's
    queries over a history of `context_lengths[r]` tokens.

    Each request owns ceil(ctx / bs) distinct pool blocks drawn without
    replacement from the whole pool; the step's K/V are new values whose
    slots the operator writes.  `window` selects sliding-window visibility.
    """

    device = torch.device(device)
    gen = torch.Generator().manual_seed(seed)
    need = [-(-c // block_size) for c in context_lengths]
    if sum(need) > num_blocks:
        raise ValueError("pool too small for the batch")
    chosen = torch.randperm(num_blocks, generator=gen)[: sum(need)]
    width = max(need) if need else 1
    table = torch.zeros((len(context_lengths), max(width, 1)), dtype=torch.int64)
    cursor = 0
    for r, n in enumerate(need):
        table[r, :n] = chosen[cursor : cursor + n]
        cursor += n
    positions, qsl = [], [0]
    for c, q in zip(context_lengths, query_lengths):
        positions.extend(range(c - q, c))
        qsl.append(qsl[-1] + q)
    pos = torch.tensor(positions, dtype=torch.int64)
    req_of_tok = torch.repeat_interleave(torch.arange(len(context_lengths)), torch.tensor(query_lengths))
    slots = table[req_of_tok, pos // block_size] * block_size + pos % block_size
    starts = torch.zeros_like(pos) if window is None else (pos - (window - 1)).clamp(min=0)
    num_tokens = len(positions)
    qkv_gen = torch.Generator().manual_seed(seed + 1)
    query = torch.randn((num_tokens, num_q_heads, head_dim), generator=qkv_gen).to(dtype)
    key = torch.randn((num_tokens, num_kv_heads, head_dim), generator=qkv_gen).to(dtype)
    value = torch.randn((num_tokens, num_kv_heads, head_dim), generator=qkv_gen).to(dtype)
    if cache is None:
        cache = torch.empty((2, num_blocks, block_size, num_kv_heads, head_dim), dtype=dtype, device=device)
        if fill_cache:
            if device.type == "cuda":
                fill_normal_(cache, seed + 2)
            else:
                cache.copy_(torch.randn(cache.shape, generator=torch.Generator().manual_seed(seed + 2)))
    md = AttentionMetadata(
        query_positions=pos.to(device),
        query_context_start_positions=starts.to(device),
        query_start_locations=torch.tensor(qsl, dtype=torch.int64, device=device),
        context_lengths=torch.tensor(context_lengths, dtype=torch.int64, device=device),
        block_table=table.to(device),
        slot_mapping=slots.to(device),
        block_size=block_size,
    )
    return PagedBatch(
        query=query.to(device),
        key=key.to(device),
        value=value.to(device),
        cache=cache,
        metadata=md,
        context_lengths=list(context_lengths),
        query_lengths=list(query_lengths),
    )


def uniform_lengths(n: int, lo: int, hi: int, seed: int) -> list[int]:
    gen = torch.Generator().manual_seed(seed)
    return torch.randint(lo, hi + 1, (n,), generator=gen).tolist()
