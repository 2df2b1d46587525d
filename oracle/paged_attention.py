"""CPU oracle for the paged-attention hot path — TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, the algorithm of micro-vLLM's readable
reference attention backend so that the CUDA kernels of ``micro_vllm_b200``
can be checked against it.  It is imported only by ``tests/``, by
``__graft_entry__.smoke()`` and by the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py``.  The product path never calls it: the operator in
``micro_vllm_b200`` raises when its CUDA library is missing instead of
falling back here.

Parity pin: ``tests/golden/make_golden.py`` ran the reference's own
``ReferenceAttentionOperator`` and ``write_kv_cache`` (imported from the
reference source tree) on seeded inputs and stored inputs and outputs under
``tests/golden/``; ``tests/test_oracle.py`` checks this restatement
against those vectors and against the reference tests' known answers.

Reference functions restated here (paths inside the reference project):

* ``map_cache_slots``          — src/micro_vllm/attention/attention.py:31-41
* spec ``context_start``        — src/micro_vllm/attention/spec.py:18-51
* ``write_kv_cache``           — src/micro_vllm/attention/operators/reference.py:84-98
* ``gather_kv_cache``          — src/micro_vllm/attention/operators/reference.py:101-138
* ``ReferenceAttentionOperator.forward``
                               — src/micro_vllm/attention/operators/reference.py:14-81

Two deliberate, documented differences, both taken from the reference's
Triton backend (src/micro_vllm/attention/operators/triton_paged.py) because
the engine's CUDA-graph padding relies on them
(src/micro_vllm/worker/model_runner.py:78-122):

* a negative slot in ``slot_mapping`` writes nothing (the readable reference
  raises ``IndexError`` from ``index_copy_``; the Triton kernel masks the
  store, triton_paged.py:37-39,62-68);
* output rows of tokens that belong to no request (zero-length padded
  requests) are zero (the readable reference leaves them uninitialised via
  ``torch.empty_like``; the Triton wrapper zero-fills, triton_paged.py:343).
"""

from __future__ import annotations

import math
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class OracleMetadata:
    """numpy mirror of ``AttentionMetadata`` (attention/attention.py:12-28)."""

    query_positions: np.ndarray  # int64 [T]
    query_context_start_positions: np.ndarray  # int64 [T]
    query_start_locations: np.ndarray  # int64 [R+1]
    context_lengths: np.ndarray  # int64 [R]
    block_table: np.ndarray  # int64 [R, W]
    slot_mapping: np.ndarray  # int64 [T]
    block_size: int

    @property
    def num_requests(self) -> int:
        return int(self.context_lengths.shape[0])


def full_context_start(position: int) -> int:
    """FullAttentionSpec.context_start (spec.py:18-23)."""

    return 0


def sliding_window_context_start(position: int, window_size: int) -> int:
    """SlidingWindowSpec.context_start (spec.py:26-37)."""

    return max(0, position - window_size + 1)


def chunked_local_context_start(position: int, chunk_size: int) -> int:
    """ChunkedLocalSpec.context_start (spec.py:40-51)."""

    return (position // chunk_size) * chunk_size


def map_cache_slots(
    positions: np.ndarray, block_table_row: np.ndarray, block_size: int
) -> np.ndarray:
    """Logical positions -> flattened physical slots (attention.py:31-41).

    Like ``index_select`` in the reference, an out-of-range logical block
    raises ``IndexError``.
    """

    positions = np.asarray(positions, dtype=np.int64)
    logical_blocks = positions // block_size
    offsets = positions % block_size
    if logical_blocks.size and (
        logical_blocks.min() < 0 or logical_blocks.max() >= block_table_row.shape[0]
    ):
        raise IndexError("logical block outside the block table")
    physical = np.asarray(block_table_row, dtype=np.int64)[logical_blocks]
    return physical * block_size + offsets


def write_kv_cache(
    key: np.ndarray,
    value: np.ndarray,
    layer_kv_cache: np.ndarray,
    slot_mapping: np.ndarray,
) -> None:
    """Scatter K/V rows into ``layer_kv_cache[2, NB, bs, Hkv, D]`` in place.

    Restates reference.py:84-98: the cache is viewed as ``[2, NB*bs, Hkv, D]``
    and row ``slot_mapping[t]`` of plane 0/1 receives ``key[t]``/``value[t]``.
    Negative slots are skipped (Triton-backend semantics, see module doc);
    slots past the pool raise ``IndexError`` as ``index_copy_`` does.
    """

    flat = layer_kv_cache.reshape(2, -1, *layer_kv_cache.shape[3:])
    slots = np.asarray(slot_mapping, dtype=np.int64)
    if slots.size and slots.max() >= flat.shape[1]:
        raise IndexError("slot outside the KV pool")
    keep = slots >= 0
    flat[0][slots[keep]] = key[keep]
    flat[1][slots[keep]] = value[keep]


def gather_kv_cache(
    layer_kv_cache: np.ndarray, md: OracleMetadata
) -> list[tuple[np.ndarray, np.ndarray]]:
    """Per-request visible K/V history (reference.py:101-138).

    Request r sees logical positions ``[ctx_start(first query), ctx_len)``.
    """

    flat = layer_kv_cache.reshape(2, -1, *layer_kv_cache.shape[3:])
    histories = []
    for r in range(md.num_requests):
        qs = int(md.query_start_locations[r])
        start = int(md.query_context_start_positions[qs])
        length = int(md.context_lengths[r])
        positions = np.arange(start, length, dtype=np.int64)
        slots = map_cache_slots(positions, md.block_table[r], md.block_size)
        if slots.size and (slots.min() < 0 or slots.max() >= flat.shape[1]):
            raise IndexError("physical slot outside the KV pool")
        histories.append((flat[0][slots], flat[1][slots]))
    return histories


def _attend_request(
    query: np.ndarray,
    layer_kv_cache: np.ndarray,
    md: OracleMetadata,
    r: int,
    scale: float,
) -> tuple[int, int, np.ndarray | None]:
    """Attention for one request in fp32 (reference.py:31-79)."""

    qs = int(md.query_start_locations[r])
    qe = int(md.query_start_locations[r + 1])
    if qe <= qs:
        return qs, qe, None
    flat = layer_kv_cache.reshape(2, -1, *layer_kv_cache.shape[3:])
    start = int(md.query_context_start_positions[qs])
    length = int(md.context_lengths[r])
    positions = np.arange(start, length, dtype=np.int64)
    slots = map_cache_slots(positions, md.block_table[r], md.block_size)
    keys = flat[0][slots].astype(np.float32)  # [n, Hkv, D]
    values = flat[1][slots].astype(np.float32)
    q = query[qs:qe].astype(np.float32)  # [L, Hq, D]
    num_q, num_heads, head_dim = q.shape
    num_kv_heads = keys.shape[1]
    group = num_heads // num_kv_heads
    n = keys.shape[0]
    if n == 0:
        return qs, qe, np.zeros((num_q, num_heads, head_dim), np.float32)

    # [Hkv, G*L, D] x [Hkv, D, n] -> [Hkv, G*L, n]; row = g*L + l.
    qh = q.reshape(num_q, num_kv_heads, group, head_dim).transpose(1, 2, 0, 3)
    qh = qh.reshape(num_kv_heads, group * num_q, head_dim)
    scores = np.matmul(qh, keys.transpose(1, 2, 0))
    scores = scores.reshape(num_kv_heads, group, num_q, n)

    # Mask keys outside [ctx_start(q), pos(q)] (reference.py:49-68).
    qpos = md.query_positions[qs:qe].astype(np.int64)
    qstart = md.query_context_start_positions[qs:qe].astype(np.int64)
    hidden = (positions[None, :] < qstart[:, None]) | (positions[None, :] > qpos[:, None])
    scores = np.where(hidden[None, None], np.float32(-np.inf), scores)

    # softmax(scores * scale) in fp32 (reference.py:69-73); a fully hidden
    # row yields NaN exactly as torch.softmax does.
    scaled = scores * np.float32(scale)
    with np.errstate(invalid="ignore"):
        row_max = scaled.max(axis=-1, keepdims=True)
        weights = np.exp(scaled - row_max)
        weights = weights / weights.sum(axis=-1, keepdims=True)

    # [Hkv, G*L, n] x [Hkv, n, D] -> [Hkv, G, L, D] -> [L, Hq, D]
    out = np.matmul(
        weights.reshape(num_kv_heads, group * num_q, n).astype(np.float32),
        values.transpose(1, 0, 2),
    )
    out = out.reshape(num_kv_heads, group, num_q, head_dim).transpose(2, 0, 1, 3)
    return qs, qe, out.reshape(num_q, num_heads, head_dim)


def paged_attention(
    query: np.ndarray,
    key: np.ndarray,
    value: np.ndarray,
    layer_kv_cache: np.ndarray,
    md: OracleMetadata,
    *,
    write: bool = True,
    out_dtype: np.dtype | None = None,
    num_threads: int = 1,
) -> np.ndarray:
    """``ReferenceAttentionOperator.forward`` restated (reference.py:14-81).

    Writes K/V first (so the current chunk sees itself), then computes, for
    every query token, softmax(q.K^T * 1/sqrt(D)) . V over the keys visible
    to it, with GQA head ``h`` reading KV head ``h // (Hq/Hkv)``.  Math is
    fp32; the result is cast to ``out_dtype`` (default: the query dtype).
    ``num_threads`` > 1 runs independent requests on a thread pool (numpy
    releases the GIL inside matmul); it changes no arithmetic.
    """

    if write:
        write_kv_cache(key, value, layer_kv_cache, md.slot_mapping)
    scale = 1.0 / math.sqrt(query.shape[-1])
    out_dtype = query.dtype if out_dtype is None else out_dtype
    output = np.zeros(query.shape, dtype=out_dtype)

    def run(r: int) -> None:
        qs, qe, out = _attend_request(query, layer_kv_cache, md, r, scale)
        if out is not None:
            output[qs:qe] = out.astype(out_dtype)

    if num_threads <= 1:
        for r in range(md.num_requests):
            run(r)
    else:
        with ThreadPoolExecutor(num_threads) as pool:
            list(pool.map(run, range(md.num_requests)))
    return output


def build_metadata(
    query_positions_per_request: list[list[int]],
    block_tables: list[list[int]],
    *,
    block_size: int,
    context_start=full_context_start,
    null_block: int = 0,
) -> OracleMetadata:
    """Assemble metadata the way the reference tests and ModelRunner do.

    Flattened positions, prefix-sum ``query_start_locations``,
    ``context_lengths = last position + 1``, block tables padded with
    ``null_block`` (model_runner.py:871-900) and slots from
    ``map_cache_slots`` (model_runner.py:833-869).
    """

    positions = [p for req in query_positions_per_request for p in req]
    qsl = [0]
    for req in query_positions_per_request:
        qsl.append(qsl[-1] + len(req))
    width = max((len(t) for t in block_tables), default=0)
    table = np.full((len(block_tables), max(width, 1)), null_block, dtype=np.int64)
    for i, t in enumerate(block_tables):
        table[i, : len(t)] = t
    slots = []
    for req, t in zip(query_positions_per_request, block_tables):
        row = np.asarray(t, dtype=np.int64)
        slots.extend(map_cache_slots(np.asarray(req, np.int64), row, block_size).tolist())
    return OracleMetadata(
        query_positions=np.asarray(positions, dtype=np.int64),
        query_context_start_positions=np.asarray(
            [context_start(p) for p in positions], dtype=np.int64
        ),
        query_start_locations=np.asarray(qsl, dtype=np.int64),
        context_lengths=np.asarray(
            [req[-1] + 1 if req else 0 for req in query_positions_per_request],
            dtype=np.int64,
        ),
        block_table=table,
        slot_mapping=np.asarray(slots, dtype=np.int64),
        block_size=block_size,
    )
