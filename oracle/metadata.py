"""CPU oracle of the reference's per-step metadata build — TEST INFRASTRUCTURE ONLY.

numpy restatement of how the reference model runner turns a scheduler plan
into the batch tensors its attention layers read:

* ``ModelRunner._flatten_model_input`` (src/micro_vllm/worker/
  model_runner.py:751-831): input ids, positions, query start locations,
  context lengths, sampling rows, in plan order;
* ``_build_slot_mapping`` (model_runner.py:833-869) with ``map_cache_slots``
  (src/micro_vllm/attention/attention.py:31-41);
* ``_build_block_table`` (model_runner.py:871-900): rows padded with the
  null block id to the longest request;
* ``Attention.build_metadata`` (attention.py:56-85) with the specs of
  src/micro_vllm/attention/spec.py;
* ``_CudaGraphExecution.copy_input`` (model_runner.py:78-122): the padding
  to a captured capacity.

Only ``tests/`` and ``bench.py``'s CPU baseline import it.  Pinned by
``tests/golden/make_golden_metadata.py``, which ran the reference's own
methods on seeded plans.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class PlannedRequest:
    """The fields of a ScheduledRequest (core/scheduler_output.py) the build reads."""

    input_token_ids: tuple[int, ...]
    num_computed_tokens: int
    num_scheduled_tokens: int
    requires_sampling: bool
    block_ids: tuple[tuple[int, ...], ...]  # one tuple per cache group


def context_start(spec: tuple[str, int], position: int) -> int:
    """``AttentionSpec.context_start`` (spec.py): full, sliding window, chunked local."""

    kind, param = spec
    if kind == "full":
        return 0
    if kind == "sliding":
        return max(0, position - param + 1)
    if kind == "chunked":
        return (position // param) * param
    raise ValueError(kind)


def build(
    requests: list[PlannedRequest], block_size: int, null_block_id: int, specs: list[tuple[str, int]]
) -> dict[str, object]:
    """The unpadded batch: shared arrays plus one (block_table, slot_mapping,
    context_starts) triple per cache group."""

    ids = [t for r in requests for t in r.input_token_ids]
    positions = np.array(
        [p for r in requests for p in range(r.num_computed_tokens, r.num_computed_tokens + r.num_scheduled_tokens)],
        np.int64,
    )
    qsl = np.zeros(len(requests) + 1, np.int64)
    qsl[1:] = np.cumsum([r.num_scheduled_tokens for r in requests])
    ctx = np.array([r.num_computed_tokens + r.num_scheduled_tokens for r in requests], np.int64)
    rows = np.array([qsl[i + 1] - 1 for i, r in enumerate(requests) if r.requires_sampling], np.int64)
    groups = []
    for g, spec in enumerate(specs):
        width = max((len(r.block_ids[g]) for r in requests), default=0)
        table = np.full((len(requests), width), null_block_id, np.int64)
        slots = []
        for i, r in enumerate(requests):
            blocks = np.asarray(r.block_ids[g], np.int64)
            table[i, : len(blocks)] = blocks
            pos = np.arange(r.num_computed_tokens, r.num_computed_tokens + r.num_scheduled_tokens)
            slots.append(blocks[pos // block_size] * block_size + pos % block_size)  # IndexError past the table
        slot_mapping = np.concatenate(slots) if slots else np.zeros(0, np.int64)
        starts = np.array([context_start(spec, int(p)) for p in positions], np.int64)
        groups.append({"block_table": table, "slot_mapping": slot_mapping.astype(np.int64), "context_starts": starts})
    return {
        "input_ids": np.array(ids, np.int64),
        "positions": positions,
        "query_start_locations": qsl,
        "context_lengths": ctx,
        "sampling_rows": rows,
        "groups": groups,
    }


def pad(batch: dict[str, object], token_capacity: int, request_capacity: int, table_width: int,
        null_block_id: int) -> dict[str, object]:
    """``_CudaGraphExecution.copy_input``: the batch written into capacity-sized
    buffers (input ids, positions and starts 0, query start locations
    ``num_tokens``, context lengths 0, block table null, slots -1)."""

    t = len(batch["positions"])
    r = len(batch["context_lengths"])

    def into(n, fill, src):
        out = np.full(n, fill, np.int64)
        out[: len(src)] = src
        return out

    groups = []
    for grp in batch["groups"]:
        table = np.full((request_capacity, table_width), null_block_id, np.int64)
        src = grp["block_table"]
        table[: src.shape[0], : src.shape[1]] = src
        groups.append({
            "block_table": table,
            "slot_mapping": into(token_capacity, -1, grp["slot_mapping"]),
            "context_starts": into(token_capacity, 0, grp["context_starts"]),
        })
    return {
        "input_ids": into(token_capacity, 0, batch["input_ids"]),
        "positions": into(token_capacity, 0, batch["positions"]),
        "query_start_locations": into(request_capacity + 1, t, batch["query_start_locations"]),
        "context_lengths": into(request_capacity, 0, batch["context_lengths"]),
        "sampling_rows": batch["sampling_rows"],
        "groups": groups,
        "num_requests": r,
    }
