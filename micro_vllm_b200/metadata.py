"""Device-side build of a step's model input (``mvb_build_metadata``).

The reference model runner turns a scheduler plan into batch tensors on the
host (src/micro_vllm/worker/model_runner.py:724-900): Python loops for the
positions, query start locations, context lengths and sampling rows; per
request a ``torch.tensor`` of its block ids and a device ``arange`` for its
slot mapping (``map_cache_slots``, attention/attention.py:31-41); per request
a row copy into the null-padded block table; and per cache group a host loop
over positions for the visibility starts (``Attention.build_metadata``,
attention.py:56-85).  With a captured CUDA graph, ``copy_input``
(model_runner.py:78-122) then copies everything into the graph's fixed
buffers, padded to the captured capacity.

``DeviceMetadataBuilder.build(plan)`` reads the same plan fields, packs the
per-request counts, token ids and block ids into one pinned int32 buffer,
issues ONE host-to-device copy and one ``mvb_build_metadata`` launch per
cache group, and returns the same tensors (int64, on the device).  Built with
capacities, it writes into fixed-address buffers padded exactly as
``copy_input`` pads them, so a captured graph replays on them directly.
"""

from __future__ import annotations

import itertools
from dataclasses import dataclass

import numpy as np
import torch

from micro_vllm_b200 import _lib
from micro_vllm_b200.attention import AttentionMetadata


def spec_code(spec) -> tuple[int, int]:
    """(MVB_SPEC_*, parameter) of a visibility spec of this package or of the
    reference (attention/spec.py), recognised by its fields."""

    window = getattr(spec, "window_size", None)
    if isinstance(window, int) and window > 0:
        return _lib.MVB_SPEC_SLIDING_WINDOW, window
    chunk = getattr(spec, "chunk_size", None)
    if isinstance(chunk, int) and chunk > 0:
        return _lib.MVB_SPEC_CHUNKED_LOCAL, chunk
    if type(spec).__name__ == "FullAttentionSpec":
        return _lib.MVB_SPEC_FULL, 0
    raise ValueError(f"{type(spec).__name__} has no device form (full, sliding window, chunked local)")


@dataclass(frozen=True, slots=True, eq=False)
class StepInput:
    """The reference's ModelInput (model_runner.py:50-66): the batch tensors
    one step's model forward reads."""

    input_ids: torch.Tensor
    positions: torch.Tensor
    layer_attention_metadata: tuple[AttentionMetadata, ...]
    request_ids: tuple[str, ...]
    sampling_row_indices: torch.Tensor


class DeviceMetadataBuilder:
    """Builds ``StepInput`` from a scheduler plan with one upload and one
    launch per cache group.

    ``layer_specs``: the visibility spec of every layer in model order
    (``model.layer_attentions[i].spec``); layers with equal specs share a
    cache group, numbered in order of first appearance, as
    ``build_kv_cache_topology`` (core/kv_cache_spec.py:52-80) numbers them.
    The plan is read through the fields of the reference's SchedulerOutput
    (``scheduled_requests``; per request ``request_id``, ``input_token_ids``,
    ``num_computed_tokens``, ``num_scheduled_tokens``, ``requires_sampling``,
    ``block_tables[group].block_ids``).

    With ``token_capacity`` / ``request_capacity`` / ``table_width`` set, the
    outputs are fixed-address buffers of those sizes, padded as
    ``_CudaGraphExecution.copy_input`` pads them (the block table is
    ``table_width`` wide for every group)."""

    __slots__ = (
        "device", "block_size", "null_block_id", "group_of_layer", "group_codes",
        "token_capacity", "request_capacity", "table_width", "_fixed", "_slots", "_next", "status",
    )

    def __init__(
        self,
        layer_specs,
        block_size: int,
        null_block_id: int,
        device: torch.device | str,
        *,
        token_capacity: int | None = None,
        request_capacity: int | None = None,
        table_width: int | None = None,
    ) -> None:
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise RuntimeError("DeviceMetadataBuilder requires a CUDA device (no CPU fallback)")
        if block_size <= 0:
            raise ValueError("block_size must be positive")
        self.block_size = int(block_size)
        self.null_block_id = int(null_block_id)
        codes: list[tuple[int, int]] = []
        group_of_layer = []
        for spec in layer_specs:
            code = spec_code(spec)
            if code not in codes:
                codes.append(code)
            group_of_layer.append(codes.index(code))
        if not codes:
            raise ValueError("at least one layer spec is required")
        self.group_codes = tuple(codes)
        self.group_of_layer = tuple(group_of_layer)
        caps = (token_capacity, request_capacity, table_width)
        if any(c is not None for c in caps) and any(c is None for c in caps):
            raise ValueError("token_capacity, request_capacity and table_width go together")
        self.token_capacity, self.request_capacity, self.table_width = caps
        self._fixed = None
        if token_capacity is not None:
            self._fixed = self._allocate(token_capacity, request_capacity, [table_width] * len(codes))
        # Two staging slots (pinned host buffer, device buffer, upload event),
        # so the next step can be staged while the current one is launched.
        self._slots = [_Staging(self.device), _Staging(self.device)]
        self._next = 0
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)

    def _allocate(self, t: int, r: int, widths: list[int]) -> dict:
        i64 = dict(dtype=torch.int64, device=self.device)
        return {
            "input_ids": torch.empty(t, **i64),
            "positions": torch.empty(t, **i64),
            "qsl": torch.empty(r + 1, **i64),
            "ctx": torch.empty(r, **i64),
            "rows": torch.empty(r, **i64),
            "groups": [(torch.empty(t, **i64), torch.empty(t, **i64), torch.empty((r, w), **i64))
                       for w in widths],
        }

    def read_status(self) -> int:
        """Return and clear the device status bits (synchronises)."""

        value = int(self.status.item())
        self.status.zero_()
        return value

    def build(self, plan, /) -> StepInput:
        """``stage(plan)`` then ``launch`` of it."""

        return self.launch(self.stage(plan))

    def build_empty(self) -> StepInput:
        """The fixed buffers holding a batch of no requests, padded as
        ``copy_input`` pads (model_runner.py:78-122): zero token ids,
        positions, context lengths and visibility starts, query start
        locations 0, null-block tables, slots -1.  This is the state a graph
        is captured on (``_make_cuda_graph_input``, model_runner.py:387-463)."""

        if self._fixed is None:
            raise ValueError("build_empty needs a builder with capacities")
        out = self._fixed
        for name in ("input_ids", "positions", "qsl", "ctx"):
            out[name].zero_()
        for starts, slots, table in out["groups"]:
            starts.zero_()
            slots.fill_(-1)
            table.fill_(self.null_block_id)
        return StepInput(
            input_ids=out["input_ids"],
            positions=out["positions"],
            layer_attention_metadata=tuple(self._group_metadata(out)[g] for g in self.group_of_layer),
            request_ids=tuple(f"__cuda_graph__-{i}" for i in range(self.request_capacity)),
            sampling_row_indices=out["rows"][:0],
        )

    def _group_metadata(self, out: dict) -> list[AttentionMetadata]:
        return [
            AttentionMetadata(
                query_positions=out["positions"], query_context_start_positions=starts,
                query_start_locations=out["qsl"], context_lengths=out["ctx"], block_table=table,
                slot_mapping=slots, block_size=self.block_size,
            )
            for starts, slots, table in out["groups"]
        ]

    def stage(self, plan, /) -> "StagedPlan":
        """Pack the plan into pinned memory and start its upload (one copy).

        The staged plan must be launched before two more plans are staged."""

        requests = tuple(plan.scheduled_requests)
        r = len(requests)
        ng = len(self.group_codes)
        computed = np.fromiter((q.num_computed_tokens for q in requests), np.int64, r)
        scheduled = np.fromiter((q.num_scheduled_tokens for q in requests), np.int64, r)
        flags = np.fromiter((bool(q.requires_sampling) for q in requests), np.uint8, r)
        tables = [[q.block_tables[g].block_ids for q in requests] for g in range(ng)]
        counts = [np.fromiter((len(b) for b in tb), np.int64, r) for tb in tables]
        t = int(scheduled.sum())
        nblocks = [int(c.sum()) for c in counts]
        if r and (computed.min() < 0 or scheduled.min() < 0):
            raise ValueError("token counts must be non-negative")
        if r and int((computed + scheduled).max()) >= 2**31:
            raise ValueError("context lengths must be below 2^31")
        if max([t, *nblocks]) >= 2**31:
            raise ValueError("a step holds fewer than 2^31 tokens and block ids")

        # One pinned int32 buffer: computed | scheduled | counts per group |
        # flags (bytes) | token ids | block ids per group.
        off_counts = 2 * r
        off_flags = off_counts + ng * r
        off_tokens = off_flags + (r + 3) // 4
        off_blocks = [off_tokens + t]
        for n in nblocks:
            off_blocks.append(off_blocks[-1] + n)
        total = off_blocks[-1]
        slot = self._slots[self._next]
        self._next ^= 1
        host = slot.reserve(total)
        host[:r] = computed
        host[r:2 * r] = scheduled
        for g in range(ng):
            host[off_counts + g * r: off_counts + (g + 1) * r] = counts[g]
        host[off_flags:off_tokens].view(np.uint8)[:r] = flags
        host[off_tokens:off_tokens + t] = np.fromiter(
            itertools.chain.from_iterable(q.input_token_ids for q in requests), np.int64, t)
        for g in range(ng):
            host[off_blocks[g]:off_blocks[g + 1]] = np.fromiter(
                itertools.chain.from_iterable(tables[g]), np.int64, nblocks[g])
        slot.upload(total, torch.cuda.current_stream(self.device))
        return StagedPlan(
            base=slot.dev.data_ptr(), num_requests=r, num_tokens=t, num_sampled=int(flags.sum()),
            num_block_ids=tuple(nblocks), widths=tuple(int(c.max()) if r else 0 for c in counts),
            off_counts=off_counts, off_flags=off_flags, off_tokens=off_tokens, off_blocks=tuple(off_blocks),
            request_ids=tuple(q.request_id for q in requests), bytes=4 * total,
        )

    def launch(self, staged: "StagedPlan", /) -> StepInput:
        """One ``mvb_build_metadata`` launch per cache group on the current stream."""

        r, t, s = staged.num_requests, staged.num_tokens, staged.num_sampled
        if self._fixed is None:
            out = self._allocate(t, r, list(staged.widths))
            t_cap, r_cap = t, r
        else:
            out = self._fixed
            t_cap, r_cap = self.token_capacity, self.request_capacity
            wmax = max(staged.widths, default=0)
            if t > t_cap or r > r_cap or wmax > self.table_width:
                raise ValueError(
                    f"step ({t} tokens, {r} requests, {wmax} blocks) exceeds the "
                    f"builder's capacity ({t_cap}, {r_cap}, {self.table_width})")
        lib = _lib.load()
        stream = torch.cuda.current_stream(self.device).cuda_stream
        ptr = lambda off: staged.base + 4 * off  # noqa: E731
        for g, (kind, param) in enumerate(self.group_codes):
            starts, slots, table = out["groups"][g]
            first = g == 0  # the shared tensors are written once
            rc = lib.mvb_build_metadata(
                ptr(0), ptr(r), ptr(staged.off_counts + g * r), ptr(staged.off_blocks[g]),
                ptr(staged.off_flags) if first else None, ptr(staged.off_tokens),
                r, t, staged.num_block_ids[g], s if first else 0, r_cap, t_cap,
                table.shape[1], table.stride(0) if table.numel() else table.shape[1],
                self.block_size, self.null_block_id, kind, param,
                out["input_ids"].data_ptr() if first else None,
                out["positions"].data_ptr() if first else None,
                starts.data_ptr(),
                out["qsl"].data_ptr() if first else None,
                out["ctx"].data_ptr() if first else None,
                table.data_ptr() if table.numel() else None,
                slots.data_ptr(),
                out["rows"].data_ptr() if first and s else None,
                self.status.data_ptr(), stream,
            )
            _lib.check(rc, "b200 metadata build")
        group_md = self._group_metadata(out)
        return StepInput(
            input_ids=out["input_ids"],
            positions=out["positions"],
            layer_attention_metadata=tuple(group_md[g] for g in self.group_of_layer),
            request_ids=staged.request_ids,
            sampling_row_indices=out["rows"][:s],
        )


@dataclass(frozen=True, slots=True)
class StagedPlan:
    """A plan packed and uploaded by ``DeviceMetadataBuilder.stage``: int32
    word offsets of each section in the device staging buffer."""

    base: int
    num_requests: int
    num_tokens: int
    num_sampled: int
    num_block_ids: tuple[int, ...]
    widths: tuple[int, ...]
    off_counts: int
    off_flags: int
    off_tokens: int
    off_blocks: tuple[int, ...]
    request_ids: tuple[str, ...]
    bytes: int


class _Staging:
    """A pinned host buffer, its device twin and the event of its last upload."""

    __slots__ = ("host", "dev", "uploaded")

    def __init__(self, device: torch.device) -> None:
        self.host = torch.empty(0, dtype=torch.int32).pin_memory()
        self.dev = torch.empty(0, dtype=torch.int32, device=device)
        self.uploaded: torch.cuda.Event | None = None

    def reserve(self, words: int) -> np.ndarray:
        if self.uploaded is not None:
            self.uploaded.synchronize()  # the last upload has left the pinned buffer
        if self.host.numel() < words:
            self.host = torch.empty(max(words, 2 * self.host.numel()), dtype=torch.int32).pin_memory()
        return self.host.numpy()

    def upload(self, words: int, stream: torch.cuda.Stream) -> None:
        if self.dev.numel() < words:
            self.dev = torch.empty(self.host.numel(), dtype=self.host.dtype, device=self.dev.device)
        self.dev[:words].copy_(self.host[:words], non_blocking=True)
        self.uploaded = torch.cuda.Event()
        self.uploaded.record(stream)
