"""Attention metadata and visibility specs, mirroring the reference's types.

``AttentionMetadata`` has the reference's seven fields with the same meaning
(src/micro_vllm/attention/attention.py:12-28), so either class can be handed
to ``B200PagedAttentionOperator``.  The specs mirror
src/micro_vllm/attention/spec.py:18-51.  ``Attention.build_metadata``
computes per-query visibility starts with tensor ops on the metadata's own
device instead of the reference's per-position host loop
(attention.py:56-85), so building metadata needs no device-to-host copy.
"""

from __future__ import annotations

from abc import ABC, abstractmethod
from dataclasses import dataclass

import torch


@dataclass(frozen=True, slots=True, eq=False)
class AttentionMetadata:
    """Flattened queries, visibility bounds, and paged-cache inputs."""

    query_positions: torch.Tensor
    query_context_start_positions: torch.Tensor
    query_start_locations: torch.Tensor
    context_lengths: torch.Tensor
    block_table: torch.Tensor
    slot_mapping: torch.Tensor
    block_size: int

    @property
    def num_requests(self) -> int:
        return self.context_lengths.numel()


def map_cache_slots(
    positions: torch.Tensor, block_table: torch.Tensor, block_size: int
) -> torch.Tensor:
    """Logical positions -> flattened physical slots (attention.py:31-41)."""

    physical_blocks = block_table.index_select(0, positions // block_size)
    return physical_blocks * block_size + positions % block_size


@dataclass(frozen=True, slots=True)
class AttentionSpec(ABC):
    """First key visible to one absolute query position."""

    @abstractmethod
    def context_start(self, query_position: int) -> int:
        """Inclusive start of the query's visible key interval."""

    @abstractmethod
    def context_starts(self, query_positions: torch.Tensor) -> torch.Tensor:
        """``context_start`` applied elementwise on the tensor's device."""


@dataclass(frozen=True, slots=True)
class FullAttentionSpec(AttentionSpec):
    """The complete causal history."""

    def context_start(self, query_position: int) -> int:
        return 0

    def context_starts(self, query_positions: torch.Tensor) -> torch.Tensor:
        return torch.zeros_like(query_positions)


@dataclass(frozen=True, slots=True)
class SlidingWindowSpec(AttentionSpec):
    """At most ``window_size`` keys, including the query token."""

    window_size: int

    def __post_init__(self) -> None:
        if type(self.window_size) is not int or self.window_size <= 0:
            raise ValueError("window_size must be a positive integer")

    def context_start(self, query_position: int) -> int:
        return max(0, query_position - self.window_size + 1)

    def context_starts(self, query_positions: torch.Tensor) -> torch.Tensor:
        return (query_positions - (self.window_size - 1)).clamp_(min=0)


@dataclass(frozen=True, slots=True)
class ChunkedLocalSpec(AttentionSpec):
    """The causal prefix within one aligned local chunk."""

    chunk_size: int

    def __post_init__(self) -> None:
        if type(self.chunk_size) is not int or self.chunk_size <= 0:
            raise ValueError("chunk_size must be a positive integer")

    def context_start(self, query_position: int) -> int:
        return (query_position // self.chunk_size) * self.chunk_size

    def context_starts(self, query_positions: torch.Tensor) -> torch.Tensor:
        return torch.div(query_positions, self.chunk_size, rounding_mode="floor") * self.chunk_size


def context_starts_for(spec, query_positions: torch.Tensor) -> torch.Tensor:
    """Visibility starts for any spec object.

    Specs of this module, and the reference's specs recognised by their
    fields, are evaluated as tensor ops; any other spec goes through its
    ``context_start`` per position as the reference does.
    """

    if isinstance(spec, AttentionSpec):
        return spec.context_starts(query_positions)
    window = getattr(spec, "window_size", None)
    if isinstance(window, int):
        return SlidingWindowSpec(window).context_starts(query_positions)
    chunk = getattr(spec, "chunk_size", None)
    if isinstance(chunk, int):
        return ChunkedLocalSpec(chunk).context_starts(query_positions)
    if type(spec).__name__ == "FullAttentionSpec":
        return torch.zeros_like(query_positions)
    return torch.tensor(
        [spec.context_start(p) for p in query_positions.tolist()],
        dtype=query_positions.dtype,
        device=query_positions.device,
    )


class Attention:
    """Own an operator and the metadata semantics it consumes
    (attention.py:44-101)."""

    def __init__(self, spec, operator_name: str = "b200_paged") -> None:
        from micro_vllm_b200.operators import get_attention_operator_class

        self.spec = spec
        self.operator = get_attention_operator_class(operator_name)()

    def build_metadata(
        self,
        *,
        query_positions: torch.Tensor,
        query_start_locations: torch.Tensor,
        context_lengths: torch.Tensor,
        block_table: torch.Tensor,
        slot_mapping: torch.Tensor,
        block_size: int,
    ) -> AttentionMetadata:
        return AttentionMetadata(
            query_positions=query_positions,
            query_context_start_positions=context_starts_for(self.spec, query_positions),
            query_start_locations=query_start_locations,
            context_lengths=context_lengths,
            block_table=block_table,
            slot_mapping=slot_mapping,
            block_size=block_size,
        )

    def __call__(self, query, key, value, layer_kv_cache, metadata, /) -> torch.Tensor:
        return self.operator(query, key, value, layer_kv_cache, metadata)
