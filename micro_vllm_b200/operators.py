"""The ``b200_paged`` attention operator and its registry.

Mirrors the reference's operator contract (src/micro_vllm/attention/operators/base.py:10-40)
and registry (registry.py:24-50).  ``B200PagedAttentionOperator.forward``
is one call into ``mvb_attention_forward`` of ``libmvb200.so``: the KV
scatter, then paged attention, on the current CUDA stream, with no host
synchronisation — so the call can be captured in a CUDA graph once its
workspace exists (see ``reserve``).
"""

from __future__ import annotations

import math
from abc import ABC, abstractmethod

import torch

from micro_vllm_b200 import _lib

OPERATOR_NAME = "b200_paged"

_DTYPES = {
    torch.float16: _lib.MVB_DTYPE_F16,
    torch.bfloat16: _lib.MVB_DTYPE_BF16,
    torch.float32: _lib.MVB_DTYPE_F32,
}


class AttentionOperator(ABC):
    """Compute attention from Q/K/V tensors and semantic metadata
    (base.py:10-40): positional-only arguments, returns the output."""

    def __call__(self, query, key, value, layer_kv_cache, metadata, /) -> torch.Tensor:
        return self.forward(query, key, value, layer_kv_cache, metadata)

    @abstractmethod
    def forward(self, query, key, value, layer_kv_cache, metadata, /) -> torch.Tensor:
        """Compute attention for one layer."""


class _DeviceState:
    """Per-device workspace and status word, owned by the operator."""

    __slots__ = ("workspace", "capacity", "status")

    def __init__(self, device: torch.device) -> None:
        self.workspace: torch.Tensor | None = None
        self.capacity = (0, 0, 0, 0, 0)  # tokens, requests, Hq, Hkv, D
        self.status = torch.zeros(1, dtype=torch.int32, device=device)


def _meta(t: torch.Tensor, device: torch.device, name: str) -> torch.Tensor:
    if t.dtype != torch.int64:
        raise ValueError(f"metadata.{name} must be torch.int64")
    if t.device != device:
        raise ValueError(f"metadata.{name} must be on {device}")
    return t if t.is_contiguous() else t.contiguous()


class B200PagedAttentionOperator(AttentionOperator):
    """CUDA paged attention for B200 (sm_100a), fp16 / bf16 / fp32."""

    def __init__(self) -> None:
        self._lib = _lib.load()
        self._devices: dict[int, _DeviceState] = {}

    # -- workspace -------------------------------------------------------
    def _state(self, device: torch.device) -> _DeviceState:
        idx = device.index if device.index is not None else torch.cuda.current_device()
        st = self._devices.get(idx)
        if st is None:
            st = self._devices[idx] = _DeviceState(torch.device("cuda", idx))
        return st

    def reserve(
        self,
        device: torch.device | str,
        *,
        max_num_tokens: int,
        max_num_requests: int,
        num_q_heads: int,
        num_kv_heads: int,
        head_dim: int,
    ) -> None:
        """Allocate the workspace for batches up to these sizes now, so
        later calls (and CUDA-graph captures) allocate nothing."""

        self._workspace(torch.device(device), max_num_tokens, max_num_requests, num_q_heads, num_kv_heads, head_dim)

    def _workspace(self, device, tokens, requests, hq, hkv, d) -> tuple[torch.Tensor, _DeviceState]:
        st = self._state(device)
        cap = st.capacity
        fits = (
            st.workspace is not None
            and cap[2:] == (hq, hkv, d)
            and tokens <= cap[0]
            and requests <= cap[1]
        )
        if not fits:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError(
                    "b200_paged workspace too small during CUDA-graph capture; "
                    "call reserve() with the capture sizes first"
                )
            same_shape = cap[2:] == (hq, hkv, d)
            new_tokens = max(tokens, cap[0] if same_shape else 0, 1)
            new_requests = max(requests, 2 * cap[1] if same_shape else 0, 64)
            nbytes = self._lib.mvb_paged_attention_workspace_size(new_tokens, new_requests, hq, hkv, d)
            st.workspace = torch.empty(nbytes, dtype=torch.uint8, device=st.status.device)
            st.capacity = (new_tokens, new_requests, hq, hkv, d)
        return st.workspace, st

    def read_status(self, device: torch.device | str | None = None) -> int:
        """Return and clear the device status bits (synchronises)."""

        st = self._state(torch.device(device) if device is not None else torch.device("cuda"))
        value = int(st.status.item())
        st.status.zero_()
        return value

    # -- forward ---------------------------------------------------------
    def forward(self, query, key, value, layer_kv_cache, metadata, /) -> torch.Tensor:
        for t in (query, key, value, layer_kv_cache):
            if t.device.type != "cuda":
                raise RuntimeError("b200_paged attention requires CUDA tensors")
        dtype = _DTYPES.get(query.dtype)
        if dtype is None:
            raise ValueError(
                "b200_paged attention supports torch.float16, torch.bfloat16 and torch.float32"
            )
        if not (key.dtype == value.dtype == layer_kv_cache.dtype == query.dtype):
            raise ValueError("query, key, value and layer_kv_cache must share one dtype")
        if query.dim() != 3 or key.dim() != 3 or value.dim() != 3 or layer_kv_cache.dim() != 5:
            raise ValueError("expected query/key/value [T,H,D] and layer_kv_cache [2,NB,bs,Hkv,D]")
        num_tokens, num_q_heads, head_dim = query.shape
        _, num_blocks, block_size, num_kv_heads, cache_dim = layer_kv_cache.shape
        if key.shape != (num_tokens, num_kv_heads, head_dim) or value.shape != key.shape:
            raise ValueError("key/value must be [num_tokens, num_kv_heads, head_dim]")
        if cache_dim != head_dim or layer_kv_cache.shape[0] != 2:
            raise ValueError("layer_kv_cache must be [2, num_blocks, block_size, num_kv_heads, head_dim]")
        if block_size != metadata.block_size:
            raise ValueError("layer_kv_cache block size differs from metadata.block_size")
        if num_q_heads % num_kv_heads != 0:
            raise ValueError("num_q_heads must be a multiple of num_kv_heads")
        if not layer_kv_cache.is_contiguous():
            raise ValueError("layer_kv_cache must be contiguous")
        device = query.device
        if query.stride(2) != 1:
            query = query.contiguous()
        md_pos = _meta(metadata.query_positions, device, "query_positions")
        md_start = _meta(metadata.query_context_start_positions, device, "query_context_start_positions")
        md_qsl = _meta(metadata.query_start_locations, device, "query_start_locations")
        md_ctx = _meta(metadata.context_lengths, device, "context_lengths")
        md_slots = _meta(metadata.slot_mapping, device, "slot_mapping")
        table = metadata.block_table
        if table.dtype != torch.int64 or table.device != device:
            raise ValueError("metadata.block_table must be torch.int64 on the query's device")
        if table.dim() != 2 or (table.shape[1] > 1 and table.stride(1) != 1):
            table = table.reshape(md_ctx.numel(), -1).contiguous()
        num_requests = md_ctx.numel()

        output = torch.empty((num_tokens, num_q_heads, head_dim), dtype=query.dtype, device=device)
        workspace, st = self._workspace(device, num_tokens, num_requests, num_q_heads, num_kv_heads, head_dim)
        stream = torch.cuda.current_stream(device).cuda_stream
        rc = self._lib.mvb_attention_forward(
            query.data_ptr(), query.stride(0), query.stride(1),
            key.data_ptr(), _lib.strides3(key.stride()),
            value.data_ptr(), _lib.strides3(value.stride()),
            output.data_ptr(), layer_kv_cache.data_ptr(),
            num_blocks, block_size, num_kv_heads, head_dim,
            md_pos.data_ptr(), md_start.data_ptr(), md_qsl.data_ptr(), md_ctx.data_ptr(),
            table.data_ptr(), table.stride(0) if table.shape[1] > 0 else 0, table.shape[1],
            md_slots.data_ptr(), num_tokens, num_requests, num_q_heads,
            1.0 / math.sqrt(head_dim), dtype,
            workspace.data_ptr(), workspace.numel(), st.status.data_ptr(), stream,
        )
        _lib.check(rc, "b200_paged attention")
        return output


    # -- attention over a cache that already holds this step's keys/values
    def attend(self, query, layer_kv_cache, metadata) -> torch.Tensor:
        """Paged attention of ``query`` over ``layer_kv_cache`` without the KV
        write (reference.py:26-81 after its write_kv_cache line): for callers
        whose prologue (``qk_norm_rope_and_write``) wrote the keys and values."""

        for t in (query, layer_kv_cache):
            if t.device.type != "cuda":
                raise RuntimeError("b200_paged attention requires CUDA tensors")
        dtype = _DTYPES.get(query.dtype)
        if dtype is None or layer_kv_cache.dtype != query.dtype:
            raise ValueError("query and layer_kv_cache must share a float16/bfloat16/float32 dtype")
        if query.dim() != 3 or layer_kv_cache.dim() != 5 or not layer_kv_cache.is_contiguous():
            raise ValueError("expected query [T,H,D] and a contiguous layer_kv_cache [2,NB,bs,Hkv,D]")
        num_tokens, num_q_heads, head_dim = query.shape
        _, num_blocks, block_size, num_kv_heads, cache_dim = layer_kv_cache.shape
        if cache_dim != head_dim or block_size != metadata.block_size:
            raise ValueError("layer_kv_cache does not match the query / metadata")
        if num_q_heads % num_kv_heads != 0:
            raise ValueError("num_q_heads must be a multiple of num_kv_heads")
        device = query.device
        if query.stride(2) != 1:
            query = query.contiguous()
        md_pos = _meta(metadata.query_positions, device, "query_positions")
        md_start = _meta(metadata.query_context_start_positions, device, "query_context_start_positions")
        md_qsl = _meta(metadata.query_start_locations, device, "query_start_locations")
        md_ctx = _meta(metadata.context_lengths, device, "context_lengths")
        table = metadata.block_table
        if table.dtype != torch.int64 or table.device != device:
            raise ValueError("metadata.block_table must be torch.int64 on the query's device")
        if table.dim() != 2 or (table.shape[1] > 1 and table.stride(1) != 1):
            table = table.reshape(md_ctx.numel(), -1).contiguous()
        num_requests = md_ctx.numel()
        output = torch.empty((num_tokens, num_q_heads, head_dim), dtype=query.dtype, device=device)
        workspace, st = self._workspace(device, num_tokens, num_requests, num_q_heads, num_kv_heads, head_dim)
        rc = self._lib.mvb_paged_attention(
            query.data_ptr(), query.stride(0), query.stride(1), output.data_ptr(),
            layer_kv_cache.data_ptr(), num_blocks, block_size, num_kv_heads, head_dim,
            md_pos.data_ptr(), md_start.data_ptr(), md_qsl.data_ptr(), md_ctx.data_ptr(),
            table.data_ptr(), table.stride(0) if table.shape[1] > 0 else 0, table.shape[1],
            num_tokens, num_requests, num_q_heads, 1.0 / math.sqrt(head_dim), dtype,
            workspace.data_ptr(), workspace.numel(), st.status.data_ptr(),
            torch.cuda.current_stream(device).cuda_stream,
        )
        _lib.check(rc, "b200_paged attention")
        return output


def write_kv_cache(key, value, layer_kv_cache, metadata) -> None:
    """The KV scatter alone (reference.py:84-98), for ModelRunner-side writes."""

    lib = _lib.load()
    dtype = _DTYPES.get(key.dtype)
    if key.device.type != "cuda" or layer_kv_cache.device.type != "cuda":
        raise RuntimeError("b200_paged write_kv_cache requires CUDA tensors")
    if dtype is None or value.dtype != key.dtype or layer_kv_cache.dtype != key.dtype:
        raise ValueError("key, value and layer_kv_cache must share a float16/bfloat16/float32 dtype")
    if not layer_kv_cache.is_contiguous():
        raise ValueError("layer_kv_cache must be contiguous")
    _, num_blocks, block_size, num_kv_heads, head_dim = layer_kv_cache.shape
    slots = _meta(metadata.slot_mapping, key.device, "slot_mapping")
    stream = torch.cuda.current_stream(key.device).cuda_stream
    rc = lib.mvb_reshape_and_cache(
        key.data_ptr(), _lib.strides3(key.stride()), value.data_ptr(), _lib.strides3(value.stride()),
        layer_kv_cache.data_ptr(), num_blocks, block_size, num_kv_heads, head_dim,
        slots.data_ptr(), key.shape[0], dtype, None, stream,
    )
    _lib.check(rc, "b200_paged write_kv_cache")


_OPERATOR_CLASSES = {OPERATOR_NAME: B200PagedAttentionOperator}


def get_attention_operator_class(name: str) -> type[AttentionOperator]:
    """Registered operator class by name (registry.py:24-50 semantics)."""

    try:
        return _OPERATOR_CLASSES[name]
    except KeyError as error:
        raise ValueError(
            f"unsupported attention operator {name!r}; supported operators: {list(_OPERATOR_CLASSES)!r}"
        ) from error
