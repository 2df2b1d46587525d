"""Fused Qwen3 attention prologue: q/k RMSNorm + RoPE + KV-cache write.

In the reference, a Qwen3 layer runs, between its projections and the
attention operator (src/micro_vllm/models/qwen.py:89-98): ``q_norm`` and
``k_norm`` (RMSNorm, src/micro_vllm/layers/normalization.py:15-22), the
rotary embedding (src/micro_vllm/layers/rotary_embedding.py:22-52), then the
operator, which first writes the step's keys and values into the paged cache
(src/micro_vllm/attention/operators/reference.py:84-98).  ``mvb_qk_norm_rope_and_cache``
does all of that in one launch; the attention that follows reads the cache
through ``B200PagedAttentionOperator.attend`` (no second write).

A layer that used

    query, key = rotary(positions, q_norm(query), k_norm(key))
    out = attention(query, key, value, layer_kv_cache, metadata)

uses

    prologue = Qwen3AttentionPrologue.from_modules(q_norm, k_norm, rotary)
    out = operator.attend(prologue(positions, query, key, value, layer_kv_cache, metadata),
                          layer_kv_cache, metadata)
"""

from __future__ import annotations

import torch

from micro_vllm_b200 import _lib
from micro_vllm_b200.operators import _DTYPES, _meta


def rotary_inverse_frequencies(head_dim: int, base: float, device) -> torch.Tensor:
    """``1 / base ** (arange(0, D, 2) / D)`` in fp32 on ``device``, the
    expression of rotary_embedding.py:29-38, so the kernel's angles equal the
    reference's bit for bit on the same device."""

    idx = torch.arange(0, head_dim, 2, dtype=torch.float32, device=device)
    return 1.0 / (base ** (idx / head_dim))


def qk_norm_rope_and_write(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    positions: torch.Tensor,
    q_weight: torch.Tensor,
    k_weight: torch.Tensor,
    eps: float,
    inv_freq: torch.Tensor,
    layer_kv_cache: torch.Tensor,
    metadata,
    *,
    status: torch.Tensor | None = None,
) -> torch.Tensor:
    """Normalise and rotate ``query`` [T, Hq, D] and ``key`` [T, Hkv, D],
    write the rotated key and ``value`` into ``layer_kv_cache`` at
    ``metadata.slot_mapping``; return the rotated query (a new tensor)."""

    for t in (query, key, value, layer_kv_cache, positions, q_weight, k_weight, inv_freq):
        if t.device.type != "cuda":
            raise RuntimeError("b200_paged prologue requires CUDA tensors")
    dtype = _DTYPES.get(query.dtype)
    if dtype not in (_lib.MVB_DTYPE_F16, _lib.MVB_DTYPE_BF16):
        raise ValueError("b200_paged prologue supports torch.float16 and torch.bfloat16")
    if not (key.dtype == value.dtype == layer_kv_cache.dtype == q_weight.dtype == k_weight.dtype == query.dtype):
        raise ValueError("query, key, value, the norm weights and layer_kv_cache must share one dtype")
    if query.dim() != 3 or key.dim() != 3 or value.dim() != 3 or layer_kv_cache.dim() != 5:
        raise ValueError("expected query/key/value [T,H,D] and layer_kv_cache [2,NB,bs,Hkv,D]")
    num_tokens, num_q_heads, head_dim = query.shape
    _, num_blocks, block_size, num_kv_heads, cache_dim = layer_kv_cache.shape
    if key.shape != (num_tokens, num_kv_heads, head_dim) or value.shape != key.shape:
        raise ValueError("key/value must be [num_tokens, num_kv_heads, head_dim]")
    if cache_dim != head_dim or not layer_kv_cache.is_contiguous():
        raise ValueError("layer_kv_cache must be a contiguous [2, NB, bs, Hkv, D] tensor")
    if q_weight.shape != (head_dim,) or k_weight.shape != (head_dim,):
        raise ValueError("q_weight / k_weight must be [head_dim]")
    if inv_freq.dtype != torch.float32 or inv_freq.shape != (head_dim // 2,):
        raise ValueError("inv_freq must be float32 [head_dim // 2]")
    device = query.device
    pos = _meta(positions, device, "positions")
    slots = _meta(metadata.slot_mapping, device, "slot_mapping")
    q_weight, k_weight, inv_freq = q_weight.contiguous(), k_weight.contiguous(), inv_freq.contiguous()
    q_out = torch.empty((num_tokens, num_q_heads, head_dim), dtype=query.dtype, device=device)
    lib = _lib.load()
    rc = lib.mvb_qk_norm_rope_and_cache(
        query.data_ptr(), _lib.strides3(query.stride()),
        key.data_ptr(), _lib.strides3(key.stride()),
        value.data_ptr(), _lib.strides3(value.stride()),
        q_out.data_ptr(), q_weight.data_ptr(), k_weight.data_ptr(), float(eps),
        inv_freq.data_ptr(), pos.data_ptr(), layer_kv_cache.data_ptr(),
        num_blocks, block_size, num_kv_heads, head_dim, slots.data_ptr(), num_tokens,
        num_q_heads, dtype, None if status is None else status.data_ptr(),
        torch.cuda.current_stream(device).cuda_stream,
    )
    _lib.check(rc, "b200_paged prologue")
    return q_out


class Qwen3AttentionPrologue:
    """The q_norm / k_norm / rotary triple of ``Qwen3Attention`` (qwen.py:62-64)
    plus the KV write, as one call."""

    def __init__(self, q_weight: torch.Tensor, k_weight: torch.Tensor, eps: float, base: float) -> None:
        self.q_weight, self.k_weight, self.eps, self.base = q_weight, k_weight, float(eps), float(base)
        self._inv_freq: dict[torch.device, torch.Tensor] = {}

    @classmethod
    def from_modules(cls, q_norm, k_norm, rotary) -> "Qwen3AttentionPrologue":
        """From the reference's RMSNorm (``weight``, ``variance_epsilon``) and
        RotaryEmbedding (``base``) modules."""

        if q_norm.variance_epsilon != k_norm.variance_epsilon:
            raise ValueError("q_norm and k_norm must share one epsilon")
        return cls(q_norm.weight.detach(), k_norm.weight.detach(), q_norm.variance_epsilon, rotary.base)

    def inv_freq(self, device: torch.device, head_dim: int) -> torch.Tensor:
        t = self._inv_freq.get(device)
        if t is None or t.numel() != head_dim // 2:
            t = self._inv_freq[device] = rotary_inverse_frequencies(head_dim, self.base, device)
        return t

    def __call__(self, positions, query, key, value, layer_kv_cache, metadata) -> torch.Tensor:
        return qk_norm_rope_and_write(
            query, key, value, positions, self.q_weight, self.k_weight, self.eps,
            self.inv_freq(query.device, query.shape[-1]), layer_kv_cache, metadata,
        )
