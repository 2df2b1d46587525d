"""B200 (sm_100a) paged-attention backend for micro-vLLM.

The hot path of micro-vLLM's attention-operator layer — the KV-cache scatter
and paged attention over that cache, plus the fused q/k-norm + RoPE + KV-write
prologue of a Qwen3 layer, the device-side build of a step's metadata, and a
batched device sampler — as hand-written CUDA behind a C ABI
(include/mvb200.h, ``libmvb200.so``), with a Python operator that mirrors
the reference's ``AttentionOperator`` interface.
"""

from micro_vllm_b200.attention import (  # noqa: F401
    Attention,
    AttentionMetadata,
    AttentionSpec,
    ChunkedLocalSpec,
    FullAttentionSpec,
    SlidingWindowSpec,
    map_cache_slots,
)
from micro_vllm_b200.metadata import DeviceMetadataBuilder, StepInput  # noqa: F401
from micro_vllm_b200.operators import (  # noqa: F401
    OPERATOR_NAME,
    AttentionOperator,
    B200PagedAttentionOperator,
    get_attention_operator_class,
    write_kv_cache,
)
from micro_vllm_b200.prologue import (  # noqa: F401
    Qwen3AttentionPrologue,
    qk_norm_rope_and_write,
    rotary_inverse_frequencies,
)
from micro_vllm_b200.sampling import B200Sampler, sample_tokens  # noqa: F401

__all__ = [
    "Attention",
    "AttentionMetadata",
    "AttentionOperator",
    "AttentionSpec",
    "B200PagedAttentionOperator",
    "B200Sampler",
    "ChunkedLocalSpec",
    "DeviceMetadataBuilder",
    "FullAttentionSpec",
    "OPERATOR_NAME",
    "Qwen3AttentionPrologue",
    "SlidingWindowSpec",
    "StepInput",
    "get_attention_operator_class",
    "map_cache_slots",
    "qk_norm_rope_and_write",
    "rotary_inverse_frequencies",
    "sample_tokens",
    "write_kv_cache",
]
