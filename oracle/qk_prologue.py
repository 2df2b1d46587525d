"""CPU oracle of the Qwen3 attention prologue — TEST INFRASTRUCTURE ONLY.

numpy restatement of what the reference does between the Q/K/V projections
and the attention operator of a Qwen3 layer: per-head RMSNorm of the query
and key heads, rotary position embedding of both, then the KV-cache write
the attention operator performs first.  It checks the fused CUDA kernel
``mvb_qk_norm_rope_and_cache``; only ``tests/`` import it.

Parity pin: ``tests/golden/make_golden_prologue.py`` ran the reference's own
``RMSNorm``, ``RotaryEmbedding`` and ``write_kv_cache`` (imported from the
reference source tree) on seeded inputs; ``tests/test_oracle.py`` checks
this restatement against those vectors and the reference tests' known
answers.

Reference code restated here (paths inside the reference project):

* ``Qwen3Attention.forward`` q/k norm then rope — src/micro_vllm/models/qwen.py:74-98
* ``RMSNorm.forward``                          — src/micro_vllm/layers/normalization.py:15-22
* ``rotate_half``                              — src/micro_vllm/layers/rotary_embedding.py:7-11
* ``RotaryEmbedding.forward``                  — src/micro_vllm/layers/rotary_embedding.py:22-52
* ``write_kv_cache``                           — src/micro_vllm/attention/operators/reference.py:84-98

Arithmetic follows the reference's dtypes step by step: the statistics and
the rotation in fp32, the normalised activations rounded to the model dtype
before the weight multiply (computed in fp32, rounded again), the rotated
values rounded to the model dtype.  bf16 rounding is emulated on fp32 bits
(round to nearest even), as numpy has no bf16 type.
"""

from __future__ import annotations

import numpy as np

from oracle.paged_attention import write_kv_cache


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """fp32 values rounded to ``dtype`` ("f16", "bf16" or "f32"), as fp32."""

    x = np.asarray(x, dtype=np.float32)
    if dtype == "f32":
        return x
    if dtype == "f16":
        return x.astype(np.float16).astype(np.float32)
    if dtype == "bf16":
        bits = x.view(np.uint32).astype(np.uint64)
        nan = np.isnan(x)
        rounded = (bits + 0x7FFF + ((bits >> 16) & 1)) & 0xFFFF0000
        out = rounded.astype(np.uint32).view(np.float32).copy()
        out[nan] = np.float32("nan")
        return out
    raise ValueError(f"unsupported dtype {dtype}")


def rms_norm(x: np.ndarray, weight: np.ndarray, eps: float, dtype: str) -> np.ndarray:
    """``RMSNorm.forward`` (normalization.py:15-22) over the last axis."""

    xf = np.asarray(x, dtype=np.float32)
    variance = np.mean(xf * xf, axis=-1, keepdims=True, dtype=np.float32)
    normed = xf * (np.float32(1.0) / np.sqrt(variance + np.float32(eps), dtype=np.float32))
    normed = round_to(normed, dtype)
    return round_to(np.asarray(weight, np.float32) * normed, dtype)


def inverse_frequencies(head_dim: int, base: float) -> np.ndarray:
    """``1 / base ** (arange(0, D, 2) / D)`` in fp32 (rotary_embedding.py:29-38)."""

    idx = np.arange(0, head_dim, 2, dtype=np.float32)
    return (np.float32(1.0) / np.power(np.float32(base), idx / np.float32(head_dim))).astype(np.float32)


def rotate_half(x: np.ndarray) -> np.ndarray:
    """``rotate_half`` (rotary_embedding.py:7-11)."""

    half = x.shape[-1] // 2
    return np.concatenate((-x[..., half:], x[..., :half]), axis=-1)


def rope(positions: np.ndarray, x: np.ndarray, inv_freq: np.ndarray, dtype: str) -> np.ndarray:
    """Rotation of ``RotaryEmbedding.forward`` (rotary_embedding.py:39-52) for
    one of query or key, ``x`` [T, H, D] holding ``dtype`` values."""

    freqs = np.outer(np.asarray(positions).astype(np.float32), inv_freq).astype(np.float32)
    angles = np.concatenate((freqs, freqs), axis=-1)[:, None, :]
    cos, sin = np.cos(angles).astype(np.float32), np.sin(angles).astype(np.float32)
    xf = np.asarray(x, np.float32)
    rotated = (xf * cos).astype(np.float32) + (rotate_half(xf) * sin).astype(np.float32)
    return round_to(rotated, dtype)


def qk_norm_rope_and_cache(
    query: np.ndarray,
    key: np.ndarray,
    value: np.ndarray,
    positions: np.ndarray,
    q_weight: np.ndarray,
    k_weight: np.ndarray,
    eps: float,
    inv_freq: np.ndarray,
    cache: np.ndarray,
    slot_mapping: np.ndarray,
    dtype: str,
) -> np.ndarray:
    """The fused prologue: returns the normalised, rotated query [T, Hq, D]
    and writes the normalised, rotated key and the value into ``cache``
    ([2, NB, bs, Hkv, D], in place) at ``slot_mapping`` (negative slots write
    nothing, as the Triton write kernel, triton_paged.py:37-39)."""

    q = rope(positions, rms_norm(query, q_weight, eps, dtype), inv_freq, dtype)
    k = rope(positions, rms_norm(key, k_weight, eps, dtype), inv_freq, dtype)
    write_kv_cache(k, np.asarray(value, np.float32), cache, np.asarray(slot_mapping, np.int64))
    return q
