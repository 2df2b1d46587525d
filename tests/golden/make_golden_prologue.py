"""Generate the Qwen3 attention-prologue golden vectors from the real reference.

Run once, in a container that has the micro-vLLM source tree:

    python tests/golden/make_golden_prologue.py /path/to/micro-vllm

It imports ``micro_vllm`` from ``<path>/src`` and runs, on the CPU, the
reference's own ``RMSNorm`` (src/micro_vllm/layers/normalization.py:15-22)
as ``q_norm``/``k_norm``, ``RotaryEmbedding`` (src/micro_vllm/layers/
rotary_embedding.py:22-52) and ``write_kv_cache`` (src/micro_vllm/attention/
operators/reference.py:84-98) in the order ``Qwen3Attention.forward`` uses
them (src/micro_vllm/models/qwen.py:74-98), in fp16 and bf16.  Each case is
``prologue_<name>.npz``: inputs and outputs as raw 16-bit patterns, the
positions, the RMSNorm weights, the rotary inverse frequencies the reference
computes, and the post-write cache.  Nothing on the GPU box reads the
reference tree.
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def _bits(t) -> np.ndarray:
    import torch

    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def make_case(torch, mv, name: str, *, dtype, tokens: int, hq: int, hkv: int, base: float,
              eps: float, max_pos: int, seed: int) -> dict:
    RMSNorm, RotaryEmbedding = mv["RMSNorm"], mv["RotaryEmbedding"]
    write_kv_cache, AttentionMetadata = mv["write_kv_cache"], mv["AttentionMetadata"]
    g = torch.Generator().manual_seed(seed)
    d, bs, nb = 128, 16, 2
    # Projection outputs with a spread of scales, as a trained model's are.
    query = (torch.randn((tokens, hq, d), generator=g) * 3.0).to(dtype)
    key = (torch.randn((tokens, hkv, d), generator=g) * 3.0).to(dtype)
    value = torch.randn((tokens, hkv, d), generator=g).to(dtype)
    positions = torch.randint(0, max_pos, (tokens,), generator=g, dtype=torch.int64)
    positions[0] = 0
    positions[1] = max_pos - 1
    q_norm, k_norm = RMSNorm(d, eps=eps), RMSNorm(d, eps=eps)
    with torch.no_grad():
        q_norm.weight.copy_(0.5 + torch.rand(d, generator=g))
        k_norm.weight.copy_(0.5 + torch.rand(d, generator=g))
    q_norm, k_norm = q_norm.to(dtype), k_norm.to(dtype)
    rotary = RotaryEmbedding(d, base=base)
    slots = torch.randperm(nb * bs, generator=g)[:tokens].to(torch.int64)
    slots[3] = -1  # graph padding: writes nothing
    cache = torch.randn((2, nb, bs, hkv, d), generator=g).to(dtype)
    cache_before = cache.clone()
    with torch.no_grad():
        q_out, k_out = rotary(positions, q_norm(query), k_norm(key))
        keep = slots >= 0  # index_copy_ rejects -1; the padding row is dropped
        md = AttentionMetadata(
            query_positions=positions[keep], query_context_start_positions=positions[keep] * 0,
            query_start_locations=torch.tensor([0, int(keep.sum())]),
            context_lengths=torch.tensor([1]), block_table=torch.zeros((1, 1), dtype=torch.int64),
            slot_mapping=slots[keep], block_size=bs,
        )
        write_kv_cache(k_out[keep], value[keep], cache, md)
    idx = torch.arange(0, d, 2, dtype=torch.float32)
    inv_freq = (1.0 / (base ** (idx / d))).numpy().astype(np.float32)
    return {
        "dtype": "f16" if dtype == torch.float16 else "bf16",
        "query": _bits(query), "key": _bits(key), "value": _bits(value),
        "positions": positions.numpy(), "slot_mapping": slots.numpy(),
        "q_weight": _bits(q_norm.weight.data), "k_weight": _bits(k_norm.weight.data),
        "eps": np.float32(eps), "base": np.float64(base), "inv_freq": inv_freq,
        "cache_before": _bits(cache_before), "q_out": _bits(q_out), "cache_after": _bits(cache),
        "block_size": np.int64(bs),
    }


def main(ref_root: str) -> None:
    sys.path.insert(0, str(Path(ref_root) / "src"))
    import torch
    from micro_vllm.attention.attention import AttentionMetadata
    from micro_vllm.attention.operators.reference import write_kv_cache
    from micro_vllm.layers.normalization import RMSNorm
    from micro_vllm.layers.rotary_embedding import RotaryEmbedding

    mv = dict(RMSNorm=RMSNorm, RotaryEmbedding=RotaryEmbedding, write_kv_cache=write_kv_cache,
              AttentionMetadata=AttentionMetadata)
    cases = {
        # Qwen3-0.6B attention: 16/8 heads, theta 1e6, eps 1e-6.
        "qwen3_f16": dict(dtype=torch.float16, tokens=24, hq=16, hkv=8, base=1e6, eps=1e-6,
                          max_pos=4096, seed=1),
        "qwen3_bf16": dict(dtype=torch.bfloat16, tokens=24, hq=16, hkv=8, base=1e6, eps=1e-6,
                           max_pos=4096, seed=2),
        # Llama-3-8B-shaped GQA at long positions.
        "gqa4_long_f16": dict(dtype=torch.float16, tokens=20, hq=32, hkv=8, base=5e5, eps=1e-5,
                              max_pos=131072, seed=3),
    }
    manifest = {}
    for name, kw in cases.items():
        arrays = make_case(torch, mv, name, **kw)
        np.savez_compressed(HERE / f"prologue_{name}.npz", **arrays)
        manifest[name] = {k: v for k, v in kw.items() if k != "dtype"} | {"dtype": arrays["dtype"]}
    (HERE / "prologue_manifest.json").write_text(json.dumps(manifest, indent=1) + "\n")
    print("wrote", ", ".join(manifest))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_golden_prologue.py <micro-vllm source tree>")
    main(sys.argv[1])
