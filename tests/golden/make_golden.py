"""Generate the golden vectors under tests/golden/ from the real reference.

Run once, in a container that has the micro-vLLM source tree:

    python tests/golden/make_golden.py /path/to/micro-vllm

It imports ``micro_vllm`` from ``<path>/src`` and runs the reference's own
``ReferenceAttentionOperator`` (src/micro_vllm/attention/operators/reference.py:14-81)
and ``write_kv_cache`` (reference.py:84-98) in fp32 on the CPU.  Inputs are
seeded numpy draws rounded to fp16-representable values, so the same fixture
also drives the fp16 CUDA path bit-for-bit on its inputs.  Each case is one
``<name>.npz`` holding the inputs (fp16, exact), the metadata, the cache
before the call, the reference's fp32 output and a SHA-256 of the reference's
full post-write cache (fp32 bytes).  ``manifest.json`` lists the cases.
Nothing on the GPU box reads the reference tree: tests load only these files.
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))

from _golden import cache_digest  # noqa: E402


def _rng(seed: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(seed))


def _normal16(rng: np.random.Generator, shape) -> np.ndarray:
    """N(0,1) draws rounded to fp16 and widened back to fp32."""

    return rng.standard_normal(shape).astype(np.float16).astype(np.float32)


def _slots(positions, table_row, block_size):
    return [table_row[p // block_size] * block_size + p % block_size for p in positions]


def _run_reference(torch, mv, case: dict) -> dict:
    """Run ReferenceAttentionOperator on one case; return expected arrays."""

    AttentionMetadata = mv["AttentionMetadata"]
    op = mv["ReferenceAttentionOperator"]()
    md = AttentionMetadata(
        query_positions=torch.from_numpy(case["query_positions"]),
        query_context_start_positions=torch.from_numpy(case["query_context_start_positions"]),
        query_start_locations=torch.from_numpy(case["query_start_locations"]),
        context_lengths=torch.from_numpy(case["context_lengths"]),
        block_table=torch.from_numpy(case["block_table"]),
        slot_mapping=torch.from_numpy(case["slot_mapping"]),
        block_size=int(case["block_size"]),
    )
    cache = torch.from_numpy(case["cache_before"].copy())
    out = op(
        torch.from_numpy(case["query"]),
        torch.from_numpy(case["key"]),
        torch.from_numpy(case["value"]),
        cache,
        md,
    )
    return {"expected_output": out.numpy().copy(), "expected_cache": cache.numpy().copy()}


def _prefill_history(torch, mv, cache, table_rows, lengths, rng, block_size):
    """Write K/V history for positions [0, length) of each request via the
    reference's write_kv_cache (reference.py:84-98)."""

    AttentionMetadata = mv["AttentionMetadata"]
    write = mv["write_kv_cache"]
    num_kv_heads, head_dim = cache.shape[3], cache.shape[4]
    for row, length in zip(table_rows, lengths):
        if length == 0:
            continue
        k = _normal16(rng, (length, num_kv_heads, head_dim))
        v = _normal16(rng, (length, num_kv_heads, head_dim))
        slots = np.asarray(_slots(range(length), row, block_size), np.int64)
        md = AttentionMetadata(
            query_positions=torch.arange(length),
            query_context_start_positions=torch.zeros(length, dtype=torch.int64),
            query_start_locations=torch.tensor([0, length]),
            context_lengths=torch.tensor([length]),
            block_table=torch.tensor([row]),
            slot_mapping=torch.from_numpy(slots),
            block_size=block_size,
        )
        t = torch.from_numpy(cache)
        write(torch.from_numpy(k), torch.from_numpy(v), t, md)


def _case(
    torch,
    mv,
    *,
    name: str,
    seed: int,
    num_q_heads: int,
    num_kv_heads: int,
    head_dim: int,
    block_size: int,
    num_blocks: int,
    requests: list[dict],
    pad_block: int,
    cache_fill: float = 0.0,
    extra_tokens: int = 0,
    description: str,
) -> dict:
    """Build one case.

    Each request dict has ``table`` (block ids), ``history`` (positions
    already in the cache before the call), ``positions`` (query positions of
    this call) and optionally ``starts`` (per-query visibility starts; default
    0) and ``context_length`` (default last position + 1).
    """

    rng = _rng(seed)
    cache = np.full(
        (2, num_blocks, block_size, num_kv_heads, head_dim), cache_fill, dtype=np.float32
    )
    _prefill_history(
        torch, mv, cache, [r["table"] for r in requests], [r["history"] for r in requests], rng, block_size
    )
    positions, starts, slots, qsl, ctx = [], [], [], [0], []
    for r in requests:
        positions += list(r["positions"])
        starts += list(r.get("starts", [0] * len(r["positions"])))
        slots += _slots(r["positions"], r["table"], block_size)
        qsl.append(qsl[-1] + len(r["positions"]))
        ctx.append(r.get("context_length", (r["positions"][-1] + 1) if r["positions"] else 0))
    # Graph-capture style padding tokens (model_runner.py:78-122): position 0,
    # start 0, slot -1, owned by no request.
    positions += [0] * extra_tokens
    starts += [0] * extra_tokens
    slots += [-1] * extra_tokens
    width = max(len(r["table"]) for r in requests)
    table = np.full((len(requests), width), pad_block, dtype=np.int64)
    for i, r in enumerate(requests):
        table[i, : len(r["table"])] = r["table"]
    num_tokens = len(positions)
    case = {
        "query": _normal16(rng, (num_tokens, num_q_heads, head_dim)),
        "key": _normal16(rng, (num_tokens, num_kv_heads, head_dim)),
        "value": _normal16(rng, (num_tokens, num_kv_heads, head_dim)),
        "query_positions": np.asarray(positions, np.int64),
        "query_context_start_positions": np.asarray(starts, np.int64),
        "query_start_locations": np.asarray(qsl, np.int64),
        "context_lengths": np.asarray(ctx, np.int64),
        "block_table": table,
        "slot_mapping": np.asarray(slots, np.int64),
        "block_size": np.asarray(block_size, np.int64),
        "cache_before": cache,
    }
    # The reference operator raises on slot -1 (index_copy_); padding rows
    # are therefore run through it with those tokens removed, and the
    # expected padding rows are zero (Triton-backend semantics).
    if extra_tokens:
        live = num_tokens - extra_tokens
        trimmed = dict(case)
        for key in ("query", "key", "value", "query_positions", "query_context_start_positions", "slot_mapping"):
            trimmed[key] = case[key][:live]
        trimmed["query_start_locations"] = np.minimum(case["query_start_locations"], live)
        expected = _run_reference(torch, mv, _drop_empty_requests(trimmed))
        out = np.zeros(case["query"].shape, np.float32)
        out[:live] = expected["expected_output"]
        expected["expected_output"] = out
    else:
        expected = _run_reference(torch, mv, case)
    stored = {k: v for k, v in case.items()}
    for key in ("query", "key", "value", "cache_before"):
        stored[key] = case[key].astype(np.float16)  # exact: values are fp16-representable
    stored["expected_output"] = expected["expected_output"].astype(np.float32)
    stored["expected_cache_sha256"] = np.asarray(cache_digest(expected["expected_cache"]))
    np.savez_compressed(HERE / f"{name}.npz", **stored)
    return {
        "name": name,
        "description": description,
        "seed": seed,
        "shape": {"Hq": num_q_heads, "Hkv": num_kv_heads, "D": head_dim, "bs": block_size, "NB": num_blocks},
        "num_tokens": num_tokens,
        "num_requests": len(requests),
    }


def _drop_empty_requests(case: dict) -> dict:
    """Remove zero-length requests before calling the readable reference,
    which would index past the token arrays for them (reference.py:114-118)."""

    qsl = case["query_start_locations"]
    keep = [i for i in range(len(qsl) - 1) if qsl[i + 1] > qsl[i]]
    out = dict(case)
    out["query_start_locations"] = np.asarray([qsl[i] for i in keep] + [qsl[keep[-1] + 1]], np.int64)
    out["context_lengths"] = case["context_lengths"][keep]
    out["block_table"] = case["block_table"][keep]
    return out


def main(reference_root: str) -> None:
    sys.path.insert(0, str(Path(reference_root) / "src"))
    import torch

    from micro_vllm.attention.attention import AttentionMetadata
    from micro_vllm.attention.operators.reference import (
        ReferenceAttentionOperator,
        write_kv_cache,
    )

    torch.set_num_threads(1)
    mv = {
        "AttentionMetadata": AttentionMetadata,
        "ReferenceAttentionOperator": ReferenceAttentionOperator,
        "write_kv_cache": write_kv_cache,
    }
    manifest = []

    # 4 decode sequences, ctx {17,33,64,100}, 16/8/128,
    # bs 16, pool of 64 blocks with block tables drawn from a permutation of
    # blocks 0..62 (block 63 is the null/padding block).
    perm = _rng(0).permutation(63).tolist()
    lengths = [17, 33, 64, 100]
    tables, cursor = [], 0
    for n in lengths:
        nb = -(-n // 16)
        tables.append(perm[cursor : cursor + nb])
        cursor += nb
    manifest.append(
        _case(
            torch, mv, name="config1_decode", seed=1, num_q_heads=16, num_kv_heads=8, head_dim=128,
            block_size=16, num_blocks=64, pad_block=63,
            requests=[{"table": t, "history": n - 1, "positions": [n - 1]} for t, n in zip(tables, lengths)],
            description="BASELINE config 1: decode step, history written first via write_kv_cache",
        )
    )
    # Mixed chunked prefill with prefix-cache hit + decode + fresh prefill.
    manifest.append(
        _case(
            torch, mv, name="mixed_chunked", seed=3, num_q_heads=4, num_kv_heads=2, head_dim=128,
            block_size=16, num_blocks=24, pad_block=23,
            requests=[
                {"table": [5, 9, 2], "history": 21, "positions": list(range(21, 40))},
                {"table": [7, 11, 3, 0], "history": 52, "positions": [52]},
                {"table": [13, 1, 17], "history": 0, "positions": list(range(0, 35))},
                {"table": [4, 19], "history": 16, "positions": list(range(16, 18))},
            ],
            description="chunked prefill over a cached prefix, a decode, a fresh prefill and a 2-token chunk",
        )
    )
    # Reference spike test shapes: ragged multi-request with -1 padded block
    # table and per-query visibility starts (tests/benchmarks/test_spike_triton_paged.py:215-319).
    for hq, hkv, d in ((4, 4, 8), (4, 2, 8), (7, 1, 8), (4, 1, 7), (16, 8, 128)):
        manifest.append(
            _case(
                torch, mv, name=f"ragged_{hq}_{hkv}_{d}", seed=4, num_q_heads=hq, num_kv_heads=hkv,
                head_dim=d, block_size=2, num_blocks=6, pad_block=-1,
                requests=[
                    {"table": [3, 1, 5], "history": 0, "positions": [0, 1, 2, 3, 4], "starts": [0, 0, 1, 1, 2]},
                    {"table": [4, 0], "history": 2, "positions": [2], "starts": [0]},
                ],
                description="ragged MHA/GQA/MQA, non-power-of-two group, odd head_dim, -1 table padding",
            )
        )
    # Graph padding: a zero-length request and a slot -1 token over a NaN
    # sentinel cache (tests/attention/operators/test_triton_paged.py:180-247).
    manifest.append(
        _case(
            torch, mv, name="graph_padding", seed=5, num_q_heads=4, num_kv_heads=2, head_dim=16,
            block_size=3, num_blocks=7, pad_block=0, cache_fill=float("nan"), extra_tokens=1,
            requests=[
                {"table": [6, 1, 4], "history": 0, "positions": [0, 1, 2]},
                {"table": [0, 0, 0], "history": 0, "positions": [], "context_length": 0},
            ],
            description="CUDA-graph padding: zero-length request, slot -1, NaN sentinel cache",
        )
    )
    # Sliding-window and chunked-local visibility, chunked prefill then decode
    # (test_triton_paged.py:252-292), one call per chunk.
    for spec_name, start_fn in (
        ("sliding3", lambda p: max(0, p - 3 + 1)),
        ("chunked4", lambda p: (p // 4) * 4),
    ):
        for ci, (s, e) in enumerate(((0, 3), (3, 6), (6, 7), (7, 8))):
            manifest.append(
                _case(
                    torch, mv, name=f"{spec_name}_chunk{ci}", seed=10 + ci, num_q_heads=4, num_kv_heads=2,
                    head_dim=16, block_size=3, num_blocks=7, pad_block=0,
                    requests=[{"table": [6, 1, 4], "history": s, "positions": list(range(s, e)),
                               "starts": [start_fn(p) for p in range(s, e)]}],
                    description=f"{spec_name} visibility, chunk [{s},{e}) over a history of {s} tokens",
                )
            )
    # Sliding window at the production shape, long enough to cross blocks.
    manifest.append(
        _case(
            torch, mv, name="sliding40_qwen", seed=20, num_q_heads=16, num_kv_heads=8, head_dim=128,
            block_size=16, num_blocks=16, pad_block=15,
            requests=[
                {"table": [3, 8, 1, 12, 6], "history": 60, "positions": list(range(60, 70)),
                 "starts": [max(0, p - 40 + 1) for p in range(60, 70)]},
                {"table": [2, 9, 14], "history": 44, "positions": [44],
                 "starts": [max(0, 44 - 40 + 1)]},
            ],
            description="sliding window 40 at 16/8/128, chunk + decode",
        )
    )
    (HERE / "manifest.json").write_text(json.dumps(manifest, indent=1) + "\n")
    print(f"wrote {len(manifest)} cases")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_golden.py <micro-vllm source tree>")
    main(sys.argv[1])
