"""Generate the metadata-build golden vectors from the real reference.

    python tests/golden/make_golden_metadata.py /path/to/micro-vllm

Imports ``micro_vllm`` from ``<path>/src`` and runs, on the CPU, the
reference's own ``ModelRunner._build_model_input`` (worker/model_runner.py:
724-900: block tables, slot mappings, flattened batch, per-group
``Attention.build_metadata``) and ``_CudaGraphExecution.copy_input``
(model_runner.py:78-122) on seeded scheduler plans, the runner set up as the
reference's own tests set it up (tests/worker/test_model_runner.py:34-53).
``metadata_cases.npz`` holds, per case, the plan as flat arrays and every
tensor the reference produced; ``metadata_manifest.json`` lists the cases.
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent

NULL_BLOCK = 4095
NUM_BLOCKS = 4096


def make_cases(rng: np.random.Generator) -> list[dict]:
    """Plans as plain dicts: specs per layer, block size, requests."""

    cases = []

    # A mixed step over a hybrid model: full, sliding-window and chunked-local
    # layers (three cache groups).  Decodes, chunked-prefill chunks without
    # sampling, fresh prefills, requests crossing block boundaries.
    reqs = []
    for i in range(14):
        kind = i % 3
        if kind == 0:  # decode
            computed, scheduled, sample = int(rng.integers(0, 300)), 1, True
        elif kind == 1:  # a middle chunk of a chunked prefill
            computed, scheduled, sample = int(rng.integers(1, 200)), int(rng.integers(2, 70)), False
        else:  # the last (or only) chunk of a prefill
            computed, scheduled, sample = int(rng.choice([0, 0, 16, 33])), int(rng.integers(1, 90)), True
        reqs.append((computed, scheduled, sample))
    cases.append({"name": "hybrid_mixed", "block_size": 16,
                  "layer_specs": [("full", 0), ("sliding", 24), ("full", 0), ("chunked", 32)],
                  "requests": reqs, "extra_blocks": 2, "pad": (37, 5, 3)})

    # A decode-only step of 256 requests, block size 16, one full group.
    reqs = [(int(c), 1, True) for c in rng.integers(0, 700, size=256)]
    cases.append({"name": "decode256", "block_size": 16, "layer_specs": [("full", 0)],
                  "requests": reqs, "extra_blocks": 0, "pad": (64, 32, 8)})

    # Small blocks, long chunks: many blocks per request, sliding window only.
    reqs = [(int(rng.integers(0, 40)), int(rng.integers(1, 40)), bool(rng.integers(0, 2))) for _ in range(9)]
    cases.append({"name": "sliding_bs4", "block_size": 4, "layer_specs": [("sliding", 5)],
                  "requests": reqs, "extra_blocks": 1, "pad": (3, 2, 0)})
    return cases


def main(ref_root: str) -> None:
    sys.path.insert(0, str(Path(ref_root) / "src"))
    import torch
    from micro_vllm.attention.attention import Attention, AttentionMetadata
    from micro_vllm.attention.spec import ChunkedLocalSpec, FullAttentionSpec, SlidingWindowSpec
    from micro_vllm.config import CacheConfig, LLMConfig, ModelConfig
    from micro_vllm.core.kv_cache_spec import build_kv_cache_topology
    from micro_vllm.core.scheduler_output import CacheGroupBlockTable, ScheduledRequest, SchedulerOutput
    from micro_vllm.worker.model_runner import ModelInput, ModelRunner, _CudaGraphExecution

    def make_spec(kind, param):
        return {"full": FullAttentionSpec, "sliding": SlidingWindowSpec, "chunked": ChunkedLocalSpec}[kind](
            *(() if kind == "full" else (param,)))

    class _InputModel:
        def __init__(self, layer_attentions):
            self.layer_attentions = layer_attentions

    rng = np.random.default_rng(11)
    arrays: dict[str, np.ndarray] = {}
    manifest = []
    for case in make_cases(rng):
        name, bs = case["name"], case["block_size"]
        attentions = tuple(Attention(make_spec(*s), "reference") for s in case["layer_specs"])
        topology = build_kv_cache_topology(tuple(a.spec for a in attentions))
        group_specs = [
            next(s for s, a in zip(case["layer_specs"], attentions) if a.spec == g.attention_spec)
            for g in topology.groups
        ]
        runner = ModelRunner(LLMConfig(
            model_config=ModelConfig(model="unused", device=torch.device("cpu")),
            cache_config=CacheConfig(block_size=bs, num_blocks=8),
        ))
        runner._model = _InputModel(attentions)
        runner._kv_cache_topology = topology

        scheduled = []
        flat = {"computed": [], "scheduled": [], "sample": [], "token_ids": []}
        group_blocks = [[] for _ in group_specs]
        group_counts = [[] for _ in group_specs]
        for i, (computed, n, sample) in enumerate(case["requests"]):
            tokens = tuple(int(t) for t in rng.integers(0, 151936, size=n))
            needed = (computed + n + bs - 1) // bs + case["extra_blocks"] * (i % 2)
            tables = []
            for g, (kind, param) in enumerate(group_specs):
                ids = [int(b) for b in rng.choice(NULL_BLOCK, size=needed, replace=False)]
                if kind == "sliding":  # blocks wholly before the window are released to the null block
                    first_visible = max(0, computed - param + 1) // bs
                    ids[:first_visible] = [NULL_BLOCK] * first_visible
                tables.append(CacheGroupBlockTable(tuple(ids)))
                group_blocks[g].extend(ids)
                group_counts[g].append(len(ids))
            scheduled.append(ScheduledRequest(
                request_id=f"r{i}", input_token_ids=tokens, num_computed_tokens=computed,
                num_scheduled_tokens=n, requires_sampling=sample, block_tables=tuple(tables),
            ))
            flat["computed"].append(computed)
            flat["scheduled"].append(n)
            flat["sample"].append(int(sample))
            flat["token_ids"].extend(tokens)
        plan = SchedulerOutput(tuple(scheduled))
        mi = runner._build_model_input(plan, NULL_BLOCK)
        group_md = []
        for g in topology.groups:
            md = mi.layer_attention_metadata[g.layer_indices[0]]
            group_md.append(md)

        # Padded copy into a captured capacity, through the reference's copy_input.
        extra_t, extra_r, extra_w = case["pad"]
        t_cap = mi.input_ids.numel() + extra_t
        r_cap = len(scheduled) + extra_r
        shared_qsl = torch.zeros(r_cap + 1, dtype=torch.int64)
        shared_ctx = torch.zeros(r_cap, dtype=torch.int64)
        shared_pos = torch.zeros(t_cap, dtype=torch.int64)
        widths = [md.block_table.shape[1] + extra_w for md in group_md]
        target_groups = [
            AttentionMetadata(
                query_positions=shared_pos,
                query_context_start_positions=torch.zeros(t_cap, dtype=torch.int64),
                query_start_locations=shared_qsl, context_lengths=shared_ctx,
                block_table=torch.zeros((r_cap, w), dtype=torch.int64),
                slot_mapping=torch.zeros(t_cap, dtype=torch.int64), block_size=bs,
            )
            for w in widths
        ]
        layer_targets = [None] * topology.num_layers
        for gi, g in enumerate(topology.groups):
            for li in g.layer_indices:
                layer_targets[li] = target_groups[gi]
        target = ModelInput(
            input_ids=torch.zeros(t_cap, dtype=torch.int64), positions=shared_pos,
            layer_attention_metadata=tuple(layer_targets), request_ids=(),
            sampling_row_indices=torch.zeros(0, dtype=torch.int64),
        )
        _CudaGraphExecution(graph=None, model_input=target, hidden_states=None,
                            null_block_id=NULL_BLOCK).copy_input(mi)

        p = f"{name}/"
        arrays[p + "computed"] = np.array(flat["computed"], np.int32)
        arrays[p + "scheduled"] = np.array(flat["scheduled"], np.int32)
        arrays[p + "sample"] = np.array(flat["sample"], np.uint8)
        arrays[p + "token_ids"] = np.array(flat["token_ids"], np.int32)
        arrays[p + "input_ids"] = mi.input_ids.numpy()
        arrays[p + "positions"] = mi.positions.numpy()
        arrays[p + "query_start_locations"] = group_md[0].query_start_locations.numpy()
        arrays[p + "context_lengths"] = group_md[0].context_lengths.numpy()
        arrays[p + "sampling_rows"] = mi.sampling_row_indices.numpy()
        arrays[p + "pad/input_ids"] = target.input_ids.numpy()
        arrays[p + "pad/positions"] = target.positions.numpy()
        arrays[p + "pad/query_start_locations"] = shared_qsl.numpy()
        arrays[p + "pad/context_lengths"] = shared_ctx.numpy()
        for g, md in enumerate(group_md):
            q = f"{p}g{g}/"
            arrays[q + "block_counts"] = np.array(group_counts[g], np.int32)
            arrays[q + "block_ids"] = np.array(group_blocks[g], np.int32)
            arrays[q + "block_table"] = md.block_table.numpy()
            arrays[q + "slot_mapping"] = md.slot_mapping.numpy()
            arrays[q + "context_starts"] = md.query_context_start_positions.numpy()
            arrays[q + "pad/block_table"] = target_groups[g].block_table.numpy()
            arrays[q + "pad/slot_mapping"] = target_groups[g].slot_mapping.numpy()
            arrays[q + "pad/context_starts"] = target_groups[g].query_context_start_positions.numpy()
        manifest.append({
            "name": name, "block_size": bs, "null_block_id": NULL_BLOCK,
            "group_specs": [list(s) for s in group_specs],
            "token_capacity": t_cap, "request_capacity": r_cap, "table_widths": widths,
        })
    np.savez_compressed(HERE / "metadata_cases.npz", **arrays)
    (HERE / "metadata_manifest.json").write_text(json.dumps(manifest, indent=1) + "\n")
    print("wrote metadata_cases.npz:", ", ".join(c["name"] for c in manifest))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_golden_metadata.py <micro-vllm source tree>")
    main(sys.argv[1])
