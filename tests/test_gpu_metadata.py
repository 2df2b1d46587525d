"""The device metadata build (``mvb_build_metadata``) against the reference.

* every tensor the reference's ``ModelRunner._build_model_input`` produced
  (golden, tests/golden/make_golden_metadata.py), bit-exact, and the padded
  tensors of its ``_CudaGraphExecution.copy_input`` from a fixed-capacity
  builder whose buffers held an earlier, larger step;
* seeded random plans (up to the 16384-request limit) against the oracle;
* the error paths: a position past its block ids, inconsistent counts,
  capacity overflow, too many requests;
* metadata from the builder drives the attention operator to the same
  output as metadata built the reference's way.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from _golden import BlockIds, Plan, PlanRequest, load_metadata_case, metadata_manifest
from micro_vllm_b200 import (
    B200PagedAttentionOperator,
    ChunkedLocalSpec,
    DeviceMetadataBuilder,
    FullAttentionSpec,
    SlidingWindowSpec,
)
from micro_vllm_b200 import AttentionMetadata, _lib
from oracle.metadata import PlannedRequest
from oracle.metadata import build as oracle_build

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def _spec(kind: str, param: int):
    return {"full": lambda: FullAttentionSpec(), "sliding": lambda: SlidingWindowSpec(param),
            "chunked": lambda: ChunkedLocalSpec(param)}[kind]()


def _planned(plan) -> list[PlannedRequest]:
    return [
        PlannedRequest(q.input_token_ids, q.num_computed_tokens, q.num_scheduled_tokens, q.requires_sampling,
                       tuple(t.block_ids for t in q.block_tables))
        for q in plan.scheduled_requests
    ]


def _np(t: torch.Tensor) -> np.ndarray:
    return t.cpu().numpy()


def _check_step(step, expected: dict, groups: int, layer_of_group: list[int], prefix: str = "") -> None:
    pre = prefix
    np.testing.assert_array_equal(_np(step.input_ids), expected[pre + "input_ids"])
    np.testing.assert_array_equal(_np(step.positions), expected[pre + "positions"])
    for g in range(groups):
        md = step.layer_attention_metadata[layer_of_group[g]]
        np.testing.assert_array_equal(_np(md.query_start_locations), expected[pre + "query_start_locations"])
        np.testing.assert_array_equal(_np(md.context_lengths), expected[pre + "context_lengths"])
        gp = f"g{g}/{pre}"
        np.testing.assert_array_equal(_np(md.block_table), expected[gp + "block_table"], err_msg=f"g{g}")
        np.testing.assert_array_equal(_np(md.slot_mapping), expected[gp + "slot_mapping"], err_msg=f"g{g}")
        np.testing.assert_array_equal(
            _np(md.query_context_start_positions), expected[gp + "context_starts"], err_msg=f"g{g}")
        assert md.query_positions is step.positions


def _layers(entry) -> tuple[list, list[int]]:
    """One layer per group (in group order) plus a repeat of group 0."""

    specs = [_spec(*s) for s in entry["group_specs"]]
    return specs + [specs[0]], list(range(len(specs)))


@pytest.mark.parametrize("entry", metadata_manifest(), ids=lambda e: e["name"])
def test_build_matches_reference_golden(entry) -> None:
    plan, z = load_metadata_case(entry)
    specs, layer_of_group = _layers(entry)
    builder = DeviceMetadataBuilder(specs, entry["block_size"], entry["null_block_id"], DEV)
    step = builder.build(plan)
    _check_step(step, z, len(entry["group_specs"]), layer_of_group)
    np.testing.assert_array_equal(_np(step.sampling_row_indices), z["sampling_rows"])
    assert step.request_ids == tuple(q.request_id for q in plan.scheduled_requests)
    assert step.layer_attention_metadata[-1] is step.layer_attention_metadata[0]
    assert builder.read_status() == 0


def _random_plan(rng: np.random.Generator, num_requests: int, groups: int, block_size: int,
                 num_blocks: int, long: bool = False) -> Plan:
    reqs = []
    for i in range(num_requests):
        if rng.random() < 0.7:
            computed, n = int(rng.integers(0, 4096 if long else 900)), 1
        else:
            computed, n = int(rng.integers(0, 300)), int(rng.integers(1, 200))
        need = -(-(computed + n) // block_size) + int(rng.integers(0, 3))
        tables = tuple(BlockIds(tuple(int(b) for b in rng.integers(0, num_blocks, size=need)))
                       for _ in range(groups))
        reqs.append(PlanRequest(f"q{i}", tuple(int(t) for t in rng.integers(0, 151936, size=n)), computed, n,
                                bool(rng.random() < 0.8), tables))
    return Plan(tuple(reqs))


@pytest.mark.parametrize("entry", metadata_manifest(), ids=lambda e: e["name"])
def test_fixed_capacity_build_pads_as_copy_input(entry) -> None:
    plan, z = load_metadata_case(entry)
    specs, layer_of_group = _layers(entry)
    width = entry["table_widths"][0]
    builder = DeviceMetadataBuilder(
        specs, entry["block_size"], entry["null_block_id"], DEV, token_capacity=entry["token_capacity"],
        request_capacity=entry["request_capacity"], table_width=width)
    # An earlier step fills every request row and table cell; the golden step
    # must overwrite or pad all of them.
    groups = len(entry["group_specs"])
    full_rows = tuple(BlockIds(tuple(range(1, width + 1))) for _ in range(groups))
    dirty = Plan(tuple(
        PlanRequest(f"d{i}", (7,), i % (width * entry["block_size"]), 1, True, full_rows)
        for i in range(entry["request_capacity"])
    ))
    first = builder.build(dirty)
    step = builder.build(plan)
    assert step.input_ids.data_ptr() == first.input_ids.data_ptr()  # fixed addresses
    _check_step(step, z, groups, layer_of_group, prefix="pad/")
    np.testing.assert_array_equal(_np(step.sampling_row_indices), z["sampling_rows"])
    assert builder.read_status() == 0


@pytest.mark.parametrize("num_requests,groups,block_size", [(1, 1, 16), (7, 3, 16), (256, 1, 16),
                                                            (1000, 2, 8), (4096, 1, 16), (16384, 1, 32)])
def test_random_plans_match_the_oracle(num_requests, groups, block_size) -> None:
    rng = np.random.default_rng(num_requests + groups)
    plan = _random_plan(rng, num_requests, groups, block_size, 1 << 20, long=num_requests == 256)
    kinds = [("full", 0), ("sliding", 129), ("chunked", 64)][:groups]
    builder = DeviceMetadataBuilder([_spec(*k) for k in kinds], block_size, (1 << 20) - 1, DEV)
    step = builder.build(plan)
    exp = oracle_build(_planned(plan), block_size, (1 << 20) - 1, kinds)
    np.testing.assert_array_equal(_np(step.input_ids), exp["input_ids"])
    np.testing.assert_array_equal(_np(step.positions), exp["positions"])
    np.testing.assert_array_equal(_np(step.sampling_row_indices), exp["sampling_rows"])
    for g in range(groups):
        md = step.layer_attention_metadata[g]
        np.testing.assert_array_equal(_np(md.query_start_locations), exp["query_start_locations"])
        np.testing.assert_array_equal(_np(md.context_lengths), exp["context_lengths"])
        for key, t in (("block_table", md.block_table), ("slot_mapping", md.slot_mapping),
                       ("context_starts", md.query_context_start_positions)):
            np.testing.assert_array_equal(_np(t), exp["groups"][g][key], err_msg=f"g{g} {key}")
    assert builder.read_status() == 0


def test_empty_plan() -> None:
    builder = DeviceMetadataBuilder([FullAttentionSpec()], 16, 9, DEV)
    step = builder.build(Plan(()))
    md = step.layer_attention_metadata[0]
    assert md.block_table.shape == (0, 0) and md.query_start_locations.tolist() == [0]
    assert step.input_ids.numel() == 0 and step.sampling_row_indices.numel() == 0
    assert builder.read_status() == 0


def test_position_past_the_block_ids_sets_status() -> None:
    """The reference raises IndexError (map_cache_slots); the device writes
    slot -1 and sets MVB_STATUS_POSITION_PAST_TABLE."""

    plan = Plan((
        PlanRequest("a", (1,), 4, 1, True, (BlockIds((2,)),)),
        PlanRequest("b", (2, 3), 0, 2, True, (BlockIds((5,)),)),
    ))
    builder = DeviceMetadataBuilder([FullAttentionSpec()], 4, 7, DEV)
    step = builder.build(plan)
    assert step.layer_attention_metadata[0].slot_mapping.tolist() == [-1, 20, 21]
    assert builder.read_status() == _lib.MVB_STATUS_POSITION_PAST_TABLE
    with pytest.raises(IndexError):
        oracle_build(_planned(plan), 4, 7, [("full", 0)])


def _raw_build(counts_sum_override: int | None = None, table_width: int = 4):
    """Three requests through the C ABI directly, the token total optionally wrong."""

    i32 = dict(dtype=torch.int32, device=DEV)
    computed = torch.tensor([0, 5, 9], **i32)
    scheduled = torch.tensor([2, 1, 3], **i32)
    nblk = torch.tensor([1, 2, 3], **i32)
    ids = torch.tensor([10, 11, 12, 13, 14, 15], **i32)
    t_cap, r_cap = 8, 4
    out = {k: torch.full((n,), 123, dtype=torch.int64, device=DEV) for k, n in
           (("pos", t_cap), ("start", t_cap), ("slot", t_cap), ("qsl", r_cap + 1), ("ctx", r_cap))}
    table = torch.full((r_cap, table_width), 123, dtype=torch.int64, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    lib = _lib.load()
    num_tokens = 6 if counts_sum_override is None else counts_sum_override
    rc = lib.mvb_build_metadata(
        computed.data_ptr(), scheduled.data_ptr(), nblk.data_ptr(), ids.data_ptr(), None, None,
        3, num_tokens, 6, 0, r_cap, t_cap, table_width, table_width, 4, 99, _lib.MVB_SPEC_FULL, 0,
        None, out["pos"].data_ptr(), out["start"].data_ptr(), out["qsl"].data_ptr(), out["ctx"].data_ptr(),
        table.data_ptr(), out["slot"].data_ptr(), None, status.data_ptr(),
        torch.cuda.current_stream(DEV).cuda_stream)
    return rc, out, table, status


def test_c_abi_build_and_inconsistent_counts() -> None:
    rc, out, table, status = _raw_build()
    assert rc == _lib.MVB_OK and int(status.item()) == 0
    assert out["pos"].tolist() == [0, 1, 5, 9, 10, 11, 0, 0]
    assert out["slot"].tolist() == [40, 41, 49, 61, 62, 63, -1, -1]
    assert out["qsl"].tolist() == [0, 2, 3, 6, 6] and out["ctx"].tolist() == [2, 6, 12, 0]
    assert table.tolist() == [[10, 99, 99, 99], [11, 12, 99, 99], [13, 14, 15, 99], [99, 99, 99, 99]]
    # Totals that disagree with the counts: padding only, and the status bit.
    rc, out, table, status = _raw_build(counts_sum_override=5)
    assert rc == _lib.MVB_OK and int(status.item()) == _lib.MVB_STATUS_INCONSISTENT_COUNTS
    assert out["slot"].tolist() == [-1] * 8 and out["qsl"].tolist() == [0, 5, 5, 5, 5]  # an empty batch
    assert table.tolist() == [[99] * 4] * 4
    # A request with more block ids than the table is wide.
    rc, out, table, status = _raw_build(table_width=2)
    assert int(status.item()) == _lib.MVB_STATUS_INCONSISTENT_COUNTS
    # Argument checks.
    lib = _lib.load()
    assert lib.mvb_build_metadata(None, None, None, None, None, None, 1, 0, 0, 0, 1, 0, 0, 0, 4, 0, 0, 0,
                                  *([None] * 10)) == _lib.MVB_ERR_INVALID_ARGUMENT
    assert lib.mvb_build_metadata(None, None, None, None, None, None, 0, 0, 0, 0, 0, 0, 0, 0, 4, 0, 1, 0,
                                  *([None] * 10)) == _lib.MVB_ERR_INVALID_ARGUMENT  # window 0
    dummy = ctypes.c_void_p(torch.zeros(1, device=DEV).data_ptr())
    assert lib.mvb_build_metadata(dummy, dummy, dummy, None, None, None, 16385, 0, 0, 0, 16385, 0, 0, 0, 4,
                                  0, 0, 0, *([None] * 10)) == _lib.MVB_ERR_UNSUPPORTED_SHAPE


def test_capacity_overflow_raises() -> None:
    builder = DeviceMetadataBuilder([FullAttentionSpec()], 16, 9, DEV, token_capacity=4, request_capacity=2,
                                    table_width=2)
    plan = Plan(tuple(PlanRequest(f"r{i}", (1, 2, 3), 0, 3, True, (BlockIds((i,)),)) for i in range(2)))
    with pytest.raises(ValueError):
        builder.build(plan)


def test_builder_metadata_drives_the_operator() -> None:
    """Attention over a 64-request mixed step: metadata from the builder and
    metadata built the reference's way give bit-identical outputs."""

    rng = np.random.default_rng(5)
    bs, nb, hq, hkv, d = 16, 4096, 16, 8, 128
    free = iter(rng.permutation(nb - 1).tolist())  # every slot written once
    reqs = []
    for i in range(64):
        computed, n = (int(rng.integers(0, 900)), 1) if i % 3 else (int(rng.integers(0, 300)), 150)
        blocks = tuple(next(free) for _ in range(-(-(computed + n) // bs)))
        reqs.append(PlanRequest(f"q{i}", (0,) * n, computed, n, True, (BlockIds(blocks),)))
    plan = Plan(tuple(reqs))
    builder = DeviceMetadataBuilder([SlidingWindowSpec(300)], bs, nb - 1, DEV)
    step = builder.build(plan)
    exp = oracle_build(_planned(plan), bs, nb - 1, [("sliding", 300)])
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(DEV)  # noqa: E731
    ref_md = AttentionMetadata(
        query_positions=t(exp["positions"]), query_context_start_positions=t(exp["groups"][0]["context_starts"]),
        query_start_locations=t(exp["query_start_locations"]), context_lengths=t(exp["context_lengths"]),
        block_table=t(exp["groups"][0]["block_table"]), slot_mapping=t(exp["groups"][0]["slot_mapping"]),
        block_size=bs)
    g = torch.Generator(device=DEV).manual_seed(1)
    n = step.positions.numel()
    q = torch.randn((n, hq, d), generator=g, device=DEV).half()
    k = torch.randn((n, hkv, d), generator=g, device=DEV).half()
    v = torch.randn((n, hkv, d), generator=g, device=DEV).half()
    cache = torch.randn((2, nb, bs, hkv, d), generator=g, device=DEV).half()
    cache2 = cache.clone()
    op = B200PagedAttentionOperator()
    out = op(q, k, v, cache, step.layer_attention_metadata[0])
    ref = op(q, k, v, cache2, ref_md)
    assert torch.equal(out, ref) and torch.equal(cache, cache2)
    assert builder.read_status() == 0


def test_pinned_staging_round_trip() -> None:
    """One pinned buffer, one copy: the device views hold the host tensors."""

    from micro_vllm_b200.staging import PinnedStaging

    g = torch.Generator().manual_seed(2)
    host = {"a": torch.randn((3, 5), generator=g).half(), "b": torch.arange(7), "c": torch.randn(1, generator=g)}
    st = PinnedStaging(DEV)
    st.pack(host)
    for _ in range(2):
        d = st.upload()
        for k, t in host.items():
            assert torch.equal(d[k].cpu(), t) and d[k].device == DEV
        host["b"] = host["b"] + 1
        st.pack(host)
    with pytest.raises(ValueError):
        st.pack({"a": torch.zeros(2)})


def test_upload_pipeline_steps_in_order() -> None:
    """Double-buffered uploads and read-backs: every step sees its own inputs
    and every host result is its own step's, with slow kernels in between
    (a slot is not overwritten while its step still reads it)."""

    from micro_vllm_b200.staging import UploadPipeline

    steps, n = 6, 4096
    g = torch.Generator().manual_seed(5)
    inputs = [{"x": torch.randn(n, generator=g), "y": torch.full((n,), float(i))} for i in range(steps)]
    outs = [torch.empty(n).pin_memory() for _ in range(steps)]
    pipe = UploadPipeline(DEV)
    for i in range(steps):
        pipe.slot(i).pack(inputs[i])  # waits for the slot's previous upload on the host
        d = pipe.upload(i)
        torch.cuda._sleep(2_000_000)  # a long step: the next upload runs beside it
        result = d["x"] * 2 + d["y"]
        pipe.download(i, result, outs[i])
    pipe.drain()
    torch.cuda.synchronize(DEV)
    for i in range(steps):
        assert torch.equal(outs[i], inputs[i]["x"] * 2 + inputs[i]["y"])


def test_upload_pipeline_drives_the_operator() -> None:
    """The benchmark's end-to-end path: a decode step's q/k/v and metadata
    from pinned host memory through the pipeline give the same output, bit
    for bit, as the operator on device inputs."""

    from micro_vllm_b200 import B200PagedAttentionOperator
    from micro_vllm_b200.staging import UploadPipeline
    from micro_vllm_b200.workloads import paged_batch

    ctx = [37, 300, 1, 129, 64]
    batch = paged_batch(context_lengths=ctx, query_lengths=[1] * len(ctx), num_q_heads=16, num_kv_heads=8,
                        head_dim=128, block_size=16, num_blocks=256, dtype=torch.float16, device=DEV, seed=3)
    op = B200PagedAttentionOperator()
    md = batch.metadata
    ref = op(batch.query, batch.key, batch.value, batch.cache, md).cpu()
    host = {"q": batch.query.cpu(), "k": batch.key.cpu(), "v": batch.value.cpu(),
            "pos": md.query_positions.cpu(), "start": md.query_context_start_positions.cpu(),
            "qsl": md.query_start_locations.cpu(), "ctx": md.context_lengths.cpu(),
            "table": md.block_table.cpu(), "slots": md.slot_mapping.cpu()}
    pipe = UploadPipeline(DEV)
    pipe.slot(0).pack(host)
    pipe.slot(1).pack(host)
    outs = [torch.empty(ref.shape, dtype=ref.dtype).pin_memory() for _ in range(4)]
    for i in range(4):
        d = pipe.upload(i)
        emd = AttentionMetadata(query_positions=d["pos"], query_context_start_positions=d["start"],
                                query_start_locations=d["qsl"], context_lengths=d["ctx"],
                                block_table=d["table"], slot_mapping=d["slots"], block_size=16)
        pipe.download(i, op(d["q"], d["k"], d["v"], batch.cache, emd), outs[i])
    pipe.drain()
    torch.cuda.synchronize(DEV)
    for o in outs:
        assert torch.equal(o, ref)
