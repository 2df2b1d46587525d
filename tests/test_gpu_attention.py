"""Parity of the CUDA path with the oracle and the reference's golden vectors.

Everything here goes through the C ABI (``libmvb200.so``) via the
``b200_paged`` operator.  Tolerances (from the build's contract):
  * KV-cache scatter: bit-exact;
  * fp16 / bf16 attention: |out - ref| <= 2e-3 + 1e-2 * |ref| against an
    fp32 reference computed on the same (rounded) inputs;
  * fp32 attention (exact CUDA-core kernel): 1e-5.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from _golden import cache_digest, case_names, load_case
from _oracle_bridge import assert_close, oracle_subset, snapshot_pages
from micro_vllm_b200 import AttentionMetadata, B200PagedAttentionOperator, write_kv_cache
from micro_vllm_b200 import _lib
from micro_vllm_b200.workloads import paged_batch, uniform_lengths
from oracle import OracleMetadata, paged_attention, write_kv_cache as oracle_write

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-2
DEV = torch.device("cuda", 0)


def _case_on_device(case: dict, dtype: torch.dtype):
    t = lambda name: torch.from_numpy(np.ascontiguousarray(case[name]))  # noqa: E731
    md = AttentionMetadata(
        query_positions=t("query_positions").to(DEV),
        query_context_start_positions=t("query_context_start_positions").to(DEV),
        query_start_locations=t("query_start_locations").to(DEV),
        context_lengths=t("context_lengths").to(DEV),
        block_table=t("block_table").to(DEV),
        slot_mapping=t("slot_mapping").to(DEV),
        block_size=case["block_size"],
    )
    conv = lambda name: torch.from_numpy(case[name].astype(np.float32)).to(DEV, dtype)  # noqa: E731
    return conv("query"), conv("key"), conv("value"), conv("cache_before"), md


def _oracle_md(case: dict) -> OracleMetadata:
    return OracleMetadata(
        query_positions=case["query_positions"],
        query_context_start_positions=case["query_context_start_positions"],
        query_start_locations=case["query_start_locations"],
        context_lengths=case["context_lengths"],
        block_table=case["block_table"],
        slot_mapping=case["slot_mapping"],
        block_size=case["block_size"],
    )


@pytest.mark.parametrize("name", case_names())
def test_golden_fp16_matches_reference(name: str) -> None:
    """fp16 inputs equal the fixture's exactly; compare to the reference's
    fp32 output, and the written cache bit-for-bit to the reference's."""

    case = load_case(name)
    q, k, v, cache, md = _case_on_device(case, torch.float16)
    out = B200PagedAttentionOperator()(q, k, v, cache, md)
    torch.cuda.synchronize()
    assert out.dtype == torch.float16 and out.shape == q.shape
    assert_close(out, case["expected_output"], ATOL, RTOL)
    assert cache_digest(cache.float().cpu().numpy()) == case["expected_cache_sha256"]


@pytest.mark.parametrize("name", case_names())
def test_golden_fp32_matches_reference_tightly(name: str) -> None:
    case = load_case(name)
    q, k, v, cache, md = _case_on_device(case, torch.float32)
    out = B200PagedAttentionOperator()(q, k, v, cache, md)
    torch.cuda.synchronize()
    assert_close(out, case["expected_output"], 1e-5, 1e-5)
    assert cache_digest(cache.cpu().numpy()) == case["expected_cache_sha256"]


@pytest.mark.parametrize("name", case_names())
def test_golden_bf16_matches_oracle(name: str) -> None:
    case = load_case(name)
    q, k, v, cache, md = _case_on_device(case, torch.bfloat16)
    # The oracle sees exactly the bf16-rounded values the kernel sees.
    qn, kn, vn, cn = (x.float().cpu().numpy() for x in (q, k, v, cache))
    expected = paged_attention(qn, kn, vn, cn, _oracle_md(case))
    out = B200PagedAttentionOperator()(q, k, v, cache, md)
    torch.cuda.synchronize()
    assert_close(out, expected, ATOL, RTOL)
    assert np.array_equal(cache.float().cpu().numpy(), cn, equal_nan=True)


def _run_and_check(batch, rows=None, atol=ATOL, rtol=RTOL, op=None):
    rows = list(range(batch.num_requests)) if rows is None else rows
    snap = snapshot_pages(batch.cache, batch.metadata.block_table, batch.context_lengths, rows)
    op = op or B200PagedAttentionOperator()
    out = op(batch.query, batch.key, batch.value, batch.cache, batch.metadata)
    torch.cuda.synchronize()
    expected, tok = oracle_subset(batch, rows, snap)
    assert_close(out[torch.tensor(tok, device=DEV)], expected, atol, rtol)
    return out


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("num_q_heads,num_kv_heads", [(16, 8), (32, 8), (8, 8), (64, 8), (14, 2)])
def test_decode_batch_matches_oracle(dtype, num_q_heads, num_kv_heads) -> None:
    """Split-KV decode with long and short contexts (many splits, merges)."""

    ctx = uniform_lengths(24, 1, 3000, seed=num_q_heads) + [1, 16, 17, 4096]
    batch = paged_batch(
        context_lengths=ctx, query_lengths=[1] * len(ctx), num_q_heads=num_q_heads,
        num_kv_heads=num_kv_heads, head_dim=128, block_size=16, num_blocks=20000,
        dtype=dtype, device=DEV, seed=7,
    )
    _run_and_check(batch)


def test_config4_long_context_decode_matches_oracle() -> None:
    """BASELINE config 4 on one GPU: 64 sequences at Hq 32 / Hkv 8 (group 4),
    contexts U[4096, 8192], bf16, pages drawn over a 40 GB pool (block ids
    past 2^19, byte offsets past 2^35).  The kernel runs the whole batch (the
    stream-K shares cut long requests into many segments); a spread of rows
    is checked against the oracle."""

    ctx = uniform_lengths(64, 4096, 8192, seed=1000)
    nb = int(40e9) // (2 * 16 * 8 * 128 * 2)
    batch = paged_batch(
        context_lengths=ctx, query_lengths=[1] * 64, num_q_heads=32, num_kv_heads=8, head_dim=128,
        block_size=16, num_blocks=nb, dtype=torch.bfloat16, device=DEV, seed=2000,
    )
    order = sorted(range(64), key=lambda r: ctx[r])
    rows = sorted(set(order[:4] + order[-4:] + list(range(0, 64, 4))))
    _run_and_check(batch, rows)
    del batch
    torch.cuda.empty_cache()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_config3_full_mixed_batch_matches_oracle(dtype) -> None:
    """BASELINE config 3 at full size, in one call: 8 prefill chunks of 2048
    new tokens over cached prefixes U[0, 1024] plus 120 decodes at contexts
    U[256, 2048], 16/8/128 (the bench's seeds).  Checked: every decode and
    the prefill chunks with the shortest and the longest prefix (every
    token of each)."""

    prefix = uniform_lengths(8, 0, 1024, seed=31)
    dec_ctx = uniform_lengths(120, 256, 2048, seed=32)
    ctx = [p + 2048 for p in prefix] + dec_ctx
    qlen = [2048] * 8 + [1] * 120
    nb = sum(-(-c // 16) for c in ctx) + 64
    batch = paged_batch(
        context_lengths=ctx, query_lengths=qlen, num_q_heads=16, num_kv_heads=8, head_dim=128,
        block_size=16, num_blocks=nb, dtype=dtype, device=DEV, seed=33,
    )
    rows = sorted({min(range(8), key=lambda r: prefix[r]), max(range(8), key=lambda r: prefix[r])}) + list(range(8, 128))
    _run_and_check(batch, rows)


@pytest.mark.parametrize("block_size", [1, 5, 8, 32, 64])
def test_decode_any_block_size(block_size: int) -> None:
    ctx = uniform_lengths(12, 1, 700, seed=block_size)
    nb = sum(-(-c // block_size) for c in ctx) + 50
    batch = paged_batch(
        context_lengths=ctx, query_lengths=[1] * len(ctx), num_q_heads=16, num_kv_heads=8,
        head_dim=128, block_size=block_size, num_blocks=nb, dtype=torch.float16, device=DEV, seed=3,
    )
    _run_and_check(batch)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_mixed_prefill_and_decode_batch(dtype) -> None:
    """Chunked prefill over cached prefixes (prefix-cache hits), short
    multi-token chunks that still fit the decode tile, and decodes."""

    ctx = [2048 + 300, 700, 40, 1500, 5, 999, 64, 129]
    qlen = [2048, 1, 4, 3, 5, 1, 64, 2]
    batch = paged_batch(
        context_lengths=ctx, query_lengths=qlen, num_q_heads=16, num_kv_heads=8, head_dim=128,
        block_size=16, num_blocks=4000, dtype=dtype, device=DEV, seed=11,
    )
    _run_and_check(batch)


@pytest.mark.parametrize("window", [1, 7, 40, 600])
def test_sliding_window_decode_and_chunks(window: int) -> None:
    ctx = [1000, 37, 600, 2500, 3]
    qlen = [1, 4, 1, 33, 3]
    batch = paged_batch(
        context_lengths=ctx, query_lengths=qlen, num_q_heads=16, num_kv_heads=8, head_dim=128,
        block_size=16, num_blocks=2000, dtype=torch.float16, device=DEV, seed=window, window=window,
    )
    _run_and_check(batch)


def test_graph_padding_rows_are_zero_and_cache_untouched() -> None:
    """test_triton_paged.py:180-247 at the production head shape: a
    zero-length request, slot -1 and tokens owned by no request."""

    bs, nb = 16, 40
    cache = torch.full((2, nb, bs, 8, 128), float("nan"), dtype=torch.float16, device=DEV)
    q = torch.randn((6, 16, 128), dtype=torch.float16, device=DEV)
    k = torch.randn((6, 8, 128), dtype=torch.float16, device=DEV)
    v = torch.randn((6, 8, 128), dtype=torch.float16, device=DEV)
    table = torch.tensor([[7, 3, 39], [39, 39, 39], [39, 39, 39]], device=DEV)
    md = AttentionMetadata(
        query_positions=torch.tensor([0, 1, 2, 0, 0, 0], device=DEV),
        query_context_start_positions=torch.zeros(6, dtype=torch.int64, device=DEV),
        query_start_locations=torch.tensor([0, 3, 3, 3], device=DEV),
        context_lengths=torch.tensor([3, 0, 0], device=DEV),
        block_table=table,
        slot_mapping=torch.tensor([112, 113, 114, -1, -1, -1], device=DEV),
        block_size=bs,
    )
    before = cache.clone()
    out = B200PagedAttentionOperator()(q, k, v, cache, md)
    torch.cuda.synchronize()
    assert torch.all(out[3:] == 0)
    changed = ~(torch.isnan(before) & torch.isnan(cache)) & (before != cache)
    assert changed.view(2, -1, 8, 128)[:, [112, 113, 114]].all()
    changed.view(2, -1, 8, 128)[:, [112, 113, 114]] = False
    assert not changed.any()
    qn, kn, vn = (x[:3].float().cpu().numpy() for x in (q, k, v))
    cn = np.full((2, nb, bs, 8, 128), np.nan, np.float32)
    omd = OracleMetadata(
        query_positions=np.array([0, 1, 2]), query_context_start_positions=np.zeros(3, np.int64),
        query_start_locations=np.array([0, 3]), context_lengths=np.array([3]),
        block_table=np.array([[7, 3, 39]]), slot_mapping=np.array([112, 113, 114]), block_size=bs,
    )
    assert_close(out[:3], paged_attention(qn, kn, vn, cn, omd, out_dtype=np.float32), ATOL, RTOL)


def test_out_of_range_block_ids_are_never_read() -> None:
    """A block id past the pool is excluded (and reported) instead of read."""

    bs, nb = 16, 8
    cache = torch.randn((2, nb, bs, 8, 128), dtype=torch.float16, device=DEV)
    q = torch.randn((1, 16, 128), dtype=torch.float16, device=DEV)
    kv = torch.randn((1, 8, 128), dtype=torch.float16, device=DEV)
    md = AttentionMetadata(
        query_positions=torch.tensor([40], device=DEV),
        query_context_start_positions=torch.zeros(1, dtype=torch.int64, device=DEV),
        query_start_locations=torch.tensor([0, 1], device=DEV),
        context_lengths=torch.tensor([41], device=DEV),
        block_table=torch.tensor([[2, 1 << 40, 5]], device=DEV),
        slot_mapping=torch.tensor([5 * bs + 8], device=DEV),
        block_size=bs,
    )
    op = B200PagedAttentionOperator()
    out = op(q, kv, kv, cache, md)
    assert op.read_status(DEV) & _lib.MVB_STATUS_BLOCK_OUT_OF_RANGE
    assert torch.isfinite(out.float()).all()


@pytest.mark.parametrize("head_dim", [7, 64, 128])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_kv_write_is_bit_exact_for_strided_inputs(head_dim: int, dtype) -> None:
    """tests/benchmarks/test_spike_triton_paged.py:84-129: key is a strided
    view (every other element), slots cross pages, -1 is skipped."""

    bs, nb, hkv = 4, 6, 3
    storage = torch.randn((5, hkv, head_dim * 2), device=DEV).to(dtype)
    key = storage[..., ::2]
    value = torch.randn((5, hkv, head_dim), device=DEV).to(dtype)
    slots = torch.tensor([7, 2, -1, 8, 23], device=DEV)
    cache = torch.randn((2, nb, bs, hkv, head_dim), device=DEV).to(dtype)
    expected = cache.float().cpu().numpy().copy()
    oracle_write(key.float().cpu().numpy(), value.float().cpu().numpy(), expected, slots.cpu().numpy())
    md = AttentionMetadata(
        query_positions=torch.zeros(5, dtype=torch.int64, device=DEV),
        query_context_start_positions=torch.zeros(5, dtype=torch.int64, device=DEV),
        query_start_locations=torch.tensor([0, 5], device=DEV),
        context_lengths=torch.tensor([1], device=DEV),
        block_table=torch.zeros((1, 1), dtype=torch.int64, device=DEV),
        slot_mapping=slots,
        block_size=bs,
    )
    write_kv_cache(key, value, cache, md)
    torch.cuda.synchronize()
    assert np.array_equal(cache.float().cpu().numpy(), expected)


def test_kv_write_at_decode_scale_is_bit_exact() -> None:
    """256 tokens x 8 heads x 128 scattered over a 20k-page pool."""

    bs, nb = 16, 20000
    gen = torch.Generator().manual_seed(5)
    slots = torch.randperm(nb * bs, generator=gen)[:256].to(DEV)
    key = torch.randn((256, 8, 128), device=DEV, dtype=torch.float16)
    value = torch.randn((256, 8, 128), device=DEV, dtype=torch.float16)
    cache = torch.zeros((2, nb, bs, 8, 128), device=DEV, dtype=torch.float16)
    md = AttentionMetadata(
        query_positions=torch.zeros(256, dtype=torch.int64, device=DEV),
        query_context_start_positions=torch.zeros(256, dtype=torch.int64, device=DEV),
        query_start_locations=torch.tensor([0, 256], device=DEV),
        context_lengths=torch.tensor([1], device=DEV),
        block_table=torch.zeros((1, 1), dtype=torch.int64, device=DEV),
        slot_mapping=slots,
        block_size=bs,
    )
    write_kv_cache(key, value, cache, md)
    flat = cache.view(2, -1, 8, 128)
    assert torch.equal(flat[0, slots], key) and torch.equal(flat[1, slots], value)
    assert int((flat != 0).any(dim=(2, 3)).sum()) == 2 * 256


def test_physical_placement_does_not_change_the_output() -> None:
    """Size-independent property at the benchmark's batch shape: the same
    logical contexts stored in two different page placements give
    bit-identical outputs (placement only changes addresses)."""

    ctx = uniform_lengths(256, 512, 4096, seed=0)
    kw = dict(context_lengths=ctx, query_lengths=[1] * 256, num_q_heads=16, num_kv_heads=8,
              head_dim=128, block_size=16, dtype=torch.float16, device=DEV)
    a = paged_batch(num_blocks=40000, seed=1, **kw)
    b = paged_batch(num_blocks=41000, seed=1, fill_cache=False, **kw)
    # Copy a's logical pages into b's placement.
    ta, tb = a.metadata.block_table, b.metadata.block_table
    for r, c in enumerate(ctx):
        n = -(-c // 16)
        b.cache[:, tb[r, :n]] = a.cache[:, ta[r, :n]]
    op = B200PagedAttentionOperator()
    out_a = op(a.query, a.key, a.value, a.cache, a.metadata)
    out_b = op(b.query, b.key, b.value, b.cache, b.metadata)
    torch.cuda.synchronize()
    assert torch.equal(out_a, out_b)
    # And a sample of sequences against the oracle at this size.
    rows = [0, 17, 99, 255]
    snap_batch = paged_batch(num_blocks=40000, seed=1, **kw)
    _run_and_check(snap_batch, rows=rows, op=op)


def _nan_fill_page_tails(batch) -> None:
    """Poison the unused slots after each request's context in its last page
    (and nothing the operator reads as a visible key)."""

    bs = batch.metadata.block_size
    table = batch.metadata.block_table.cpu()
    for r, c in enumerate(batch.context_lengths):
        if c % bs:
            page = int(table[r, (c - 1) // bs])
            batch.cache[:, page, c % bs:] = float("nan")


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("num_q_heads,num_kv_heads", [(16, 8), (32, 8), (8, 8), (64, 8), (16, 2)])
def test_prefill_tensor_core_path_matches_oracle(dtype, num_q_heads, num_kv_heads) -> None:
    """Chunked prefill on the tcgen05 kernel: fresh prompts, chunks over a
    cached prefix (prefix-cache hits), chunk lengths that are not a multiple
    of the query tile, NaN-poisoned page tails."""

    ctx = [700, 1500, 300, 129, 2100, 64]
    qlen = [700, 333, 300, 65, 1024, 64]
    batch = paged_batch(
        context_lengths=ctx, query_lengths=qlen, num_q_heads=num_q_heads,
        num_kv_heads=num_kv_heads, head_dim=128, block_size=16, num_blocks=2000,
        dtype=dtype, device=DEV, seed=num_q_heads + num_kv_heads,
    )
    _nan_fill_page_tails(batch)
    out = _run_and_check(batch)
    assert torch.isfinite(out.float()).all()


@pytest.mark.parametrize("block_size", [32, 48, 256])
def test_prefill_tensor_core_path_other_page_sizes(block_size: int) -> None:
    ctx = [900, 257, 1200]
    qlen = [900, 100, 17]
    nb = sum(-(-c // block_size) for c in ctx) + 8
    batch = paged_batch(
        context_lengths=ctx, query_lengths=qlen, num_q_heads=16, num_kv_heads=8, head_dim=128,
        block_size=block_size, num_blocks=nb, dtype=torch.float16, device=DEV, seed=block_size,
    )
    _run_and_check(batch)


@pytest.mark.parametrize("window", [1, 50, 300])
def test_prefill_sliding_window_on_tensor_cores(window: int) -> None:
    ctx = [1000, 640]
    qlen = [1000, 200]
    batch = paged_batch(
        context_lengths=ctx, query_lengths=qlen, num_q_heads=16, num_kv_heads=8, head_dim=128,
        block_size=16, num_blocks=200, dtype=torch.bfloat16, device=DEV, seed=window, window=window,
    )
    _nan_fill_page_tails(batch)
    _run_and_check(batch)


def test_prefill_bf16_values_beyond_fp16_range() -> None:
    """bf16 values far outside fp16's range (|v| up to 1e5, in different
    128-key tiles of a cached prefix and in a freshly written row) and
    values below fp16's normal range: the tcgen05 kernel keeps V in bf16 and
    P as P_hi + P_lo, so these must come out within the tolerance of the
    oracle like any other value."""

    ctx = [1000, 700, 900]
    qlen = [400, 700, 300]
    batch = paged_batch(
        context_lengths=ctx, query_lengths=qlen, num_q_heads=16, num_kv_heads=8, head_dim=128,
        block_size=16, num_blocks=400, dtype=torch.bfloat16, device=DEV, seed=77,
    )
    table = batch.metadata.block_table.cpu()
    # Request 0: cached prefix keys with values past the fp16 maximum in two
    # different 128-key tiles, and tiny ones in a third.
    for pos, val in ((5, 7.0e4), (300, -1.0e5), (450, 3.0e-6)):
        page, off = int(table[0, pos // 16]), pos % 16
        batch.cache[1, page, off, 2] = val
    # Request 1 (fresh prompt): one written value past the fp16 maximum.
    batch.value[400 + 123, 5] = 9.0e4
    _run_and_check(batch)


def test_a_decode_wait_that_runs_out_is_reported_and_the_next_call_is_correct() -> None:
    """The kernels' bounded waits, exercised without a fault: a one-shot hook
    (mvb_debug_arm_decode_stall) makes decode CTA 0's producer issue nothing
    for the second tile of its share and limits every wait of that launch to
    20 000 polls.  No copy is in flight for the skipped stage; the consumers'
    wait for it runs out, the launch sets MVB_STATUS_WAIT_TIMEOUT, lets its
    issued copies land and returns.  The context stays usable: the next call
    on the same operator and workspace matches the oracle with a clean
    status."""

    ctx = uniform_lengths(48, 500, 2000, seed=5)
    batch = paged_batch(
        context_lengths=ctx, query_lengths=[1] * 48, num_q_heads=16, num_kv_heads=8, head_dim=128,
        block_size=16, num_blocks=8000, dtype=torch.float16, device=DEV, seed=55,
    )
    op = B200PagedAttentionOperator()
    lib = _lib.load()
    assert op.read_status(DEV) == 0
    assert lib.mvb_debug_arm_decode_stall(0, 1, 20000) == _lib.MVB_OK
    op(batch.query, batch.key, batch.value, batch.cache, batch.metadata)
    assert op.read_status(DEV) & _lib.MVB_STATUS_WAIT_TIMEOUT
    _run_and_check(batch, op=op)
    assert op.read_status(DEV) == 0
    # Disarming works too: an armed-then-disarmed hook changes nothing.
    assert lib.mvb_debug_arm_decode_stall(0, 1, 20000) == _lib.MVB_OK
    assert lib.mvb_debug_arm_decode_stall(0, 1, 0) == _lib.MVB_OK
    _run_and_check(batch, op=op)
    assert op.read_status(DEV) == 0


def test_prefill_repeated_calls_reuse_the_workspace() -> None:
    """Several different mixed batches through one operator instance (the
    persistent kernels' barrier phases and work cursors restart cleanly)."""

    op = B200PagedAttentionOperator()
    for seed in range(4):
        ctx = uniform_lengths(6, 1, 1500, seed=seed) + [800]
        qlen = [min(c, q) for c, q in zip(ctx, uniform_lengths(6, 1, 300, seed=seed + 9))] + [800]
        batch = paged_batch(
            context_lengths=ctx, query_lengths=qlen, num_q_heads=16, num_kv_heads=8, head_dim=128,
            block_size=16, num_blocks=1000, dtype=torch.float16, device=DEV, seed=100 + seed,
        )
        _run_and_check(batch, op=op)
