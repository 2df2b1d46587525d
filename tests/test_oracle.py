"""Pin the CPU oracle before trusting it.

1. Against every golden vector produced by the reference's own
   ``ReferenceAttentionOperator`` (tests/golden/make_golden.py): outputs
   within 1e-5 (both are fp32 math; only summation order differs) and the
   full post-write cache bit-exact (SHA-256 of its fp32 bytes).
2. Against the known answers in the reference's operator tests
   (tests/attention/operators/test_reference.py in the reference project),
   restated here on the oracle.
"""

from __future__ import annotations

import math

import numpy as np
import pytest

from _golden import cache_digest, case_names, load_case, oracle_metadata
from oracle import (
    OracleMetadata,
    build_metadata,
    chunked_local_context_start,
    gather_kv_cache,
    paged_attention,
    sliding_window_context_start,
    write_kv_cache,
)


@pytest.mark.parametrize("name", case_names())
def test_oracle_matches_reference_golden_vectors(name: str) -> None:
    case = load_case(name)
    cache = case["cache_before"].astype(np.float32)
    out = paged_attention(
        case["query"].astype(np.float32),
        case["key"].astype(np.float32),
        case["value"].astype(np.float32),
        cache,
        oracle_metadata(case),
    )
    np.testing.assert_allclose(out, case["expected_output"], atol=1e-5, rtol=1e-5)
    assert cache_digest(cache) == case["expected_cache_sha256"]


def test_oracle_thread_pool_changes_nothing() -> None:
    case = load_case("mixed_chunked")
    args = [case[k].astype(np.float32) for k in ("query", "key", "value")]
    serial = paged_attention(*args, case["cache_before"].astype(np.float32), oracle_metadata(case))
    threaded = paged_attention(
        *args, case["cache_before"].astype(np.float32), oracle_metadata(case), num_threads=4
    )
    assert np.array_equal(serial, threaded)


def _md(**kw) -> OracleMetadata:
    kw.setdefault("query_context_start_positions", np.zeros_like(kw["query_positions"]))
    return OracleMetadata(**{k: (np.asarray(v, np.int64) if k != "block_size" else v) for k, v in kw.items()})


def test_visibility_start_known_answer() -> None:
    """test_reference.py:114-139 — keys before the visibility start are
    hidden; the two visible values 20 and 30 with equal scores give 25."""

    cache = np.zeros((2, 2, 2, 1, 1), np.float32)
    flat = cache.reshape(2, 4, 1, 1)
    flat[0, 0], flat[1, 0], flat[0, 1], flat[1, 1] = 1, 100, 1, 20
    md = _md(
        query_positions=[2],
        query_context_start_positions=[1],
        query_start_locations=[0, 1],
        context_lengths=[3],
        block_table=[[0, 1]],
        slot_mapping=[2],
        block_size=2,
    )
    out = paged_attention(
        np.ones((1, 1, 1), np.float32),
        np.ones((1, 1, 1), np.float32),
        np.full((1, 1, 1), 30.0, np.float32),
        cache,
        md,
    )
    assert out.shape == (1, 1, 1) and abs(float(out[0, 0, 0]) - 25.0) < 1e-6


def test_write_uses_flattened_physical_slots() -> None:
    """test_reference.py:157-178."""

    cache = np.zeros((2, 2, 4, 2, 2), np.float32)
    key = np.array([[[1, 2], [3, 4]], [[5, 6], [7, 8]]], np.float32)
    value = key + 10
    write_kv_cache(key, value, cache, np.array([1, 6]))
    flat = cache.reshape(2, 8, 2, 2)
    assert np.array_equal(flat[0, 1], key[0]) and np.array_equal(flat[0, 6], key[1])
    assert np.array_equal(flat[1, 1], value[0]) and np.array_equal(flat[1, 6], value[1])
    assert np.count_nonzero(flat[:, [0, 2, 3, 4, 5, 7]]) == 0


def test_write_skips_negative_slots_and_rejects_slots_past_the_pool() -> None:
    cache = np.full((2, 2, 2, 1, 2), 7.0, np.float32)
    key = np.ones((2, 1, 2), np.float32)
    write_kv_cache(key, key + 1, cache, np.array([-1, 3]))
    flat = cache.reshape(2, 4, 1, 2)
    assert np.all(flat[:, :3] == 7.0) and np.all(flat[0, 3] == 1) and np.all(flat[1, 3] == 2)
    with pytest.raises(IndexError):
        write_kv_cache(key, key, cache, np.array([0, 4]))


def test_gather_handles_each_request_independently() -> None:
    """test_reference.py:202-232."""

    cache = np.full((2, 5, 2, 1, 1), 99.0, np.float32)
    flat = cache.reshape(2, 10, 1, 1)
    flat[0, [6, 7, 2, 8], 0, 0] = [10, 11, 12, 20]
    flat[1, [6, 7, 2, 8], 0, 0] = [110, 111, 112, 120]
    md = _md(
        query_positions=[1, 2, 0],
        query_start_locations=[0, 2, 3],
        context_lengths=[3, 1],
        block_table=[[3, 1, 0], [4, 0, 0]],
        slot_mapping=[7, 2, 8],
        block_size=2,
    )
    hist = gather_kv_cache(cache, md)
    assert [k.flatten().tolist() for k, _ in hist] == [[10, 11, 12], [20]]
    assert [v.flatten().tolist() for _, v in hist] == [[110, 111, 112], [120]]


def test_gather_reads_only_the_minimum_contiguous_context() -> None:
    """test_reference.py:298-322: gathering starts at the first query's
    visibility start."""

    cache = np.zeros((2, 4, 2, 1, 1), np.float32)
    flat = cache.reshape(2, 8, 1, 1)
    flat[0, [1, 6, 7], 0, 0] = [3, 4, 5]
    flat[1, [1, 6, 7], 0, 0] = [13, 14, 15]
    md = _md(
        query_positions=[4, 5],
        query_context_start_positions=[3, 4],
        query_start_locations=[0, 2],
        context_lengths=[6],
        block_table=[[2, 0, 3]],
        slot_mapping=[6, 7],
        block_size=2,
    )
    ((k, v),) = gather_kv_cache(cache, md)
    assert k.flatten().tolist() == [3, 4, 5] and v.flatten().tolist() == [13, 14, 15]


def dense_attention(q, k, v, positions=None, starts=None) -> np.ndarray:
    """Dense masked attention over a contiguous history (the reference
    tests' ``dense_causal_attention``, test_reference.py:325-360)."""

    t, hq, d = q.shape
    g = hq // k.shape[1]
    kk = np.repeat(k, g, axis=1).astype(np.float64)
    vv = np.repeat(v, g, axis=1).astype(np.float64)
    pos = np.arange(t) if positions is None else np.asarray(positions)
    st = np.zeros_like(pos) if starts is None else np.asarray(starts)
    kpos = np.arange(k.shape[0])
    s = np.einsum("qhd,khd->hqk", q.astype(np.float64), kk) / math.sqrt(d)
    hidden = (kpos[None, :] < st[:, None]) | (kpos[None, :] > pos[:, None])
    s = np.where(hidden[None], -np.inf, s)
    w = np.exp(s - s.max(-1, keepdims=True))
    w /= w.sum(-1, keepdims=True)
    return np.einsum("hqk,khd->qhd", w, vv)


def _linspace_tensors(t, hq=4, hkv=2, d=3):
    """The reference tests' ``make_attention_tensors`` (test_reference.py:428-460)."""

    q = np.linspace(-0.8, 0.9, t * hq * d, dtype=np.float32).reshape(t, hq, d)
    k = np.linspace(0.7, -0.6, t * hkv * d, dtype=np.float32).reshape(t, hkv, d)
    v = np.linspace(-1.0, 1.0, t * hkv * d, dtype=np.float32).reshape(t, hkv, d)
    return q, k, v


@pytest.mark.parametrize("hkv", [4, 2, 1])
def test_full_prefill_matches_dense_mha_gqa_mqa(hkv: int) -> None:
    """test_reference.py:463-497."""

    q = np.arange(24, dtype=np.float32).reshape(3, 4, 2) / 10
    k = np.arange(3 * hkv * 2, dtype=np.float32).reshape(3, hkv, 2) / 20
    v = k + 1
    cache = np.zeros((2, 3, 2, hkv, 2), np.float32)
    md = _md(
        query_positions=[0, 1, 2],
        query_start_locations=[0, 3],
        context_lengths=[3],
        block_table=[[2, 0]],
        slot_mapping=[4, 5, 0],
        block_size=2,
    )
    out = paged_attention(q, k, v, cache, md)
    np.testing.assert_allclose(out, dense_attention(q, k, v), atol=1e-6, rtol=1e-6)


@pytest.mark.parametrize(
    "start_fn",
    [
        lambda p: sliding_window_context_start(p, 2),
        lambda p: sliding_window_context_start(p, 6),
        lambda p: chunked_local_context_start(p, 2),
        lambda p: chunked_local_context_start(p, 6),
    ],
)
def test_bounded_prefill_matches_dense_mask(start_fn) -> None:
    """test_reference.py:500-549."""

    q, k, v = _linspace_tensors(9)
    cache = np.zeros((2, 5, 4, 2, 3), np.float32)
    md = build_metadata([list(range(9))], [[4, 1, 3]], block_size=4, context_start=start_fn)
    out = paged_attention(q, k, v, cache, md)
    expected = dense_attention(q, k, v, md.query_positions, md.query_context_start_positions)
    np.testing.assert_allclose(out, expected, atol=1e-6, rtol=1e-6)


def test_low_precision_dtype_is_restored() -> None:
    """test_reference.py:552-575."""

    q = np.array([[[1.0, 2.0]]], np.float16)
    k = np.array([[[2.0, 1.0]]], np.float16)
    v = np.array([[[3.0, 4.0]]], np.float16)
    cache = np.zeros((2, 1, 2, 1, 2), np.float16)
    md = _md(
        query_positions=[0], query_start_locations=[0, 1], context_lengths=[1],
        block_table=[[0]], slot_mapping=[0], block_size=2,
    )
    out = paged_attention(q, k, v, cache, md)
    assert out.dtype == np.float16 and np.array_equal(out, v)


def test_chunked_prefill_and_decode_match_full_prefill() -> None:
    """test_reference.py:607-643 and :695-748."""

    q, k, v = _linspace_tensors(6)
    table = [4, 1, 3]
    full = paged_attention(
        q, k, v, np.zeros((2, 5, 2, 2, 3), np.float32),
        build_metadata([list(range(6))], [table], block_size=2),
    )
    cache = np.zeros((2, 5, 2, 2, 3), np.float32)
    pieces = [
        paged_attention(q[s:e], k[s:e], v[s:e], cache, build_metadata([list(range(s, e))], [table], block_size=2))
        for s, e in ((0, 3), (3, 4), (4, 5), (5, 6))
    ]
    expected = dense_attention(q, k, v)
    np.testing.assert_allclose(full, expected, atol=1e-6, rtol=1e-6)
    np.testing.assert_allclose(np.concatenate(pieces), expected, atol=1e-6, rtol=1e-6)


def test_shared_prefix_gives_identical_attention() -> None:
    """test_reference.py:923-968."""

    pq, pk, pv = _linspace_tensors(2, hq=2, hkv=1)
    cache = np.zeros((2, 3, 2, 1, 3), np.float32)
    paged_attention(pq, pk, pv, cache, build_metadata([[0, 1]], [[0]], block_size=2))
    q, k, v = _linspace_tensors(1, hq=2, hkv=1)
    q, k, v = q + 0.25, k - 0.15, v + 0.35
    out = paged_attention(
        np.concatenate((q, q)), np.concatenate((k, k)), np.concatenate((v, v)), cache,
        build_metadata([[2], [2]], [[0, 1], [0, 2]], block_size=2),
    )
    expected = dense_attention(np.concatenate((pq, q)), np.concatenate((pk, k)), np.concatenate((pv, v)))[-1]
    np.testing.assert_allclose(out[0], expected, atol=1e-6, rtol=1e-6)
    np.testing.assert_allclose(out[1], expected, atol=1e-6, rtol=1e-6)


def test_padding_rows_are_zero_and_empty_visibility_is_nan() -> None:
    cache = np.zeros((2, 2, 2, 1, 2), np.float32)
    q = np.ones((3, 1, 2), np.float32)
    md = _md(
        query_positions=[0, 1, 0],
        query_context_start_positions=[0, 5, 0],  # token 1 sees nothing
        query_start_locations=[0, 2, 2],
        context_lengths=[2, 0],
        block_table=[[0, 1], [1, 1]],
        slot_mapping=[0, 1, -1],
        block_size=2,
    )
    out = paged_attention(q, q, q, cache, md)
    assert np.all(np.isfinite(out[0])) and np.all(np.isnan(out[1])) and np.all(out[2] == 0)


# ---------------------------------------------------------------- Qwen3 attention prologue
from _golden import PROLOGUE_CASES, from_bits, load_prologue_case, within_ulps  # noqa: E402
from oracle.qk_prologue import inverse_frequencies, qk_norm_rope_and_cache, rms_norm, rope  # noqa: E402


@pytest.mark.parametrize("name", PROLOGUE_CASES)
def test_prologue_oracle_matches_reference_golden(name: str) -> None:
    """q/k RMSNorm + RoPE + KV write against the reference's own modules
    (tests/golden/make_golden_prologue.py): every element within two ulps of
    the model dtype (the variance is summed in another order, and a one-ulp
    change of the normalised value can pass through the weight multiply and
    the rotation), all but a handful exactly equal."""

    z = load_prologue_case(name)
    dt = str(z["dtype"])
    q, k, v = (from_bits(z[n], dt) for n in ("query", "key", "value"))
    cache = from_bits(z["cache_before"], dt).copy()
    out = qk_norm_rope_and_cache(
        q, k, v, z["positions"], from_bits(z["q_weight"], dt), from_bits(z["k_weight"], dt),
        float(z["eps"]), z["inv_freq"], cache, z["slot_mapping"], dt,
    )
    expected_q, expected_cache = from_bits(z["q_out"], dt), from_bits(z["cache_after"], dt)
    assert within_ulps(out, expected_q, dt, 2, rotated=True).all()
    assert np.mean(out != expected_q) < 1e-3
    assert within_ulps(cache, expected_cache, dt, 2, rotated=True).all()
    # numpy's float32 power may differ from torch's by an ulp, which is why
    # the kernel takes the inverse frequencies computed with torch exactly as
    # the reference computes them (rotary_embedding.py:29-38).
    np.testing.assert_allclose(inverse_frequencies(128, float(z["base"])), z["inv_freq"], rtol=3e-7)


def test_prologue_rms_norm_kat() -> None:
    """normalization test: fp16 [512, -384, 256, -128] equals the fp32
    formula rounded to fp16 (tests/layers/test_normalization.py:16-33)."""

    x = np.array([[[512.0, -384.0, 256.0, -128.0]]], np.float32)
    eps = 1e-6
    expected = (x * (1.0 / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps))).astype(np.float16)
    out = rms_norm(x, np.ones(4, np.float32), eps, "f16")
    np.testing.assert_array_equal(out, expected.astype(np.float32))


def test_prologue_rope_is_a_rotation_of_half_pairs() -> None:
    """RoPE rotates each pair (x_i, x_{i+D/2}) by pos * inv_freq_i (the
    transformers comparison of tests/layers/test_rotary_embedding.py:35-52)."""

    pos = np.array([5, 1, 127])
    x = np.linspace(-1.0, 1.0, 3 * 4 * 8, dtype=np.float32).reshape(3, 4, 8)
    inv = inverse_frequencies(8, 50_000.0)
    out = rope(pos, x, inv, "f32")
    z = (x[..., :4] + 1j * x[..., 4:]) * np.exp(1j * (pos[:, None, None] * inv[None, None, :]))
    np.testing.assert_allclose(out[..., :4], z.real, atol=1e-6)
    np.testing.assert_allclose(out[..., 4:], z.imag, atol=1e-6)


# ---------------------------------------------------------------- sampler
from _golden import SAMPLER_TIE_ROW, load_sampler_cases  # noqa: E402
from oracle.sampler import greedy, kept_and_probabilities  # noqa: E402


def test_sampler_oracle_matches_reference_golden() -> None:
    """Greedy tokens (ties: first index) and the sets top-k / top-p keep,
    against the reference's Sampler and filters (make_golden_sampler.py)."""

    z = load_sampler_cases()
    assert [greedy(r) for r in z["logits"]] == z["greedy"].tolist()
    for c in range(len(z["temperature"])):
        k = int(z["top_k"][c])
        for r, row in enumerate(z["logits"]):
            kept, probs = kept_and_probabilities(row, float(z["temperature"][c]), k or None, float(z["top_p"][c]))
            if r == SAMPLER_TIE_ROW:
                assert kept.sum() == z["kept"][c, r].sum()
            else:
                np.testing.assert_array_equal(kept, z["kept"][c, r])
            assert abs(probs.sum() - 1.0) < 1e-9 and np.all(probs[~kept] == 0)


def test_sampler_oracle_reference_test_cases() -> None:
    """sampler tests: top-p keeps the boundary token (test_sampler.py:127-143),
    top-k keeps the largest (:96-111), top-k >= vocab filters nothing (:114-124)."""

    kept, _ = kept_and_probabilities(np.array([3.0, 2.0, 0.0, -1.0]), 1.0, None, 0.8)
    assert kept.tolist() == [True, True, False, False]
    kept, _ = kept_and_probabilities(np.array([0.0, 1.0, 2.0, 3.0, 4.0]), 1.0, 2, 1.0)
    assert kept.tolist() == [False, False, False, True, True]
    kept, _ = kept_and_probabilities(np.array([0.0, 1.0, 2.0]), 1.0, 3, 1.0)
    assert kept.all()


def test_race_oracle_is_torch_multinomial_with_the_same_generator() -> None:
    """oracle.sampler.race_token with q drawn by a generator seeded as the
    reference seeds its own equals torch.multinomial(probabilities, 1,
    generator) on the reference's filtered softmax (sampler.py:48-61), for
    every policy.  (CPU generator here; the GPU tests run the CUDA one.)"""

    import torch

    from oracle.sampler import race_token

    rng = np.random.default_rng(5)
    vocab = 6000
    for trial in range(60):
        logits = (rng.standard_normal(vocab) * rng.uniform(0.5, 4.0)).astype(np.float32)
        temp, k, p = [(0.8, None, 1.0), (1.0, 40, 1.0), (1.3, None, 0.9), (0.7, 500, 0.95)][trial % 4]
        kept, _ = kept_and_probabilities(logits, temp, k, p)
        x = torch.from_numpy(logits) / temp
        probs = torch.softmax(x.masked_fill(~torch.from_numpy(kept), -torch.inf), dim=-1)
        seed = (2**62 + 977 * trial) % 2**63
        g = torch.Generator()
        g.manual_seed(seed)
        want = int(torch.multinomial(probs, num_samples=1, generator=g).item())
        g = torch.Generator()
        g.manual_seed(seed)
        q = torch.empty_like(probs).exponential_(1, generator=g).numpy()
        assert race_token(logits, temp, kept, q) == want, trial


# ---------------------------------------------------------------- metadata build
from _golden import BlockIds, PlanRequest, load_metadata_case, metadata_manifest  # noqa: E402
from oracle.metadata import PlannedRequest  # noqa: E402
from oracle.metadata import build as build_step  # noqa: E402
from oracle.metadata import pad as pad_step  # noqa: E402


def _planned(plan) -> list[PlannedRequest]:
    return [
        PlannedRequest(q.input_token_ids, q.num_computed_tokens, q.num_scheduled_tokens, q.requires_sampling,
                       tuple(t.block_ids for t in q.block_tables))
        for q in plan.scheduled_requests
    ]


@pytest.mark.parametrize("entry", metadata_manifest(), ids=lambda e: e["name"])
def test_metadata_oracle_matches_reference_golden(entry) -> None:
    """Every tensor of the reference's ModelRunner._build_model_input and of
    _CudaGraphExecution.copy_input (make_golden_metadata.py), bit-exact."""

    plan, z = load_metadata_case(entry)
    specs = [tuple(s) for s in entry["group_specs"]]
    batch = build_step(_planned(plan), entry["block_size"], entry["null_block_id"], specs)
    for key in ("input_ids", "positions", "query_start_locations", "context_lengths", "sampling_rows"):
        np.testing.assert_array_equal(batch[key], z[key], err_msg=key)
    for g, grp in enumerate(batch["groups"]):
        for key in ("block_table", "slot_mapping", "context_starts"):
            np.testing.assert_array_equal(grp[key], z[f"g{g}/{key}"], err_msg=f"g{g} {key}")
    padded = pad_step(batch, entry["token_capacity"], entry["request_capacity"], entry["table_widths"][0],
                      entry["null_block_id"])
    for key in ("input_ids", "positions", "query_start_locations", "context_lengths"):
        np.testing.assert_array_equal(padded[key], z["pad/" + key], err_msg="pad " + key)
    for g, grp in enumerate(padded["groups"]):
        for key in ("block_table", "slot_mapping", "context_starts"):
            np.testing.assert_array_equal(grp[key], z[f"g{g}/pad/{key}"], err_msg=f"pad g{g} {key}")


def _req(tokens, computed, sample, *tables):
    return PlannedRequest(tuple(tokens), computed, len(tokens), sample, tuple(tuple(t) for t in tables))


def test_metadata_oracle_reference_test_cases() -> None:
    """Known answers of the reference's runner tests (tests/worker/
    test_model_runner.py:213-520), restated on the oracle."""

    full = [("full", 0)]
    b = build_step([_req((10, 11, 12), 0, True, (0,))], 4, 7, full)  # :213-235
    assert b["positions"].tolist() == [0, 1, 2] and b["query_start_locations"].tolist() == [0, 3]
    assert b["context_lengths"].tolist() == [3] and b["sampling_rows"].tolist() == [2]
    b = build_step([_req((12, 13), 2, False, (0,))], 4, 7, full)  # :256-268
    assert b["positions"].tolist() == [2, 3] and b["sampling_rows"].tolist() == []
    b = build_step([_req((20,), 4, True, (0, 1)), _req((30, 31, 32), 0, False, (2,))], 4, 7, full)  # :271-293
    assert b["input_ids"].tolist() == [20, 30, 31, 32] and b["positions"].tolist() == [4, 0, 1, 2]
    assert b["query_start_locations"].tolist() == [0, 1, 4] and b["context_lengths"].tolist() == [5, 3]
    assert b["sampling_rows"].tolist() == [0]
    b = build_step([_req((10,), 3, True, (0,)), _req((20, 21), 5, True, (0, 1))], 4, 7, full)  # :296-313
    assert b["sampling_rows"].tolist() == [0, 2]
    b = build_step([_req((10,), 4, False, (2, 3, 4), (7, 7, 5))], 2, 7, [("full", 0), ("sliding", 3)])  # :316-380
    assert b["groups"][0]["context_starts"].tolist() == [0] and b["groups"][1]["context_starts"].tolist() == [2]
    assert b["groups"][0]["block_table"].tolist() == [[2, 3, 4]]
    assert b["groups"][1]["block_table"].tolist() == [[7, 7, 5]]
    assert b["groups"][0]["slot_mapping"].tolist() == [8] and b["groups"][1]["slot_mapping"].tolist() == [10]
    b = build_step([_req((10, 11), 3, False, (2, 5))], 4, 7, full)  # :383-402
    assert b["groups"][0]["slot_mapping"].tolist() == [11, 20]
    b = build_step([_req((10,), 4, False, (0, 3)), _req((20, 21), 1, False, (6,))], 4, 7, full)  # :405-430
    assert b["groups"][0]["slot_mapping"].tolist() == [12, 25, 26]
    b = build_step([_req((10,), 0, False, (2,)), _req((20,), 4, False, (3, 5, 6))], 4, 7, full)  # :455-485
    assert b["groups"][0]["block_table"].tolist() == [[2, 7, 7], [3, 5, 6]]
    b = build_step([], 4, 7, full)  # :508-518
    assert b["groups"][0]["block_table"].shape == (0, 0)
    with pytest.raises(IndexError):  # a position past the request's blocks
        build_step([_req((10,), 4, False, (2,))], 4, 7, full)


def test_metadata_spec_codes_and_builder_needs_cuda() -> None:
    from micro_vllm_b200 import ChunkedLocalSpec, DeviceMetadataBuilder, FullAttentionSpec, SlidingWindowSpec
    from micro_vllm_b200 import _lib
    from micro_vllm_b200.metadata import spec_code

    assert spec_code(FullAttentionSpec()) == (_lib.MVB_SPEC_FULL, 0)
    assert spec_code(SlidingWindowSpec(7)) == (_lib.MVB_SPEC_SLIDING_WINDOW, 7)
    assert spec_code(ChunkedLocalSpec(64)) == (_lib.MVB_SPEC_CHUNKED_LOCAL, 64)

    class Odd:
        def context_start(self, p):
            return p

    with pytest.raises(ValueError):
        spec_code(Odd())
    with pytest.raises(RuntimeError):
        DeviceMetadataBuilder([FullAttentionSpec()], 16, 0, "cpu")
    assert BlockIds((1,)).block_ids == (1,) and PlanRequest("a", (), 0, 0, False, ()).request_id == "a"
