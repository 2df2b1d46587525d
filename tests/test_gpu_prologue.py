"""Parity of the fused Qwen3 attention prologue (``mvb_qk_norm_rope_and_cache``).

Against the reference's own RMSNorm / RotaryEmbedding / write_kv_cache
(golden vectors from tests/golden/make_golden_prologue.py) and against the
oracle (oracle/qk_prologue.py) on larger seeded batches.  Tolerances:
  * the rotated query and key: within two ulps of the model dtype at the
    magnitude of the larger of the element and its rotation partner (the
    variance is summed in another order, sin/cos may differ by an ulp, and a
    one-ulp change of the normalised value passes through the weight multiply
    and the rotation, whose sum can cancel); all but a few per mille exactly
    equal;
  * the value rows and every cache byte the write does not touch: bit-exact.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from _golden import PROLOGUE_CASES, from_bits, load_prologue_case, within_ulps
from micro_vllm_b200 import (
    AttentionMetadata,
    B200PagedAttentionOperator,
    Qwen3AttentionPrologue,
    qk_norm_rope_and_write,
    rotary_inverse_frequencies,
)
from micro_vllm_b200 import _lib
from oracle import build_metadata, paged_attention
from oracle.qk_prologue import qk_norm_rope_and_cache

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
TORCH_DTYPE = {"f16": torch.float16, "bf16": torch.bfloat16}


def _dev_bits(bits: np.ndarray, dt: str) -> torch.Tensor:
    """Raw 16-bit patterns as a device tensor of the model dtype."""

    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(TORCH_DTYPE[dt]).to(DEV)


def _metadata(slots: torch.Tensor, block_size: int) -> AttentionMetadata:
    n = slots.numel()
    return AttentionMetadata(
        query_positions=torch.zeros(n, dtype=torch.int64, device=DEV),
        query_context_start_positions=torch.zeros(n, dtype=torch.int64, device=DEV),
        query_start_locations=torch.tensor([0, n], device=DEV),
        context_lengths=torch.tensor([1], device=DEV),
        block_table=torch.zeros((1, 1), dtype=torch.int64, device=DEV),
        slot_mapping=slots, block_size=block_size,
    )


@pytest.mark.parametrize("name", PROLOGUE_CASES)
def test_prologue_matches_reference_golden(name: str) -> None:
    z = load_prologue_case(name)
    dt = str(z["dtype"])
    q, k, v = (_dev_bits(z[n], dt) for n in ("query", "key", "value"))
    cache = _dev_bits(z["cache_before"], dt)
    slots = torch.from_numpy(z["slot_mapping"]).to(DEV)
    q_out = qk_norm_rope_and_write(
        q, k, v, torch.from_numpy(z["positions"]).to(DEV), _dev_bits(z["q_weight"], dt),
        _dev_bits(z["k_weight"], dt), float(z["eps"]), torch.from_numpy(z["inv_freq"]).to(DEV),
        cache, _metadata(slots, int(z["block_size"])),
    )
    torch.cuda.synchronize()
    got_q = q_out.float().cpu().numpy()
    got_cache = cache.float().cpu().numpy()
    exp_q, exp_cache = from_bits(z["q_out"], dt), from_bits(z["cache_after"], dt)
    assert within_ulps(got_q, exp_q, dt, 2, rotated=True).all()
    assert np.mean(got_q != exp_q) < 5e-3
    # Keys within two ulps; values and untouched slots bit-exact.
    assert within_ulps(got_cache[0], exp_cache[0], dt, 2, rotated=True).all()
    np.testing.assert_array_equal(got_cache[1], exp_cache[1])


def _random_case(dtype: torch.dtype, tokens: int, hq: int, hkv: int, seed: int, lead: int = 0):
    g = torch.Generator().manual_seed(seed)
    d, bs, nb = 128, 16, 64
    # q, k, v as views of one fused projection output (strided rows); `lead`
    # extra elements in front of each row leave rows only 8-byte aligned.
    fused = (torch.randn((tokens, lead + (hq + 2 * hkv) * d), generator=g) * 2.0).to(dtype).to(DEV)
    q = fused[:, lead : lead + hq * d].unflatten(1, (hq, d))
    k = fused[:, lead + hq * d : lead + (hq + hkv) * d].unflatten(1, (hkv, d))
    v = fused[:, lead + (hq + hkv) * d :].unflatten(1, (hkv, d))
    positions = torch.randint(0, 100_000, (tokens,), generator=g).to(DEV)
    slots = torch.randperm(nb * bs, generator=g)[:tokens].to(DEV)
    slots[5] = -1
    q_w = (0.5 + torch.rand(d, generator=g)).to(dtype).to(DEV)
    k_w = (0.5 + torch.rand(d, generator=g)).to(dtype).to(DEV)
    cache = torch.randn((2, nb, bs, hkv, d), generator=g).to(dtype).to(DEV)
    return q, k, v, positions, slots, q_w, k_w, cache, bs


def _oracle(q, k, v, positions, slots, q_w, k_w, eps, inv_freq, cache, dt):
    np_cache = cache.float().cpu().numpy()
    out = qk_norm_rope_and_cache(
        q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy(),
        positions.cpu().numpy(), q_w.float().cpu().numpy(), k_w.float().cpu().numpy(), eps,
        inv_freq.cpu().numpy(), np_cache, slots.cpu().numpy(), dt,
    )
    return out, np_cache


@pytest.mark.parametrize("dt", ["f16", "bf16"])
@pytest.mark.parametrize("hq,hkv,lead", [(16, 8, 0), (32, 8, 0), (8, 8, 0), (14, 2, 0), (15, 3, 0),
                                         (16, 8, 4), (15, 3, 4)])
def test_prologue_matches_oracle_on_strided_views(dt: str, hq: int, hkv: int, lead: int) -> None:
    """lead 0: 16-byte rows (two rows per warp instruction; 15/3 puts a query
    and a key row, then a key and a value row, in one instruction); lead 4:
    8-byte rows (one row per warp instruction)."""

    q, k, v, positions, slots, q_w, k_w, cache, bs = _random_case(TORCH_DTYPE[dt], 300, hq, hkv, hq + hkv, lead)
    inv = rotary_inverse_frequencies(128, 1e6, DEV)
    exp_q, exp_cache = _oracle(q, k, v, positions, slots, q_w, k_w, 1e-6, inv, cache, dt)
    q_out = qk_norm_rope_and_write(q, k, v, positions, q_w, k_w, 1e-6, inv, cache, _metadata(slots, bs))
    torch.cuda.synchronize()
    got_q, got_cache = q_out.float().cpu().numpy(), cache.float().cpu().numpy()
    assert within_ulps(got_q, exp_q, dt, 2, rotated=True).all()
    assert np.mean(got_q != exp_q) < 5e-3
    assert within_ulps(got_cache[0], exp_cache[0], dt, 2, rotated=True).all()
    np.testing.assert_array_equal(got_cache[1], exp_cache[1])


def test_prologue_then_attend_matches_the_reference_order() -> None:
    """Prologue + attention over the written cache equals the oracle doing
    norm, rope, write and attention (qwen.py:89-98 order) within the
    attention tolerance."""

    dtype, dt = torch.float16, "f16"
    ctx = [40, 130, 7]
    tables = [[0, 1, 2], [3, 4, 5, 6, 7, 8, 9, 10, 11], [12]]
    nb, bs, hq, hkv, d = 16, 16, 16, 8, 128
    g = torch.Generator().manual_seed(11)
    positions_l = [list(range(c)) for c in ctx]
    md_np = build_metadata(positions_l, tables, block_size=bs)
    tokens = int(md_np.query_start_locations[-1])
    q = (torch.randn((tokens, hq, d), generator=g) * 2).to(dtype).to(DEV)
    k = (torch.randn((tokens, hkv, d), generator=g) * 2).to(dtype).to(DEV)
    v = torch.randn((tokens, hkv, d), generator=g).to(dtype).to(DEV)
    q_w = (0.5 + torch.rand(d, generator=g)).to(dtype).to(DEV)
    k_w = (0.5 + torch.rand(d, generator=g)).to(dtype).to(DEV)
    cache = torch.zeros((2, nb, bs, hkv, d), dtype=dtype, device=DEV)
    md = AttentionMetadata(
        query_positions=torch.from_numpy(md_np.query_positions).to(DEV),
        query_context_start_positions=torch.from_numpy(md_np.query_context_start_positions).to(DEV),
        query_start_locations=torch.from_numpy(md_np.query_start_locations).to(DEV),
        context_lengths=torch.from_numpy(md_np.context_lengths).to(DEV),
        block_table=torch.from_numpy(md_np.block_table).to(DEV),
        slot_mapping=torch.from_numpy(md_np.slot_mapping).to(DEV), block_size=bs,
    )
    prologue = Qwen3AttentionPrologue(q_w, k_w, 1e-6, 1e6)
    op = B200PagedAttentionOperator()
    out = op.attend(prologue(md.query_positions, q, k, v, cache, md), cache, md)
    torch.cuda.synchronize()
    inv = rotary_inverse_frequencies(d, 1e6, DEV)
    oq, ocache = _oracle(q, k, v, md.query_positions, md.slot_mapping, q_w, k_w, 1e-6, inv,
                         torch.zeros_like(cache), dt)
    # The oracle's attention reads the keys the oracle prologue wrote.
    np_k = ocache[0].reshape(-1, hkv, d)[md_np.slot_mapping]
    np_v = ocache[1].reshape(-1, hkv, d)[md_np.slot_mapping]
    expected = paged_attention(oq, np_k, np_v, np.zeros_like(ocache), md_np)
    np.testing.assert_allclose(out.float().cpu().numpy(), expected, atol=2e-3, rtol=1e-2)


def test_prologue_reports_slots_past_the_pool_and_rejects_bad_inputs() -> None:
    q, k, v, positions, slots, q_w, k_w, cache, bs = _random_case(torch.float16, 20, 16, 8, 3)
    slots[7] = cache.shape[1] * bs + 5  # past the pool: skipped, status bit
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    inv = rotary_inverse_frequencies(128, 1e6, DEV)
    qk_norm_rope_and_write(q, k, v, positions, q_w, k_w, 1e-6, inv, cache, _metadata(slots, bs), status=status)
    torch.cuda.synchronize()
    assert int(status.item()) & _lib.MVB_STATUS_SLOT_OUT_OF_RANGE
    with pytest.raises(ValueError):
        qk_norm_rope_and_write(q.float(), k.float(), v.float(), positions, q_w.float(), k_w.float(),
                               1e-6, inv, cache.float(), _metadata(slots, bs))
    with pytest.raises(ValueError):  # head_dim 64 is not supported by the fused kernel
        qk_norm_rope_and_write(q[..., :64], k[..., :64], v[..., :64], positions, q_w[:64], k_w[:64],
                               1e-6, inv[:32], cache[..., :64].contiguous(), _metadata(slots, bs))
    with pytest.raises(RuntimeError):
        qk_norm_rope_and_write(q.cpu(), k.cpu(), v.cpu(), positions.cpu(), q_w.cpu(), k_w.cpu(),
                               1e-6, inv.cpu(), cache.cpu(), _metadata(slots, bs))


def test_prologue_large_batch_positions_and_writes() -> None:
    """8192 tokens (max_num_batched_tokens of BASELINE config 5) at the
    Qwen3 shape: spot-check rows against the oracle."""

    q, k, v, positions, slots, q_w, k_w, cache, bs = _random_case(torch.bfloat16, 1000, 16, 8, 21)
    big = 8192
    reps = math.ceil(big / 1000)
    q, k, v = (t.repeat(reps, 1, 1)[:big].contiguous() for t in (q, k, v))
    positions = positions.repeat(reps)[:big]
    cache = torch.zeros((2, 600, bs, 8, 128), dtype=torch.bfloat16, device=DEV)
    slots = torch.randperm(600 * bs, device=DEV)[:big]
    inv = rotary_inverse_frequencies(128, 1e6, DEV)
    q_out = qk_norm_rope_and_write(q, k, v, positions, q_w, k_w, 1e-6, inv, cache, _metadata(slots, bs))
    torch.cuda.synchronize()
    rows = torch.tensor([0, 1, 999, 4095, 8191], device=DEV)
    exp_q, exp_cache = _oracle(q[rows], k[rows], v[rows], positions[rows], torch.arange(5, device=DEV),
                               q_w, k_w, 1e-6, inv, torch.zeros((2, 1, 5, 8, 128), dtype=torch.bfloat16), "bf16")
    assert within_ulps(q_out[rows].float().cpu().numpy(), exp_q, "bf16", 2, rotated=True).all()
    flat = cache.view(2, -1, 8, 128)
    got_k = flat[0, slots[rows]].float().cpu().numpy()
    assert within_ulps(got_k, exp_cache[0].reshape(5, 8, 128), "bf16", 2, rotated=True).all()
    assert torch.equal(flat[1, slots[rows]], v[rows])
