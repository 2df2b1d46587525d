"""The batched device sampler (``mvb_sample``) against the reference's policy.

* greedy rows: bit-exact tokens (the first index of the largest logit) —
  against the reference Sampler's own output (golden) and the oracle;
* stochastic rows: every draw lies in the set the reference's top-k / top-p
  filters keep (golden), and the empirical distribution of many draws matches
  the oracle's probabilities (a chi-square bound at fixed seeds);
* a (seed, sample index) pair gives the same token whatever the other rows;
* rows with Exp(1) noise run torch.multinomial's exponential race: the
  oracle's token on every kernel path, and with the noise drawn from
  generators seeded as the reference seeds its own, the reference Sampler's
  token ids.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from _golden import SAMPLER_TIE_ROW, load_sampler_cases
from micro_vllm_b200.sampling import B200Sampler, sample_tokens
from oracle.sampler import greedy, kept_and_probabilities

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def _rows(n, temperature, top_k=0, top_p=1.0, seed=0, index=None):
    t = lambda v, dt: torch.full((n,), v, dtype=dt, device=DEV)  # noqa: E731
    idx = torch.arange(n, device=DEV) if index is None else index
    return t(temperature, torch.float32), t(top_k, torch.int32), t(top_p, torch.float32), t(seed, torch.int64), idx


def test_greedy_matches_reference_golden_and_oracle_in_every_dtype() -> None:
    z = load_sampler_cases()
    logits = torch.from_numpy(z["logits"]).to(DEV)
    n = logits.shape[0]
    got = sample_tokens(logits, *_rows(n, 0.0)).cpu().numpy()
    np.testing.assert_array_equal(got, z["greedy"])
    for dtype in (torch.float16, torch.bfloat16):
        low = logits.to(dtype)
        got = sample_tokens(low, *_rows(n, 0.0)).cpu().numpy()
        assert got.tolist() == [greedy(r) for r in low.float().cpu().numpy()]


@pytest.mark.parametrize("case", range(6))
def test_draws_stay_in_the_reference_kept_set(case: int) -> None:
    z = load_sampler_cases()
    logits = torch.from_numpy(z["logits"]).to(DEV)
    rows, draws = logits.shape[0], 256
    big = logits.repeat_interleave(draws, dim=0)
    index = torch.arange(rows * draws, device=DEV)
    temp, k, p = float(z["temperature"][case]), int(z["top_k"][case]), float(z["top_p"][case])
    got = sample_tokens(big, *_rows(rows * draws, temp, k, p, seed=123, index=index)).cpu().numpy()
    got = got.reshape(rows, draws)
    for r in range(rows):
        if r == SAMPLER_TIE_ROW:
            kept, _ = kept_and_probabilities(z["logits"][r], temp, k or None, p)
        else:
            kept = z["kept"][case, r]
        assert kept[got[r]].all(), (case, r)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_distribution_of_draws_matches_the_filtered_softmax(dtype) -> None:
    g = torch.Generator().manual_seed(3)
    vocab, draws = 40, 40000
    logits = (torch.randn(vocab, generator=g) * 1.5).to(dtype)
    row = logits.to(DEV).expand(draws, vocab)
    for temp, k, p in ((1.0, 0, 1.0), (0.8, 12, 1.0), (1.2, 0, 0.9), (1.0, 20, 0.7)):
        got = sample_tokens(row, *_rows(draws, temp, k, p, seed=99)).cpu().numpy()
        kept, probs = kept_and_probabilities(logits.float().numpy(), temp, k or None, p)
        assert kept[got].all()
        counts = np.bincount(got, minlength=vocab)[kept]
        expected = probs[kept] * draws
        chi2 = float(((counts - expected) ** 2 / expected).sum())
        dof = int(kept.sum()) - 1
        assert chi2 < dof + 6 * np.sqrt(2 * dof) + 10, (temp, k, p, chi2, dof)


def test_seed_and_index_fix_the_token_whatever_the_other_rows() -> None:
    logits = torch.zeros((3, 64), device=DEV)
    t = torch.tensor([0.0, 1.0, 1.0], device=DEV)
    k = torch.zeros(3, dtype=torch.int32, device=DEV)
    p = torch.ones(3, device=DEV)
    seed = torch.tensor([0, 11, 11], dtype=torch.int64, device=DEV)
    index = torch.tensor([0, 4, 4], dtype=torch.int64, device=DEV)
    mixed = sample_tokens(logits, t, k, p, seed, index).cpu()
    alone = sample_tokens(logits[1:2], t[1:2], k[1:2], p[1:2], seed[1:2], index[1:2]).cpu()
    assert mixed[1] == mixed[2] == alone[0]
    seqs = []
    for s in (11, 29):
        idx = torch.arange(16, device=DEV)
        seqs.append(sample_tokens(torch.zeros((16, 64), device=DEV), *_rows(16, 1.0, seed=s, index=idx)).cpu())
    assert not torch.equal(seqs[0], seqs[1])


def test_sampler_interface_mirrors_the_reference() -> None:
    """B200Sampler(logits, request_ids, sampling_params, sample_indices) with
    the reference tests' cases (tests/sampling/test_sampler.py)."""

    class Params:  # the reference SamplingParams' fields the sampler reads
        def __init__(self, temperature=0.0, top_k=None, top_p=1.0, seed=None):
            self.temperature, self.top_k, self.top_p, self.seed = temperature, top_k, top_p, seed

    from micro_vllm_b200.sampling import _output_types

    # The reference's own ModelRunnerOutput when micro_vllm is loaded in this
    # process (its scheduler consumes it), else this package's mirror.
    output_type, token_type = _output_types()
    s = B200Sampler()
    logits = torch.tensor([[0.0, 1.0, 3.0], [4.0, 2.0, 1.0], [0.0, 5.0, 1.0]], device=DEV)
    out = s(logits, ("third", "first", "second"), (Params(),) * 3, (0, 0, 0))
    assert out == output_type((token_type("third", 2), token_type("first", 0), token_type("second", 1)))
    assert s(torch.empty((0, 4), device=DEV), (), (), ()) == output_type()
    tie = torch.tensor([[1.0, 3.0, 3.0, 2.0]], device=DEV)
    assert s(tie, ("r",), (Params(),), (0,)).sampled_tokens[0].token_id == 1
    topk = torch.tensor([[0.0, 1.0, 2.0, 3.0, 4.0]], device=DEV)
    got = {s(topk, ("r",), (Params(1.0, 2, 1.0, 0),), (i,)).sampled_tokens[0].token_id for i in range(32)}
    assert got and got <= {3, 4}
    topp = torch.tensor([[3.0, 2.0, 0.0, -1.0]], device=DEV)
    got = {s(topp, ("r",), (Params(1.0, None, 0.8, 0),), (i,)).sampled_tokens[0].token_id for i in range(32)}
    assert got and got <= {0, 1}
    few = torch.tensor([[0.0, 1.0, 2.0]], device=DEV)
    a = s(few, ("r",), (Params(1.0, None, 1.0, 9),), (0,))
    b = s(few, ("r",), (Params(1.0, 3, 1.0, 9),), (0,))
    assert a == b


def test_vocab_scale_batch() -> None:
    """256 rows of a 151936-token vocabulary (Qwen3): greedy exact, top-k/top-p
    draws inside their kept sets."""

    g = torch.Generator(device=DEV).manual_seed(1)
    rows, vocab = 256, 151936
    logits = torch.randn((rows, vocab), generator=g, device=DEV).half()
    temp = torch.where(torch.arange(rows, device=DEV) % 2 == 0, 0.0, 0.9).float()
    k = torch.where(torch.arange(rows, device=DEV) % 4 == 1, 40, 0).int()
    p = torch.where(torch.arange(rows, device=DEV) % 4 == 3, 0.92, 1.0).float()
    seed = torch.arange(rows, device=DEV) * 7
    idx = torch.arange(rows, device=DEV)
    got = sample_tokens(logits, temp, k, p, seed, idx).cpu().numpy()
    host = logits.float().cpu().numpy()
    for r in range(rows):
        if r % 2 == 0:
            assert got[r] == greedy(host[r])
        else:
            kept, _ = kept_and_probabilities(host[r], 0.9, int(k[r]) or None, float(p[r]))
            assert kept[got[r]]


@pytest.mark.parametrize("case", ["large_k", "flat_top_p", "k_and_p_large"])
def test_multi_pass_paths_keep_the_reference_set(case) -> None:
    """Cuts whose boundary holds more than the 2048 tokens sorted in shared
    memory: the digit-refinement passes and the draw over the whole row."""

    g = torch.Generator(device=DEV).manual_seed(21)
    vocab, rows = 50000, 64
    scale = 0.05 if case != "large_k" else 1.0  # nearly flat: the top-p boundary bin is crowded
    logits = (torch.randn((1, vocab), generator=g, device=DEV) * scale).expand(rows, vocab)
    k, p = {"large_k": (3000, 1.0), "flat_top_p": (0, 0.5), "k_and_p_large": (20000, 0.7)}[case]
    got = sample_tokens(logits, *_rows(rows, 1.0, k, p, seed=5)).cpu().numpy()
    kept, _ = kept_and_probabilities(logits[0].float().cpu().numpy(), 1.0, k or None, p)
    assert kept[got].all()
    again = sample_tokens(logits, *_rows(rows, 1.0, k, p, seed=5)).cpu().numpy()
    assert (got == again).all()
    assert len(set(got.tolist())) > 8  # the draws spread over the kept set


def test_exact_ties_beyond_the_shared_memory_set() -> None:
    """10000 equal logits: top-k 100 keeps the first 100 indices; top-p 0.5
    keeps indices 0..5000 (mass before each <= 0.5); ties in index order."""

    rows, vocab = 128, 10000
    logits = torch.zeros((rows, vocab), device=DEV)
    got = sample_tokens(logits, *_rows(rows, 1.0, 100, 1.0, seed=3)).cpu().numpy()
    assert got.max() < 100 and len(set(got.tolist())) > 20
    got = sample_tokens(logits, *_rows(rows, 1.0, 0, 0.5, seed=3)).cpu().numpy()
    assert got.max() <= 5000 and got.max() > 1000
    got = sample_tokens(logits, *_rows(rows, 1.0, 3000, 0.1, seed=3)).cpu().numpy()
    assert got.max() <= 300  # top-k 3000, then 10 % of its mass: indices 0..300


def _cuda_noise(seeds_and_indices, vocab):
    """Exp(1) rows as the reference's torch.multinomial draws them: one
    generator on the logits' device per row, seeded (seed + index) mod 2^63."""

    noise = torch.empty((len(seeds_and_indices), vocab), dtype=torch.float32, device=DEV)
    for r, (seed, index) in enumerate(seeds_and_indices):
        g = torch.Generator(device=DEV)
        g.manual_seed((seed + index) % 2**63)
        noise[r].exponential_(1.0, generator=g)
    return noise


@pytest.mark.parametrize(
    "policy",
    ["temperature", "top_k_small", "top_p", "k_and_p", "large_k", "flat_top_p", "k_and_p_large"],
)
def test_noise_rows_run_the_exponential_race_of_the_oracle(policy) -> None:
    """mvb_sample_with_noise: a row with noise returns oracle.race_token over
    the reference's kept set, on every path of the kernel (the shared-memory
    candidate sets and the whole-row passes); rows without noise still draw
    from their kept set."""

    from oracle.sampler import race_token

    temp, k, p, scale, vocab = {
        "temperature": (0.8, 0, 1.0, 3.0, 151936),
        "top_k_small": (1.0, 50, 1.0, 3.0, 151936),
        "top_p": (1.1, 0, 0.9, 3.0, 151936),
        "k_and_p": (0.9, 40, 0.9, 3.0, 151936),
        "large_k": (1.0, 3000, 1.0, 1.0, 50000),
        "flat_top_p": (1.0, 0, 0.5, 0.05, 50000),
        "k_and_p_large": (1.0, 20000, 0.7, 0.05, 50000),
    }[policy]
    rows = 12
    g = torch.Generator(device=DEV).manual_seed(41)
    logits = (torch.randn((rows, vocab), generator=g, device=DEV) * scale).to(torch.bfloat16)
    pairs = [(1000 + 7 * r, 3 * r) for r in range(rows)]
    noise = _cuda_noise(pairs[: rows // 2 * 2 : 2], vocab)  # even rows only
    noise_row = torch.tensor([r // 2 if r % 2 == 0 else -1 for r in range(rows)], dtype=torch.int32, device=DEV)
    args = _rows(rows, temp, k, p, seed=5)
    got = sample_tokens(logits, *args, noise=noise, noise_row=noise_row).cpu().numpy()
    host, q = logits.float().cpu().numpy(), noise.cpu().numpy()
    for r in range(rows):
        kept, _ = kept_and_probabilities(host[r], temp, k or None, p)
        assert kept[got[r]], (policy, r)
        if r % 2 == 0:
            assert got[r] == race_token(host[r], temp, kept, q[r // 2]), (policy, r)
    with pytest.raises(ValueError):
        sample_tokens(logits, *args, noise=noise, noise_row=None)


def test_seeded_rows_give_the_reference_sampler_tokens() -> None:
    """The reference's own Sampler (torch.multinomial with its seeded CUDA
    generator) and B200Sampler on the same Qwen3-vocabulary logits: every
    greedy and every seeded stochastic row gets the same token id.  fp32
    logits: with bf16's 256 values per octave, equal logits at a top-k
    boundary are common, and torch.topk keeps an unspecified one of them."""

    from _reference import require_reference

    require_reference()
    from micro_vllm.sampling.params import SamplingParams
    from micro_vllm.sampling.sampler import Sampler

    rows, vocab = 40, 151936
    g = torch.Generator(device=DEV).manual_seed(8)
    logits = torch.randn((rows, vocab), generator=g, device=DEV) * 2.5
    policies = [(0.0, None, 1.0), (0.7, None, 1.0), (1.0, 50, 1.0), (1.2, None, 0.9), (0.9, 40, 0.8)]
    params = tuple(
        SamplingParams(max_tokens=8, temperature=t, top_k=k, top_p=p, seed=None if t == 0.0 else 31 * r + 2**40)
        for r, (t, k, p) in ((r, policies[r % len(policies)]) for r in range(rows))
    )
    ids = tuple(f"req{r}" for r in range(rows))
    indices = tuple(5 * r + 1 for r in range(rows))
    want = [t.token_id for t in Sampler()(logits, ids, params, indices).sampled_tokens]
    got = [t.token_id for t in B200Sampler()(logits, ids, params, indices).sampled_tokens]
    assert got == want
    # Without the reference's streams the tokens are the kernel's own draws.
    own = [t.token_id for t in B200Sampler(reference_streams=False)(logits, ids, params, indices).sampled_tokens]
    assert own != want
