"""CPU oracle of the reference sampler's row policy — TEST INFRASTRUCTURE ONLY.

numpy restatement of ``Sampler._sample_row`` and its filters
(src/micro_vllm/sampling/sampler.py:39-87) for checking the device sampler
``mvb_sample``: the greedy token, the set of tokens top-k / top-p keep and
the probabilities of the multinomial draw over that set.  Only ``tests/``
import it.  Pinned by ``tests/golden/make_golden_sampler.py``, which ran the
reference's own ``Sampler`` (greedy rows) and ``_apply_top_k`` /
``_apply_top_p`` on seeded logits.

Ties: torch.topk and torch.sort leave the order of equal values open; this
restatement (and the kernel) keeps the lowest indices first.
"""

from __future__ import annotations

import numpy as np


def greedy(logits: np.ndarray) -> int:
    """``logits.argmax()`` — the first index of the largest value (sampler.py:45-46)."""

    return int(np.argmax(np.asarray(logits, np.float32)))


def kept_and_probabilities(
    logits: np.ndarray, temperature: float, top_k: int | None, top_p: float
) -> tuple[np.ndarray, np.ndarray]:
    """(kept mask, probabilities) of a stochastic row (sampler.py:48-51, 64-87)."""

    x = np.asarray(logits, np.float32) / np.float32(temperature)
    v = x.shape[-1]
    order = np.lexsort((np.arange(v), -x.astype(np.float64)))  # descending value, then index
    kept = np.ones(v, bool)
    if top_k is not None and top_k < v:  # _apply_top_k (sampler.py:64-69)
        kept[:] = False
        kept[order[:top_k]] = True
    if top_p != 1.0:  # _apply_top_p (sampler.py:72-80)
        m = x[kept].max()
        p = np.where(kept, np.exp((x - m).astype(np.float64)), 0.0)
        p /= p.sum()
        sp = p[order]
        before = np.cumsum(sp) - sp
        remove = before > top_p
        kept[order[remove]] = False
    m = x[kept].max()
    probs = np.where(kept, np.exp((x - m).astype(np.float64)), 0.0)
    return kept, probs / probs.sum()


def race_token(logits: np.ndarray, temperature: float, kept: np.ndarray, q: np.ndarray) -> int:
    """The token ``torch.multinomial(probabilities, 1, generator)`` returns
    (sampler.py:55-61), restated as the exponential race torch runs for one
    sample: argmax(probabilities / q), q = ``empty_like(probabilities)
    .exponential_(1, generator)``, the first index among equal ratios.
    probabilities = exp(x - max x) over the kept set with x = logit / T in
    fp32; the softmax denominator is common to every token and is left out
    (the winner changes only where the two best ratios agree to within
    fp32 rounding)."""

    x = np.asarray(logits, np.float32) / np.float32(temperature)
    m = x[kept].max()
    e = np.where(kept, np.exp((x - m).astype(np.float32)), np.float32(0.0)).astype(np.float32)
    return int(np.argmax(e / np.asarray(q, np.float32)))
