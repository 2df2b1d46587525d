"""Batched device sampler (``mvb_sample``): the next token of every row at once.

The reference samples row by row (src/micro_vllm/sampling/sampler.py:14-61),
each row ending in ``.item()`` — one host synchronisation per request per
step.  ``B200Sampler`` keeps the same call signature and per-row policy
(greedy argmax; temperature, top-k, top-p, seeded multinomial) and runs all
rows in one kernel; the host reads the token ids once.  ``sample_tokens``
returns them on the device without any synchronisation.

Random draws.  A row whose request carries a seed takes the reference's
own stream: ``torch.multinomial(probabilities, 1, generator)`` is the
exponential race argmax(probabilities / q) with q = Exp(1) noise from the
generator, so ``B200Sampler`` draws q with a ``torch.Generator`` seeded as
the reference seeds it ((seed + sample index) mod 2^63, on the logits'
device) and the kernel runs the race over the row's kept set
(``mvb_sample_with_noise``): the reference's token, unless the two best
ratios agree to within fp32 rounding.  A row without a seed (the reference
draws a random one) takes the kernel's own Philox4x32-10 stream keyed by a
random seed, with no per-row noise to generate.
"""

from __future__ import annotations

import secrets
import sys
from dataclasses import dataclass

import torch

from micro_vllm_b200 import _lib
from micro_vllm_b200.operators import _DTYPES


@dataclass(frozen=True, slots=True)
class SampledToken:
    """Mirror of the reference's SampledToken (executor/interface.py)."""

    request_id: str
    token_id: int


@dataclass(frozen=True, slots=True)
class SamplerOutput:
    """Mirror of the reference's ModelRunnerOutput (executor/interface.py)."""

    sampled_tokens: tuple[SampledToken, ...] = ()


def sample_tokens(
    logits: torch.Tensor,
    temperature: torch.Tensor,
    top_k: torch.Tensor,
    top_p: torch.Tensor,
    seed: torch.Tensor,
    sample_index: torch.Tensor,
    out: torch.Tensor | None = None,
    noise: torch.Tensor | None = None,
    noise_row: torch.Tensor | None = None,
) -> torch.Tensor:
    """Token ids (device int64 [rows]) for ``logits`` [rows, vocab].

    Per-row device tensors: ``temperature`` float32 (0: greedy), ``top_k``
    int32 (<= 0: none), ``top_p`` float32 (1: none), ``seed`` int64 (used as
    an unsigned 64-bit key) and ``sample_index`` int64.  With ``noise``
    (float32 [n, vocab], Exp(1) values) and ``noise_row`` (int32 [rows]), a
    stochastic row r with 0 <= noise_row[r] < n takes the exponential race
    against noise[noise_row[r]] instead of the Philox draw."""

    if logits.device.type != "cuda":
        raise RuntimeError("b200_paged sampler requires CUDA tensors")
    dtype = _DTYPES.get(logits.dtype)
    if dtype is None:
        raise ValueError("b200_paged sampler supports float16, bfloat16 and float32 logits")
    if logits.dim() != 2:
        raise ValueError("logits must be [rows, vocab]")
    if logits.stride(1) != 1:
        logits = logits.contiguous()
    rows, vocab = logits.shape
    dev = logits.device
    expect = ((temperature, torch.float32), (top_k, torch.int32), (top_p, torch.float32),
              (seed, torch.int64), (sample_index, torch.int64))
    for t, dt in expect:
        if t.dtype != dt or t.shape != (rows,) or t.device != dev:
            raise ValueError(f"per-row sampling tensors must be {dt} [{rows}] on {dev}")
    if noise is not None:
        if (noise.dtype != torch.float32 or noise.dim() != 2 or noise.shape[1] != vocab
                or noise.stride(1) != 1 or noise.device != dev):
            raise ValueError(f"noise must be float32 [n, {vocab}] rows on {dev}")
        if noise_row is None or noise_row.dtype != torch.int32 or noise_row.shape != (rows,) \
                or noise_row.device != dev:
            raise ValueError(f"noise_row must be int32 [{rows}] on {dev}")
    if out is None:
        out = torch.empty(rows, dtype=torch.int64, device=dev)
    if rows == 0:
        return out
    lib = _lib.load()
    rc = lib.mvb_sample_with_noise(
        logits.data_ptr(), logits.stride(0), rows, vocab, dtype,
        temperature.contiguous().data_ptr(), top_k.contiguous().data_ptr(),
        top_p.contiguous().data_ptr(), seed.contiguous().data_ptr(),
        sample_index.contiguous().data_ptr(),
        None if noise is None else noise.data_ptr(), vocab if noise is None else noise.stride(0),
        0 if noise is None else noise.shape[0],
        None if noise is None else noise_row.contiguous().data_ptr(), out.data_ptr(),
        torch.cuda.current_stream(dev).cuda_stream,
    )
    _lib.check(rc, "b200_paged sampler")
    return out


class B200Sampler:
    """``Sampler.__call__(logits, request_ids, sampling_params, sample_indices)``
    (sampler.py:14-37) with every row sampled in one launch.  Accepts the
    reference's SamplingParams (or anything with ``temperature``, ``top_k``,
    ``top_p`` and ``seed``); a row without a seed gets a random one, as the
    reference draws ``secrets.randbits(63)`` (sampler.py:51-53).

    ``reference_streams`` (default on): a seeded stochastic row draws its
    Exp(1) noise from a ``torch.Generator`` on the logits' device seeded with
    (seed + sample index) mod 2^63, as the reference's generator
    (sampler.py:52-61), so it gets the reference's token; one generator and
    one noise launch per such row.  Off: every row takes the kernel's Philox
    draw (the same distribution, another stream, no per-row launches)."""

    __slots__ = ("reference_streams",)

    def __init__(self, reference_streams: bool = True) -> None:
        self.reference_streams = bool(reference_streams)

    def __call__(self, logits, request_ids, sampling_params, sample_indices, /) -> SamplerOutput:
        rows = len(request_ids)
        if rows == 0:
            return _output_types()[0]()
        dev = logits.device
        temperature = torch.tensor([float(p.temperature) for p in sampling_params], dtype=torch.float32)
        top_k = torch.tensor([0 if p.top_k is None else int(p.top_k) for p in sampling_params],
                             dtype=torch.int32)
        top_p = torch.tensor([float(p.top_p) for p in sampling_params], dtype=torch.float32)
        seed = torch.tensor(
            [(p.seed if p.seed is not None else secrets.randbits(63)) for p in sampling_params],
            dtype=torch.int64,
        )
        index = torch.tensor([int(i) for i in sample_indices], dtype=torch.int64)
        packed = [t.to(dev, non_blocking=True) for t in (temperature, top_k, top_p, seed, index)]
        noise, noise_row = self._reference_noise(logits, sampling_params, sample_indices)
        tokens = sample_tokens(logits, *packed, noise=noise, noise_row=noise_row).cpu()  # the one host read
        output_type, token_type = _output_types()
        return output_type(tuple(token_type(r, int(t)) for r, t in zip(request_ids, tokens.tolist())))


    def _reference_noise(self, logits, sampling_params, sample_indices):
        """(noise [n, vocab], noise_row [rows]) for the seeded stochastic rows,
        or (None, None): each noise row is what ``torch.empty_like(p)
        .exponential_(1, generator)`` gives inside the reference's
        ``torch.multinomial`` for that row's generator."""

        if not self.reference_streams:
            return None, None
        seeded = [j for j, p in enumerate(sampling_params) if p.seed is not None and float(p.temperature) > 0.0]
        if not seeded:
            return None, None
        dev = logits.device
        noise = torch.empty((len(seeded), logits.shape[-1]), dtype=torch.float32, device=dev)
        row_of = [-1] * len(sampling_params)
        for n, j in enumerate(seeded):
            generator = torch.Generator(device=dev)
            generator.manual_seed((int(sampling_params[j].seed) + int(sample_indices[j])) % (2**63))
            noise[n].exponential_(1.0, generator=generator)
            row_of[j] = n
        return noise, torch.tensor(row_of, dtype=torch.int32).to(dev, non_blocking=True)


def _output_types() -> tuple[type, type]:
    """The reference's ``ModelRunnerOutput`` / ``SampledToken``
    (executor/interface.py:9-24) when micro_vllm is loaded in this process
    (its scheduler reads them), else this module's mirrors.  micro_vllm is
    not imported here: importing it loads transformers."""

    interface = sys.modules.get("micro_vllm.executor.interface")
    if interface is not None:
        return interface.ModelRunnerOutput, interface.SampledToken
    return SamplerOutput, SampledToken
