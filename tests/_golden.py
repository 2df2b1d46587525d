"""Loading helpers for the golden vectors in tests/golden/.

The vectors were produced by ``tests/golden/make_golden.py`` from the
reference's own ``ReferenceAttentionOperator``; see that script.
"""

from __future__ import annotations

import hashlib
import json
from pathlib import Path

import numpy as np

GOLDEN_DIR = Path(__file__).resolve().parent / "golden"


def cache_digest(cache: np.ndarray) -> str:
    """SHA-256 of a cache's fp32 bytes with NaNs canonicalised."""

    c = np.ascontiguousarray(cache, dtype=np.float32).copy()
    c[np.isnan(c)] = np.float32("nan")
    return hashlib.sha256(c.tobytes()).hexdigest()


def case_names() -> list[str]:
    manifest = json.loads((GOLDEN_DIR / "manifest.json").read_text())
    return [entry["name"] for entry in manifest]


def load_case(name: str) -> dict:
    """Return one case as a dict of numpy arrays (inputs widened to fp32)."""

    with np.load(GOLDEN_DIR / f"{name}.npz") as data:
        case = {k: data[k] for k in data.files}
    case["block_size"] = int(case["block_size"])
    case["expected_cache_sha256"] = str(case["expected_cache_sha256"])
    return case


def oracle_metadata(case: dict):
    from oracle import OracleMetadata

    return OracleMetadata(
        query_positions=case["query_positions"],
        query_context_start_positions=case["query_context_start_positions"],
        query_start_locations=case["query_start_locations"],
        context_lengths=case["context_lengths"],
        block_table=case["block_table"],
        slot_mapping=case["slot_mapping"],
        block_size=case["block_size"],
    )


# ---------------------------------------------------------------- prologue
PROLOGUE_CASES = ("qwen3_f16", "qwen3_bf16", "gqa4_long_f16")


def from_bits(bits, dtype: str):
    """Raw 16-bit patterns of ``dtype`` ("f16" or "bf16") as fp32 values."""

    b = np.asarray(bits, np.uint16)
    if dtype == "f16":
        return b.view(np.float16).astype(np.float32)
    return (b.astype(np.uint32) << 16).view(np.float32)


def load_prologue_case(name: str) -> dict:
    with np.load(GOLDEN_DIR / f"prologue_{name}.npz") as z:
        return {k: z[k] for k in z.files}


def within_ulps(actual, expected, dtype: str, ulps: int = 1, rotated: bool = False) -> np.ndarray:
    """Elementwise: |actual - expected| is at most ``ulps`` units in the last
    place of ``dtype`` at the larger magnitude (or both equal, NaN included).
    ``rotated``: the values are RoPE outputs over the last axis."""

    a, e = np.asarray(actual, np.float64), np.asarray(expected, np.float64)
    mag = np.maximum(np.abs(a), np.abs(e))
    if rotated:
        # A rotated element is x*cos + partner*sin, partner = column c ^ D/2:
        # its rounding error scales with the larger of the two, not with the
        # (possibly cancelled) result.
        d = e.shape[-1]
        mag = np.maximum(mag, np.abs(e[..., np.arange(d) ^ (d // 2)]))
    mant = 10 if dtype == "f16" else 7
    ulp = np.where(mag > 0, 2.0 ** (np.floor(np.log2(np.maximum(mag, 1e-30))) - mant), 2.0 ** -24)
    ulp = np.maximum(ulp, 2.0 ** -24 if dtype == "f16" else 2.0 ** -133)
    return (np.abs(a - e) <= ulps * ulp) | (a == e) | (np.isnan(a) & np.isnan(e))


# ---------------------------------------------------------------- sampler
SAMPLER_TIE_ROW = 2  # two equal maxima: the filters' tie order is left open by torch


def load_sampler_cases() -> dict:
    with np.load(GOLDEN_DIR / "sampler_cases.npz") as z:
        d = {k: z[k] for k in z.files}
    d["kept"] = np.unpackbits(d["kept"], axis=-1)[..., : d["logits"].shape[1]].astype(bool)
    return d


# ---- metadata build (tests/golden/make_golden_metadata.py) ----

from dataclasses import dataclass as _dataclass  # noqa: E402


@_dataclass(frozen=True)
class BlockIds:
    """CacheGroupBlockTable's one field."""

    block_ids: tuple


@_dataclass(frozen=True)
class PlanRequest:
    """The ScheduledRequest fields (core/scheduler_output.py) a step's build reads."""

    request_id: str
    input_token_ids: tuple
    num_computed_tokens: int
    num_scheduled_tokens: int
    requires_sampling: bool
    block_tables: tuple


@_dataclass(frozen=True)
class Plan:
    """SchedulerOutput's ``scheduled_requests``."""

    scheduled_requests: tuple


def metadata_manifest() -> list[dict]:
    return json.loads((GOLDEN_DIR / "metadata_manifest.json").read_text())


def load_metadata_case(entry: dict) -> tuple[Plan, dict]:
    """(plan, the reference's tensors as numpy) of one golden case."""

    z = np.load(GOLDEN_DIR / "metadata_cases.npz")
    p = entry["name"] + "/"
    ng = len(entry["group_specs"])
    computed, scheduled = z[p + "computed"], z[p + "scheduled"]
    sample, tokens = z[p + "sample"], z[p + "token_ids"]
    blocks = []
    for g in range(ng):
        counts, ids = z[f"{p}g{g}/block_counts"], z[f"{p}g{g}/block_ids"]
        offs = np.concatenate([[0], np.cumsum(counts)])
        blocks.append([tuple(int(b) for b in ids[offs[i]:offs[i + 1]]) for i in range(len(counts))])
    qsl = np.concatenate([[0], np.cumsum(scheduled)])
    reqs = tuple(
        PlanRequest(
            request_id=f"r{i}", input_token_ids=tuple(int(x) for x in tokens[qsl[i]:qsl[i + 1]]),
            num_computed_tokens=int(computed[i]), num_scheduled_tokens=int(scheduled[i]),
            requires_sampling=bool(sample[i]),
            block_tables=tuple(BlockIds(blocks[g][i]) for g in range(ng)),
        )
        for i in range(len(computed))
    )
    expected = {k[len(p):]: z[k] for k in z.files if k.startswith(p)}
    return Plan(reqs), expected
