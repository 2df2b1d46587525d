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
