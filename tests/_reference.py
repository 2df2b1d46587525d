"""Access to the reference package (micro_vllm) for integration tests.

The reference is installed into ``baseline/_ref`` (``__graft_entry__.build``
does it from the reference's source tree when that tree is present); tests
that drive the reference's own engine or runner skip when it is absent.
"""

from __future__ import annotations

import importlib
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
REFERENCE_SITE = ROOT / "baseline" / "_ref"


def require_reference():
    """Import and return the ``micro_vllm`` package, or skip the test."""

    if REFERENCE_SITE.is_dir() and str(REFERENCE_SITE) not in sys.path:
        sys.path.append(str(REFERENCE_SITE))
    try:
        return importlib.import_module("micro_vllm")
    except ImportError as error:
        pytest.skip(f"reference package micro_vllm not installed under baseline/_ref ({error})")
