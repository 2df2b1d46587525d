"""Shared pytest configuration.

Markers: ``gpu`` tests need a CUDA device and the built CUDA library; the
rest run on the CPU (oracle, host logic, library exports, gloo ranks).
"""

from __future__ import annotations

import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
for path in (ROOT, ROOT / "tests"):
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))


def pytest_configure(config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
