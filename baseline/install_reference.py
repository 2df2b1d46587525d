"""Install the reference package (micro_vllm, pure Python) into baseline/_ref.

    python baseline/install_reference.py <reference source tree>

The config-5 engine measurement (bench.py) and the integration tests drive
the reference's own scheduler, engine loop and model with this repository's
operator plugged in; they import micro_vllm from baseline/_ref, which travels
with the repository to the GPU box (it is git-ignored, not copied from the
source tree at run time).  The source tree is copied to a temporary
directory first (pip writes build files beside the sources).  Dependencies
are not resolved (--no-deps): the reference pins torch<2.9 and
transformers<5, and its code runs on the newer installed versions.
"""

from __future__ import annotations

import shutil
import subprocess
import sys
import tempfile
from pathlib import Path

TARGET = Path(__file__).resolve().parent / "_ref"


def install(source: str | Path, target: Path = TARGET) -> Path:
    source = Path(source).resolve()
    if not (source / "pyproject.toml").is_file():
        raise FileNotFoundError(f"{source} is not the reference's source tree (no pyproject.toml)")
    with tempfile.TemporaryDirectory() as tmp:
        copy = Path(tmp) / "src_tree"
        shutil.copytree(source, copy, ignore=shutil.ignore_patterns(".git", "__pycache__"))
        staging = Path(tmp) / "target"
        subprocess.run(
            [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation", "--no-deps",
             "--quiet", "--target", str(staging), str(copy)],
            check=True,
        )
        if target.exists():
            shutil.rmtree(target)
        shutil.copytree(staging, target)
    return target


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit(__doc__)
    print(install(sys.argv[1]))
