"""Build ``libmvb200.so`` (the C-ABI CUDA library) in-tree for sm_100a.

    python -m micro_vllm_b200.build [--force] [--verbose]

Every ``csrc/*.cu`` file is compiled by nvcc with
``-gencode arch=compute_100a,code=sm_100a`` into ``_build/`` (in parallel),
then linked into ``micro_vllm_b200/libmvb200.so`` with the static CUDA
runtime.  The library exports only the ``extern "C"`` symbols declared in
``include/mvb200.h``.  Rebuilds only when a source or header is newer than
the library.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
BUILD = PKG / "_build"
LIB = PKG / "libmvb200.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    *ARCH_FLAGS,
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC,-fvisibility=hidden",
    "-I",
    str(INCLUDE),
    "-I",
    str(CSRC),
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put CUDA's bin directory on PATH")


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _inputs() -> list[Path]:
    return [*_sources(), *CSRC.glob("*.cuh"), *CSRC.glob("*.h"), *INCLUDE.glob("*.h")]


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    lib_time = LIB.stat().st_mtime
    return all(p.stat().st_mtime <= lib_time for p in _inputs())


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    """Compile and link the library; return its path."""

    if not force and up_to_date():
        return LIB
    BUILD.mkdir(exist_ok=True)
    compiler = nvcc()
    extra = ["-Xptxas", "-v"] if ptxas_verbose else []

    def compile_one(src: Path) -> Path:
        obj = BUILD / (src.stem + ".o")
        cmd = [compiler, *NVCC_FLAGS, *extra, "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
        if (verbose or ptxas_verbose) and res.stderr:
            print(res.stderr, flush=True)
        return obj

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as pool:
        objs = list(pool.map(compile_one, _sources()))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [compiler, *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs)]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    tmp.replace(LIB)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true", help="print registers/spills per kernel")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose, ptxas_verbose=args.ptxas_verbose))


if __name__ == "__main__":
    main()
