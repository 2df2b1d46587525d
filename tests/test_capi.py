"""The C-ABI library loads and exports every symbol include/mvb200.h declares.

CPU-only: no call here launches device work.  The argument checks that
return before any CUDA call are exercised too.
"""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from micro_vllm_b200 import _lib
from micro_vllm_b200.build import LIB, build

HEADER = Path(__file__).resolve().parent.parent / "include" / "mvb200.h"


def declared_symbols() -> list[str]:
    text = HEADER.read_text()
    return re.findall(r"^MVB_API\s+[\w\s\*]+?\b(mvb_\w+)\s*\(", text, flags=re.M)


@pytest.fixture(scope="module")
def lib() -> ctypes.CDLL:
    build()
    return _lib.load()


def test_header_and_binding_declare_the_same_entry_points() -> None:
    names = declared_symbols()
    assert len(names) == len(set(names)) >= 7
    assert set(names) == set(_lib.SIGNATURES)


def test_library_exports_every_declared_symbol(lib) -> None:
    for name in declared_symbols():
        assert hasattr(lib, name), name


def test_library_exports_nothing_else() -> None:
    import subprocess

    out = subprocess.run(["nm", "-D", "--defined-only", str(LIB)], capture_output=True, text=True, check=True)
    exported = {line.split()[-1] for line in out.stdout.splitlines() if line.split()[-1].startswith("mvb_")}
    assert exported == set(declared_symbols())


def test_version_and_status_strings(lib) -> None:
    assert lib.mvb_version() >= 1
    assert lib.mvb_status_string(0) == b"ok"
    assert lib.mvb_status_string(_lib.MVB_ERR_WORKSPACE_TOO_SMALL) == b"workspace too small"
    assert lib.mvb_last_cuda_error() == 0


def test_workspace_size_is_host_arithmetic(lib) -> None:
    small = lib.mvb_paged_attention_workspace_size(1, 1, 16, 8, 128)
    big = lib.mvb_paged_attention_workspace_size(8192, 256, 16, 8, 128)
    assert 0 < small < big
    assert lib.mvb_paged_attention_workspace_size(-1, 1, 16, 8, 128) == 0


def test_argument_checks_return_before_touching_the_device(lib) -> None:
    strides = _lib.strides3((1024, 128, 1))
    # Unknown dtype.
    rc = lib.mvb_reshape_and_cache(None, strides, None, strides, None, 1, 16, 8, 128, None, 1, 7, None, None)
    assert rc == _lib.MVB_ERR_UNSUPPORTED_DTYPE
    # Non-positive block size.
    rc = lib.mvb_reshape_and_cache(None, strides, None, strides, None, 1, 0, 8, 128, None, 1, 0, None, None)
    assert rc == _lib.MVB_ERR_INVALID_ARGUMENT
    # Zero tokens is a no-op.
    rc = lib.mvb_reshape_and_cache(None, strides, None, strides, None, 1, 16, 8, 128, None, 0, 0, None, None)
    assert rc == _lib.MVB_OK
    # Head ratio that is not an integer.
    rc = lib.mvb_paged_attention(
        None, 0, 0, None, None, 1, 16, 3, 128, None, None, None, None, None, 0, 0,
        1, 1, 16, 1.0, 0, None, 0, None, None,
    )
    assert rc == _lib.MVB_ERR_UNSUPPORTED_SHAPE
    rc = lib.mvb_paged_attention(
        None, 0, 0, None, None, 1, 16, 8, 128, None, None, None, None, None, 0, 0,
        0, 0, 16, 1.0, 0, None, 0, None, None,
    )
    assert rc == _lib.MVB_OK
    # Sampler noise: rows without noise_row, or noise rows shorter than the
    # vocabulary, are rejected before anything runs; no rows is a no-op.
    fake = ctypes.c_void_p(16)
    rc = lib.mvb_sample_with_noise(None, 0, 1, 100, 0, None, None, None, None, None,
                                   fake, 100, 1, None, None, None)
    assert rc == _lib.MVB_ERR_INVALID_ARGUMENT
    rc = lib.mvb_sample_with_noise(None, 0, 1, 100, 0, None, None, None, None, None,
                                   fake, 99, 1, fake, None, None)
    assert rc == _lib.MVB_ERR_INVALID_ARGUMENT
    rc = lib.mvb_sample_with_noise(None, 0, 0, 100, 0, None, None, None, None, None,
                                   None, 0, 0, None, None, None)
    assert rc == _lib.MVB_OK
    rc = lib.mvb_sample_with_noise(None, 0, 1, 100, 9, None, None, None, None, None,
                                   None, 0, 0, None, None, None)
    assert rc == _lib.MVB_ERR_UNSUPPORTED_DTYPE


def test_operator_rejects_cpu_tensors() -> None:
    """Mirrors tests/benchmarks/test_spike_triton_paged.py:58-82: no CPU fallback."""

    import torch

    from micro_vllm_b200 import AttentionMetadata, B200PagedAttentionOperator

    token = torch.zeros((1, 1, 16), dtype=torch.float16)
    cache = torch.zeros((2, 1, 1, 1, 16), dtype=torch.float16)
    md = AttentionMetadata(
        query_positions=torch.tensor((0,)),
        query_context_start_positions=torch.tensor((0,)),
        query_start_locations=torch.tensor((0, 1)),
        context_lengths=torch.tensor((1,)),
        block_table=torch.tensor(((0,),)),
        slot_mapping=torch.tensor((0,)),
        block_size=1,
    )
    with pytest.raises(RuntimeError, match="b200_paged attention requires CUDA tensors"):
        B200PagedAttentionOperator()(token, token, token, cache, md)


def test_registry_resolves_the_operator_and_rejects_unknown_names() -> None:
    from micro_vllm_b200 import B200PagedAttentionOperator, get_attention_operator_class

    assert get_attention_operator_class("b200_paged") is B200PagedAttentionOperator
    with pytest.raises(ValueError, match=r"unsupported attention operator 'unknown'.*b200_paged"):
        get_attention_operator_class("unknown")


def test_pinned_staging_needs_cuda() -> None:
    import pytest
    from micro_vllm_b200.staging import PinnedStaging, UploadPipeline

    with pytest.raises(RuntimeError):
        PinnedStaging("cpu")
    with pytest.raises(RuntimeError, match="CUDA device"):
        UploadPipeline("cpu")


def test_layer_stages_reject_cpu_tensors() -> None:
    """The fused layer stages, like the attention operator, have no CPU path."""

    import torch

    from micro_vllm_b200.layers import rms_norm, silu_mul

    x = torch.zeros((2, 64), dtype=torch.float16)
    with pytest.raises(ValueError):
        rms_norm(x, torch.ones(64, dtype=torch.float16), 1e-6)
    with pytest.raises(ValueError):
        silu_mul(torch.zeros((2, 128), dtype=torch.float16), 64)
