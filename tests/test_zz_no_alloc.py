"""mvb_paged_attention_no_alloc against mvb_paged_attention.

The no-allocation entry point serves callers that cannot allocate device
memory (an arena-owning plugin host, an allocation-free serving loop, a
binding without CUDA memory management): it runs the same kernels on a
scratch region built into the library instead of a caller workspace.  This
file is named so pytest collects it last; it passes alone in a fresh process
and after the other tests.
"""

from __future__ import annotations

import math

import pytest
import torch

from micro_vllm_b200 import _lib
from micro_vllm_b200.build import build
from micro_vllm_b200.workloads import paged_batch, uniform_lengths

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-2
DEV = torch.device("cuda", 0)


def _common_args(batch, out: torch.Tensor) -> tuple:
    md = batch.metadata
    q = batch.query
    return (
        q.data_ptr(), q.stride(0), q.stride(1), out.data_ptr(),
        batch.cache.data_ptr(), batch.cache.shape[1], md.block_size,
        batch.cache.shape[3], q.shape[2],
        md.query_positions.data_ptr(), md.query_context_start_positions.data_ptr(),
        md.query_start_locations.data_ptr(), md.context_lengths.data_ptr(),
        md.block_table.data_ptr(), md.block_table.stride(0), md.block_table.shape[1],
        q.shape[0], batch.num_requests, q.shape[1], 1.0 / math.sqrt(q.shape[2]),
        _lib.MVB_DTYPE_F16 if q.dtype == torch.float16 else _lib.MVB_DTYPE_BF16,
    )


def test_no_alloc_entry_point_matches_the_workspace_entry_point() -> None:
    build()
    lib = _lib.load()
    stream = torch.cuda.current_stream(DEV).cuda_stream
    # Two different batches in a row through the shared scratch region; both
    # have long contexts cut across CTAs (partials merged through counters
    # that must start from zero on every call) and multi-token chunks.
    batches = [
        paged_batch(
            context_lengths=uniform_lengths(96, 1, 3000, seed=1) + [700, 40],
            query_lengths=[1] * 96 + [3, 4], num_q_heads=16, num_kv_heads=8, head_dim=128,
            block_size=16, num_blocks=30000, dtype=torch.float16, device=DEV, seed=21,
        ),
        paged_batch(
            context_lengths=uniform_lengths(40, 200, 4096, seed=2) + [65],
            query_lengths=[1] * 40 + [64], num_q_heads=32, num_kv_heads=8, head_dim=128,
            block_size=16, num_blocks=20000, dtype=torch.bfloat16, device=DEV, seed=22,
        ),
    ]
    for batch in batches:
        q = batch.query
        nbytes = lib.mvb_paged_attention_workspace_size(
            q.shape[0], batch.num_requests, q.shape[1], batch.cache.shape[3], q.shape[2]
        )
        workspace = torch.empty(nbytes, dtype=torch.uint8, device=DEV)
        expected = torch.empty_like(q)
        actual = torch.full_like(q, float("nan"))
        rc = lib.mvb_paged_attention(
            *_common_args(batch, expected), workspace.data_ptr(), workspace.numel(), None, stream
        )
        assert rc == _lib.MVB_OK
        rc = lib.mvb_paged_attention_no_alloc(*_common_args(batch, actual), None, stream)
        assert rc == _lib.MVB_OK
        torch.cuda.synchronize(DEV)
        torch.testing.assert_close(actual, expected, atol=ATOL, rtol=RTOL)


def test_no_alloc_entry_point_rejects_batches_beyond_its_region() -> None:
    build()
    lib = _lib.load()
    # Ten million requests on the tensor-core path need far more than the
    # built-in 24 MiB: refused before anything is launched, so small valid
    # buffers stand in for the batch's.
    buf = torch.zeros(1 << 16, dtype=torch.int64, device=DEV)
    p = buf.data_ptr()
    stream = torch.cuda.current_stream(DEV).cuda_stream
    rc = lib.mvb_paged_attention_no_alloc(
        p, 2048, 128, p, p, 1, 16, 8, 128, p, p, p, p, p, 1, 1,
        10_000_000, 10_000_000, 16, 1.0, _lib.MVB_DTYPE_F16, None, stream,
    )
    assert rc == _lib.MVB_ERR_WORKSPACE_TOO_SMALL
    # Invalid arguments get the code mvb_paged_attention gives them, whatever the size.
    for dtype, expected in ((7, _lib.MVB_ERR_UNSUPPORTED_DTYPE), (_lib.MVB_DTYPE_F16, _lib.MVB_ERR_INVALID_ARGUMENT)):
        args = (None, 0, 0, None, None, 1, 16, 8, 128, None, None, None, None, None, 0, 0,
                1, 10_000_000, 16, 1.0, dtype)
        assert lib.mvb_paged_attention(*args, None, 0, None, None) == expected
        assert lib.mvb_paged_attention_no_alloc(*args, None, None) == expected


def test_no_alloc_entry_point_on_the_exact_path() -> None:
    """fp32 and head_dim 64 run the exact CUDA-core kernel, which uses no
    scratch: the no-allocation entry point gives the same rows."""

    build()
    lib = _lib.load()
    stream = torch.cuda.current_stream(DEV).cuda_stream
    for dtype, head_dim in ((torch.float32, 128), (torch.float16, 64)):
        batch = paged_batch(
            context_lengths=uniform_lengths(12, 1, 600, seed=5) + [90], query_lengths=[1] * 12 + [30],
            num_q_heads=8, num_kv_heads=2, head_dim=head_dim, block_size=16, num_blocks=1000,
            dtype=dtype, device=DEV, seed=31,
        )
        args = list(_common_args(batch, batch.query))
        code = {torch.float32: _lib.MVB_DTYPE_F32, torch.float16: _lib.MVB_DTYPE_F16}[dtype]
        outs = []
        for entry in ("mvb_paged_attention", "mvb_paged_attention_no_alloc"):
            out = torch.full_like(batch.query, float("nan"))
            args[3] = out.data_ptr()
            args[-1] = code
            tail = (None, 0, None, stream) if entry == "mvb_paged_attention" else (None, stream)
            assert getattr(lib, entry)(*args, *tail) == _lib.MVB_OK
            outs.append(out)
        torch.cuda.synchronize(DEV)
        torch.testing.assert_close(outs[1], outs[0], atol=0, rtol=0)
