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
    # Ten million requests need far more than the built-in 24 MiB.
    rc = lib.mvb_paged_attention_no_alloc(
        None, 0, 0, None, None, 1, 16, 8, 128, None, None, None, None, None, 0, 0,
        1, 10_000_000, 16, 1.0, _lib.MVB_DTYPE_F16, None, None,
    )
    assert rc == _lib.MVB_ERR_WORKSPACE_TOO_SMALL
