"""Test infrastructure: the CPU oracle of the paged-attention hot path.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
legs import this package.  The product (``micro_vllm_b200``) never does.
"""

from oracle.paged_attention import (  # noqa: F401
    OracleMetadata,
    build_metadata,
    chunked_local_context_start,
    full_context_start,
    gather_kv_cache,
    map_cache_slots,
    paged_attention,
    sliding_window_context_start,
    write_kv_cache,
)
