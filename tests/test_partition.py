"""Sequence partitioning over GPUs and the replica launcher (CPU, gloo).

The multi-GPU path of the backend is N independent replicas, each with its
own KV pool and whole sequences; these tests run that host-side logic with
world_size 2 on gloo, the oracle standing in for each rank's kernel.
"""

from __future__ import annotations

import numpy as np
import pytest

from micro_vllm_b200.partition import imbalance, partition_sequences, sequence_work
from micro_vllm_b200.replicas import ReplicaFailure, launch_replicas


def test_partition_covers_every_sequence_once_and_is_deterministic() -> None:
    rng = np.random.default_rng(0)
    work = rng.integers(512, 4097, size=256).tolist()
    for ranks in (1, 2, 4, 8):
        a = partition_sequences(work, ranks)
        b = partition_sequences(list(work), ranks)
        assert a == b
        seen = sorted(i for s in a for i in s.indices)
        assert seen == list(range(256))
        assert [s.work for s in a] == [sum(work[i] for i in s.indices) for s in a]
        assert imbalance(a) < 1.01


def test_partition_edge_cases() -> None:
    assert partition_sequences([], 3) == [
        type(partition_sequences([], 1)[0])(rank=r, indices=(), work=0) for r in range(3)
    ]
    shards = partition_sequences([5], 4)
    assert sum(len(s.indices) for s in shards) == 1
    with pytest.raises(ValueError):
        partition_sequences([1], 0)
    assert sequence_work(100, 1) == 101


def test_two_gloo_ranks_partition_and_gather_match_one_process(tmp_path) -> None:
    from _replica_worker import global_batch, shard_and_attend
    from oracle import paged_attention

    result = tmp_path / "out.npy"
    launch_replicas(shard_and_attend, 2, args=(str(result),), timeout=120)
    ctx, tables, cache, q, k, v, md = global_batch()
    expected = paged_attention(q, k, v, cache.copy(), md)
    np.testing.assert_array_equal(np.load(result), expected)


def test_a_failing_rank_is_reported() -> None:
    from _replica_worker import fail_on_rank_one

    with pytest.raises(ReplicaFailure) as info:
        launch_replicas(fail_on_rank_one, 2, timeout=60)
    assert info.value.failed[1].startswith("exit code")
    # Rank 0 is either done already or stopped because rank 1 failed.
    assert info.value.failed.get(0, "stopped after rank 1 failed") == "stopped after rank 1 failed"


def test_a_hung_rank_is_detected_and_stopped() -> None:
    from _replica_worker import hang_on_rank_one

    with pytest.raises(ReplicaFailure) as info:
        launch_replicas(hang_on_rank_one, 2, timeout=20)
    # Rank 1 never joins; rank 0's barrier times out with an error (exit
    # code), which ends the job and stops rank 1.
    assert info.value.failed[0].startswith("exit code")
    assert info.value.failed[1] == "stopped after rank 0 failed"


def test_a_rank_that_never_finishes_times_out() -> None:
    """No collective to fail: the launcher's own deadline stops the rank."""

    from _replica_worker import sleep_on_rank_one

    with pytest.raises(ReplicaFailure) as info:
        launch_replicas(sleep_on_rank_one, 2, timeout=8)
    assert info.value.failed == {1: "timed out after 8s"}


def test_an_early_failure_is_reported_before_the_timeout() -> None:
    """Rank 1 exits non-zero at once while rank 0 waits in a collective: the
    launcher reports it and stops rank 0 without waiting for the timeout."""

    import time

    from _replica_worker import fail_fast_while_rank_zero_waits

    start = time.monotonic()
    with pytest.raises(ReplicaFailure) as info:
        launch_replicas(fail_fast_while_rank_zero_waits, 2, timeout=240)
    assert time.monotonic() - start < 60
    assert info.value.failed[1].startswith("exit code")
    assert info.value.failed[0] == "stopped after rank 1 failed"
