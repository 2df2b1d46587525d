"""Per-GPU replica processes with failure detection on the host.

One process per GPU (rank), each owning its own KV pool and its share of
whole sequences (``partition.partition_sequences``).  The launcher starts
the ranks with the ``spawn`` method (safe after CUDA initialisation), gives
each the torch.distributed rendezvous environment, and watches them from the
host: a rank that raises (non-zero exit code) or never finishes (join
timeout, then terminate/kill) is reported in one ``ReplicaFailure`` instead
of leaving the job hanging.  Collectives inside the ranks should use a short
process-group timeout so survivors of a failed rank end with an error too.
"""

from __future__ import annotations

import multiprocessing as mp
import os
import socket
import time
import traceback
from typing import Callable


class ReplicaFailure(RuntimeError):
    """One or more ranks failed or timed out."""

    def __init__(self, failed: dict[int, str]) -> None:
        self.failed = dict(failed)
        detail = ", ".join(f"rank {r}: {why}" for r, why in sorted(failed.items()))
        super().__init__(f"replica ranks failed: {detail}")


def free_port() -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(target: Callable, rank: int, world_size: int, port: int, args: tuple) -> None:
    os.environ.update(
        MASTER_ADDR="127.0.0.1",
        MASTER_PORT=str(port),
        RANK=str(rank),
        LOCAL_RANK=str(rank),
        WORLD_SIZE=str(world_size),
    )
    try:
        target(rank, world_size, *args)
    except BaseException:
        traceback.print_exc()
        os._exit(1)


def launch_replicas(
    target: Callable, world_size: int, *, args: tuple = (), timeout: float = 600.0
) -> None:
    """Run ``target(rank, world_size, *args)`` in ``world_size`` processes.

    Returns when every rank exited 0; raises ``ReplicaFailure`` naming each
    rank that exited non-zero or was still running after ``timeout`` seconds
    (those are terminated, then killed).
    """

    ctx = mp.get_context("spawn")
    port = free_port()
    procs = [
        ctx.Process(target=_rank_main, args=(target, r, world_size, port, args), daemon=False)
        for r in range(world_size)
    ]
    for p in procs:
        p.start()
    deadline = time.monotonic() + timeout
    failed: dict[int, str] = {}
    for r, p in enumerate(procs):
        p.join(max(0.0, deadline - time.monotonic()))
    for r, p in enumerate(procs):
        if p.is_alive():
            failed[r] = f"timed out after {timeout:.0f}s"
            p.terminate()
            p.join(5)
            if p.is_alive():
                p.kill()
                p.join(5)
        elif p.exitcode != 0:
            failed[r] = f"exit code {p.exitcode}"
    if failed:
        raise ReplicaFailure(failed)
