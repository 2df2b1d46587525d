"""Per-GPU replica processes with failure detection on the host.

One process per GPU (rank), each owning its own KV pool and its share of
whole sequences (``partition.partition_sequences``).  The launcher starts
the ranks with the ``spawn`` method (safe after CUDA initialisation), gives
each the torch.distributed rendezvous environment, and watches them from the
host: a rank that raises (non-zero exit code) or never finishes (join
timeout, then terminate/kill) is reported in one ``ReplicaFailure`` instead
of leaving the job hanging.  The launcher waits on all ranks at once: the
first rank to exit non-zero is reported at once and the others are stopped,
even when they are blocked in a collective waiting for it.  Collectives
inside the ranks should still use a short process-group timeout.
"""

from __future__ import annotations

import multiprocessing as mp
from multiprocessing.connection import wait
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
    running = {p.sentinel: r for r, p in enumerate(procs)}
    # Watch every rank at once: the first one to exit non-zero ends the job
    # now, not after the ranks it leaves blocked in a collective time out.
    while running and not failed:
        left = deadline - time.monotonic()
        if left <= 0:
            break
        for sentinel in wait(list(running), timeout=left):
            r = running.pop(sentinel)
            procs[r].join()
            if procs[r].exitcode != 0:
                failed[r] = f"exit code {procs[r].exitcode}"
    first_failure = min(failed) if failed else None
    for r in running.values():
        p = procs[r]
        failed[r] = (f"timed out after {timeout:.0f}s" if first_failure is None
                     else f"stopped after rank {first_failure} failed")
        p.terminate()
        p.join(5)
        if p.is_alive():
            p.kill()
            p.join(5)
    if failed:
        raise ReplicaFailure(failed)
