"""Benchmark of the b200_paged attention hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--dtype fp16|bf16] [--ctx uniform|fixed4096]
                    [--workload decode|llama8b|mixed|prologue|layers|sample|metadata|engine]
                    [--no-engine] [--no-engine-baselines] [--no-triton]

Workload (Qwen3-0.6B attention shape): 256 decode
sequences per GPU, context lengths uniform in [512, 4096] (or all 4096),
16 query / 8 KV heads, head_dim 128, block_size 16, N(0,1) K/V in ONE
layer's paged cache sized to 80% of HBM, block tables drawn at random
without replacement over the whole pool.  A step is one
``AttentionOperator.forward`` — the KV scatter of the step's new tokens and
split-KV paged decode over the whole context.  Each GPU holds its own pool
and its own 256 sequences (whole sequences are partitioned over GPUs, no
collective on the data path): weak scaling.

Metric: algorithmic HBM bytes of paged decode per second (GB/s) —
sum(ctx) * Hkv * D * 2 (K and V) * elsize + Q and O (2 * B * Hq * D * elsize)
+ block-table entries (8 B per page).  Inputs are larger than L2 (about
2.4 GB of KV per step against a 126 MB L2), so no flush is needed.

The same line also carries ``reference_gpu`` (the reference's own Triton
kernel, ``triton_paged_attention``, timed against this step on the same batch
in interleaved CUDA-event samples; fp16 only), ``reference_sdpa`` (the
reference's SDPA backend, ``paged_sdpa_attention``, on the same batch) and
``engine``: BASELINE config
5, output tokens/s of the reference's own engine (scheduler, KV block manager,
engine loop, Qwen3 model, installed under baseline/_ref) with ``b200_paged``
and ``B200ModelRunner``, on a random-init Qwen3-0.6B in fp16: 512 requests,
prompts U[128,1024], 256 greedy output tokens each, partitioned over the
ranks (strong scaling, ``engine.value``), plus each rank serving its own 512
requests at N > 1 (weak scaling, ``engine.weak``); at N = 1 the reference's
fastest engine configuration (``triton_paged`` with CUDA graphs) runs the
same job (``engine.reference_engine``).

``--impl reference`` times the reference algorithm on the host CPU (the
numpy port in oracle/, all host threads) on a bounded sample of the same
workload and reports the same metric.

Other workloads (parity and supplementary lines, not the default):
``--workload llama8b`` is BASELINE config 4 (32/8 heads, 64 seqs/GPU, ctx
U[4096,8192], bf16) with the same metric; ``--workload mixed`` is config 3
(8 chunked prefills of 2048 tokens over cached prefixes + 120 decodes, bf16)
and reports the prefill kernel's tensor throughput in TFLOP/s; ``--workload
prologue`` times the fused Qwen3 q/k-norm + RoPE + KV-write kernel on one
8192-token step (config 5's max_num_batched_tokens) in GB/s; ``--workload
layers`` the fused decoder-layer stages (RMSNorm after the residual add,
silu * up) on the same step in GB/s; ``--workload sample`` the batched
sampler on 256 rows of a 151936-token vocabulary (GB/s
of logits); ``--workload metadata`` the device build of a config-2 step's
metadata (us per step, lower is better); ``--workload engine`` the config-5
measurement alone.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

NUM_Q_HEADS, NUM_KV_HEADS, HEAD_DIM, BLOCK_SIZE = 16, 8, 128, 16
BATCH_PER_GPU = 256
POOL_FRACTION = 0.8
# ncu dram__bytes_read.sum + dram__bytes_write.sum of one paged_decode_kernel
# launch over its algorithmic bytes, per workload, from captures of the same
# batches on a 4 GB pool (summaries under profiles/).  bench scales the ratio
# to the launch it times.
# ncu dram read+write bytes of one paged_prefill_kernel launch on the config-3
# prefill chunks (same seeds, 1 GB pool).
PREFILL_TRAFFIC = {"fp16": 396.8e6, "bf16": 339.023e6 + 46.738e6}
DECODE_TRAFFIC_RATIO = {"config2": (2.527153 + 0.011768) / 2.5180, "config4": (1.613162 + 0.007385) / 1.6100}


class DecodeShape:
    """One decode workload of BASELINE.json: config 2 (Qwen3-0.6B attention,
    256 seqs/GPU, ctx U[512,4096] or 4096) or config 4 (Llama-3-8B GQA, 32/8
    heads, 64 seqs/GPU, ctx U[4096,8192])."""

    def __init__(self, args) -> None:
        self.key = "config4" if args.workload == "llama8b" else "config2"
        if args.workload == "llama8b":
            self.name, self.hq, self.batch = "BASELINE config 4: Llama-3-8B GQA long decode", 32, 64
            self.lo, self.hi, self.default_dtype = 4096, 8192, "bf16"
            self.ctx_label = "U[4096,8192]"
        else:
            self.name, self.hq, self.batch = "BASELINE config 2: paged decode", NUM_Q_HEADS, BATCH_PER_GPU
            self.lo, self.hi, self.default_dtype = 512, 4096, "fp16"
            self.ctx_label = "U[512,4096]" if args.ctx == "uniform" else "4096"
        self.fixed = args.workload != "llama8b" and args.ctx == "fixed4096"
        self.dtype = args.dtype or self.default_dtype

    def lengths(self, n: int, seed: int) -> list[int]:
        from micro_vllm_b200.workloads import uniform_lengths

        return [4096] * n if self.fixed else uniform_lengths(n, self.lo, self.hi, seed)

    def bytes(self, ctx: list[int], elsize: int) -> int:
        return decode_bytes(ctx, elsize, self.hq)

    def label(self) -> str:
        return (f"{self.name}, {self.batch} seqs/GPU, ctx {self.ctx_label}, Hq {self.hq} / Hkv {NUM_KV_HEADS}, "
                f"D {HEAD_DIM}, bs {BLOCK_SIZE}")


def parse_args() -> argparse.Namespace:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--dtype", choices=("fp16", "bf16"), default=None,
                    help="default: the workload's own (fp16 for config 2, bf16 for configs 3 and 4)")
    ap.add_argument("--ctx", choices=("uniform", "fixed4096"), default="uniform")
    ap.add_argument("--cpu-sample-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer end-to-end leg")
    ap.add_argument("--workload",
                    choices=("decode", "mixed", "llama8b", "prologue", "layers", "sample", "metadata", "engine"),
                    default="decode",
                    help="decode: BASELINE config 2 (headline, with the config-5 engine object); "
                         "mixed: config 3 (prefill + decode); engine: config 5 alone")
    ap.add_argument("--no-triton", action="store_true",
                    help="skip the reference's GPU backends (Triton kernel, SDPA) timed beside ours "
                         "on the decode batch")
    ap.add_argument("--no-engine", action="store_true",
                    help="decode workload without the config-5 engine measurement")
    ap.add_argument("--engine-requests", type=int, default=512)
    ap.add_argument("--engine-max-tokens", type=int, default=256)
    ap.add_argument("--no-engine-baselines", action="store_true",
                    help="skip the reference engine configurations timed beside ours at N=1")
    ap.add_argument("--pool-gb", type=float, default=None,
                    help="pool size in GB instead of 80%% of HBM (small cases for ncu captures)")
    return ap.parse_args()


def decode_bytes(ctx: list[int], elsize: int, num_q_heads: int = NUM_Q_HEADS) -> int:
    """Algorithmic HBM bytes of one paged decode launch."""

    kv = sum(ctx) * NUM_KV_HEADS * HEAD_DIM * 2 * elsize
    qo = 2 * len(ctx) * num_q_heads * HEAD_DIM * elsize
    table = sum(-(-c // BLOCK_SIZE) for c in ctx) * 8
    return kv + qo + table


def write_bytes(n: int, elsize: int) -> int:
    """Algorithmic bytes of the KV scatter: read new K/V, write them."""

    return 2 * 2 * n * NUM_KV_HEADS * HEAD_DIM * elsize


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples of this GPU's clocks during the timed region."""

    FIELDS = (
        "clocks.sm,clocks.max.sm,clocks_event_reasons.active,"
        "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
        "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"
    )

    def __init__(self, gpu_index: int) -> None:
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def start(self) -> None:
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True,
            )
            threading.Thread(target=self._read, daemon=True).start()
        except OSError:
            self.proc = None

    def _read(self) -> None:
        assert self.proc is not None and self.proc.stdout is not None
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def wait_first(self, timeout: float = 10.0) -> None:
        """Block until the first sample has arrived (bounded): nvidia-smi
        takes up to seconds to start, longer with one per rank, and a timed
        region of a few milliseconds would otherwise end before it."""

        end = time.monotonic() + timeout
        while self.proc is not None and not self.lines and time.monotonic() < end:
            if self.proc.poll() is not None:
                return
            time.sleep(0.02)

    def stop(self) -> dict:
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        sm, mx, reasons = [], 0.0, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                mx = max(mx, float(parts[1]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[3:7]):
                if flag.lower() in ("active", "1", "yes"):
                    reasons.add(name)
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": mx or None,
            "reasons": sorted(reasons),
            "samples": len(sm),
        }


# ---------------------------------------------------------------- CPU
def cpu_baseline(args, dtype_size: int, seconds: float) -> dict:
    """The reference algorithm (numpy port of ReferenceAttentionOperator,
    oracle/paged_attention.py) on the host cores, on a bounded sample: the
    first sequences of the same workload, repeated for about `seconds`."""

    import numpy as np

    from oracle import build_metadata, paged_attention

    cores = os.cpu_count() or 1
    shape = DecodeShape(args)
    sample = min(32, shape.batch)
    ctx = shape.lengths(shape.batch, seed=0)[:sample]
    rng = np.random.default_rng(0)
    tables, cursor = [], 0
    for c in ctx:
        n = -(-c // BLOCK_SIZE)
        tables.append(list(range(cursor, cursor + n)))
        cursor += n
    cache = rng.standard_normal((2, cursor, BLOCK_SIZE, NUM_KV_HEADS, HEAD_DIM), dtype=np.float32)
    md = build_metadata([[c - 1] for c in ctx], tables, block_size=BLOCK_SIZE)
    q = rng.standard_normal((sample, shape.hq, HEAD_DIM), dtype=np.float32)
    k = rng.standard_normal((sample, NUM_KV_HEADS, HEAD_DIM), dtype=np.float32)
    v = rng.standard_normal((sample, NUM_KV_HEADS, HEAD_DIM), dtype=np.float32)
    from threadpoolctl import threadpool_limits

    # Requests run on `cores` threads; one BLAS thread each avoids oversubscription.
    with threadpool_limits(limits=1):
        paged_attention(q, k, v, cache, md, num_threads=cores)  # warm-up
        calls, t0 = 0, time.perf_counter()
        while True:
            paged_attention(q, k, v, cache, md, num_threads=cores)
            calls += 1
            elapsed = time.perf_counter() - t0
            if elapsed >= seconds or calls >= 1000:
                break
    per_call = elapsed / calls
    return {
        "value": shape.bytes(ctx, dtype_size) / per_call / 1e9,
        "unit": "GB/s",
        "cores": cores,
        "kind": "port",
        "sample": (
            f"{sample} of the {shape.batch} decode sequences (ctx {shape.ctx_label}), fp32 numpy port of "
            f"ReferenceAttentionOperator, {calls} calls in {elapsed:.1f}s, "
            f"{per_call * 1e3:.1f} ms/call; bytes counted at {dtype_size}-byte elements like the GPU line"
        ),
    }


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    elsize = 2
    cpu = cpu_baseline(args, elsize, seconds=max(2.0, args.cpu_sample_seconds / 2))
    # Steps: repeated bounded samples; time each as one step.
    values = []
    for _ in range(max(1, min(args.steps, 3))):
        values.append(cpu_baseline(args, elsize, seconds=2.0)["value"])
    value = statistics.median(values + [cpu["value"]])
    line = {
        "impl": "reference",
        "metric": "paged_decode_hbm_GBps",
        "value": value,
        "unit": "GB/s",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": {
            "workload": DecodeShape(args).label(),
            "sample_sequences": min(32, DecodeShape(args).batch),
        },
        "cpu_baseline": cpu,
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- ranks
def init_ranks():
    """(world size, rank, this rank's device); one NCCL process group for the
    job (torchrun's environment), created once, with a short timeout so
    ranks waiting on a failed one end with an error."""

    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1 and not dist.is_initialized():
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    return world, rank, dev


def finish_ranks() -> None:
    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()


def _reduce(value: float, op: str, dev) -> float:
    """MAX / MIN / SUM of a host number over the ranks (identity at N=1)."""

    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()):
        return value
    t = torch.tensor([value], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op={"max": dist.ReduceOp.MAX, "min": dist.ReduceOp.MIN, "sum": dist.ReduceOp.SUM}[op])
    return float(t.item())


# ---------------------------------------------------------------- GPU
def triton_comparator(batch, ours, dev, samples: int = 10, launches: int = 5) -> dict:
    """The reference's own GPU kernel on the same batch and pool:
    ``triton_paged_attention`` (src/micro_vllm/attention/operators/triton_paged.py:328-389
    in the reference project: its one-launch KV write, then one program per
    block of query rows walking the whole context), timed against ``ours``
    (the full operator step) in interleaved CUDA-event samples with a
    rotating order, the method of the reference's benchmarks/spike_triton_paged.py:309-415."""

    import statistics as st

    import torch

    if batch.query.dtype != torch.float16:
        return {"unavailable": "the reference's Triton operator supports torch.float16 only"}
    sys.path.insert(0, str(ROOT / "baseline" / "_ref"))
    try:
        from micro_vllm.attention.operators.triton_paged import triton_paged_attention
    except Exception as exc:  # micro_vllm or triton missing
        return {"unavailable": f"{type(exc).__name__}: {exc}"}

    md = batch.metadata

    def theirs():
        return triton_paged_attention(batch.query, batch.key, batch.value, batch.cache, md)

    out_ref, out_ours = theirs(), ours()
    torch.cuda.synchronize(dev)
    diff = (out_ref.float() - out_ours.float()).abs().max().item()
    ops = {"ours": ours, "triton": theirs}
    for _ in range(3):
        for fn in ops.values():
            fn()
    torch.cuda.synchronize(dev)
    times = {name: [] for name in ops}
    names = list(ops)
    for i in range(samples):
        for name in names[i % 2:] + names[:i % 2]:
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for _ in range(launches):
                ops[name]()
            b.record()
            b.synchronize()
            times[name].append(a.elapsed_time(b) / launches)
    t_ours, t_theirs = st.median(times["ours"]), st.median(times["triton"])
    return {
        "impl": "triton_paged_attention, the reference's Triton kernel (KV write + paged attention), "
                "compiled here by Triton for this GPU",
        "ms_per_step": t_theirs,
        "ours_ms_per_step": t_ours,
        "speedup_ours_over_triton": t_theirs / t_ours,
        "max_abs_diff_vs_ours": diff,
        "method": f"interleaved CUDA-event samples, rotating order, {samples} samples x {launches} launches, "
                  "medians",
    }


def sdpa_comparator(batch, ours, dev, calls: int = 3, launches: int = 10) -> dict:
    """The reference's SDPA backend on the same batch and pool:
    ``paged_sdpa_attention`` (src/micro_vllm/attention/operators/sdpa.py:82-114
    in the reference project: its KV write, a gather of each request's
    history with host reads per request, then one PyTorch SDPA call per
    request).  The path synchronises the host per request, so each call is
    timed whole with CUDA events (median of ``calls``); ``ours`` is timed
    beside it as the median of ``launches`` back-to-back steps."""

    import statistics as st

    import torch

    sys.path.insert(0, str(ROOT / "baseline" / "_ref"))
    try:
        from micro_vllm.attention.operators.sdpa import paged_sdpa_attention
    except Exception as exc:  # micro_vllm missing
        return {"unavailable": f"{type(exc).__name__}: {exc}"}

    md = batch.metadata

    def theirs():
        return paged_sdpa_attention(batch.query, batch.key, batch.value, batch.cache, md)

    out_ref, out_ours = theirs(), ours()
    torch.cuda.synchronize(dev)
    diff = (out_ref.float() - out_ours.float()).abs().max().item()
    del out_ref
    times = []
    for _ in range(calls):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        theirs()
        b.record()
        b.synchronize()
        times.append(a.elapsed_time(b))
    mine = []
    for _ in range(launches):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        ours()
        b.record()
        b.synchronize()
        mine.append(a.elapsed_time(b))
    t_theirs, t_ours = st.median(times), st.median(mine)
    return {
        "impl": "paged_sdpa_attention, the reference's SDPA backend (KV write, per-request gather, "
                "PyTorch SDPA per request)",
        "ms_per_step": t_theirs,
        "ours_ms_per_step": t_ours,
        "speedup_ours_over_sdpa": t_theirs / t_ours,
        "max_abs_diff_vs_ours": diff,
        "method": f"CUDA events around whole calls (host-synchronised per request), medians of "
                  f"{calls} calls and of {launches} steps of ours",
    }


def run_ours(args) -> dict:
    import torch
    import torch.distributed as dist

    from micro_vllm_b200 import AttentionMetadata, B200PagedAttentionOperator
    from micro_vllm_b200 import _lib
    from micro_vllm_b200.workloads import paged_batch, pool_blocks_for_fraction

    world, rank, dev = init_ranks()
    local = dev.index
    shape = DecodeShape(args)
    hq = shape.hq
    dtype = torch.float16 if shape.dtype == "fp16" else torch.bfloat16
    elsize = 2

    # The global batch (shape.batch sequences per GPU) is split over the ranks
    # by whole sequences, longest-first to the least-loaded rank.
    from micro_vllm_b200.partition import partition_sequences, sequence_work

    global_ctx = shape.lengths(shape.batch * world, seed=1000)
    shards = partition_sequences([sequence_work(c) for c in global_ctx], world)
    ctx = [global_ctx[i] for i in shards[rank].indices]
    local_batch = len(ctx)
    if args.pool_gb is None:
        nb = pool_blocks_for_fraction(POOL_FRACTION, BLOCK_SIZE, NUM_KV_HEADS, HEAD_DIM, dtype, dev)
    else:
        nb = int(args.pool_gb * 1e9) // (2 * BLOCK_SIZE * NUM_KV_HEADS * HEAD_DIM * elsize)
    batch = paged_batch(
        context_lengths=ctx, query_lengths=[1] * local_batch, num_q_heads=hq,
        num_kv_heads=NUM_KV_HEADS, head_dim=HEAD_DIM, block_size=BLOCK_SIZE, num_blocks=nb,
        dtype=dtype, device=dev, seed=2000 + rank,
    )
    op = B200PagedAttentionOperator()
    op.reserve(dev, max_num_tokens=local_batch, max_num_requests=local_batch,
               num_q_heads=hq, num_kv_heads=NUM_KV_HEADS, head_dim=HEAD_DIM)
    stream = torch.cuda.current_stream(dev)

    def barrier() -> None:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    step = lambda: op(batch.query, batch.key, batch.value, batch.cache, batch.metadata)  # noqa: E731

    # Attention-only entry point (plan + decode), to time the decode kernel.
    md = batch.metadata
    ws, st = op._workspace(dev, local_batch, local_batch, hq, NUM_KV_HEADS, HEAD_DIM)
    out_buf = torch.empty_like(batch.query)
    lib = _lib.load()
    attn_args = (
        batch.query.data_ptr(), batch.query.stride(0), batch.query.stride(1), out_buf.data_ptr(),
        batch.cache.data_ptr(), nb, BLOCK_SIZE, NUM_KV_HEADS, HEAD_DIM,
        md.query_positions.data_ptr(), md.query_context_start_positions.data_ptr(),
        md.query_start_locations.data_ptr(), md.context_lengths.data_ptr(),
        md.block_table.data_ptr(), md.block_table.stride(0), md.block_table.shape[1],
        local_batch, local_batch, hq, 1.0 / math.sqrt(HEAD_DIM),
        _lib.MVB_DTYPE_F16 if dtype == torch.float16 else _lib.MVB_DTYPE_BF16,
        ws.data_ptr(), ws.numel(), st.status.data_ptr(), stream.cuda_stream,
    )

    def attention_only() -> None:
        _lib.check(lib.mvb_paged_attention(*attn_args), "bench attention")

    for _ in range(max(args.warmup, 3)):
        step()
        attention_only()
    barrier()

    # ---- timed region: K full forward steps ----
    clocks = ClockSampler(local)
    clocks.start()
    clocks.wait_first()
    t_start, t_stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    # A ~100 us spin keeps the GPU busy while the host enqueues the start
    # event and the first step, so the timed region holds device work only.
    torch.cuda._sleep(200_000)
    t_start.record(stream)
    for _ in range(args.steps):
        step()
    t_stop.record(stream)
    barrier()
    step_ms = max_over_ranks(t_start.elapsed_time(t_stop) / args.steps)

    # ---- decode kernel alone (plan + decode launches) ----
    barrier()
    a_start, a_stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda._sleep(200_000)
    a_start.record(stream)
    for _ in range(args.steps):
        attention_only()
    a_stop.record(stream)
    barrier()
    clock_info = clocks.stop()
    attn_ms = max_over_ranks(a_start.elapsed_time(a_stop) / args.steps)

    # ---- the reference's own GPU kernel on the same batch (rank 0) ----
    comparator = sdpa = None
    if rank == 0 and not args.no_triton:
        comparator = triton_comparator(batch, step, dev)
        torch.cuda.synchronize(dev)
        sdpa = sdpa_comparator(batch, step, dev)
        torch.cuda.synchronize(dev)
        torch.cuda.empty_cache()
    barrier()

    # ---- end to end through the public operator with host buffers ----
    # The step's host inputs are packed into one pinned buffer (the
    # caller-side staging a serving loop keeps) and uploaded with one copy;
    # the output is read back into pinned memory.  Pipelined: two staging
    # slots, the upload and the read-back on their own streams, so step i's
    # kernels overlap step i+1's upload and step i-1's read-back (every
    # step's copies stay inside the timed region).  Serial: the same copies
    # and the step one after the other on one stream.
    from micro_vllm_b200.staging import PinnedStaging, UploadPipeline

    host = {
        "q": batch.query.cpu(), "k": batch.key.cpu(), "v": batch.value.cpu(),
        "pos": md.query_positions.cpu(), "start": md.query_context_start_positions.cpu(),
        "qsl": md.query_start_locations.cpu(), "ctx": md.context_lengths.cpu(),
        "table": md.block_table.cpu(), "slots": md.slot_mapping.cpu(),
    }
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    out_hosts = [torch.empty(batch.query.shape, dtype=dtype).pin_memory() for _ in range(2)]
    d2h = out_hosts[0].numel() * out_hosts[0].element_size()

    def run_op(d) -> torch.Tensor:
        emd = AttentionMetadata(
            query_positions=d["pos"], query_context_start_positions=d["start"],
            query_start_locations=d["qsl"], context_lengths=d["ctx"], block_table=d["table"],
            slot_mapping=d["slots"], block_size=BLOCK_SIZE,
        )
        return op(d["q"], d["k"], d["v"], batch.cache, emd)

    staging = PinnedStaging(dev)
    staging.pack(host)

    # Every step packs its host inputs into pinned memory (the caller-side
    # staging of a serving loop) inside the timed region, then uploads them.
    def serial_step(i: int) -> None:
        staging.pack(host)
        out_hosts[0].copy_(run_op(staging.upload()), non_blocking=True)

    pipe = UploadPipeline(dev)

    def pipelined_step(i: int) -> None:
        pipe.slot(i).pack(host)
        out = run_op(pipe.upload(i))
        pipe.download(i, out, out_hosts[i % 2])

    def e2e_time(fn, finish=None) -> float:
        for i in range(3):
            fn(i)
        if finish is not None:
            finish()
        barrier()
        e_start, e_stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e_start.record(stream)
        for i in range(args.steps):
            fn(i)
        if finish is not None:
            finish()  # the last read-back inside the timed region
        e_stop.record(stream)
        barrier()
        return max_over_ranks(e_start.elapsed_time(e_stop) / args.steps)

    e2e_ms = serial_ms = float("nan")
    if not args.no_e2e:
        serial_ms = e2e_time(serial_step)
        e2e_ms = e2e_time(pipelined_step, pipe.drain)

    attn_bytes = shape.bytes(ctx, elsize)  # this rank's share
    step_bytes_all = shape.bytes(global_ctx, elsize)  # the whole job
    value = step_bytes_all / (step_ms * 1e-3) / 1e9
    peaks_path = ROOT / "MEASURED_PEAKS.json"
    peak, peak_src = 6650.0, "fallback"
    if peaks_path.exists():
        peak, peak_src = float(json.loads(peaks_path.read_text())["hbm_gbs"]), "measured"
    achieved = attn_bytes / (attn_ms * 1e-3) / 1e9
    ratio = DECODE_TRAFFIC_RATIO.get(shape.key)
    traffic = None if ratio is None else attn_bytes * ratio
    traffic_src = (
        None if ratio is None else
        f"ncu dram read+write of paged_decode_kernel on this workload's batch (4 GB pool) = {ratio:.4f} x "
        "algorithmic bytes, scaled to this launch's algorithmic bytes"
    )
    line = {
        "metric": "paged_decode_hbm_GBps",
        "value": value,
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": max(args.warmup, 3),
        "ms_per_step": step_ms,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f16" if dtype == torch.float16 else "bf16",
        "data": "synthetic",
        "config": {
            "workload": (
                f"{shape.label()}, pool {POOL_FRACTION:.0%} of HBM ({nb} blocks), random block tables; "
                "step = KV scatter + decode"
            ),
            "global_batch": shape.batch * world,
            "parallelism": f"whole-sequence LPT partition over {world} GPU replicas, no data-path collective",
            "l2": "inputs larger than L2 (KV per step about %.2f GB vs 126 MB L2); no flush" % (attn_bytes / 1e9),
            "bytes_per_step_per_gpu": attn_bytes,
        },
        "roofline": {
            "bound": "hbm",
            "achieved": achieved,
            "peak": peak,
            "unit": "GB/s",
            "frac": achieved / peak,
            "traffic": traffic,
            "traffic_source": traffic_src,
            "peak_source": peak_src,
            "kernel": "paged_decode_kernel (timed with its planner launch, attention-only entry point)",
            "ms_per_launch": attn_ms,
        },
        "e2e": {
            "value": step_bytes_all / (e2e_ms * 1e-3) / 1e9,
            "unit": "GB/s",
            "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h,
            "ms_per_step": e2e_ms,
            "what": "B200PagedAttentionOperator.forward on this step's q/k/v and metadata, packed from "
                    "pageable host tensors into one pinned buffer and uploaded with one copy, output read "
                    "back to pinned host memory, all inside the timed region; packing and copies of step "
                    "i+1 / i-1 overlap step i's kernels (UploadPipeline)",
            "serial": {"value": step_bytes_all / (serial_ms * 1e-3) / 1e9, "ms_per_step": serial_ms,
                       "what": "the same packing, copies and step one after the other on one stream"},
        },
        "gpu_launches": 4 * args.steps * world,
        "clocks": clock_info,
    }
    if world > 1:
        line["config"]["shard_imbalance"] = max(s.work for s in shards) / (sum(s.work for s in shards) / world)
    if comparator is not None:
        if "ms_per_step" in comparator:
            comparator["value"] = attn_bytes / (comparator["ms_per_step"] * 1e-3) / 1e9
            comparator["unit"] = "GB/s"
        line["reference_gpu"] = comparator
    if sdpa is not None:
        if "ms_per_step" in sdpa:
            sdpa["value"] = attn_bytes / (sdpa["ms_per_step"] * 1e-3) / 1e9
            sdpa["unit"] = "GB/s"
        line["reference_sdpa"] = sdpa
    if rank == 0 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(args, elsize, args.cpu_sample_seconds)
    return line


# ---------------------------------------------------------------- config 5
ENGINE_CHECKPOINT = "/tmp/mvb200_random_qwen3_0_6b_seed0"


def _engine_config(path, operator: str, graphs: bool, args):
    import torch
    from micro_vllm.config import CacheConfig, LLMConfig, ModelConfig, SchedulerConfig
    from micro_vllm_b200.integration import register

    register()  # b200_paged may take CUDA graphs: ModelConfig checks at construction
    return LLMConfig(
        model_config=ModelConfig(model=str(path), attention_operator=operator, enable_cuda_graph=graphs,
                                 device="cuda", dtype=torch.float16),
        scheduler_config=SchedulerConfig(max_num_batched_tokens=8192, max_num_seqs=512, max_model_len=1280),
        cache_config=CacheConfig(block_size=16, gpu_memory_utilization=0.9),
    )


def _engine_once(name: str, operator: str, graphs: bool, options, requests, args, dev, then=None) -> dict:
    """Initialise one worker, warm it with one full run of the same
    requests (the reference's benchmarks/benchmark_engine.py runs two warm-up
    repetitions of the workload by default: a first run pays one-time costs,
    cuBLAS's first use of each new GEMM shape among them, 30-100 ms on some
    prefill steps), then time the requests to completion through a fresh
    Engine."""

    import gc

    import torch
    from micro_vllm_b200.engine import build_worker, fresh_engine, run_engine

    # Every rank takes the same collectives whatever fails: one MIN after
    # the set-up (the start barrier of the timed run) and, with a second
    # run, one MAX before it (its start barrier); none inside the runs.
    t0 = time.perf_counter()
    worker = config = run = second = None
    error = None
    try:
        config = _engine_config(ENGINE_CHECKPOINT, operator, graphs, args)
        worker = build_worker(config, options)
        run_engine(fresh_engine(worker, config), requests, dev)
    except Exception as exc:
        error = f"{type(exc).__name__}: {exc}"
    init_s = time.perf_counter() - t0
    try:
        if _reduce(0.0 if error else 1.0, "min", dev) < 1.0:
            error = error or "another rank failed to set up its engine"
        else:
            try:
                run = run_engine(fresh_engine(worker, config), requests, dev)
            except Exception as exc:
                error = f"{type(exc).__name__}: {exc}"
        if then is not None:
            _reduce(0.0, "max", dev)
            if error is None:
                try:
                    second = run_engine(fresh_engine(worker, config), then, dev)
                except Exception as exc:
                    error = f"{type(exc).__name__}: {exc}"
    finally:
        if worker is not None:
            worker.shutdown()
        del worker
        gc.collect()
        torch.cuda.empty_cache()
    if error is not None:
        raise RuntimeError(error)
    return {"name": name, "seconds": run.seconds, "wall_seconds": run.wall_seconds, "steps": run.steps,
            "output_tokens": run.output_tokens, "prompt_tokens": run.prompt_tokens, "init_seconds": init_s,
            "outputs": run.outputs,
            **({"then": {"seconds": second.seconds, "output_tokens": second.output_tokens}} if second else {})}


def engine_measure(args) -> dict:
    """output tokens/s of the reference's own engine
    (scheduler, KV block manager, engine loop, Qwen3 model) with the
    ``b200_paged`` operator and ``B200ModelRunner``, on a random-init
    Qwen3-0.6B in fp16.  The 512 requests are partitioned over the ranks
    longest-first on prompt + max_tokens (one engine replica per GPU, no
    collective on the data path): strong scaling of a fixed job.  Each rank
    times its Engine.step loop with CUDA events; the job time is the max over
    ranks.  At N=1 the reference's fastest engine configuration
    (``triton_paged`` with CUDA graphs, its stock runner) runs the same job."""

    import traceback

    world, rank, dev = init_ranks()
    sys.path.insert(0, str(ROOT / "baseline" / "_ref"))
    error = None
    try:
        from micro_vllm_b200.engine import QWEN3_0_6B, RunnerOptions, engine_requests, write_random_checkpoint
        from micro_vllm_b200.partition import partition_sequences

        if rank == 0 and not (Path(ENGINE_CHECKPOINT) / "config.json").exists():
            write_random_checkpoint(ENGINE_CHECKPOINT + ".tmp", QWEN3_0_6B, seed=0)
            os.replace(ENGINE_CHECKPOINT + ".tmp", ENGINE_CHECKPOINT)
    except Exception as exc:  # the reference is not installed, or the checkpoint failed
        error = f"{type(exc).__name__}: {exc}"
    if _reduce(0.0 if error else 1.0, "min", dev) < 1.0:
        return {"unavailable": error or "another rank could not prepare the engine"}

    import torch

    # Eight engine processes share the host: keep each one's CPU ops on a
    # few threads (the scheduler and engine loop are single-threaded Python).
    torch.set_num_threads(max(1, (os.cpu_count() or 1) // world))
    requests = engine_requests(args.engine_requests, max_tokens=args.engine_max_tokens, seed=0)
    shards = partition_sequences([len(r.prompt_token_ids) + r.max_tokens for r in requests], world)
    mine = [requests[i] for i in shards[rank].indices]
    # Weak scaling beside it: every replica serves its own stream of the
    # same size (other seeds); at N=1 it is the same job.
    own = engine_requests(args.engine_requests, max_tokens=args.engine_max_tokens, seed=1000 + rank)
    result = weak = None
    try:
        result = _engine_once("b200", "b200_paged", True, RunnerOptions(), mine, args, dev,
                              then=own if world > 1 else None)
        weak = result.pop("then", None)
    except Exception:
        error = traceback.format_exc(limit=3).strip().splitlines()[-1]
    if _reduce(0.0 if error else 1.0, "min", dev) < 1.0:
        return {"unavailable": error or "another rank failed in the engine run"}
    seconds = _reduce(result["seconds"], "max", dev)
    wall = _reduce(result["wall_seconds"], "max", dev)
    tokens = _reduce(float(result["output_tokens"]), "sum", dev)
    steps = _reduce(float(result["steps"]), "max", dev)
    weak_line = None
    if world > 1:
        weak_seconds = _reduce(weak["seconds"], "max", dev)
        weak_tokens = _reduce(float(weak["output_tokens"]), "sum", dev)
        weak_line = {
            "value": weak_tokens / weak_seconds, "unit": "tokens/s", "scaling": "weak",
            "seconds": weak_seconds, "output_tokens": int(weak_tokens),
            "what": f"each of the {world} replicas serves its own {len(own)} requests (same distribution, "
                    "seed 1000 + rank): the N=1 job per GPU",
        }
    out = {
        "metric": "engine output tokens/s (BASELINE config 5)",
        "value": tokens / seconds,
        "unit": "tokens/s",
        "n_gpus": world,
        "scaling": "strong",
        "seconds": seconds,
        "wall_seconds": wall,
        "output_tokens": int(tokens),
        "max_steps_over_ranks": int(steps),
        "config": {
            "model": "Qwen3-0.6B shape (28 layers, hidden 1024, 16/8 heads, head_dim 128, MLP 3072, vocab 151936), "
                     "random init N(0, 0.02) seed 0, fp16",
            "requests": len(requests),
            "prompt_len": "U[128,1024] token ids U[1,151935]",
            "max_tokens": args.engine_max_tokens,
            "sampling": "greedy, ignore_eos",
            "max_num_batched_tokens": 8192, "max_num_seqs": 512, "max_model_len": 1280, "block_size": 16,
            "cuda_graphs": True,
            "attention_operator": "b200_paged",
            "runner": "B200ModelRunner: device metadata build, batched device sampler, fused Qwen3 prologue",
            "partition": f"LPT on prompt + max_tokens over {world} engine replicas, no data-path collective",
            "requests_per_rank_max": max(len(sh.indices) for sh in shards),
        },
        "timing": "CUDA events around each rank's Engine.step loop (synchronised at both ends), max over ranks; "
                  "wall_seconds is the host clock around the same loop; each engine (ours and the reference's) "
                  "first runs the same requests once untimed (warm-up)",
    }
    if weak_line is not None:
        out["weak"] = weak_line
    if world == 1 and not args.no_engine_baselines:
        try:
            ref = _engine_once("triton_paged", "triton_paged", True, None, mine, args, dev)
            out["reference_engine"] = {
                "value": ref["output_tokens"] / ref["seconds"], "unit": "tokens/s", "seconds": ref["seconds"],
                "steps": ref["steps"],
                "what": "the reference's stock ModelRunner with attention_operator='triton_paged' and CUDA "
                        "graphs (its fastest engine configuration), same model, requests and limits",
            }
        except Exception:
            out["reference_engine"] = {"unavailable": traceback.format_exc(limit=3).strip().splitlines()[-1]}
    return out


def run_engine_workload(args) -> None:
    """``--workload engine``: the config-5 measurement as its own line."""

    world, rank, dev = init_ranks()
    eng = engine_measure(args)
    finish_ranks()
    if rank != 0:
        return
    line = {
        "metric": "engine_output_tokens_per_s",
        "value": eng.get("value"),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f16",
        "data": "synthetic",
        "config": {"workload": "BASELINE config 5: engine, random-init Qwen3-0.6B, 512 requests"},
        "engine": eng,
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- config 3
def prefill_flops(prefix: list[int], new: list[int], num_q_heads: int, head_dim: int) -> int:
    """Algorithmic flops of causal attention for chunks of `new` tokens over
    `prefix` cached tokens: 4*D per visible (query, key) pair per head."""

    pairs = sum(l * p + l * (l + 1) // 2 for p, l in zip(prefix, new))
    return 4 * head_dim * num_q_heads * pairs


def run_mixed(args) -> None:
    """8 prefill chunks of 2048 new tokens over cached
    prefixes U[0,1024] + 120 decodes at ctx U[256,2048], 16/8/128, bf16.
    Reports the prefill kernel's tensor throughput (prefill requests alone,
    attention-only entry point) and the whole mixed step's time."""

    import torch

    from micro_vllm_b200 import B200PagedAttentionOperator
    from micro_vllm_b200 import _lib
    from micro_vllm_b200.workloads import paged_batch, uniform_lengths

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    # Config 3 is specified in bf16 (the default here); --dtype fp16 runs the
    # same batch in fp16 (the prefill target is quoted against fp16 peak).
    dtype = torch.float16 if args.dtype == "fp16" else torch.bfloat16
    prefix = uniform_lengths(8, 0, 1024, seed=31)
    new = [2048] * 8
    dec_ctx = uniform_lengths(120, 256, 2048, seed=32)
    ctx = [p + n for p, n in zip(prefix, new)] + dec_ctx
    qlen = new + [1] * 120
    need = sum(-(-c // BLOCK_SIZE) for c in ctx)
    nb = max(need + 64, int((args.pool_gb or 4.0) * 1e9) // (2 * BLOCK_SIZE * NUM_KV_HEADS * HEAD_DIM * 2))
    mixed = paged_batch(context_lengths=ctx, query_lengths=qlen, num_q_heads=NUM_Q_HEADS,
                        num_kv_heads=NUM_KV_HEADS, head_dim=HEAD_DIM, block_size=BLOCK_SIZE,
                        num_blocks=nb, dtype=dtype, device=dev, seed=33)
    prefill_only = paged_batch(context_lengths=ctx[:8], query_lengths=qlen[:8], num_q_heads=NUM_Q_HEADS,
                               num_kv_heads=NUM_KV_HEADS, head_dim=HEAD_DIM, block_size=BLOCK_SIZE,
                               num_blocks=nb, dtype=dtype, device=dev, seed=34)
    op = B200PagedAttentionOperator()
    lib = _lib.load()
    stream = torch.cuda.current_stream(dev)

    def attention_only(batch, out):
        md = batch.metadata
        ws, st = op._workspace(dev, batch.query.shape[0], batch.num_requests, NUM_Q_HEADS, NUM_KV_HEADS, HEAD_DIM)
        rc = lib.mvb_paged_attention(
            batch.query.data_ptr(), batch.query.stride(0), batch.query.stride(1), out.data_ptr(),
            batch.cache.data_ptr(), batch.cache.shape[1], BLOCK_SIZE, NUM_KV_HEADS, HEAD_DIM,
            md.query_positions.data_ptr(), md.query_context_start_positions.data_ptr(),
            md.query_start_locations.data_ptr(), md.context_lengths.data_ptr(),
            md.block_table.data_ptr(), md.block_table.stride(0), md.block_table.shape[1],
            batch.query.shape[0], batch.num_requests, NUM_Q_HEADS, 1.0 / math.sqrt(HEAD_DIM),
            _lib.MVB_DTYPE_BF16 if dtype == torch.bfloat16 else _lib.MVB_DTYPE_F16,
            ws.data_ptr(), ws.numel(), st.status.data_ptr(), stream.cuda_stream)
        _lib.check(rc, "bench attention")

    def timed(fn, steps):
        for _ in range(max(args.warmup, 3)):
            fn()
        torch.cuda.synchronize(dev)
        torch.cuda._sleep(200_000)  # GPU busy while the host enqueues the first launch
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(steps):
            fn()
        b.record(stream)
        torch.cuda.synchronize(dev)
        return a.elapsed_time(b) / steps

    out_p = torch.empty_like(prefill_only.query)
    # Write the prefill chunks' K/V once so the attention-only timing sees the real cache.
    op(prefill_only.query, prefill_only.key, prefill_only.value, prefill_only.cache, prefill_only.metadata)
    clocks = ClockSampler(dev.index)
    clocks.start()
    clocks.wait_first()
    prefill_ms = timed(lambda: attention_only(prefill_only, out_p), args.steps)
    mixed_ms = timed(lambda: op(mixed.query, mixed.key, mixed.value, mixed.cache, mixed.metadata), args.steps)
    clock_info = clocks.stop()
    flops = prefill_flops(prefix, new, NUM_Q_HEADS, HEAD_DIM)
    dtype_name = "bf16" if dtype == torch.bfloat16 else "fp16"
    achieved = flops / (prefill_ms * 1e-3) / 1e12
    peaks_path = ROOT / "MEASURED_PEAKS.json"
    peak, peak_src = 1590.0, "fallback"
    if peaks_path.exists():
        peak, peak_src = float(json.loads(peaks_path.read_text())["bf16_tflops"]), "measured"
    dec_bytes = decode_bytes(dec_ctx, 2)
    line = {
        "metric": "prefill_attn_TFLOPs",
        "value": achieved,
        "unit": "TFLOP/s",
        "n_gpus": 1,
        "steps": args.steps,
        "warmup": max(args.warmup, 3),
        "ms_per_step": prefill_ms,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16" if dtype == torch.bfloat16 else "f16",
        "data": "synthetic",
        "config": {
            "workload": "BASELINE config 3: 8 prefill chunks x 2048 new tokens over cached prefixes "
                        "U[0,1024] + 120 decodes ctx U[256,2048], 16/8/128, bs 16, causal",
            "prefix_tokens": prefix,
            "prefill_flops": flops,
            "l2": "prefill re-reads K/V per query tile from L2/HBM; no flush",
        },
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "traffic": PREFILL_TRAFFIC.get(dtype_name),
                     "traffic_source": "ncu dram read+write of paged_prefill_kernel on this batch (1 GB pool)"
                     if dtype_name in PREFILL_TRAFFIC else None, "peak_source": peak_src,
                     "kernel": "paged_prefill_kernel (with planner; prefill requests only)"},
        "mixed_step": {"ms": mixed_ms, "decode_bytes": dec_bytes,
                       "note": "scatter of 16504 tokens + plan + decode (120 seqs) + prefill (8 chunks)"},
        "gpu_launches": 4 * args.steps,
        "clocks": clock_info,
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- prologue
def run_layers(args) -> None:
    """The fused decoder-layer stages (mvb_rms_norm with the residual add,
    mvb_silu_mul) on an 8192-token step of the Qwen3-0.6B shape (hidden
    1024, intermediate 3072), fp16 unless --dtype; each timed alone, the L2
    evicted before every timed launch."""

    import torch

    from micro_vllm_b200.layers import rms_norm, silu_mul

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    dtype = torch.bfloat16 if args.dtype == "bf16" else torch.float16
    tokens, hidden, inter = 8192, 1024, 3072
    g = torch.Generator(device=dev).manual_seed(11)
    x = torch.randn((tokens, hidden), generator=g, device=dev).to(dtype)
    residual = torch.randn((tokens, hidden), generator=g, device=dev).to(dtype)
    weight = (0.5 + torch.rand(hidden, generator=g, device=dev)).to(dtype)
    gate_up = torch.randn((tokens, 2 * inter), generator=g, device=dev).to(dtype)
    stream = torch.cuda.current_stream(dev)
    flush = torch.ones(64 * 1024 * 1024, dtype=torch.float32, device=dev)  # 256 MB read between launches
    ops = {
        "rms_norm_add": (lambda: rms_norm(x, weight, 1e-6, residual=residual), 4 * tokens * hidden * 2),
        "silu_mul": (lambda: silu_mul(gate_up, inter), 3 * tokens * inter * 2),
    }
    for fn, _ in ops.values():
        for _ in range(max(args.warmup, 3)):
            fn()
    torch.cuda.synchronize(dev)
    clocks = ClockSampler(dev.index)
    clocks.start()
    clocks.wait_first()
    results = {}
    for name, (fn, byts) in ops.items():
        total = 0.0
        for _ in range(args.steps):
            flush.max()
            torch.cuda._sleep(1_000_000)  # ~0.5 ms: the GPU stays busy while the host launches
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            fn()
            b.record(stream)
            torch.cuda.synchronize(dev)
            total += a.elapsed_time(b)
        ms = total / args.steps
        results[name] = {"ms": ms, "bytes": byts, "GBps": byts / (ms * 1e-3) / 1e9}
    clock_info = clocks.stop()
    peak, peak_src = _hbm_peak()
    all_bytes = sum(r["bytes"] for r in results.values())
    all_ms = sum(r["ms"] for r in results.values())
    value = all_bytes / (all_ms * 1e-3) / 1e9
    line = {
        "metric": "fused_layer_stages_GBps", "value": value, "unit": "GB/s", "n_gpus": 1,
        "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": all_ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16" if dtype == torch.float16 else "bf16",
        "data": "synthetic",
        "config": {"workload": f"RMSNorm after the residual add and silu(gate) * up, {tokens} tokens, "
                               f"hidden {hidden}, intermediate {inter} (one Qwen3-0.6B layer's stages)",
                   "l2": "L2 evicted (256 MB read) before every timed launch"},
        "roofline": {"bound": "hbm", "achieved": value, "peak": peak, "unit": "GB/s", "frac": value / peak,
                     "traffic": None, "peak_source": peak_src, "kernels": {
                         name: {"GBps": r["GBps"], "frac": r["GBps"] / peak, "ms": r["ms"],
                                "bytes_per_launch": r["bytes"]} for name, r in results.items()}},
        "gpu_launches": 2 * args.steps, "clocks": clock_info,
    }
    print(json.dumps(line), flush=True)


def run_prologue(args) -> None:
    """Fused q/k RMSNorm + RoPE + KV write (mvb_qk_norm_rope_and_cache) on an
    8192-token step at the Qwen3-0.6B attention shape, fp16 unless --dtype."""

    import numpy as np
    import torch

    from micro_vllm_b200 import AttentionMetadata, qk_norm_rope_and_write, rotary_inverse_frequencies

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    dtype = torch.bfloat16 if args.dtype == "bf16" else torch.float16
    tokens, hq, hkv, d, bs = 8192, NUM_Q_HEADS, NUM_KV_HEADS, HEAD_DIM, BLOCK_SIZE
    g = torch.Generator(device=dev).manual_seed(7)
    qkv = torch.randn((tokens, (hq + 2 * hkv) * d), generator=g, device=dev).to(dtype)
    q = qkv[:, : hq * d].view(tokens, hq, d)
    k = qkv[:, hq * d : (hq + hkv) * d].view(tokens, hkv, d)
    v = qkv[:, (hq + hkv) * d :].view(tokens, hkv, d)
    nb = int((args.pool_gb or 8.0) * 1e9) // (2 * bs * hkv * d * 2)
    cache = torch.empty((2, nb, bs, hkv, d), dtype=dtype, device=dev)
    slots = torch.randperm(nb * bs, generator=g, device=dev)[:tokens]
    positions = torch.randint(0, 8192, (tokens,), generator=g, device=dev)
    q_w = (0.5 + torch.rand(d, generator=g, device=dev)).to(dtype)
    k_w = (0.5 + torch.rand(d, generator=g, device=dev)).to(dtype)
    inv = rotary_inverse_frequencies(d, 1e6, dev)
    md = AttentionMetadata(
        query_positions=positions, query_context_start_positions=positions * 0,
        query_start_locations=torch.tensor([0, tokens], device=dev),
        context_lengths=torch.tensor([1], device=dev),
        block_table=torch.zeros((1, 1), dtype=torch.int64, device=dev), slot_mapping=slots, block_size=bs,
    )
    step = lambda: qk_norm_rope_and_write(q, k, v, positions, q_w, k_w, 1e-6, inv, cache, md)  # noqa: E731
    stream = torch.cuda.current_stream(dev)
    # The step's 134 MB barely exceeds the 126 MB L2: evict it between steps
    # by reading a 256 MB buffer (a read leaves no dirty lines to write back
    # during the timed kernel, as a write-based flush would).
    flush = torch.ones(64 * 1024 * 1024, dtype=torch.float32, device=dev)
    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize(dev)
    clocks = ClockSampler(dev.index)
    clocks.start()
    clocks.wait_first()
    def timed(fn) -> float:
        # The flush, then a ~0.5 ms spin that keeps the GPU busy while the
        # host enqueues the start event, runs the Python wrapper and
        # launches: the events bracket the kernel, not the host's launch path.
        total = 0.0
        for _ in range(args.steps):
            flush.max()
            torch.cuda._sleep(1_000_000)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            fn()
            b.record(stream)
            torch.cuda.synchronize(dev)
            total += a.elapsed_time(b)
        return total / args.steps

    ms = timed(step)
    clock_info = clocks.stop()
    rows = hq + 2 * hkv
    byts = 2 * tokens * rows * d * 2  # read q, k, v; write q_out, k, v
    achieved = byts / (ms * 1e-3) / 1e9
    # A plain device copy moving the same bytes (half read, half written),
    # timed the same way: what HBM gives a transfer of this size.
    src = torch.empty(byts // 2, dtype=torch.uint8, device=dev)
    dst = torch.empty_like(src)
    copy_ms = timed(lambda: dst.copy_(src))
    copy_gbs = byts / (copy_ms * 1e-3) / 1e9
    peaks_path = ROOT / "MEASURED_PEAKS.json"
    peak, peak_src = 6650.0, "fallback"
    if peaks_path.exists():
        peak, peak_src = float(json.loads(peaks_path.read_text())["hbm_gbs"]), "measured"
    line = {
        "metric": "qk_norm_rope_cache_GBps", "value": achieved, "unit": "GB/s", "n_gpus": 1,
        "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16" if dtype == torch.float16 else "bf16",
        "data": "synthetic",
        "config": {"workload": "fused Qwen3 attention prologue: q/k RMSNorm + RoPE + KV write, "
                               f"{tokens} tokens, 16/8/128, random slots over a {nb}-block pool",
                   "l2": "L2 evicted (256 MB read) before every timed step"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": None, "peak_source": peak_src,
                     "kernel": "qk_prologue_kernel", "bytes_per_launch": byts,
                     "same_size_copy": {"GBps": copy_gbs, "frac": achieved / copy_gbs,
                                        "what": "torch copy_ of %d MB into %d MB, L2 evicted, timed alike"
                                                % (byts // 2 // 1000000, byts // 2 // 1000000)}},
        "gpu_launches": args.steps, "clocks": clock_info,
    }
    print(json.dumps(line), flush=True)


def _hbm_peak() -> tuple[float, str]:
    peaks_path = ROOT / "MEASURED_PEAKS.json"
    if peaks_path.exists():
        return float(json.loads(peaks_path.read_text())["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# ---------------------------------------------------------------- sampler
def run_sample(args) -> None:
    """Batched device sampler (mvb_sample): one token for each of 256 rows of a
    151936-token vocabulary (Qwen3; one row per decode sequence of config 2),
    bf16 logits unless --dtype; a quarter of the rows greedy, a quarter top-k
    50, a quarter top-p 0.9, a quarter both, temperature 0.8."""

    import numpy as np
    import torch

    from micro_vllm_b200 import sample_tokens

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    dtype = torch.float16 if args.dtype == "fp16" else torch.bfloat16
    rows, vocab = BATCH_PER_GPU, 151936
    g = torch.Generator(device=dev).manual_seed(9)
    logits = (torch.randn((rows, vocab), generator=g, device=dev) * 2.0).to(dtype)
    r = torch.arange(rows, device=dev)
    temperature = torch.where(r % 4 == 0, 0.0, 0.8).float()
    top_k = torch.where((r % 4 == 1) | (r % 4 == 3), 50, 0).int()
    top_p = torch.where(r % 4 >= 2, 0.9, 1.0).float()
    seed, index = r * 7 + 1, r.clone()
    out = torch.empty(rows, dtype=torch.int64, device=dev)
    step = lambda: sample_tokens(logits, temperature, top_k, top_p, seed, index, out=out)  # noqa: E731
    stream = torch.cuda.current_stream(dev)
    # 78 MB of logits fit in the 126 MB L2: evict them before every timed step
    # by reading a 256 MB buffer.
    flush = torch.ones(64 * 1024 * 1024, dtype=torch.float32, device=dev)
    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize(dev)
    clocks = ClockSampler(dev.index)
    clocks.start()
    clocks.wait_first()
    total = 0.0
    for _ in range(args.steps):
        flush.max()
        torch.cuda._sleep(1_000_000)  # ~0.5 ms: GPU busy while the host enqueues the event and the launch
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        step()
        b.record(stream)
        torch.cuda.synchronize(dev)
        total += a.elapsed_time(b)
    clock_info = clocks.stop()
    ms = total / args.steps
    byts = rows * vocab * logits.element_size()
    achieved = byts / (ms * 1e-3) / 1e9

    # End to end: logits from pinned host memory, tokens back to the host.
    host_logits = logits.cpu().pin_memory()
    params = [t.cpu().pin_memory() for t in (temperature, top_k, top_p, seed, index)]
    host_out = torch.empty(rows, dtype=torch.int64).pin_memory()
    h2d = host_logits.numel() * host_logits.element_size() + sum(t.numel() * t.element_size() for t in params)

    def serial_step(i: int) -> None:
        dl = host_logits.to(dev, non_blocking=True)
        dp = [t.to(dev, non_blocking=True) for t in params]
        host_out.copy_(sample_tokens(dl, *dp), non_blocking=True)

    # Pipelined: logits and parameters in one pinned buffer per slot, one
    # upload per step on its own stream, overlapping the neighbouring steps'
    # sampling and read-back.
    from micro_vllm_b200.staging import UploadPipeline

    names = ("logits", "temperature", "top_k", "top_p", "seed", "index")
    pipe = UploadPipeline(dev)
    for j in range(2):
        pipe.slot(j).pack(dict(zip(names, (host_logits, *params))))
    host_outs = [torch.empty(rows, dtype=torch.int64).pin_memory() for _ in range(2)]

    def pipelined_step(i: int) -> None:
        d = pipe.upload(i)
        pipe.download(i, sample_tokens(*(d[n] for n in names)), host_outs[i % 2])

    def e2e_time(fn, finish=None) -> float:
        for i in range(3):
            fn(i)
        if finish is not None:
            finish()
        torch.cuda.synchronize(dev)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for i in range(args.steps):
            fn(i)
        if finish is not None:
            finish()
        b.record(stream)
        torch.cuda.synchronize(dev)
        return a.elapsed_time(b) / args.steps

    serial_ms = e2e_time(serial_step)
    e2e_ms = e2e_time(pipelined_step, pipe.drain)

    # CPU baseline: the oracle's row policy (numpy) on a bounded sample of rows.
    from oracle.sampler import greedy, kept_and_probabilities

    host = logits[:32].float().cpu().numpy()
    rng = np.random.default_rng(0)
    done, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < min(args.cpu_sample_seconds, 10.0):
        i = done % len(host)
        if i % 4 == 0:
            greedy(host[i])
        else:
            kept, probs = kept_and_probabilities(host[i], 0.8, 50 if i % 4 in (1, 3) else None,
                                                 0.9 if i % 4 >= 2 else 1.0)
            rng.choice(vocab, p=probs)
        done += 1
    cpu_s = time.perf_counter() - t0
    peak, peak_src = _hbm_peak()
    line = {
        "metric": "sampler_logits_GBps", "value": achieved, "unit": "GB/s", "n_gpus": 1,
        "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16" if dtype == torch.bfloat16 else "f16",
        "data": "synthetic",
        "config": {"workload": f"batched sampler: {rows} rows x {vocab} vocab, greedy / top-k 50 / top-p 0.9 / "
                               "both, temperature 0.8, Philox draws",
                   "rows_per_s": rows / (ms * 1e-3),
                   "l2": "L2 evicted (256 MB read) before every timed step"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": None, "peak_source": peak_src,
                     "kernel": "sample_kernel", "bytes_per_launch": byts},
        "e2e": {"value": byts / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": rows * 8, "ms_per_step": e2e_ms,
                "what": "sample_tokens on logits and parameters uploaded each step from one pinned buffer "
                        "(one copy), tokens read back to pinned memory; uploads and read-backs pipelined "
                        "against the neighbouring steps (UploadPipeline)",
                "serial": {"value": byts / (serial_ms * 1e-3) / 1e9, "ms_per_step": serial_ms,
                           "what": "one copy per tensor, the step and the read-back in turn on one stream"}},
        "cpu_baseline": {"value": done * vocab * logits.element_size() / cpu_s / 1e9, "unit": "GB/s", "cores": 1,
                         "kind": "port",
                         "sample": f"{done} rows of the same logits through oracle/sampler.py (numpy) in "
                                   f"{cpu_s:.1f}s, {cpu_s / done * 1e3:.2f} ms/row"},
        "gpu_launches": args.steps, "clocks": clock_info,
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- metadata
def run_metadata(args) -> None:
    """Device-side metadata build (mvb_build_metadata) of a config-2 step: 256
    decode requests, ctx U[512,4096], block size 16, one full-attention cache
    group, block ids drawn without replacement from an 80%-of-HBM pool."""

    import numpy as np
    import torch

    from micro_vllm_b200 import DeviceMetadataBuilder, FullAttentionSpec, _lib
    from oracle.metadata import PlannedRequest
    from oracle.metadata import build as oracle_build

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    shape = DecodeShape(args)
    ctx = shape.lengths(shape.batch, seed=1000)
    pool = 2_340_000
    rng = np.random.default_rng(4)
    perm = iter(rng.permutation(pool - 1).tolist())

    class _Req:
        __slots__ = ("request_id", "input_token_ids", "num_computed_tokens", "num_scheduled_tokens",
                     "requires_sampling", "block_tables")

    class _Blocks:
        __slots__ = ("block_ids",)

    reqs = []
    for i, c in enumerate(ctx):
        q, b = _Req(), _Blocks()
        b.block_ids = tuple(next(perm) for _ in range(-(-c // BLOCK_SIZE)))
        q.request_id, q.input_token_ids = f"seq{i}", (int(rng.integers(0, 151936)),)
        q.num_computed_tokens, q.num_scheduled_tokens, q.requires_sampling = c - 1, 1, True
        q.block_tables = (b,)
        reqs.append(q)

    class _Plan:
        scheduled_requests = tuple(reqs)

    plan = _Plan()
    builder = DeviceMetadataBuilder([FullAttentionSpec()], BLOCK_SIZE, pool - 1, dev)
    stream = torch.cuda.current_stream(dev)
    for _ in range(max(args.warmup, 3)):
        builder.build(plan)
    torch.cuda.synchronize(dev)

    # Kernel alone: the packed plan already on the device, the launches
    # replayed from a CUDA graph so that the host's launch cost stays out.
    staged = builder.stage(plan)
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream(dev)
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        builder.launch(staged)  # warm the graph pool's allocations
    torch.cuda.synchronize(dev)
    with torch.cuda.graph(graph):
        for _ in range(args.steps):
            step = builder.launch(staged)
    graph.replay()
    torch.cuda.synchronize(dev)
    clocks = ClockSampler(dev.index)
    clocks.start()
    clocks.wait_first()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    graph.replay()
    b.record(stream)
    torch.cuda.synchronize(dev)
    kern_us = a.elapsed_time(b) / args.steps * 1e3
    del graph

    # End to end through the public call: pack + one upload + launch, and a
    # read of the step's last slot back to the host (a synchronisation).
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(args.steps):
        step = builder.build(plan)
        int(step.layer_attention_metadata[0].slot_mapping[-1])
    b.record(stream)
    torch.cuda.synchronize(dev)
    clock_info = clocks.stop()
    e2e_us = a.elapsed_time(b) / args.steps * 1e3
    assert builder.read_status() == 0

    r, t = len(reqs), len(reqs)
    w = max(-(-c // BLOCK_SIZE) for c in ctx)
    nblk = sum(-(-c // BLOCK_SIZE) for c in ctx)
    byts = staged.bytes + 8 * (4 * t + 2 * r + 1 + r * w + r)  # inputs read; int64 outputs written

    planned = [PlannedRequest(q.input_token_ids, q.num_computed_tokens, 1, True, (q.block_tables[0].block_ids,))
               for q in reqs]
    calls, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < min(args.cpu_sample_seconds, 5.0):
        oracle_build(planned, BLOCK_SIZE, pool - 1, [("full", 0)])
        calls += 1
    cpu_us = (time.perf_counter() - t0) / calls * 1e6
    peak, peak_src = _hbm_peak()
    achieved = byts / (kern_us * 1e-6) / 1e9
    line = {
        "metric": "metadata_build_us", "value": kern_us, "unit": "us/step", "n_gpus": 1,
        "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": kern_us / 1e3,
        "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "int64",
        "data": "synthetic",
        "config": {"workload": f"metadata of a config-2 step: {r} decode requests, ctx {shape.ctx_label}, "
                               f"{nblk} block ids, table {r}x{w}, one full-attention group",
                   "l2": "inputs and outputs under 1 MB (L2-resident): a launch-latency-bound kernel"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": None, "peak_source": peak_src, "kernel": "build_metadata_kernel",
                     "bytes_per_launch": byts,
                     "note": "a few-us kernel timed in a CUDA graph: bound by launch latency and one "
                             "grid-wide pass over sub-MB data, not bandwidth"},
        "e2e": {"value": e2e_us, "unit": "us/step", "h2d_bytes_per_step": staged.bytes, "d2h_bytes_per_step": 8,
                "what": "DeviceMetadataBuilder.build(plan) from the plan's Python objects: host packing, one "
                        "pinned upload, the launch, and a read back of the last slot"},
        "cpu_baseline": {"value": cpu_us, "unit": "us/step", "cores": 1, "kind": "port",
                         "sample": f"the whole step through oracle/metadata.py (numpy restatement of the "
                                   f"reference's host build), {calls} calls"},
        "gpu_launches": 2 * args.steps, "clocks": clock_info,
    }
    print(json.dumps(line), flush=True)
    del step


def main() -> None:
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "mixed":
        run_mixed(args)
    elif args.workload == "layers":
        run_layers(args)
    elif args.workload == "prologue":
        run_prologue(args)
    elif args.workload == "sample":
        run_sample(args)
    elif args.workload == "metadata":
        run_metadata(args)
    elif args.workload == "engine":
        run_engine_workload(args)
    else:
        line = run_ours(args)
        if not args.no_engine and args.workload == "decode":
            import gc

            import torch

            gc.collect()
            torch.cuda.empty_cache()  # the decode pool goes back before the engine sizes its cache
            line["engine"] = engine_measure(args)
        finish_ranks()
        if int(os.environ.get("RANK", "0")) == 0:
            print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
