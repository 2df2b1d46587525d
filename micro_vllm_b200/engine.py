"""The reference's engine with the B200 pieces plugged in where they fit.

Nothing of the reference is edited: ``register()`` makes ``"b200_paged"`` a
selectable operator, and ``B200ModelRunner`` derives from the reference's
``ModelRunner`` (src/micro_vllm/worker/model_runner.py:125-900), replacing
three host-side stages of its step with this package's kernels:

* ``_build_model_input`` and, under a CUDA graph, ``_CudaGraphExecution.copy_input``
  (model_runner.py:724-900, :78-122): the step's positions, token ids,
  query start locations, context lengths, padded block tables, slot
  mappings, visibility starts and sampling rows come from one pinned upload
  and one ``mvb_build_metadata`` launch per cache group
  (``DeviceMetadataBuilder``), written straight into the captured graph's
  fixed buffers with ``copy_input``'s padding;
* ``Sampler`` (sampling/sampler.py:14-61, one ``.item()`` per row): every
  row in one ``mvb_sample`` launch and one host read (``B200Sampler``);
* in Qwen3 layers, ``q_norm``, ``k_norm``, the rotary embedding and the
  operator's KV write (models/qwen.py:89-98) become one
  ``mvb_qk_norm_rope_and_cache`` launch, followed by attention over the cache
  (``B200PagedAttentionOperator.attend``);
* with ``fused_layers``, the rest of each Qwen3 decoder layer
  (models/qwen.py:136-156) runs in fewer launches: every RMSNorm as one
  ``mvb_rms_norm`` together with the residual add before it (the model's
  layer loop, models/qwen.py:220-240, carries each layer's last add into the
  next norm), q/k/v as one GEMM over their weights concatenated, gate/up as
  one GEMM and ``mvb_silu_mul`` (layers/mlp.py:19-21).  The reference's
  Linear modules keep working: their weights become views into the
  concatenated ones.

The scheduler, KV block manager, request state, engine loop and the GEMMs
are the reference's, unchanged.
``B200Worker`` is the reference ``Worker`` around a ``B200ModelRunner``
(``build_worker``); ``fresh_engine`` assembles
``Engine(Scheduler, SingleProcessExecutor(worker))`` as ``LLM.__init__`` does
(llm.py:54-77).

This module imports micro_vllm; import it only where the reference is
installed.
"""

from __future__ import annotations

import json
import math
import time
import types
from dataclasses import dataclass
from pathlib import Path
from typing import Sequence

import torch

from micro_vllm.config import LLMConfig
from micro_vllm.core.kv_cache_manager import KVCacheManager
from micro_vllm.core.scheduler import Scheduler
from micro_vllm.engine.engine import Engine
from micro_vllm.executor.single_process import SingleProcessExecutor
from micro_vllm.sampling.params import SamplingParams
from micro_vllm.worker.model_runner import ModelRunner, _CudaGraphExecution
from micro_vllm.worker.worker import Worker

from micro_vllm_b200.integration import register
from micro_vllm_b200.layers import rms_norm, silu_mul
from micro_vllm_b200.metadata import DeviceMetadataBuilder
from micro_vllm_b200.operators import B200PagedAttentionOperator
from micro_vllm_b200.prologue import Qwen3AttentionPrologue
from micro_vllm_b200.sampling import B200Sampler


@dataclass(frozen=True, slots=True)
class RunnerOptions:
    """Which reference stages ``B200ModelRunner`` replaces."""

    device_metadata: bool = True
    device_sampler: bool = True
    fused_prologue: bool = True
    fused_layers: bool = True


class B200ModelRunner(ModelRunner):
    """``ModelRunner`` with the device metadata build, the batched sampler and
    the fused Qwen3 prologue (see the module docstring)."""

    def __init__(self, config: LLMConfig, options: RunnerOptions = RunnerOptions()) -> None:
        super().__init__(config)
        self._options = options
        self._eager_builders: dict[int, DeviceMetadataBuilder] = {}
        self._graph_builders: dict[int, DeviceMetadataBuilder] = {}
        if options.device_sampler:
            self._sampler = B200Sampler()

    # -- model -------------------------------------------------------------
    def initialize_model(self) -> None:
        super().initialize_model()
        if self._options.fused_prologue:
            self._install_prologue()
            if self._options.fused_layers:
                self._install_fused_layers()

    def _b200_operators(self) -> list[B200PagedAttentionOperator]:
        seen: dict[int, B200PagedAttentionOperator] = {}
        for attention in self._model.layer_attentions:
            if isinstance(attention.operator, B200PagedAttentionOperator):
                seen.setdefault(id(attention.operator), attention.operator)
        return list(seen.values())

    def _install_prologue(self) -> None:
        """Route every Qwen3 attention module whose operator is ``b200_paged``
        through the fused prologue (fp16 / bf16 only)."""

        head_dim = self._config.model_config.values.get("head_dim")
        if self._dtype not in (torch.float16, torch.bfloat16) or head_dim != 128:
            return
        try:
            from micro_vllm.models.qwen import Qwen3Attention
        except ImportError:
            return
        for module in self._model.modules():
            if not isinstance(module, Qwen3Attention):
                continue
            if not isinstance(module.attention.operator, B200PagedAttentionOperator):
                continue
            module._b200_prologue = Qwen3AttentionPrologue.from_modules(
                module.q_norm, module.k_norm, module.rotary_embedding)
            module.forward = types.MethodType(_qwen3_attention_forward, module)

    def _install_fused_layers(self) -> None:
        """Fewer launches per Qwen3 decoder layer (module docstring), for
        layers whose attention runs the fused prologue, in fp16 / bf16, with
        bias-free projections and 16-bit norm weights of the model's dtype."""

        dtype = self._dtype
        if dtype not in (torch.float16, torch.bfloat16):
            return  # the fused kernels take 16-bit rows only
        try:
            from micro_vllm.layers.normalization import RMSNorm
            from micro_vllm.models.qwen import Qwen3DecoderLayer
        except ImportError:
            return

        def fusable_norm(norm) -> bool:
            w = norm.weight
            return w.dtype == dtype and w.dim() == 1 and w.shape[0] % 8 == 0

        with torch.no_grad():
            for layer in self._model.modules():
                if not isinstance(layer, Qwen3DecoderLayer):
                    continue
                attn, mlp = layer.self_attn, layer.mlp
                if getattr(attn, "_b200_prologue", None) is None:
                    continue
                projections = (attn.q_proj, attn.k_proj, attn.v_proj, mlp.gate_proj, mlp.up_proj)
                if any(getattr(m, "bias", None) is not None for m in projections):
                    continue
                if not (fusable_norm(layer.input_layernorm) and fusable_norm(layer.post_attention_layernorm)):
                    continue
                if mlp.gate_proj.weight.shape[0] % 8 != 0:
                    continue
                attn._b200_qkv = _concatenate_weights(attn.q_proj, attn.k_proj, attn.v_proj)
                mlp._b200_gate_up = _concatenate_weights(mlp.gate_proj, mlp.up_proj)
                mlp._b200_inter = int(mlp.gate_proj.weight.shape[0])
                attn.forward = types.MethodType(_qwen3_attention_forward_qkv, attn)
                layer.forward = types.MethodType(_qwen3_layer_forward, layer)
            for norm in self._model.modules():
                if isinstance(norm, RMSNorm) and fusable_norm(norm):
                    norm.forward = types.MethodType(_rms_norm_forward, norm)
            # With every layer fused, each layer's last residual add moves
            # into the next layer's input norm (and the last one into the
            # final norm): one launch fewer per layer.
            model = self._model
            layers = list(getattr(model, "layers", ()))
            if (layers and all(getattr(layer.mlp, "_b200_gate_up", None) is not None for layer in layers)
                    and isinstance(getattr(model, "norm", None), RMSNorm) and fusable_norm(model.norm)
                    and hasattr(model, "embed_tokens")):
                model.forward = types.MethodType(_qwen3_model_forward, model)
        torch.cuda.empty_cache()

    # -- step inputs ---------------------------------------------------------
    def _layer_specs(self) -> list:
        return [attention.spec for attention in self._model.layer_attentions]

    def _build_model_input(self, plan, null_block_id: int):
        if not self._options.device_metadata:
            return super()._build_model_input(plan, null_block_id)
        builder = self._eager_builders.get(null_block_id)
        if builder is None:
            builder = DeviceMetadataBuilder(
                self._layer_specs(), self._block_size, null_block_id, self._device)
            self._eager_builders[null_block_id] = builder
        return builder.build(plan)

    def _make_cuda_graph_input(self, num_tokens: int, num_requests: int, null_block_id: int):
        if not self._options.device_metadata:
            return super()._make_cuda_graph_input(num_tokens, num_requests, null_block_id)
        width = math.ceil(self._config.scheduler_config.max_model_len / self._block_size)
        builder = DeviceMetadataBuilder(
            self._layer_specs(), self._block_size, null_block_id, self._device,
            token_capacity=num_tokens, request_capacity=num_requests, table_width=width)
        self._graph_builders[num_tokens] = builder
        # The captured forward reads these buffers: start from copy_input's
        # padding of an empty batch (model_runner.py:78-122).
        return builder.build_empty()

    def _capture_cuda_graphs(self, layout, kv_cache_buffers):
        scheduler = self._config.scheduler_config
        values = self._config.model_config.values
        hq = int(values["num_attention_heads"])
        hkv = int(values.get("num_key_value_heads", hq))
        head_dim = int(values.get("head_dim") or int(values["hidden_size"]) // hq)
        for operator in self._b200_operators():
            operator.reserve(
                self._device, max_num_tokens=scheduler.max_num_batched_tokens,
                max_num_requests=scheduler.max_num_seqs, num_q_heads=hq,
                num_kv_heads=hkv, head_dim=head_dim)
        return super()._capture_cuda_graphs(layout, kv_cache_buffers)

    # -- one step ----------------------------------------------------------------
    def execute(self, plan, /):
        if not self._options.device_metadata:
            return super().execute(plan)
        model = self._model
        kv_cache_buffers = self._kv_cache_buffers
        if model is None or kv_cache_buffers is None:
            raise RuntimeError("model runner is not initialized")
        null_block_id = self._kv_cache_layout.num_blocks - 1
        num_tokens = sum(request.num_scheduled_tokens for request in plan.scheduled_requests)
        graph_size = self._graph_size(num_tokens)
        layer_kv_caches = self._bind_layer_kv_caches(kv_cache_buffers)
        with torch.inference_mode():
            if graph_size is None:
                model_input = self._build_model_input(plan, null_block_id)
                hidden_states = self._forward_model(model_input, layer_kv_caches)
            else:
                model_input = self._graph_builders[graph_size].build(plan)
                execution: _CudaGraphExecution = self._cuda_graph_executions[graph_size]
                execution.graph.replay()
                hidden_states = execution.hidden_states
            logits = self._compute_logits(hidden_states, model_input.sampling_row_indices)
        sampled = tuple(request for request in plan.scheduled_requests if request.requires_sampling)
        return self._sampler(
            logits,
            tuple(request.request_id for request in sampled),
            tuple(request.sampling_params for request in sampled),
            tuple(request.sample_index for request in sampled),
        )

    def _graph_size(self, num_tokens: int) -> int | None:
        if num_tokens == 0:
            return None
        for size in sorted(self._cuda_graph_executions):
            if num_tokens <= size:
                return size
        return None


def _qwen3_attention_forward(self, hidden_states, positions, layer_kv_cache, metadata):
    """``Qwen3Attention.forward`` (models/qwen.py:69-98) with q/k norm, RoPE and
    the KV write fused into one launch, then attention over the cache."""

    query = self.q_proj(hidden_states).view(-1, self.num_attention_heads, self.head_dim)
    key = self.k_proj(hidden_states).view(-1, self.num_key_value_heads, self.head_dim)
    value = self.v_proj(hidden_states).view(-1, self.num_key_value_heads, self.head_dim)
    query = self._b200_prologue(positions, query, key, value, layer_kv_cache, metadata)
    attention_output = self.attention.operator.attend(query, layer_kv_cache, metadata)
    return self.o_proj(attention_output.flatten(start_dim=1))


def _concatenate_weights(*linears) -> torch.Tensor:
    """One [sum of out features, in features] weight; each module's weight
    becomes a view of its rows, so the concatenation costs no memory."""

    joined = torch.cat([m.weight.data for m in linears], dim=0)
    row = 0
    for m in linears:
        n = m.weight.shape[0]
        m.weight.data = joined[row:row + n]
        row += n
    return joined


def _rms_norm_forward(self, hidden_states):
    """``RMSNorm.forward`` (layers/normalization.py:15-22) as one launch; rows
    the kernel does not take (another dtype than the weight's 16-bit one, an
    unaligned view) run the reference's own forward."""

    shape = hidden_states.shape
    rows = hidden_states.reshape(-1, shape[-1])
    if (hidden_states.dtype != self.weight.dtype or not hidden_states.is_cuda or rows.stride(-1) != 1
            or rows.stride(0) % 8 != 0 or rows.data_ptr() % 16 != 0):
        return type(self).forward(self, hidden_states)
    out, _ = rms_norm(rows, self.weight, self.variance_epsilon)
    return out.view(shape)


def _qwen3_attention_forward_qkv(self, hidden_states, positions, layer_kv_cache, metadata):
    """``_qwen3_attention_forward`` with q, k and v from one GEMM over the
    concatenated projection weights (views of its output feed the prologue)."""

    qkv = torch.nn.functional.linear(hidden_states, self._b200_qkv)
    nq = self.num_attention_heads * self.head_dim
    nk = self.num_key_value_heads * self.head_dim
    query = qkv[:, :nq].view(-1, self.num_attention_heads, self.head_dim)
    key = qkv[:, nq:nq + nk].view(-1, self.num_key_value_heads, self.head_dim)
    value = qkv[:, nq + nk:nq + 2 * nk].view(-1, self.num_key_value_heads, self.head_dim)
    query = self._b200_prologue(positions, query, key, value, layer_kv_cache, metadata)
    attention_output = self.attention.operator.attend(query, layer_kv_cache, metadata)
    return self.o_proj(attention_output.flatten(start_dim=1))


def _qwen3_layer_forward(self, hidden_states, positions, layer_kv_cache, metadata):
    """``Qwen3DecoderLayer.forward`` (models/qwen.py:136-156): the same sums,
    norms and products, in fewer launches."""

    x = self.input_layernorm(hidden_states)
    attention = self.self_attn(x, positions, layer_kv_cache, metadata)
    # residual + attention, and the post-attention norm of it, in one launch.
    norm = self.post_attention_layernorm
    x, hidden = rms_norm(attention, norm.weight, norm.variance_epsilon, residual=hidden_states)
    mlp = self.mlp
    gate_up = torch.nn.functional.linear(x, mlp._b200_gate_up)
    return hidden + mlp.down_proj(silu_mul(gate_up, mlp._b200_inter))


def _qwen3_layer_step(self, hidden_states, pending, positions, layer_kv_cache, metadata):
    """One fused decoder layer that leaves its MLP output unadded: returns
    (h, m) with the layer's output h + m; the caller adds them in the next
    norm.  ``pending`` is the previous layer's m (None for the first)."""

    norm = self.input_layernorm
    if pending is None:
        x, hidden = rms_norm(hidden_states, norm.weight, norm.variance_epsilon)
    else:  # residual + hidden_states of the previous layer (models/qwen.py:156)
        x, hidden = rms_norm(pending, norm.weight, norm.variance_epsilon, residual=hidden_states)
    attention = self.self_attn(x, positions, layer_kv_cache, metadata)
    norm = self.post_attention_layernorm
    x, hidden = rms_norm(attention, norm.weight, norm.variance_epsilon, residual=hidden)
    mlp = self.mlp
    gate_up = torch.nn.functional.linear(x, mlp._b200_gate_up)
    return hidden, mlp.down_proj(silu_mul(gate_up, mlp._b200_inter))


def _qwen3_model_forward(self, input_ids, positions, layer_kv_caches, layer_attention_metadata):
    """``Qwen3Model.forward`` (models/qwen.py:220-240) over fused layers, the
    residual adds carried into the following norms."""

    hidden = self.embed_tokens(input_ids)
    pending = None
    for layer, layer_kv_cache, metadata in zip(self.layers, layer_kv_caches, layer_attention_metadata,
                                               strict=True):
        hidden, pending = _qwen3_layer_step(layer, hidden, pending, positions, layer_kv_cache, metadata)
    if pending is None:
        return self.norm(hidden)
    out, _ = rms_norm(pending, self.norm.weight, self.norm.variance_epsilon, residual=hidden)
    return out


class B200Worker(Worker):
    """The reference ``Worker`` (worker/worker.py:10-54) around a ``B200ModelRunner``."""

    __slots__ = ()

    def __init__(self, config: LLMConfig, options: RunnerOptions = RunnerOptions()) -> None:
        runner = B200ModelRunner(config, options)
        runner.initialize_model()
        runner.initialize_kv_cache()
        self._config = config
        self._model_runner = runner


def build_worker(config: LLMConfig, options: RunnerOptions | None = RunnerOptions()) -> Worker:
    """A worker for ``config``: ``B200Worker`` when the operator is
    ``b200_paged`` and ``options`` is given, else the reference's ``Worker``."""

    register()
    if options is not None and config.model_config.attention_operator == "b200_paged":
        return B200Worker(config, options)
    return Worker(config)


def fresh_engine(worker: Worker, config: LLMConfig) -> Engine:
    """A new ``Engine`` (fresh Scheduler and KVCacheManager) over an initialised
    worker, as the reference's engine benchmark builds one per repetition
    (benchmarks/benchmark_engine.py:146-153)."""

    scheduler = Scheduler(config, KVCacheManager(config, worker.kv_cache_layout))
    return Engine(scheduler, SingleProcessExecutor(worker))


# -- the engine workload ---------------------------------------

QWEN3_0_6B = {
    "architectures": ["Qwen3ForCausalLM"],
    "model_type": "qwen3",
    "vocab_size": 151936,
    "hidden_size": 1024,
    "intermediate_size": 3072,
    "num_hidden_layers": 28,
    "num_attention_heads": 16,
    "num_key_value_heads": 8,
    "head_dim": 128,
    "max_position_embeddings": 40960,
    "rms_norm_eps": 1e-6,
    "rope_theta": 1000000.0,
    "hidden_act": "silu",
    "tie_word_embeddings": True,
    "attention_bias": False,
    "attention_dropout": 0.0,
    "use_sliding_window": False,
    "torch_dtype": "float16",
}


def qwen3_tensor_shapes(values: dict) -> dict[str, tuple[int, ...]]:
    """Checkpoint tensor names and shapes of a dense Qwen3 model, in the
    Hugging Face naming the reference loader maps (models/qwen.py:248-262)."""

    h = values["hidden_size"]
    i = values["intermediate_size"]
    hq, hkv, d = values["num_attention_heads"], values["num_key_value_heads"], values["head_dim"]
    shapes = {"model.embed_tokens.weight": (values["vocab_size"], h), "model.norm.weight": (h,)}
    if not values.get("tie_word_embeddings", False):
        shapes["lm_head.weight"] = (values["vocab_size"], h)
    for layer in range(values["num_hidden_layers"]):
        p = f"model.layers.{layer}."
        shapes.update({
            p + "self_attn.q_proj.weight": (hq * d, h),
            p + "self_attn.k_proj.weight": (hkv * d, h),
            p + "self_attn.v_proj.weight": (hkv * d, h),
            p + "self_attn.o_proj.weight": (h, hq * d),
            p + "self_attn.q_norm.weight": (d,),
            p + "self_attn.k_norm.weight": (d,),
            p + "mlp.gate_proj.weight": (i, h),
            p + "mlp.up_proj.weight": (i, h),
            p + "mlp.down_proj.weight": (h, i),
            p + "input_layernorm.weight": (h,),
            p + "post_attention_layernorm.weight": (h,),
        })
    return shapes


def write_random_checkpoint(path: str | Path, values: dict = QWEN3_0_6B, *, seed: int = 0,
                            dtype: torch.dtype = torch.float16, std: float = 0.02) -> Path:
    """A random-init checkpoint directory (``config.json`` + ``model.safetensors``)
    the reference loader reads: matrices N(0, std) (the Hugging Face
    initializer range), norm weights 1, drawn from one seeded CPU generator
    in name order, so the same seed gives the same model anywhere."""

    from safetensors.torch import save_file

    path = Path(path)
    path.mkdir(parents=True, exist_ok=True)
    gen = torch.Generator().manual_seed(seed)
    tensors = {}
    for name, shape in sorted(qwen3_tensor_shapes(values).items()):
        if name.endswith("norm.weight"):
            tensors[name] = torch.ones(shape, dtype=dtype)
        else:
            tensors[name] = (torch.randn(shape, generator=gen) * std).to(dtype)
    save_file(tensors, str(path / "model.safetensors"))
    (path / "config.json").write_text(json.dumps(values, indent=1, sort_keys=True))
    return path


@dataclass(frozen=True, slots=True)
class EngineRequest:
    request_id: str
    prompt_token_ids: tuple[int, ...]
    max_tokens: int


def engine_requests(num_requests: int = 512, *, prompt_range: tuple[int, int] = (128, 1024),
                    max_tokens: int = 256, vocab_size: int = 151936, seed: int = 0) -> list[EngineRequest]:
    """Seeded synthetic requests: prompt lengths U[lo, hi], token ids U[1, vocab-1]."""

    gen = torch.Generator().manual_seed(seed)
    lo, hi = prompt_range
    lengths = torch.randint(lo, hi + 1, (num_requests,), generator=gen).tolist()
    out = []
    for index, length in enumerate(lengths):
        ids = torch.randint(1, vocab_size, (length,), generator=gen).tolist()
        out.append(EngineRequest(f"request-{index}", tuple(ids), max_tokens))
    return out


@dataclass(frozen=True, slots=True)
class EngineRun:
    """One drive of the engine to completion."""

    seconds: float  # CUDA events around the loop
    wall_seconds: float  # host clock around the same loop
    steps: int
    output_tokens: int
    prompt_tokens: int
    outputs: dict[str, tuple[int, ...]]


def run_engine(engine: Engine, requests: Sequence[EngineRequest], device: torch.device,
               *, max_steps: int | None = None) -> EngineRun:
    """Add every request (greedy, ``ignore_eos``), then call ``Engine.step`` until
    none is unfinished; the time covers the step loop only, bracketed by
    CUDA events on the current stream with a device synchronisation at
    each end (the method of benchmarks/benchmark_engine.py:177-200, with the
    whole loop timed once instead of per step)."""

    for request in requests:
        engine.add_request(
            request.request_id, list(request.prompt_token_ids),
            SamplingParams(max_tokens=request.max_tokens, ignore_eos=True, temperature=0.0, seed=0),
        )
    limit = max_steps if max_steps is not None else 10 * sum(
        len(r.prompt_token_ids) + r.max_tokens for r in requests)
    outputs: dict[str, tuple[int, ...]] = {}
    stream = torch.cuda.current_stream(device)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(device)
    wall = time.perf_counter()
    start.record(stream)
    steps = 0
    while engine.has_unfinished_requests():
        if steps >= limit:
            raise RuntimeError(f"engine did not finish within {limit} steps")
        for output in engine.step():
            outputs[output.request_id] = output.output_token_ids
        steps += 1
    stop.record(stream)
    torch.cuda.synchronize(device)
    wall = time.perf_counter() - wall
    return EngineRun(
        seconds=start.elapsed_time(stop) / 1e3, wall_seconds=wall, steps=steps,
        output_tokens=sum(len(v) for v in outputs.values()),
        prompt_tokens=sum(len(r.prompt_token_ids) for r in requests),
        outputs=outputs,
    )
