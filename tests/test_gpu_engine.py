"""The reference's own engine and model runner with ``b200_paged`` plugged in.

Every test drives the reference package (installed under ``baseline/_ref``):
its Scheduler, KV block manager, Engine loop, Qwen3 model and, for the
comparison side, its stock ``ModelRunner`` with the reference operator
(src/micro_vllm/attention/operators/reference.py), all on the GPU.  The
B200 side is ``B200ModelRunner`` (device metadata build into the CUDA graph's
buffers, batched sampler, fused Qwen3 prologue) with ``b200_paged``.

The model is a small random-init Qwen3 with untied embeddings and 16/8 heads
of head_dim 128, so every step runs the tcgen05 prefill, the stream-K decode
and the fused prologue.  (With tied embeddings and the usual 0.02 init, a
random model just repeats its input token and greedy parity would be empty.)
"""

from __future__ import annotations

import pytest
import torch

from _reference import require_reference

pytestmark = pytest.mark.gpu

TINY = dict(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=4,
            tie_word_embeddings=False)


@pytest.fixture(scope="module")
def env(tmp_path_factory):
    require_reference()
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from micro_vllm_b200.engine import QWEN3_0_6B, write_random_checkpoint
    from micro_vllm_b200.integration import register

    register()
    path = write_random_checkpoint(tmp_path_factory.mktemp("tiny_qwen3"), dict(QWEN3_0_6B, **TINY),
                                   seed=1, std=0.08)
    return {"path": path, "device": torch.device("cuda", 0)}


def make_config(path, operator, graphs, dtype=torch.float16, *, max_seqs=8, max_len=512, tokens=256):
    from micro_vllm.config import CacheConfig, LLMConfig, ModelConfig, SchedulerConfig

    return LLMConfig(
        model_config=ModelConfig(model=str(path), attention_operator=operator, enable_cuda_graph=graphs,
                                 device="cuda", dtype=dtype),
        scheduler_config=SchedulerConfig(max_num_batched_tokens=tokens, max_num_seqs=max_seqs,
                                         max_model_len=max_len),
        # A fixed page count: earlier tests in the process may hold device memory.
        cache_config=CacheConfig(block_size=16, gpu_memory_utilization=0.9, num_blocks=2048),
    )


def requests(n=6, max_tokens=32, seed=3):
    from micro_vllm_b200.engine import engine_requests

    return engine_requests(n, prompt_range=(20, 300), max_tokens=max_tokens, vocab_size=TINY["vocab_size"],
                           seed=seed)


def drive(worker, config, reqs, device):
    from micro_vllm_b200.engine import fresh_engine, run_engine

    import gc

    try:
        return run_engine(fresh_engine(worker, config), reqs, device).outputs
    finally:
        worker.shutdown()
        gc.collect()
        torch.cuda.empty_cache()


def test_greedy_tokens_match_the_reference_operator(env):
    """Greedy generation through the reference engine: 6 requests, prompts of
    20-300 tokens under a 256-token step budget (chunked prefill), 32 output
    tokens each; identical with the reference operator, with ``b200_paged``
    in the stock runner, and through ``B200ModelRunner`` with CUDA graphs."""

    from micro_vllm_b200.engine import RunnerOptions, build_worker

    path, dev = env["path"], env["device"]
    reqs = requests()
    outputs = {}
    for name, operator, graphs, options in (
        ("reference", "reference", False, None),
        ("b200_stock_runner", "b200_paged", False, None),
        ("b200_runner_eager", "b200_paged", False, RunnerOptions()),
        ("b200_runner_graphs", "b200_paged", True, RunnerOptions()),
    ):
        config = make_config(path, operator, graphs)
        outputs[name] = drive(build_worker(config, options), config, reqs, dev)
    expected = outputs["reference"]
    assert all(len(v) == 32 for v in expected.values())
    assert len(set(expected.values())) == len(expected)  # a non-degenerate model
    for name, got in outputs.items():
        assert got == expected, f"{name} differs from the reference operator"


def test_fp32_model_keeps_the_reference_layers(env):
    """An fp32 model through ``B200ModelRunner``: the fused prologue and layer
    stages take 16-bit rows only, so none is installed (no RMSNorm module
    gets a replaced forward) and the model runs the reference's own layers
    over ``b200_paged``'s exact fp32 path; greedy tokens equal the reference
    operator's."""

    from micro_vllm_b200.engine import RunnerOptions, build_worker

    path, dev = env["path"], env["device"]
    reqs = requests(n=3, max_tokens=8)
    outputs = {}
    for name, operator, options in (("reference", "reference", None), ("b200_runner", "b200_paged", RunnerOptions())):
        config = make_config(path, operator, False, torch.float32)
        worker = build_worker(config, options)
        if options is not None:
            model = worker._model_runner._model
            assert not any("forward" in vars(m) for m in model.modules() if type(m).__name__ == "RMSNorm")
        outputs[name] = drive(worker, config, reqs, dev)
    assert outputs["b200_runner"] == outputs["reference"]


class ScriptedSampler:
    """Records each row's logits and returns a fixed token per (request, sample
    index), so two runners see the same token streams whatever they compute."""

    def __init__(self, vocab):
        self.vocab = vocab
        self.logits = {}

    def __call__(self, logits, request_ids, sampling_params, sample_indices, /):
        from micro_vllm.executor.interface import ModelRunnerOutput, SampledToken

        out = []
        rows = logits.float().cpu()
        for row, rid, index in zip(rows, request_ids, sample_indices):
            self.logits[(rid, index)] = row
            out.append(SampledToken(rid, (sum(map(ord, rid)) % 97 + 31 * index) % self.vocab))
        return ModelRunnerOutput(tuple(out))


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_teacher_forced_logits_match_the_reference_operator(env, dtype):
    """Every step's logits of ``B200ModelRunner`` (graphs) against the stock
    runner with the reference operator, on identical token streams."""

    from micro_vllm_b200.engine import RunnerOptions, build_worker

    path, dev = env["path"], env["device"]
    reqs = requests(n=5, max_tokens=12, seed=5)
    recorded = {}
    for name, operator, graphs, options in (
        ("reference", "reference", False, None),
        ("b200", "b200_paged", True, RunnerOptions()),
    ):
        config = make_config(path, operator, graphs, dtype)
        worker = build_worker(config, options)
        sampler = ScriptedSampler(TINY["vocab_size"])
        worker._model_runner._sampler = sampler
        drive(worker, config, reqs, dev)
        recorded[name] = sampler.logits
    assert recorded["reference"].keys() == recorded["b200"].keys()
    assert len(recorded["reference"]) == 5 * 12
    ref = torch.stack([recorded["reference"][k] for k in sorted(recorded["reference"])])
    got = torch.stack([recorded["b200"][k] for k in sorted(recorded["reference"])])
    scale = ref.abs().max().item()
    err = (got - ref).abs().max().item()
    # fp16 / bf16 activations through 4 layers: a few ulps of the logits' scale.
    tol = (4e-3 if dtype == torch.float16 else 3e-2) * scale
    assert err <= tol, f"max |logit difference| {err:.4g} > {tol:.4g} (logit scale {scale:.3g})"
    assert (got.argmax(-1) == ref.argmax(-1)).float().mean().item() >= 0.95


def _hybrid_worker(config, options, window):
    """A worker whose odd layers use a sliding window: two cache groups whose
    layers share physical page buffers (model_runner.py:707-722)."""

    from micro_vllm.attention.attention import Attention
    from micro_vllm.attention.spec import SlidingWindowSpec
    from micro_vllm.core.kv_cache_spec import build_kv_cache_topology
    from micro_vllm.worker.model_runner import ModelRunner
    from micro_vllm.worker.worker import Worker

    from micro_vllm_b200.engine import B200ModelRunner, B200Worker

    runner = B200ModelRunner(config, options) if options is not None else ModelRunner(config)
    runner.initialize_model()
    model = runner._model
    windowed = Attention(SlidingWindowSpec(window), config.model_config.attention_operator)
    attentions = list(model.layer_attentions)
    for index, layer in enumerate(model.layers):
        if index % 2:
            layer.self_attn.attention = windowed
            attentions[index] = windowed
    model.layer_attentions = tuple(attentions)
    runner._kv_cache_topology = build_kv_cache_topology(tuple(a.spec for a in attentions))
    runner.initialize_kv_cache()
    worker_class = B200Worker if options is not None else Worker
    worker = worker_class.__new__(worker_class)  # Worker.__init__ builds its own runner
    worker._config = config
    worker._model_runner = runner
    return worker


def test_cache_groups_sharing_page_buffers(env):
    """Full-attention and sliding-window layers in two cache groups, each
    pair of layers on ONE physical page buffer at its own group's block ids;
    greedy outputs equal the reference operator's."""

    from micro_vllm_b200.engine import RunnerOptions

    path, dev = env["path"], env["device"]
    reqs = requests(n=5, max_tokens=24, seed=7)
    outputs = {}
    for name, operator, graphs, options in (
        ("reference", "reference", False, None),
        ("b200", "b200_paged", True, RunnerOptions()),
    ):
        config = make_config(path, operator, graphs)
        worker = _hybrid_worker(config, options, window=40)
        layout = worker.kv_cache_layout
        assert len(layout.groups) == 2 and layout.page_layer_count == 2
        runner = worker._model_runner
        caches = runner._bind_layer_kv_caches(runner._kv_cache_buffers)
        assert caches[0] is caches[1] and caches[2] is caches[3] and caches[0] is not caches[2]
        outputs[name] = drive(worker, config, reqs, dev)
    assert outputs["b200"] == outputs["reference"]


def test_cuda_graph_replays_a_padded_mixed_batch(env, monkeypatch):
    """The reference's own graph test (tests/worker/test_model_runner_execution.py:414-486)
    with ``b200_paged`` and ``B200ModelRunner``: the metadata builder writes the
    step into the captured buffers with ``copy_input``'s padding."""

    import micro_vllm.worker.model_runner as model_runner_module
    from micro_vllm.attention.attention import Attention
    from micro_vllm.attention.spec import FullAttentionSpec
    from micro_vllm.config import CacheConfig, LLMConfig, ModelConfig, SchedulerConfig
    from micro_vllm.core.scheduler_output import CacheGroupBlockTable, ScheduledRequest, SchedulerOutput
    from micro_vllm.sampling.params import SamplingParams

    from micro_vllm_b200.engine import B200ModelRunner

    class GraphableModel(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.layer_attentions = (Attention(FullAttentionSpec(), "b200_paged"),)
            self.config = ModelConfig(model="unused", metadata={
                "architectures": ["LlamaForCausalLM"], "vocab_size": 64, "hidden_size": 8,
                "intermediate_size": 16, "num_hidden_layers": 1, "num_attention_heads": 2,
                "num_key_value_heads": 1, "max_position_embeddings": 32})
            self.embedding = torch.nn.Embedding(64, 64)
            with torch.no_grad():
                self.embedding.weight.copy_(torch.eye(64))

        def forward(self, input_ids, positions, layer_kv_caches, layer_attention_metadata):
            return self.embedding(input_ids)

        def compute_logits(self, hidden_states):
            return hidden_states

    monkeypatch.setattr(model_runner_module, "load_model", lambda config: GraphableModel())
    runner = B200ModelRunner(LLMConfig(
        model_config=ModelConfig(model="unused", device="cuda", dtype=torch.float16,
                                 attention_operator="b200_paged", enable_cuda_graph=True),
        cache_config=CacheConfig(block_size=2, num_blocks=8),
        scheduler_config=SchedulerConfig(max_num_batched_tokens=4, max_num_seqs=2, max_model_len=8),
    ))
    runner.initialize_model()
    runner.initialize_kv_cache()
    execution = runner._cuda_graph_executions[4]

    def request(rid, tokens, computed, block_ids):
        return ScheduledRequest(
            request_id=rid, input_token_ids=tokens, num_computed_tokens=computed,
            num_scheduled_tokens=len(tokens), requires_sampling=True,
            block_tables=(CacheGroupBlockTable(block_ids),), sampling_params=SamplingParams(max_tokens=4),
            sample_index=0)

    first = runner.execute(SchedulerOutput((request("first", (7,), 1, (0,)),
                                            request("second", (11, 12), 0, (1,)))))
    second = runner.execute(SchedulerOutput((request("first", (13,), 2, (0, 2)),
                                             request("second", (17, 19), 0, (1,)))))
    assert runner._cuda_graph_executions[4] is execution
    assert [s.token_id for s in first.sampled_tokens] == [7, 12]
    assert [s.token_id for s in second.sampled_tokens] == [13, 19]
    assert execution.model_input.input_ids.tolist() == [13, 17, 19, 0]
    metadata = execution.model_input.layer_attention_metadata[0]
    assert metadata.query_start_locations.tolist() == [0, 1, 3]
    assert metadata.slot_mapping[-1].item() == -1
    assert metadata.block_table.tolist() == [[0, 2, 7, 7], [1, 7, 7, 7]]
    assert metadata.context_lengths.tolist() == [3, 2]
