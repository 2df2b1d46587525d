"""Registration into the reference package, checked on the CPU.

``register()`` must make ``"b200_paged"`` selectable through the reference's
own registry and config without editing it
(src/micro_vllm/attention/operators/registry.py:24-50, config.py:45-57), and
the checkpoint writer must produce what the reference loader reads.
"""

from __future__ import annotations

import pytest
import torch

from _reference import require_reference


@pytest.fixture(scope="module")
def reference():
    return require_reference()


def test_registry_resolves_b200_paged(reference):
    from micro_vllm.attention.operators.base import AttentionOperator as ReferenceBase

    from micro_vllm_b200 import B200PagedAttentionOperator
    from micro_vllm_b200.integration import register

    registered = register()
    assert register() is registered  # idempotent
    # A name imported after register() is the wrapped lookup.
    from micro_vllm.attention.operators.registry import get_attention_operator_class

    cls = get_attention_operator_class("b200_paged")
    assert cls is registered
    assert issubclass(cls, ReferenceBase) and issubclass(cls, B200PagedAttentionOperator)
    # The other names resolve as before.
    from micro_vllm.attention.operators.reference import ReferenceAttentionOperator
    from micro_vllm.attention.operators.sdpa import SDPAAttentionOperator

    assert get_attention_operator_class("reference") is ReferenceAttentionOperator
    assert get_attention_operator_class("sdpa") is SDPAAttentionOperator
    # Unknown names keep the reference's error, with b200_paged in the list.
    with pytest.raises(ValueError, match=r"unsupported attention operator 'nope'; supported operators: .*b200_paged"):
        get_attention_operator_class("nope")
    # The package-level re-export follows.
    import micro_vllm.attention.operators as ops

    assert ops.get_attention_operator_class("b200_paged") is registered


def test_attention_builds_the_operator(reference):
    from micro_vllm.attention.attention import Attention
    from micro_vllm.attention.operators.base import AttentionOperator as ReferenceBase
    from micro_vllm.attention.spec import SlidingWindowSpec

    from micro_vllm_b200.integration import register

    register()
    attention = Attention(SlidingWindowSpec(8), "b200_paged")
    assert isinstance(attention.operator, ReferenceBase)
    # No CPU fallback: the operator refuses host tensors.
    q = torch.zeros(1, 2, 8)
    cache = torch.zeros(2, 4, 16, 1, 8)
    md = attention.build_metadata(
        query_positions=torch.zeros(1, dtype=torch.int64),
        query_start_locations=torch.tensor([0, 1]),
        context_lengths=torch.tensor([1]),
        block_table=torch.zeros((1, 1), dtype=torch.int64),
        slot_mapping=torch.zeros(1, dtype=torch.int64),
        block_size=16,
    )
    with pytest.raises(RuntimeError, match="requires CUDA tensors"):
        attention(q, q[:, :1], q[:, :1], cache, md)


def test_cuda_graph_gate(reference):
    from micro_vllm.config import ModelConfig

    from micro_vllm_b200.integration import register

    register()
    for dtype in (torch.float16, torch.bfloat16):
        cfg = ModelConfig(model="m", attention_operator="b200_paged", enable_cuda_graph=True,
                          device="cuda", dtype=dtype)
        assert cfg.enable_cuda_graph
    with pytest.raises(ValueError, match="requires a CUDA device"):
        ModelConfig(model="m", attention_operator="b200_paged", enable_cuda_graph=True, device="cpu")
    with pytest.raises(ValueError, match="float16 or torch.bfloat16"):
        ModelConfig(model="m", attention_operator="b200_paged", enable_cuda_graph=True,
                    device="cuda", dtype=torch.float32)
    # The reference's own gate is unchanged for its operators.
    with pytest.raises(ValueError, match="triton_paged"):
        ModelConfig(model="m", attention_operator="reference", enable_cuda_graph=True, device="cuda")
    with pytest.raises(ValueError, match="requires torch.float16"):
        ModelConfig(model="m", attention_operator="triton_paged", enable_cuda_graph=True,
                    device="cuda", dtype=torch.bfloat16)
    # Its other checks still run for b200_paged.
    with pytest.raises(ValueError, match="device must be"):
        ModelConfig(model="m", attention_operator="b200_paged", device="meta")


def test_sampler_output_is_the_reference_type(reference):
    from micro_vllm.executor.interface import ModelRunnerOutput, SampledToken

    from micro_vllm_b200.sampling import B200Sampler, _output_types

    assert _output_types() == (ModelRunnerOutput, SampledToken)
    assert isinstance(B200Sampler()(torch.zeros(0, 4), (), (), ()), ModelRunnerOutput)


def test_random_checkpoint_loads_through_the_reference(reference, tmp_path):
    from micro_vllm.config import CacheConfig, LLMConfig, ModelConfig, SchedulerConfig
    from micro_vllm.model_loader import load_model

    from micro_vllm_b200.engine import QWEN3_0_6B, qwen3_tensor_shapes, write_random_checkpoint

    values = dict(QWEN3_0_6B, vocab_size=64, hidden_size=32, intermediate_size=48, num_hidden_layers=2,
                  num_attention_heads=4, num_key_value_heads=2, head_dim=8)
    for tied in (True, False):
        values["tie_word_embeddings"] = tied
        path = write_random_checkpoint(tmp_path / f"m{tied}", values, seed=3, dtype=torch.float32)
        config = LLMConfig(
            model_config=ModelConfig(model=str(path), device="cpu", dtype=torch.float32),
            scheduler_config=SchedulerConfig(64, 4, 64), cache_config=CacheConfig(num_blocks=8),
        )
        model = load_model(config)
        params = dict(model.named_parameters())
        names = {n.removeprefix("model.") for n in qwen3_tensor_shapes(values)}
        assert names == set(params)  # every parameter comes from the checkpoint
        again = write_random_checkpoint(tmp_path / f"again{tied}", values, seed=3, dtype=torch.float32)
        assert (again / "model.safetensors").read_bytes() == (path / "model.safetensors").read_bytes()
        assert torch.equal(params["norm.weight"], torch.ones(32))


def test_engine_requests_are_seeded():
    from micro_vllm_b200.partition import partition_sequences

    pytest.importorskip("safetensors")
    require_reference()
    from micro_vllm_b200.engine import engine_requests

    a = engine_requests(64, seed=0)
    assert a == engine_requests(64, seed=0) and a != engine_requests(64, seed=1)
    assert all(128 <= len(r.prompt_token_ids) <= 1024 for r in a)
    assert all(1 <= t <= 151935 for r in a for t in r.prompt_token_ids)
    shards = partition_sequences([len(r.prompt_token_ids) + r.max_tokens for r in a], 8)
    assert sorted(i for s in shards for i in s.indices) == list(range(64))


def test_concatenated_projection_weights_are_shared_views(reference):
    """B200ModelRunner's fused layers run q/k/v (and gate/up) as one GEMM over
    their weights concatenated; the reference's Linear modules keep their
    weights as views into that tensor, so values and memory are unchanged."""

    from micro_vllm.layers.linear import Linear

    from micro_vllm_b200.engine import _concatenate_weights

    torch.manual_seed(0)
    q, k, v = Linear(8, 16, bias=False), Linear(8, 4, bias=False), Linear(8, 4, bias=False)
    before = [m.weight.detach().clone() for m in (q, k, v)]
    joined = _concatenate_weights(q, k, v)
    assert joined.shape == (24, 8)
    assert torch.equal(joined, torch.cat(before))
    for m, w in zip((q, k, v), before):
        assert torch.equal(m.weight, w)
        assert m.weight.untyped_storage().data_ptr() == joined.untyped_storage().data_ptr()
    x = torch.randn(3, 8)
    assert torch.equal(torch.nn.functional.linear(x, joined)[:, 16:20], k(x))


def test_seeded_rows_get_the_reference_generators_noise():
    """B200Sampler draws Exp(1) noise only for seeded stochastic rows, each
    from a generator seeded (seed + sample index) mod 2^63 on the logits'
    device, as the reference's _sample_row seeds its own (sampler.py:52-61);
    greedy rows and rows without a seed get none (noise_row -1)."""

    from micro_vllm_b200.sampling import B200Sampler

    class Params:
        def __init__(self, temperature, seed):
            self.temperature, self.top_k, self.top_p, self.seed = temperature, None, 1.0, seed

    vocab = 1000
    logits = torch.zeros((4, vocab))
    params = (Params(0.0, 5), Params(0.8, 2**63 - 1), Params(0.8, None), Params(1.0, 7))
    indices = (3, 4, 5, 6)
    noise, rows = B200Sampler()._reference_noise(logits, params, indices)
    assert rows.tolist() == [-1, 0, -1, 1]
    assert noise.shape == (2, vocab) and noise.dtype == torch.float32
    for n, (seed, index) in enumerate(((2**63 - 1, 4), (7, 6))):
        g = torch.Generator()
        g.manual_seed((seed + index) % 2**63)
        assert torch.equal(noise[n], torch.empty(vocab).exponential_(1.0, generator=g))
    assert B200Sampler(reference_streams=False)._reference_noise(logits, params, indices) == (None, None)
    assert B200Sampler()._reference_noise(logits, params[:1] + params[2:3], indices[:2]) == (None, None)


def test_patched_rms_norm_falls_back_to_the_reference_forward(reference):
    """B200ModelRunner replaces RMSNorm.forward with the one-launch kernel;
    rows that kernel does not take (here: CPU rows) still get the reference's
    own forward, unchanged."""

    import types

    from micro_vllm.layers.normalization import RMSNorm

    from micro_vllm_b200.engine import _rms_norm_forward

    torch.manual_seed(0)
    norm = RMSNorm(64, eps=1e-6)
    with torch.no_grad():
        norm.weight.copy_(0.5 + torch.rand(64))
    x = torch.randn(5, 3, 64)
    want = norm(x)
    norm.forward = types.MethodType(_rms_norm_forward, norm)
    assert torch.equal(norm(x), want)
