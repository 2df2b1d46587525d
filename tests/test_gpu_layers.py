"""mvb_rms_norm and mvb_silu_mul against the reference's own torch ops.

RMSNorm.forward (src/micro_vllm/layers/normalization.py:15-22), the residual
add before the post-attention norm (src/micro_vllm/models/qwen.py:151-154)
and SwiGLUMLP's silu(gate) * up (src/micro_vllm/layers/mlp.py:19-21) are
restated below with the reference's torch ops, step for step; the reference
module itself is compared too when micro_vllm is installed.  The residual
sum is bit-exact; normalised values may differ from torch's in the last
place where the sum of squares (added in another order) rounds differently,
and the weight product can carry that to two units in the last place of the
result, so they are held to two units and to a small share of differing
elements (the bound of the attention prologue's tests); silu * up too.
"""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from micro_vllm_b200.layers import rms_norm, silu_mul

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def reference_rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    input_dtype = x.dtype
    h = x.to(torch.float32)
    variance = h.pow(2).mean(dim=-1, keepdim=True)
    h = h * torch.rsqrt(variance + eps)
    return weight * h.to(input_dtype)


def ulps_apart(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """|a - b| in units of the last place of b's dtype at b's magnitude."""

    bits = 10 if b.dtype == torch.float16 else 7
    mag = b.float().abs().clamp_min(2.0 ** -14)
    ulp = torch.exp2(torch.floor(torch.log2(mag)) - bits)
    return (a.float() - b.float()).abs() / ulp


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("rows,hidden", [(1, 1024), (7, 1024), (64, 1024), (8192, 1024), (33, 128), (5, 4096)])
def test_rms_norm_matches_the_reference_ops(dtype, rows, hidden) -> None:
    g = torch.Generator(device=DEV).manual_seed(rows * 131 + hidden)
    x = (torch.randn((rows, hidden), generator=g, device=DEV) * 3).to(dtype)
    weight = (0.5 + torch.rand(hidden, generator=g, device=DEV)).to(dtype)
    out, total = rms_norm(x, weight, 1e-6)
    assert total.data_ptr() == x.data_ptr()  # no residual: h is x itself
    want = reference_rms_norm(x, weight, 1e-6)
    assert out.dtype == dtype and out.shape == want.shape
    d = ulps_apart(out, want)
    assert d.max().item() <= 2.0
    assert (d > 0).float().mean().item() < 2e-3


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_residual_add_then_norm_and_strided_rows(dtype) -> None:
    g = torch.Generator(device=DEV).manual_seed(5)
    rows, hidden = 300, 1024
    big = (torch.randn((rows, hidden + 64), generator=g, device=DEV) * 2).to(dtype)
    x = big[:, 32:32 + hidden]  # row stride hidden + 64
    residual = (torch.randn((rows, hidden), generator=g, device=DEV) * 4).to(dtype)
    weight = (0.5 + torch.rand(hidden, generator=g, device=DEV)).to(dtype)
    out, total = rms_norm(x, weight, 1e-6, residual=residual)
    want_total = residual + x  # the reference: residual + hidden_states
    assert torch.equal(total, want_total)
    d = ulps_apart(out, reference_rms_norm(want_total, weight, 1e-6))
    assert d.max().item() <= 2.0 and (d > 0).float().mean().item() < 2e-3


def test_rms_norm_matches_the_reference_module() -> None:
    from _reference import require_reference

    require_reference()
    from micro_vllm.layers.normalization import RMSNorm

    g = torch.Generator(device=DEV).manual_seed(9)
    module = RMSNorm(1024, eps=1e-6).to(DEV, torch.float16)
    with torch.no_grad():
        module.weight.copy_(0.5 + torch.rand(1024, generator=g, device=DEV))
    x = torch.randn((257, 1024), generator=g, device=DEV).half()
    out, _ = rms_norm(x, module.weight.detach(), module.variance_epsilon)
    with torch.no_grad():
        d = ulps_apart(out, module(x))
    assert d.max().item() <= 2.0 and (d > 0).float().mean().item() < 2e-3


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("rows", [1, 64, 4096])
def test_silu_mul_matches_the_reference_ops(dtype, rows) -> None:
    g = torch.Generator(device=DEV).manual_seed(rows)
    inter = 3072
    gate_up = (torch.randn((rows, 2 * inter), generator=g, device=DEV) * 3).to(dtype)
    out = silu_mul(gate_up, inter)
    want = F.silu(gate_up[:, :inter]) * gate_up[:, inter:]
    d = ulps_apart(out, want)
    assert d.max().item() <= 2.0 and (d > 0).float().mean().item() < 2e-3


def test_shapes_the_kernels_do_not_take_are_rejected() -> None:
    x = torch.zeros((4, 100), dtype=torch.float16, device=DEV)  # hidden not a multiple of 8
    with pytest.raises(Exception):
        rms_norm(x, torch.ones(100, dtype=torch.float16, device=DEV), 1e-6)
    with pytest.raises(ValueError):
        rms_norm(torch.zeros((4, 128), device=DEV), torch.ones(128, device=DEV), 1e-6)  # fp32
    with pytest.raises(ValueError):
        silu_mul(torch.zeros((4, 100), dtype=torch.float16, device=DEV), 64)  # too few columns
