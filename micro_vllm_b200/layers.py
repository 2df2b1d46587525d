"""RMSNorm (with its residual add) and SwiGLU's silu(gate) * up as one launch
each (``mvb_rms_norm``, ``mvb_silu_mul``).

The reference model runs RMSNorm.forward (src/micro_vllm/layers/normalization.py:15-22)
as a chain of torch kernels (cast, square, mean, add, rsqrt, multiply, cast,
multiply), the residual add before it as one more (src/micro_vllm/models/qwen.py:151-154),
and SwiGLUMLP's silu and product as two (src/micro_vllm/layers/mlp.py:19-21).
These kernels round where those torch ops round.
"""

from __future__ import annotations

import torch

from micro_vllm_b200 import _lib

_DTYPES = {torch.float16: _lib.MVB_DTYPE_F16, torch.bfloat16: _lib.MVB_DTYPE_BF16}


def _check_rows(name: str, t: torch.Tensor, hidden: int) -> None:
    if t.dim() != 2 or t.shape[1] != hidden or t.stride(1) != 1:
        raise ValueError(f"{name} must be [rows, {hidden}] with unit column stride")


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float,
             residual: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """(RMSNorm(h), h) for h = x, or h = x + residual when given; x and
    residual [rows, hidden] (row strides free), weight [hidden], one dtype."""

    dtype = _DTYPES.get(x.dtype)
    if dtype is None or x.device.type != "cuda":
        raise ValueError("rms_norm takes float16 / bfloat16 CUDA tensors")
    rows, hidden = x.shape
    _check_rows("x", x, hidden)
    if weight.shape != (hidden,) or weight.dtype != x.dtype:
        raise ValueError("weight must be [hidden] of the input's dtype")
    weight = weight.contiguous()
    out = torch.empty((rows, hidden), dtype=x.dtype, device=x.device)
    total = x
    if residual is not None:
        _check_rows("residual", residual, hidden)
        if residual.dtype != x.dtype or residual.shape[0] != rows:
            raise ValueError("residual must match x")
        total = torch.empty((rows, hidden), dtype=x.dtype, device=x.device)
    lib = _lib.load()
    rc = lib.mvb_rms_norm(
        x.data_ptr(), x.stride(0),
        None if residual is None else residual.data_ptr(), 0 if residual is None else residual.stride(0),
        None if residual is None else total.data_ptr(), out.data_ptr(), weight.data_ptr(), float(eps),
        rows, hidden, dtype, torch.cuda.current_stream(x.device).cuda_stream,
    )
    _lib.check(rc, "b200 rms_norm")
    return out, total


def silu_mul(gate_up: torch.Tensor, intermediate: int) -> torch.Tensor:
    """silu(gate_up[:, :I]) * gate_up[:, I:2I] for I = ``intermediate``."""

    dtype = _DTYPES.get(gate_up.dtype)
    if dtype is None or gate_up.device.type != "cuda":
        raise ValueError("silu_mul takes float16 / bfloat16 CUDA tensors")
    if gate_up.dim() != 2 or gate_up.stride(1) != 1 or gate_up.shape[1] < 2 * intermediate:
        raise ValueError("gate_up must be [rows, >= 2 * intermediate] with unit column stride")
    rows = gate_up.shape[0]
    out = torch.empty((rows, intermediate), dtype=gate_up.dtype, device=gate_up.device)
    lib = _lib.load()
    rc = lib.mvb_silu_mul(gate_up.data_ptr(), gate_up.stride(0), out.data_ptr(), rows, intermediate, dtype,
                          torch.cuda.current_stream(gate_up.device).cuda_stream)
    _lib.check(rc, "b200 silu_mul")
    return out
