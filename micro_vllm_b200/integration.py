"""Plug ``b200_paged`` into an installed micro-vLLM without editing its source.

The reference resolves an operator name through
``micro_vllm.attention.operators.registry.get_attention_operator_class``
(src/micro_vllm/attention/operators/registry.py:24-50), whose table is a
read-only mapping, and ``ModelConfig.__post_init__``
(src/micro_vllm/config.py:45-57) accepts CUDA-graph execution only for
``triton_paged`` in fp16.  ``register()`` wraps both in place:

* the registry function resolves ``"b200_paged"`` to a class that derives
  from the reference's own ``AttentionOperator`` (operators/base.py:10-40)
  and from ``B200PagedAttentionOperator``; every other name, and the error
  for an unknown name, behave as before (the supported list gains
  ``b200_paged``);
* ``ModelConfig`` accepts ``enable_cuda_graph=True`` with ``b200_paged`` on
  a CUDA device in fp16 or bf16 (the operator makes no host synchronisation
  and allocates nothing once its workspace is reserved).

``Attention.__init__`` (attention/attention.py:47-54) imports the registry
function when it runs, so models built after ``register()`` get the operator
through ``ModelConfig.attention_operator = "b200_paged"``.
"""

from __future__ import annotations

import functools
import threading

import torch

from micro_vllm_b200.operators import OPERATOR_NAME, B200PagedAttentionOperator

_lock = threading.Lock()
_registered: type | None = None


def reference_operator_class() -> type:
    """``B200PagedAttentionOperator`` as a subclass of the reference's
    ``AttentionOperator`` (raises ImportError when micro_vllm is absent)."""

    from micro_vllm.attention.operators.base import AttentionOperator as ReferenceBase

    if issubclass(B200PagedAttentionOperator, ReferenceBase):
        return B200PagedAttentionOperator
    return type(
        "B200PagedAttentionOperator",
        (B200PagedAttentionOperator, ReferenceBase),
        {"__module__": __name__, "__doc__": B200PagedAttentionOperator.__doc__},
    )


def register() -> type:
    """Make ``"b200_paged"`` a selectable operator of the installed micro_vllm
    (idempotent).  Returns the registered operator class."""

    global _registered
    with _lock:
        if _registered is not None:
            return _registered
        import micro_vllm.attention.operators.registry as registry
        import micro_vllm.config as config_module

        operator_class = reference_operator_class()
        original_lookup = registry.get_attention_operator_class

        @functools.wraps(original_lookup)
        def get_attention_operator_class(name: str) -> type:
            if name == OPERATOR_NAME:
                return operator_class
            try:
                return original_lookup(name)
            except ValueError as error:
                supported = [*registry._OPERATOR_CLASSES, "triton_paged", OPERATOR_NAME]
                raise ValueError(
                    f"unsupported attention operator {name!r}; supported operators: {supported!r}"
                ) from error

        registry.get_attention_operator_class = get_attention_operator_class
        # The package re-exports the function (operators/__init__.py:6-8).
        import micro_vllm.attention.operators as operators_package

        operators_package.get_attention_operator_class = get_attention_operator_class

        model_config = config_module.ModelConfig
        original_post_init = model_config.__post_init__

        @functools.wraps(original_post_init)
        def __post_init__(self) -> None:
            if self.attention_operator != OPERATOR_NAME or not self.enable_cuda_graph:
                original_post_init(self)
                return
            if torch.device(self.device).type != "cuda":
                raise ValueError("CUDA Graph execution requires a CUDA device")
            if self.dtype not in (torch.float16, torch.bfloat16):
                raise ValueError(
                    "CUDA Graph execution with b200_paged requires torch.float16 or torch.bfloat16"
                )
            # The reference's remaining checks, with its triton-only gate set aside.
            self.enable_cuda_graph = False
            try:
                original_post_init(self)
            finally:
                self.enable_cuda_graph = True

        model_config.__post_init__ = __post_init__
        _registered = operator_class
        return operator_class
