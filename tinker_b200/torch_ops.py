"""The kernel library's entry points as registered torch ops (``torch.ops.tinker.*``).

The kernels are called through ctypes, which ``torch.compile`` cannot trace: every call
would end the traced graph. Registered as custom ops with fake (shape-only)
implementations they become single opaque nodes instead, so a compiled model that
uses the ``TinKer*`` modules traces from end to end (``fullgraph=True`` works). The
module forwards switch to these ops while they are being compiled and call the
kernels directly otherwise (no dispatcher overhead in eager mode or in a CUDA graph).

Ops (all return a new tensor; none mutates its inputs):

* ``tinker::rmsnorm(x, weight, eps)`` - ``fused_rmsnorm``
* ``tinker::swiglu(gate, up)`` - ``fused_swiglu``
* ``tinker::fused_attention(q, k, v, cos, sin, heads, kv_heads, head_dim, start_pos)``
* ``tinker::swiglu_ffn(x, w_gate, w_up, w_down, residual)`` - ``TinKerSwiGLU.forward``
* ``tinker::attention(x, wq, wk, wv, wo, cos, sin, heads, kv_heads, head_dim, start_pos,
  residual)`` - ``TinKerAttention.forward`` without a KV cache
"""

from __future__ import annotations

from typing import Optional

import torch
from torch import Tensor
from torch.library import custom_op

from tinker_b200.kernels.fused_attention import fused_attention
from tinker_b200.kernels.fused_rmsnorm import fused_rmsnorm
from tinker_b200.kernels.fused_swiglu import fused_swiglu
from tinker_b200.kernels.gemm import swiglu_ffn


@custom_op("tinker::rmsnorm", mutates_args=())
def rmsnorm(x: Tensor, weight: Tensor, eps: float) -> Tensor:
    return fused_rmsnorm(x, weight, eps)


@rmsnorm.register_fake
def _rmsnorm_fake(x, weight, eps):
    return x.new_empty(x.shape)


@custom_op("tinker::swiglu", mutates_args=())
def swiglu(gate: Tensor, up: Tensor) -> Tensor:
    return fused_swiglu(gate, up)


@swiglu.register_fake
def _swiglu_fake(gate, up):
    return gate.new_empty(gate.shape)


@custom_op("tinker::fused_attention", mutates_args=())
def attention_kernel(q: Tensor, k: Tensor, v: Tensor, cos: Tensor, sin: Tensor, heads: int, kv_heads: int,
                     head_dim: int, start_pos: int) -> Tensor:
    return fused_attention(q, k, v, cos, sin, heads, kv_heads, head_dim, start_pos=start_pos)


@attention_kernel.register_fake
def _attention_kernel_fake(q, k, v, cos, sin, heads, kv_heads, head_dim, start_pos):
    return q.new_empty(q.shape[0], q.shape[1], heads * head_dim)


@custom_op("tinker::swiglu_ffn", mutates_args=())
def ffn(x: Tensor, w_gate: Tensor, w_up: Tensor, w_down: Tensor, residual: Optional[Tensor]) -> Tensor:
    return swiglu_ffn(x, w_gate, w_up, w_down, residual)


@ffn.register_fake
def _ffn_fake(x, w_gate, w_up, w_down, residual):
    return x.new_empty(*x.shape[:-1], w_down.shape[0])


@custom_op("tinker::attention", mutates_args=())
def attention(x: Tensor, wq: Tensor, wk: Tensor, wv: Tensor, wo: Tensor, cos: Tensor, sin: Tensor, heads: int,
              kv_heads: int, head_dim: int, start_pos: int, residual: Optional[Tensor]) -> Tensor:
    from tinker_b200.modules.attention import attention_forward
    return attention_forward(x, wq, wk, wv, wo, cos, sin, heads, kv_heads, head_dim, start_pos, residual)


@attention.register_fake
def _attention_fake(x, wq, wk, wv, wo, cos, sin, heads, kv_heads, head_dim, start_pos, residual):
    return x.new_empty(*x.shape[:-1], wo.shape[0])


def compiling() -> bool:
    """True while torch.compile traces the caller."""
    try:
        return torch.compiler.is_compiling()
    except AttributeError:  # torch without torch.compiler
        return False
