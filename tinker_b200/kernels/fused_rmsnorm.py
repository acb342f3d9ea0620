"""RMSNorm on the sm_100a kernel library.

Mirrors ``tinker.kernels.fused_rmsnorm`` (eb1386/TinKer
tinker/kernels/fused_rmsnorm.py:70-74): same name, arguments and result
(``x * rsqrt(mean(x^2) + eps) * weight`` in float32, one rounding to x's dtype).
The CUDA kernel reads each row once (tinker_b200/csrc/rmsnorm.cu).
"""

from __future__ import annotations

import torch

from tinker_b200 import _lib
from tinker_b200.kernels._common import call_ctx, row_stride, rows_view


def fused_rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """apply fused rmsnorm."""
    dev = _lib.require_cuda(x, weight)
    if weight.dim() != 1 or weight.shape[0] != x.shape[-1]:
        raise ValueError(f"weight shape {tuple(weight.shape)} does not match last dim {x.shape[-1]}")
    x2 = rows_view(x)
    w = weight if weight.is_contiguous() else weight.contiguous()
    y = torch.empty(x2.shape, dtype=x.dtype, device=x.device)
    with call_ctx(dev):
        _lib.check(_lib.lib().tk_rmsnorm(x2.data_ptr(), row_stride(x2), w.data_ptr(), _lib.dtype_code(w.dtype),
                                         y.data_ptr(), y.shape[1], x2.shape[0], x2.shape[1], float(eps),
                                         _lib.dtype_code(x.dtype), _lib.stream_ptr(dev)), "tk_rmsnorm", 1)
    return y.reshape(x.shape)


def fused_add_rmsnorm(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6):
    """``s = x + residual`` (in x's dtype) and ``fused_rmsnorm(s)``; returns ``(normed, s)``.

    The residual update of a pre-norm decoder block fused with the next norm;
    ``residual`` is left untouched.
    """
    dev = _lib.require_cuda(x, residual, weight)
    if x.shape != residual.shape or x.dtype != residual.dtype:
        raise ValueError("x and residual must have the same shape and dtype")
    xc, rc = x.contiguous(), residual.contiguous()
    dim = x.shape[-1]
    rows = xc.numel() // dim if dim else 0
    y = torch.empty_like(xc)
    s = torch.empty_like(xc)
    w = weight.contiguous()
    with call_ctx(dev):
        _lib.check(_lib.lib().tk_add_rmsnorm(xc.data_ptr(), rc.data_ptr(), w.data_ptr(), _lib.dtype_code(w.dtype),
                                             y.data_ptr(), s.data_ptr(), rows, dim, float(eps),
                                             _lib.dtype_code(x.dtype), _lib.stream_ptr(dev)), "tk_add_rmsnorm", 1)
    return y, s
