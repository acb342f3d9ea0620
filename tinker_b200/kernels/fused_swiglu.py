"""SwiGLU activation on the sm_100a kernel library.

Mirrors ``tinker.kernels.fused_swiglu`` (eb1386/TinKer
tinker/kernels/fused_swiglu.py:61-66): ``silu(gate) * up`` in float32 with one
rounding, including the shape assertion of the reference. In the patched
model the activation does not run as its own kernel: it is the epilogue of the
gate|up GEMM (``tinker_b200.kernels.gemm.gate_up_swiglu``).
"""

from __future__ import annotations

import torch

from tinker_b200 import _lib
from tinker_b200.kernels._common import call_ctx, row_stride, rows_view


def fused_swiglu(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """apply fused swiglu activation."""
    assert gate.shape == up.shape, "shape mismatch"
    dev = _lib.require_cuda(gate, up)
    if gate.dtype != up.dtype:
        raise TypeError("gate and up must have the same dtype")
    g2, u2 = rows_view(gate), rows_view(up)
    out = torch.empty(g2.shape, dtype=gate.dtype, device=gate.device)
    with call_ctx(dev):
        _lib.check(_lib.lib().tk_swiglu(g2.data_ptr(), row_stride(g2), u2.data_ptr(), row_stride(u2),
                                        out.data_ptr(), out.shape[1], g2.shape[0], g2.shape[1],
                                        _lib.dtype_code(gate.dtype), _lib.stream_ptr(dev)), "tk_swiglu", 1)
    return out.reshape(gate.shape)
