"""Fused SwiGLU FFN module (drop-in for eb1386/TinKer tinker/modules/feed_forward.py:9-47).

``forward`` runs the whole FFN as two tcgen05 GEMMs: gate|up with the SwiGLU
applied in the epilogue, then the down projection. The ``gate_proj`` /
``up_proj`` / ``down_proj`` submodules keep the reference's names and shapes, so
``state_dict`` stays compatible.
"""

import torch
import torch.nn as nn

from tinker_b200 import torch_ops
from tinker_b200.kernels.gemm import swiglu_ffn
from tinker_b200.modules._roles import swiglu_weights


class TinKerSwiGLU(nn.Module):
    """SwiGLU feed-forward block: down_proj(silu(gate_proj(x)) * up_proj(x)).

    args:
        hidden_size: model width
        intermediate_size: width of the gated inner layer
    """

    def __init__(self, hidden_size: int, intermediate_size: int):
        super().__init__()
        self.hidden_size = hidden_size
        self.intermediate_size = intermediate_size
        self.gate_proj = nn.Linear(hidden_size, intermediate_size, bias=False)
        self.up_proj = nn.Linear(hidden_size, intermediate_size, bias=False)
        self.down_proj = nn.Linear(intermediate_size, hidden_size, bias=False)

    def forward(self, x: torch.Tensor, residual: torch.Tensor | None = None) -> torch.Tensor:
        """``down(silu(gate(x)) * up(x))``; with ``residual`` the sum is added in the epilogue."""
        args = (x, self.gate_proj.weight, self.up_proj.weight, self.down_proj.weight, residual)
        if torch_ops.compiling():  # one opaque node for torch.compile (tinker_b200.torch_ops)
            return torch.ops.tinker.swiglu_ffn(*args)
        return swiglu_ffn(*args)

    @classmethod
    def from_module(cls, source: nn.Module) -> "TinKerSwiGLU":
        """A ``TinKerSwiGLU`` holding copies of ``source``'s gate / up / down weights (found by
        name, see ``modules._roles``); the sizes come from the gate weight's shape."""
        w = swiglu_weights(source)
        intermediate_size, hidden_size = w["gate"].shape
        module = cls(hidden_size, intermediate_size)
        with torch.no_grad():
            for role in ("gate", "up", "down"):
                getattr(module, f"{role}_proj").weight.copy_(w[role])
        return module

    def extra_repr(self) -> str:
        return f"{self.hidden_size} -> {self.intermediate_size} -> {self.hidden_size}"
