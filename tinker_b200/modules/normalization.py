"""RMSNorm module (drop-in for eb1386/TinKer tinker/modules/normalization.py:9-38).

The constructor signature and the ``weight`` / ``eps`` attributes are the reference's,
so state_dicts and code that reads them carry over; ``forward`` runs this library's
vectorised RMSNorm kernel.
"""

import torch
import torch.nn as nn

from tinker_b200 import torch_ops
from tinker_b200.kernels.fused_rmsnorm import fused_rmsnorm


class TinKerRMSNorm(nn.Module):
    """y = x / sqrt(mean(x^2) + eps) * weight over the last axis (float32 statistics).

    args:
        dim: size of the normalised (last) axis
        eps: added to the mean square
    """

    def __init__(self, dim: int, eps: float = 1e-6):
        super().__init__()
        self.dim = dim
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if torch_ops.compiling():  # one opaque node for torch.compile (tinker_b200.torch_ops)
            return torch.ops.tinker.rmsnorm(x, self.weight, float(self.eps))
        return fused_rmsnorm(x, self.weight, self.eps)

    @classmethod
    def from_module(cls, source: nn.Module) -> "TinKerRMSNorm":
        """Copy of ``source``'s weight; epsilon from its ``eps``, else ``variance_epsilon``
        (the Hugging Face name), else 1e-6."""
        eps = getattr(source, "eps", None)
        if eps is None:
            eps = getattr(source, "variance_epsilon", 1e-6)
        module = cls(source.weight.shape[0], eps)
        with torch.no_grad():
            module.weight.copy_(source.weight)
        return module

    def extra_repr(self) -> str:
        return f"{self.dim}, eps={self.eps}"
