"""The reference's import name for this package: ``import tinker`` gives tinker_b200.

Code written against eb1386/TinKer imports ``tinker`` and its submodules by path
(``from tinker.kernels import fused_rmsnorm``, ``from tinker.modules import TinKerAttention``,
``from tinker.patch import patch_model``). This package makes those imports resolve to the
B200 implementation: the public names of ``tinker/__init__.py`` (tinker/__init__.py:3-18 of
the reference) and the submodules of its hot path are the tinker_b200 ones. The reference's
GPU-config utilities (``tinker.utils``) are out of scope and not provided.
"""

import importlib
import sys

import tinker_b200 as _impl
from tinker_b200 import (  # noqa: F401
    CachedDecoder,
    KVCache,
    TinKerAttention,
    TinKerRMSNorm,
    TinKerSwiGLU,
    benchmark_model,
    optimize,
    patch_model,
)

__version__ = _impl.__version__
__all__ = ["TinKerAttention", "TinKerSwiGLU", "TinKerRMSNorm", "patch_model", "optimize", "benchmark_model",
           "KVCache", "CachedDecoder"]

_SUBMODULES = (
    "kernels", "kernels.fused_attention", "kernels.fused_rmsnorm", "kernels.fused_swiglu",
    "modules", "modules.attention", "modules.feed_forward", "modules.normalization",
    "patch", "optimize",
)
for _name in _SUBMODULES:
    _mod = importlib.import_module(f"tinker_b200.{_name}")
    sys.modules[f"{__name__}.{_name}"] = _mod
    if _name in ("kernels", "modules"):  # `tinker.optimize` stays the function, as in the reference
        setattr(sys.modules[__name__], _name, _mod)
