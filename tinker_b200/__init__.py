"""tinker_b200 - B200-native (sm_100a) fused-kernel inference path with TinKer's API.

Drop-in for eb1386/TinKer's public surface (tinker/__init__.py:3-18): the same
``TinKer*`` modules, ``patch_model``, ``optimize`` and ``benchmark_model``, plus a
KV cache for decoding (``KVCache``, ``CachedDecoder``), backed by hand-written
CUDA kernels in ``libtinker_b200.so`` (build it with ``python -m tinker_b200.build``).
"""

from tinker_b200.modules.attention import TinKerAttention
from tinker_b200.modules.feed_forward import TinKerSwiGLU
from tinker_b200.modules.normalization import TinKerRMSNorm
from tinker_b200.patch import patch_model
from tinker_b200.optimize import optimize, benchmark_model
from tinker_b200.generation import CachedDecoder, KVCache

__all__ = [
    "TinKerAttention",
    "TinKerSwiGLU",
    "TinKerRMSNorm",
    "patch_model",
    "optimize",
    "benchmark_model",
    "KVCache",
    "CachedDecoder",
]

__version__ = "0.1.0"
