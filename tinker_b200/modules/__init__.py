"""module wrappers"""

from tinker_b200.modules.attention import TinKerAttention
from tinker_b200.modules.feed_forward import TinKerSwiGLU
from tinker_b200.modules.normalization import TinKerRMSNorm

__all__ = ["TinKerAttention", "TinKerSwiGLU", "TinKerRMSNorm"]
