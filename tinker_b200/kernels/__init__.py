"""sm_100a kernels (the replacement of the reference's tinker/kernels package)."""

from tinker_b200.kernels.fused_rmsnorm import fused_rmsnorm, fused_add_rmsnorm
from tinker_b200.kernels.fused_swiglu import fused_swiglu
from tinker_b200.kernels.fused_attention import causal_attention, fused_attention, precompute_rope_tables
from tinker_b200.kernels.gemm import linear, linear_rope, gate_up_swiglu, row_sumsq, swiglu_ffn
from tinker_b200.kernels.kv_cache import kv_append, kv_attention, kv_attention_workspace

__all__ = ["fused_rmsnorm", "fused_swiglu", "fused_attention", "precompute_rope_tables",
           "fused_add_rmsnorm", "linear", "linear_rope", "causal_attention", "gate_up_swiglu", "row_sumsq",
           "swiglu_ffn", "kv_attention", "kv_append", "kv_attention_workspace"]
