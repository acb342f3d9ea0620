"""numpy forward of the reference's Llama-style decoder (test infrastructure only).

Restates the model that the reference benchmarks and patches:
``RMSNorm`` / ``SwiGLUFFN`` / ``GQAAttention`` / ``TransformerBlock`` /
``SimpleTransformer`` (benchmarks/bench_e2e.py:17-138), wrapped with the token
embedding and LM head of ``ToyTransformer`` (examples/patch_any_model.py:95-108).
Weights are passed as a dict keyed like the PyTorch ``state_dict`` of that model
(``layers.{i}.attn.q_proj.weight`` ...), so a test can hand the same tensors to
the CUDA path and to this oracle.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from oracle import ops


@dataclass(frozen=True)
class ModelConfig:
    vocab_size: int
    hidden_size: int
    num_layers: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    intermediate_size: int
    eps: float = 1e-6
    rope_theta: float = 10000.0
    tied_embeddings: bool = False
    max_seq_len: int = 2048


def _block(x: np.ndarray, w: dict, p: str, cfg: ModelConfig, cos, sin, acc) -> np.ndarray:
    """One pre-norm decoder block (benchmarks/bench_e2e.py:112-115)."""
    B, S, H = x.shape
    # attn_norm (bench_e2e.py:23-25; in fp32 the two roundings are no-ops)
    h = ops.rmsnorm(x, w[f"{p}.attn_norm.weight"], cfg.eps, acc=acc)
    q = ops.linear(h, w[f"{p}.attn.q_proj.weight"], acc=acc)
    k = ops.linear(h, w[f"{p}.attn.k_proj.weight"], acc=acc)
    v = ops.linear(h, w[f"{p}.attn.v_proj.weight"], acc=acc)
    # GQAAttention.forward (bench_e2e.py:79-94): interleaved RoPE, repeat KV, causal SDPA
    a = ops.attention(q, k, v, cos, sin, cfg.num_heads, cfg.num_kv_heads, cfg.head_dim,
                      acc=acc)
    x = x + ops.linear(a, w[f"{p}.attn.o_proj.weight"], acc=acc)
    # ffn_norm + SwiGLUFFN.forward (bench_e2e.py:35-36)
    h = ops.rmsnorm(x, w[f"{p}.ffn_norm.weight"], cfg.eps, acc=acc)
    g = ops.linear(h, w[f"{p}.ffn.gate_proj.weight"], acc=acc)
    u = ops.linear(h, w[f"{p}.ffn.up_proj.weight"], acc=acc)
    x = x + ops.linear(ops.swiglu(g, u, acc=acc), w[f"{p}.ffn.down_proj.weight"], acc=acc)
    return np.asarray(x, dtype=np.float32)


def forward_logits(weights: dict, tokens: np.ndarray, cfg: ModelConfig, acc=np.float32,
                   num_layers: int | None = None) -> np.ndarray:
    """Full forward ``tokens[B, S]`` (int) -> ``logits[B, S, vocab]`` in float32.

    ``num_layers`` lets a bounded CPU-baseline sample run fewer blocks; parity
    checks always run them all.
    """
    tokens = np.asarray(tokens)
    cos, sin = ops.rope_tables(cfg.head_dim, cfg.max_seq_len, cfg.rope_theta)
    x = np.asarray(weights["embedding.weight"], dtype=np.float32)[tokens]
    n = cfg.num_layers if num_layers is None else num_layers
    for i in range(n):
        x = _block(x, weights, f"layers.{i}", cfg, cos, sin, acc)
    x = ops.rmsnorm(x, weights["norm.weight"], cfg.eps, acc=acc)
    head = weights["embedding.weight"] if cfg.tied_embeddings else weights["output.weight"]
    return ops.linear(x, head, acc=acc)
