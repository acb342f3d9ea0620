"""The reference's own eager PyTorch decoder (test infrastructure only).

TEST INFRASTRUCTURE, like the rest of ``oracle/``: the blocks below are the model the
reference benchmarks (eb1386/TinKer benchmarks/bench_e2e.py:17-138: ``RMSNorm``,
``SwiGLUFFN``, ``GQAAttention``, ``TransformerBlock`` and the layer stack of
``SimpleTransformer``), kept with the reference's own arithmetic and wrapped with the
token embedding and LM head of examples/patch_any_model.py:95-108. They are carried
here because the reference checkout cannot travel to the GPU host. Uses:

* the CPU baseline: ``bench.py`` times this model's fp32 eager forward on the host
  cores (the reference's unpatched CPU path);
* the reference's half-precision eager error on the GPU, which the parity tests use as
  the bar the CUDA path must not be worse than;
* ``tests/golden/make_golden.py`` initialises the reference's own classes with
  ``init_weights`` and records their logits, which pins this copy (and the numpy
  oracle) to the reference.

Any config object with the fields of ``bench_model.DecoderConfig`` works. Nothing in
the product package imports this file.
"""

from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F


class RMSNorm(nn.Module):
    """bench_e2e.py:17-25: float32 statistics, result rounded to x's dtype, then times w."""

    def __init__(self, dim: int, eps: float = 1e-6):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        norm = x.float().pow(2).mean(-1, keepdim=True).add(self.eps).rsqrt()
        return (x * norm).to(x.dtype) * self.weight


class SwiGLUFFN(nn.Module):
    """bench_e2e.py:28-36."""

    def __init__(self, hidden_size: int, intermediate_size: int):
        super().__init__()
        self.gate_proj = nn.Linear(hidden_size, intermediate_size, bias=False)
        self.up_proj = nn.Linear(hidden_size, intermediate_size, bias=False)
        self.down_proj = nn.Linear(intermediate_size, hidden_size, bias=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))


class GQAAttention(nn.Module):
    """bench_e2e.py:39-94, with ``rope_theta`` kept as an attribute so that
    ``TinKerAttention.from_module`` picks it up (tinker/modules/attention.py:95-97)."""

    def __init__(self, hidden_size: int, num_heads: int, num_kv_heads: int, head_dim: int,
                 max_seq_len: int = 2048, rope_theta: float = 10000.0):
        super().__init__()
        self.hidden_size = hidden_size
        self.num_heads = num_heads
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.num_kv_groups = num_heads // num_kv_heads
        self.rope_theta = rope_theta
        self.q_proj = nn.Linear(hidden_size, num_heads * head_dim, bias=False)
        self.k_proj = nn.Linear(hidden_size, num_kv_heads * head_dim, bias=False)
        self.v_proj = nn.Linear(hidden_size, num_kv_heads * head_dim, bias=False)
        self.o_proj = nn.Linear(num_heads * head_dim, hidden_size, bias=False)
        freqs = 1.0 / (rope_theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
        angles = torch.outer(torch.arange(max_seq_len, dtype=torch.float32), freqs)
        self.register_buffer("cos_table", torch.cos(angles), persistent=False)
        self.register_buffer("sin_table", torch.sin(angles), persistent=False)

    def _apply_rope(self, x: torch.Tensor) -> torch.Tensor:
        S = x.shape[2]
        cos = self.cos_table[:S].unsqueeze(0).unsqueeze(0)
        sin = self.sin_table[:S].unsqueeze(0).unsqueeze(0)
        out = torch.empty_like(x)
        out[..., 0::2] = x[..., 0::2] * cos - x[..., 1::2] * sin
        out[..., 1::2] = x[..., 0::2] * sin + x[..., 1::2] * cos
        return out

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        B, S, _ = x.shape
        q = self.q_proj(x).view(B, S, self.num_heads, self.head_dim).permute(0, 2, 1, 3)
        k = self.k_proj(x).view(B, S, self.num_kv_heads, self.head_dim).permute(0, 2, 1, 3)
        v = self.v_proj(x).view(B, S, self.num_kv_heads, self.head_dim).permute(0, 2, 1, 3)
        q = self._apply_rope(q)
        k = self._apply_rope(k)
        if self.num_kv_groups > 1:
            k = k.repeat_interleave(self.num_kv_groups, dim=1)
            v = v.repeat_interleave(self.num_kv_groups, dim=1)
        out = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        out = out.permute(0, 2, 1, 3).contiguous().view(B, S, self.num_heads * self.head_dim)
        return self.o_proj(out)


class TransformerBlock(nn.Module):
    """bench_e2e.py:97-115 (pre-norm, residual adds in the model dtype)."""

    def __init__(self, cfg):
        super().__init__()
        self.attn_norm = RMSNorm(cfg.hidden_size, cfg.eps)
        self.attn = GQAAttention(cfg.hidden_size, cfg.num_heads, cfg.num_kv_heads, cfg.head_dim,
                                 cfg.max_seq_len, cfg.rope_theta)
        self.ffn_norm = RMSNorm(cfg.hidden_size, cfg.eps)
        self.ffn = SwiGLUFFN(cfg.hidden_size, cfg.intermediate_size)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x = x + self.attn(self.attn_norm(x))
        x = x + self.ffn(self.ffn_norm(x))
        return x


class ReferenceLM(nn.Module):
    """Embedding -> blocks -> final RMSNorm -> LM head (examples/patch_any_model.py:95-108)."""

    def __init__(self, cfg):
        super().__init__()
        self.config = cfg
        self.embedding = nn.Embedding(cfg.vocab_size, cfg.hidden_size)
        self.layers = nn.ModuleList([TransformerBlock(cfg) for _ in range(cfg.num_layers)])
        self.norm = RMSNorm(cfg.hidden_size, cfg.eps)
        self.output = nn.Linear(cfg.hidden_size, cfg.vocab_size, bias=False)
        if cfg.tied_embeddings:
            self.output.weight = self.embedding.weight

    def forward(self, tokens: torch.Tensor) -> torch.Tensor:
        x = self.embedding(tokens)
        for layer in self.layers:
            x = layer(x)
        return self.output(self.norm(x))


@torch.no_grad()
def init_weights(model: nn.Module, seed: int = 0, std: float = 0.02,
                 norm_std: float = 0.0) -> nn.Module:
    """Fill every parameter from one CPU generator, in sorted state_dict order.

    Matrices get N(0, std); RMSNorm weights get 1 (or N(1, norm_std) when
    ``norm_std > 0``). Tied parameters are filled once. Works on any module
    whose state_dict names follow the reference model (so it also initialises
    the reference's own ``SimpleTransformer``-based model identically).
    """
    gen = torch.Generator().manual_seed(seed)
    seen = set()
    named = dict(model.named_parameters(remove_duplicate=True))
    for name in sorted(named):
        p = named[name]
        if id(p) in seen:
            continue
        seen.add(id(p))
        buf = torch.empty(p.shape, dtype=torch.float32)
        if name.endswith("norm.weight"):
            if norm_std > 0:
                buf.normal_(1.0, norm_std, generator=gen)
            else:
                buf.fill_(1.0)
        else:
            buf.normal_(0.0, std, generator=gen)
        p.copy_(buf)
    return model


def build_model(cfg, seed: int = 0, device="cpu", dtype=torch.float32) -> ReferenceLM:
    """Seeded random-weight reference model, weights drawn on the CPU then moved."""
    model = ReferenceLM(cfg)
    init_weights(model, seed)
    return model.to(device=device, dtype=dtype).eval()

