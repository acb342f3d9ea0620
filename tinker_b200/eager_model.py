"""Plain-PyTorch Llama-style decoder: the user model that ``optimize()`` patches.

The blocks have the structure, attribute names and arithmetic of the model the
reference benchmarks (eb1386/TinKer benchmarks/bench_e2e.py:17-138), wrapped
with a token embedding and an LM head as in examples/patch_any_model.py:95-108.
Nothing here calls the CUDA extension: this is the *unpatched* eager model, the
reference's own eager path, and what ``patch_model`` rewrites in place.

``init_weights`` fills parameters deterministically (sorted ``state_dict``
names, one ``torch.Generator``), so the same seed gives identical weights in the
reference's own classes and in these.
"""

from __future__ import annotations

from dataclasses import dataclass, replace

import torch
import torch.nn as nn
import torch.nn.functional as F


@dataclass(frozen=True)
class DecoderConfig:
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

    def with_(self, **kw) -> "DecoderConfig":
        return replace(self, **kw)

    def num_params(self) -> int:
        h, d = self.hidden_size, self.head_dim
        attn = h * (self.num_heads * d) * 2 + h * (self.num_kv_heads * d) * 2
        ffn = 3 * h * self.intermediate_size
        layer = attn + ffn + 2 * h
        emb = self.vocab_size * h * (1 if self.tied_embeddings else 2)
        return self.num_layers * layer + h + emb


# The decoder shapes the workloads are quoted on.
LLAMA_268M = DecoderConfig(vocab_size=32000, hidden_size=1024, num_layers=18, num_heads=16,
                           num_kv_heads=4, head_dim=64, intermediate_size=2816, eps=1e-6,
                           rope_theta=10000.0, tied_embeddings=False)
QWEN25_05B_SHAPED = DecoderConfig(vocab_size=151936, hidden_size=896, num_layers=24, num_heads=14,
                                  num_kv_heads=2, head_dim=64, intermediate_size=4864, eps=1e-6,
                                  rope_theta=1e6, tied_embeddings=True)
LLAMA_1B = DecoderConfig(vocab_size=32000, hidden_size=2048, num_layers=16, num_heads=32,
                         num_kv_heads=8, head_dim=64, intermediate_size=5632, eps=1e-5,
                         rope_theta=10000.0, tied_embeddings=False)
TINY = DecoderConfig(vocab_size=256, hidden_size=128, num_layers=2, num_heads=2, num_kv_heads=1,
                     head_dim=64, intermediate_size=256, eps=1e-6, rope_theta=10000.0,
                     tied_embeddings=False, max_seq_len=256)

PRESETS = {"llama268m": LLAMA_268M, "qwen25-0.5b-shaped": QWEN25_05B_SHAPED,
           "llama1b": LLAMA_1B, "tiny": TINY}


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

    def __init__(self, cfg: DecoderConfig):
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


class DecoderLM(nn.Module):
    """Embedding -> blocks -> final RMSNorm -> LM head (examples/patch_any_model.py:95-108)."""

    def __init__(self, cfg: DecoderConfig):
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


def build_model(cfg: DecoderConfig, seed: int = 0, device="cpu", dtype=torch.float32) -> DecoderLM:
    """Seeded random-weight model, weights drawn on the CPU then moved."""
    model = DecoderLM(cfg)
    init_weights(model, seed)
    return model.to(device=device, dtype=dtype).eval()


def make_tokens(cfg: DecoderConfig, batch: int, seq: int, seed: int = 1) -> torch.Tensor:
    """Token ids uniform in [0, vocab) from their own CPU generator."""
    gen = torch.Generator().manual_seed(seed)
    return torch.randint(0, cfg.vocab_size, (batch, seq), generator=gen)
