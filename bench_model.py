"""The user model that ``bench.py`` hands to ``tinker_b200.optimize()``.

A plain PyTorch Llama-style decoder written the way a user's model would be: token
embedding, pre-norm blocks (RMSNorm -> grouped-query attention with interleaved-pair
RoPE -> residual, RMSNorm -> SwiGLU FFN -> residual), final RMSNorm, LM head (untied,
or tied to the embedding). It is the architecture the reference benchmarks and
patches (eb1386/TinKer benchmarks/bench_e2e.py:17-138 for the blocks,
examples/patch_any_model.py:95-108 for embedding and head), written independently:
RoPE by complex multiplication, grouped-query SDPA without repeating K/V. The
state_dict keys (``layers.{i}.attn.q_proj.weight`` ...) and attribute names
(``q_proj``, ``gate_proj``, ``weight``, ``eps``, ``head_dim``, ``rope_theta``) are the
ones the patcher looks for, so ``optimize`` rewrites this model exactly as it would
the reference's.

``init_weights`` fills parameters in sorted state_dict order from one CPU generator:
N(0, std) for matrices, 1 for norm weights. Any model with the same state_dict keys
gets the same weights for the same seed, so the parity tests give one set of tensors
to this model, to the CUDA path and to the oracle.
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
        per_layer = 2 * h * d * (self.num_heads + self.num_kv_heads) + 3 * h * self.intermediate_size + 2 * h
        embed = self.vocab_size * h * (1 if self.tied_embeddings else 2)
        return self.num_layers * per_layer + h + embed


# The decoder shapes the workloads are quoted on.
LLAMA_268M = DecoderConfig(vocab_size=32000, hidden_size=1024, num_layers=18, num_heads=16, num_kv_heads=4,
                           head_dim=64, intermediate_size=2816, eps=1e-6, rope_theta=10000.0)
QWEN25_05B_SHAPED = DecoderConfig(vocab_size=151936, hidden_size=896, num_layers=24, num_heads=14, num_kv_heads=2,
                                  head_dim=64, intermediate_size=4864, eps=1e-6, rope_theta=1e6,
                                  tied_embeddings=True)
LLAMA_1B = DecoderConfig(vocab_size=32000, hidden_size=2048, num_layers=16, num_heads=32, num_kv_heads=8,
                         head_dim=64, intermediate_size=5632, eps=1e-5, rope_theta=10000.0)
TINY = DecoderConfig(vocab_size=256, hidden_size=128, num_layers=2, num_heads=2, num_kv_heads=1, head_dim=64,
                     intermediate_size=256, max_seq_len=256)

PRESETS = {"llama268m": LLAMA_268M, "qwen25-0.5b-shaped": QWEN25_05B_SHAPED, "llama1b": LLAMA_1B, "tiny": TINY}


class Norm(nn.Module):
    """RMSNorm: statistics in float32, normalised value rounded to the input dtype, then scaled."""

    def __init__(self, dim: int, eps: float):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        inv_rms = torch.rsqrt(x.float().square().mean(dim=-1, keepdim=True) + self.eps)
        return self.weight * (x * inv_rms).to(x.dtype)


class MLP(nn.Module):
    """SwiGLU feed-forward: down(silu(gate x) * up x)."""

    def __init__(self, hidden: int, inner: int):
        super().__init__()
        self.gate_proj = nn.Linear(hidden, inner, bias=False)
        self.up_proj = nn.Linear(hidden, inner, bias=False)
        self.down_proj = nn.Linear(inner, hidden, bias=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        gated = F.silu(self.gate_proj(x)) * self.up_proj(x)
        return self.down_proj(gated)


def _angles(head_dim: int, max_seq_len: int, theta: float) -> torch.Tensor:
    """Rotation angle p * f_j of position p and pair j, f_j = theta^(-2j/head_dim), float32."""
    freqs = theta ** (-torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim)
    return torch.arange(max_seq_len, dtype=torch.float32)[:, None] * freqs[None, :]


class Attention(nn.Module):
    """Causal grouped-query attention; pairs (x[2j], x[2j+1]) of q and k rotate as complex numbers."""

    def __init__(self, cfg: DecoderConfig):
        super().__init__()
        self.num_heads, self.num_kv_heads, self.head_dim = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim
        self.rope_theta = cfg.rope_theta
        self.q_proj = nn.Linear(cfg.hidden_size, cfg.num_heads * cfg.head_dim, bias=False)
        self.k_proj = nn.Linear(cfg.hidden_size, cfg.num_kv_heads * cfg.head_dim, bias=False)
        self.v_proj = nn.Linear(cfg.hidden_size, cfg.num_kv_heads * cfg.head_dim, bias=False)
        self.o_proj = nn.Linear(cfg.num_heads * cfg.head_dim, cfg.hidden_size, bias=False)
        self.register_buffer("angles", _angles(cfg.head_dim, cfg.max_seq_len, cfg.rope_theta), persistent=False)

    def _apply(self, fn, recurse=True):
        angles = self.angles
        super()._apply(fn, recurse)
        self.angles = angles.to(self.q_proj.weight.device)  # the angles stay float32 under .half()
        return self

    def _rope(self, t: torch.Tensor) -> torch.Tensor:  # t: [B, heads, S, D]
        pairs = torch.view_as_complex(t.float().reshape(*t.shape[:-1], -1, 2))
        ang = self.angles[: t.shape[2]]
        return torch.view_as_real(pairs * torch.complex(ang.cos(), ang.sin())).flatten(-2).to(t.dtype)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        b, s, _ = x.shape

        def heads(proj, n):
            return proj(x).unflatten(-1, (n, self.head_dim)).transpose(1, 2)

        q = self._rope(heads(self.q_proj, self.num_heads))
        k = self._rope(heads(self.k_proj, self.num_kv_heads))
        v = heads(self.v_proj, self.num_kv_heads)
        o = F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=self.num_heads != self.num_kv_heads)
        return self.o_proj(o.transpose(1, 2).reshape(b, s, -1))


class Block(nn.Module):
    def __init__(self, cfg: DecoderConfig):
        super().__init__()
        self.attn_norm = Norm(cfg.hidden_size, cfg.eps)
        self.attn = Attention(cfg)
        self.ffn_norm = Norm(cfg.hidden_size, cfg.eps)
        self.ffn = MLP(cfg.hidden_size, cfg.intermediate_size)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        h = x + self.attn(self.attn_norm(x))
        return h + self.ffn(self.ffn_norm(h))


class DecoderLM(nn.Module):
    def __init__(self, cfg: DecoderConfig):
        super().__init__()
        self.config = cfg
        self.embedding = nn.Embedding(cfg.vocab_size, cfg.hidden_size)
        self.layers = nn.ModuleList(Block(cfg) for _ in range(cfg.num_layers))
        self.norm = Norm(cfg.hidden_size, cfg.eps)
        self.output = nn.Linear(cfg.hidden_size, cfg.vocab_size, bias=False)
        if cfg.tied_embeddings:
            self.output.weight = self.embedding.weight

    def forward(self, tokens: torch.Tensor) -> torch.Tensor:
        x = self.embedding(tokens)
        for block in self.layers:
            x = block(x)
        return self.output(self.norm(x))


@torch.no_grad()
def init_weights(model: nn.Module, seed: int = 0, std: float = 0.02) -> nn.Module:
    """Seeded fill in sorted parameter-name order (tied parameters once): N(0, std) for
    matrices, 1 for the weights of parameters whose name ends in ``norm.weight``."""
    gen = torch.Generator().manual_seed(seed)
    params = dict(model.named_parameters())  # named_parameters already drops tied duplicates
    for name in sorted(params):
        p = params[name]
        val = torch.empty(p.shape, dtype=torch.float32)
        if name.endswith("norm.weight"):
            val.fill_(1.0)
        else:
            val.normal_(0.0, std, generator=gen)
        p.copy_(val)
    return model


def build_model(cfg: DecoderConfig, seed: int = 0, device="cpu", dtype=torch.float32) -> DecoderLM:
    """A seeded random-weight model (weights drawn on the CPU, then moved and cast)."""
    return init_weights(DecoderLM(cfg), seed).to(device=device, dtype=dtype).eval()


def make_tokens(cfg: DecoderConfig, batch: int, seq: int, seed: int = 1) -> torch.Tensor:
    """Token ids uniform in [0, vocab) from their own CPU generator."""
    return torch.randint(0, cfg.vocab_size, (batch, seq), generator=torch.Generator().manual_seed(seed))
