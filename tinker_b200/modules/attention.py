"""Fused attention module (drop-in for eb1386/TinKer tinker/modules/attention.py:9-124).

``forward`` runs three kernels: the q|k|v projection as one tcgen05 GEMM over
the three weights (no concatenated copy) whose epilogue applies RoPE to the q
and k columns, the GQA causal attention reading q/k/v in place from that
output, and the o_proj GEMM. (Half-precision RoPE tables take the
``fused_attention`` path instead, which rotates on load inside attention.) The
``q_proj`` / ``k_proj`` / ``v_proj`` / ``o_proj`` submodules keep the reference's
names and shapes. The RoPE tables stay float32 when the module is cast to a
half dtype (the reference's ``model.to(dtype)`` rounds them to the model
dtype); positions are rotated with the exact float32 angles.
"""

import torch
import torch.nn as nn

from tinker_b200.kernels.fused_attention import causal_attention, fused_attention, precompute_rope_tables
from tinker_b200.kernels.gemm import linear, linear_rope
from tinker_b200.kernels.kv_cache import kv_append, kv_attention
from tinker_b200 import torch_ops
from tinker_b200.modules._roles import attention_projections

# Query rows per kv head (groups * new tokens) above which a prompt at position 0 runs on the
# tensor-core attention kernel before its keys/values are appended to the cache; below it the
# single kv_attention launch (rotate, append, attend) is cheaper.
PROMPT_MIN_ROWS = 64


class TinKerAttention(nn.Module):
    """Causal grouped-query attention with interleaved-pair RoPE on this library's kernels.

    args:
        hidden_size: model width (input and output features)
        num_heads: query heads
        num_kv_heads: key/value heads (a divisor of num_heads; 1 = MQA, num_heads = MHA)
        head_dim: features per head (default hidden_size // num_heads)
        rope_theta: RoPE frequency base
        max_seq_len: rows of the RoPE tables (the largest position + 1)
        dropout: accepted for signature compatibility; inference only, never applied
    """

    def __init__(
        self,
        hidden_size: int,
        num_heads: int,
        num_kv_heads: int,
        head_dim: int | None = None,
        rope_theta: float = 10000.0,
        max_seq_len: int = 2048,
        dropout: float = 0.0,
    ):
        super().__init__()
        self.hidden_size = hidden_size
        self.num_heads = num_heads
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim or (hidden_size // num_heads)
        self.rope_theta = rope_theta
        self.max_seq_len = max_seq_len

        self.q_proj = nn.Linear(hidden_size, num_heads * self.head_dim, bias=False)
        self.k_proj = nn.Linear(hidden_size, num_kv_heads * self.head_dim, bias=False)
        self.v_proj = nn.Linear(hidden_size, num_kv_heads * self.head_dim, bias=False)
        self.o_proj = nn.Linear(num_heads * self.head_dim, hidden_size, bias=False)

        cos_table, sin_table = precompute_rope_tables(self.head_dim, max_seq_len, rope_theta)
        self.register_buffer("cos_table", cos_table, persistent=False)
        self.register_buffer("sin_table", sin_table, persistent=False)

    def _apply(self, fn, recurse=True):
        # keep the RoPE tables in float32 across .to(dtype) / .half(); only move them
        cos, sin = self.cos_table, self.sin_table
        super()._apply(fn, recurse)
        dev = self.q_proj.weight.device
        self.cos_table = cos.to(device=dev)
        self.sin_table = sin.to(device=dev)
        return self

    def forward(self, x: torch.Tensor, start_pos: int = 0, residual: torch.Tensor | None = None,
                kv_cache=None, position: torch.Tensor | None = None) -> torch.Tensor:
        """forward pass; with ``residual`` the o_proj epilogue adds it to the output.

        ``kv_cache`` (a ``KVCacheLayer``): x holds the tokens at positions ``start_pos ..`` (or from
        the device int32 ``position[0]`` on), which attend to the cached positions before them and
        are appended to the cache."""
        if kv_cache is not None:
            a = self.cached_attention(x, self.q_proj.weight, self.k_proj.weight, self.v_proj.weight, kv_cache,
                                      start_pos, position)
            return linear(a, self.o_proj.weight, residual=residual)
        args = (x, self.q_proj.weight, self.k_proj.weight, self.v_proj.weight, self.o_proj.weight, self.cos_table,
                self.sin_table, self.num_heads, self.num_kv_heads, self.head_dim, int(start_pos), residual)
        if torch_ops.compiling():  # one opaque node for torch.compile (tinker_b200.torch_ops)
            return torch.ops.tinker.attention(*args)
        return attention_forward(*args)

    def cached_attention(self, x: torch.Tensor, wq: torch.Tensor, wk: torch.Tensor, wv: torch.Tensor, kv_cache,
                         start_pos: int = 0, position: torch.Tensor | None = None,
                         row_ssq_in: torch.Tensor | None = None, row_ssq_eps: float = 1e-6,
                         l2_prefetch=None) -> torch.Tensor:
        """q|k|v projection of x with the weights given (the module's own, or copies with an
        RMSNorm folded in, ``row_ssq_in``) and attention against ``kv_cache``, which receives the
        new keys and values. Returns the attention output [B, S, num_heads * head_dim].
        ``l2_prefetch``: tensors the projection launch pulls into L2 (``kernels.gemm.linear``).

        A prompt at position 0 with more than ``PROMPT_MIN_ROWS`` query rows per kv head takes the
        tensor-core path (RoPE in the projection epilogue, causal attention, cache append);
        everything else, decode steps included, one ``kv_attention`` kernel."""
        if (x.dim() != 3 or self.cos_table.dtype != torch.float32 or self.sin_table.dtype != torch.float32
                or self.head_dim not in (64, 128)):
            raise ValueError("KV-cache attention needs x [batch, seq, hidden], float32 RoPE tables and "
                             "head_dim 64 or 128")
        B, S, _ = x.shape
        hq = self.num_heads * self.head_dim
        hkv = self.num_kv_heads * self.head_dim
        groups = self.num_heads // self.num_kv_heads
        norm = {} if row_ssq_in is None else {"row_ssq_in": row_ssq_in, "row_ssq_eps": row_ssq_eps}
        if position is None and int(start_pos) == 0 and groups * S > PROMPT_MIN_ROWS:
            qkv = linear_rope(x, wq, wk, wv, self.cos_table, self.sin_table, self.head_dim, 0, **norm,
                              l2_prefetch=l2_prefetch)
            k, v = qkv[..., hq:hq + hkv], qkv[..., hq + hkv:]
            a = causal_attention(qkv[..., :hq], k, v, self.num_heads, self.num_kv_heads, self.head_dim)
            kv_append(k, v, kv_cache.k, kv_cache.v, 0)
            return a
        qkv = linear(x, wq, wk, wv, **norm, l2_prefetch=l2_prefetch)
        return kv_attention(qkv[..., :hq], qkv[..., hq:hq + hkv], qkv[..., hq + hkv:], self.cos_table,
                            self.sin_table, kv_cache.k, kv_cache.v, self.num_heads, self.num_kv_heads,
                            self.head_dim, start_pos, position, kv_cache.workspace(S))

    @classmethod
    def from_module(cls, source: nn.Module, rope_theta: float = 10000.0, max_seq_len: int = 2048) -> "TinKerAttention":
        """A ``TinKerAttention`` holding copies of ``source``'s q/k/v/o projection weights.

        The head layout comes from the weight shapes: ``source.head_dim`` when it has
        one, else the first of 64 and 128 that divides both the q and the k/v widths,
        else hidden / (q width / k/v width) (tinker/modules/attention.py:81-92). A
        ``rope_theta`` attribute on the source overrides the argument (:95-97)."""
        proj = attention_projections(source)
        q_rows, hidden = proj["q"].weight.shape
        kv_rows = proj["k"].weight.shape[0]
        head_dim, num_heads, num_kv_heads = _head_layout(source, hidden, q_rows, kv_rows)
        theta = getattr(source, "rope_theta", None)
        module = cls(hidden, num_heads, num_kv_heads, head_dim,
                     rope_theta=rope_theta if theta is None else theta, max_seq_len=max_seq_len)
        with torch.no_grad():
            for role in ("q", "k", "v", "o"):
                getattr(module, f"{role}_proj").weight.copy_(proj[role].weight)
        device = proj["q"].weight.device
        module.cos_table, module.sin_table = module.cos_table.to(device), module.sin_table.to(device)
        return module

    def extra_repr(self) -> str:
        return (f"hidden_size={self.hidden_size}, heads={self.num_heads}/{self.num_kv_heads} (q/kv), "
                f"head_dim={self.head_dim}, rope_theta={self.rope_theta}")


def attention_forward(x, wq, wk, wv, wo, cos_table, sin_table, num_heads: int, num_kv_heads: int, head_dim: int,
                      start_pos: int = 0, residual=None):
    """``TinKerAttention.forward`` without a KV cache: q|k|v projection, RoPE, causal GQA
    attention, o_proj (+ ``residual`` in its epilogue)."""
    hq = num_heads * head_dim
    hkv = num_kv_heads * head_dim
    if (x.dim() == 3 and cos_table.dtype == torch.float32 and sin_table.dtype == torch.float32
            and head_dim % 32 == 0 and hq % head_dim == 0):
        # RoPE in the projection epilogue, attention on the rotated q/k
        qkv = linear_rope(x, wq, wk, wv, cos_table, sin_table, head_dim, start_pos)
        attn_out = causal_attention(qkv[..., :hq], qkv[..., hq:hq + hkv], qkv[..., hq + hkv:], num_heads,
                                    num_kv_heads, head_dim)
        return linear(attn_out, wo, residual=residual)
    qkv = linear(x, wq, wk, wv)
    attn_out = fused_attention(qkv[..., :hq], qkv[..., hq:hq + hkv], qkv[..., hq + hkv:], cos_table, sin_table,
                               num_heads, num_kv_heads, head_dim, start_pos=start_pos)
    return linear(attn_out, wo, residual=residual)


def _head_layout(source: nn.Module, hidden: int, q_rows: int, kv_rows: int) -> tuple[int, int, int]:
    """(head_dim, query heads, kv heads) of a source attention module from its weight shapes."""
    head_dim = getattr(source, "head_dim", None)
    if head_dim is None:
        head_dim = next((d for d in (64, 128) if q_rows % d == 0 and kv_rows % d == 0), None)
    if head_dim is None:
        head_dim = hidden // (q_rows // kv_rows)
    return head_dim, q_rows // head_dim, kv_rows // head_dim
