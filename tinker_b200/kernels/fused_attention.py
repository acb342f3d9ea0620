"""Fused RoPE + GQA causal attention on the sm_100a kernel library.

Mirrors ``tinker.kernels.fused_attention`` (eb1386/TinKer
tinker/kernels/fused_attention.py): ``precompute_rope_tables`` (:157-162) with
the same torch arithmetic, and ``fused_attention`` (:234-238) with the same
arguments and result. Instead of the reference's three permute copies, two
in-place RoPE launches and the attention launch (:195-231), one tcgen05 kernel
reads q/k/v in their ``[batch, seq, heads * head_dim]`` projection layout,
applies RoPE on load and writes the output in that layout (the smallest
problems), or runs after one pass that rotates q and k (``tk_rope_qk``).
"""

from __future__ import annotations

import torch

from tinker_b200 import _lib
from tinker_b200.kernels._common import call_ctx


# fused_attention rotates q and k in one separate pass (tk_rope_qk) and runs the attention kernel
# without RoPE, except for the smallest problems (head_dim 64 and at most this many tokens), where
# one kernel that rotates on load saves the extra launch. Rotating on load re-reads the cos/sin
# rows of every key tile in every CTA, which costs more than the pass from there on (measured on
# B200: equal at batch 8 x seq 128, head_dim 64; the pass is 1.3-2.6x faster at seq >= 512).
ROPE_ON_LOAD_MAX_TOKENS = 1024


def _rope_on_load(batch: int, seq: int, head_dim: int) -> bool:
    return head_dim == 64 and batch * seq <= ROPE_ON_LOAD_MAX_TOKENS and seq <= 128


def precompute_rope_tables(head_dim, max_seq_len, theta=10000.0, device=None, dtype=torch.float32):
    """precompute sin/cos tables for rope."""
    freqs = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32, device=device) / head_dim))
    positions = torch.arange(max_seq_len, dtype=torch.float32, device=device)
    angles = torch.outer(positions, freqs)
    return torch.cos(angles).to(dtype), torch.sin(angles).to(dtype)


def _token_stride(t: torch.Tensor, B: int, S: int, width: int) -> tuple[torch.Tensor, int]:
    """(tensor, token stride) for a [B, S, width] input whose last dim is contiguous.

    Column slices of a fused QKV projection are used in place; anything else is
    copied to a contiguous tensor first.
    """
    if t.dim() != 3 or t.shape[0] != B or t.shape[1] != S or t.shape[2] != width:
        raise ValueError(f"expected shape ({B}, {S}, {width}), got {tuple(t.shape)}")
    st = t.stride()
    tok = st[1] if S > 1 else (st[0] if B > 1 else width)
    if (st[2] == 1 and tok >= width and tok % 8 == 0 and t.data_ptr() % 16 == 0
            and (B == 1 or S == 1 or st[0] == S * st[1])):
        return t, tok
    return t.contiguous(), width


def fused_attention(q, k, v, cos_table, sin_table, num_heads, num_kv_heads, head_dim, start_pos=0):
    """fused rope + gqa + attention.

    q: [B, S, num_heads * head_dim]; k, v: [B, S, num_kv_heads * head_dim];
    cos_table / sin_table: [max_seq_len, head_dim // 2] (float32, float16 or bfloat16).
    Returns [B, S, num_heads * head_dim] in q's dtype (float16 or bfloat16).
    """
    dev = _lib.require_cuda(q, k, v, cos_table, sin_table)
    if q.dtype not in (torch.float16, torch.bfloat16) or k.dtype != q.dtype or v.dtype != q.dtype:
        raise TypeError("fused_attention: q, k, v must all be float16 or all bfloat16")
    B, S = q.shape[0], q.shape[1]
    q3, qs = _token_stride(q, B, S, num_heads * head_dim)
    k3, ks = _token_stride(k, B, S, num_kv_heads * head_dim)
    v3, vs = _token_stride(v, B, S, num_kv_heads * head_dim)
    c = cos_table.contiguous()
    s = sin_table.contiguous()
    if c.shape != s.shape or c.dim() != 2 or c.shape[1] != head_dim // 2:
        raise ValueError(f"RoPE tables must be [max_seq_len, {head_dim // 2}], got {tuple(c.shape)}")
    if s.dtype != c.dtype:
        s = s.to(c.dtype)
    out = torch.empty(B, S, num_heads * head_dim, dtype=q.dtype, device=q.device)
    if not _rope_on_load(B, S, head_dim):
        # rotate q and k once into one [B, S, (Hq+Hkv)*D] buffer, then attention without RoPE: on
        # load, every CTA would re-read the cos/sin rows of every key tile
        hq, hkv = num_heads * head_dim, num_kv_heads * head_dim
        qk = torch.empty(B, S, hq + hkv, dtype=q.dtype, device=q.device)
        with call_ctx(dev):
            _lib.check(_lib.lib().tk_rope_qk(
                q3.data_ptr(), qs, k3.data_ptr(), ks, c.data_ptr(), s.data_ptr(), _lib.dtype_code(c.dtype),
                c.shape[0], qk.data_ptr(), hq + hkv, B, S, num_heads, num_kv_heads, head_dim, int(start_pos),
                _lib.dtype_code(q.dtype), _lib.stream_ptr(dev)), "tk_rope_qk", 1)
            _lib.check(_lib.lib().tk_causal_attention(
                qk.data_ptr(), hq + hkv, qk.data_ptr() + hq * qk.element_size(), hq + hkv, v3.data_ptr(), vs,
                out.data_ptr(), hq, B, S, num_heads, num_kv_heads, head_dim, _lib.dtype_code(q.dtype),
                _lib.stream_ptr(dev)), "tk_causal_attention", 1)
        return out
    with call_ctx(dev):
        _lib.check(_lib.lib().tk_rope_attention(
            q3.data_ptr(), qs, k3.data_ptr(), ks, v3.data_ptr(), vs, c.data_ptr(), s.data_ptr(),
            _lib.dtype_code(c.dtype), c.shape[0], out.data_ptr(), num_heads * head_dim, B, S, num_heads,
            num_kv_heads, head_dim, int(start_pos), _lib.dtype_code(q.dtype), _lib.stream_ptr(dev)),
            "tk_rope_attention", 1)
    return out


def causal_attention(q, k, v, num_heads, num_kv_heads, head_dim):
    """GQA causal attention on q and k that already carry RoPE (``linear_rope`` output slices):
    the kernel of ``fused_attention`` without the rotation. Same shapes and result layout."""
    dev = _lib.require_cuda(q, k, v)
    if q.dtype not in (torch.float16, torch.bfloat16) or k.dtype != q.dtype or v.dtype != q.dtype:
        raise TypeError("causal_attention: q, k, v must all be float16 or all bfloat16")
    B, S = q.shape[0], q.shape[1]
    q3, qs = _token_stride(q, B, S, num_heads * head_dim)
    k3, ks = _token_stride(k, B, S, num_kv_heads * head_dim)
    v3, vs = _token_stride(v, B, S, num_kv_heads * head_dim)
    out = torch.empty(B, S, num_heads * head_dim, dtype=q.dtype, device=q.device)
    with call_ctx(dev):
        _lib.check(_lib.lib().tk_causal_attention(
            q3.data_ptr(), qs, k3.data_ptr(), ks, v3.data_ptr(), vs, out.data_ptr(), num_heads * head_dim, B, S,
            num_heads, num_kv_heads, head_dim, _lib.dtype_code(q.dtype), _lib.stream_ptr(dev)),
            "tk_causal_attention", 1)
    return out
