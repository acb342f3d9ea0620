"""KV-cache attention on the sm_100a kernel library (decode steps and short chunks).

The reference has no KV cache (eb1386/TinKer README.md:102): ``TinKerAttention``
recomputes every position, and ``start_pos`` only shifts the RoPE angles
(tinker/modules/attention.py:51). ``kv_attention`` gives the rows a cached
decode step needs: for new tokens at positions ``start_pos .. start_pos+S-1`` it
returns what the reference's causal RoPE attention over the whole sequence
(tinker/kernels/fused_attention.py:176-192) returns for those rows, reading
positions ``0 .. start_pos-1`` from the cache. One kernel rotates the new q and k
rows, appends the new k/v rows to the cache and attends; ``kv_append`` only fills
the cache (after a prompt ran through ``linear_rope`` + ``causal_attention``).

Cache layout: ``k_cache`` / ``v_cache`` are ``[batch, num_kv_heads, capacity, head_dim]``
contiguous, in the model dtype, keys stored after RoPE.
"""

from __future__ import annotations

import torch

from tinker_b200 import _lib
from tinker_b200.kernels._common import call_ctx
from tinker_b200.kernels.fused_attention import _token_stride


def kv_attention_workspace(batch: int, num_heads: int, num_kv_heads: int, head_dim: int, seq: int,
                           max_kv: int) -> int:
    """Bytes of zero-filled workspace ``kv_attention`` needs for these sizes when at most
    ``max_kv`` keys are attended (the cache capacity when the position is a device tensor)."""
    n = _lib.lib().tk_kv_attention_workspace(batch, num_heads, num_kv_heads, head_dim, seq, max_kv)
    if n < 0:
        raise RuntimeError(f"tk_kv_attention_workspace: {_lib.last_error()}")
    return int(n)


def _check_cache(k_cache: torch.Tensor, v_cache: torch.Tensor, B: int, num_kv_heads: int, head_dim: int,
                 dtype: torch.dtype) -> int:
    if k_cache.dim() != 4 or k_cache.shape != v_cache.shape:
        raise ValueError("k_cache / v_cache must both be [batch, num_kv_heads, capacity, head_dim]")
    if k_cache.shape[0] != B or k_cache.shape[1] != num_kv_heads or k_cache.shape[3] != head_dim:
        raise ValueError(f"cache shape {tuple(k_cache.shape)} does not match batch {B}, "
                         f"{num_kv_heads} kv heads, head_dim {head_dim}")
    if not (k_cache.is_contiguous() and v_cache.is_contiguous()):
        raise ValueError("k_cache / v_cache must be contiguous")
    if k_cache.dtype != dtype or v_cache.dtype != dtype:
        raise TypeError("the cache must have the dtype of q, k and v")
    return k_cache.shape[2]


def kv_attention(q, k, v, cos_table, sin_table, k_cache, v_cache, num_heads, num_kv_heads, head_dim,
                 start_pos: int = 0, position: torch.Tensor | None = None,
                 workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Attention of S new tokens per sequence against the cache, appending them to it.

    q: [B, S, num_heads * head_dim], k / v: [B, S, num_kv_heads * head_dim] projections
    without RoPE (column slices of a fused projection are read in place); cos_table /
    sin_table: float32 [max_seq_len, head_dim // 2]. The new tokens sit at positions
    ``start_pos .. start_pos + S - 1``, or from ``position[0]`` on when ``position`` (a one-element
    int32 CUDA tensor) is given; then the position is read when the kernel runs, so a captured
    CUDA graph serves every step, and a position past the cache records device error 2 instead
    of raising. ``workspace``: zero-filled uint8 CUDA tensor of at least
    ``kv_attention_workspace(...)`` bytes, returned to zeros by the kernel (allocated per call
    when omitted). Returns [B, S, num_heads * head_dim] in q's dtype.
    """
    dev = _lib.require_cuda(q, k, v, cos_table, sin_table, k_cache, v_cache)
    if q.dtype not in (torch.float16, torch.bfloat16) or k.dtype != q.dtype or v.dtype != q.dtype:
        raise TypeError("kv_attention: q, k, v must all be float16 or all bfloat16")
    if cos_table.dtype != torch.float32 or sin_table.dtype != torch.float32:
        raise TypeError("kv_attention: the RoPE tables must be float32")
    B, S = q.shape[0], q.shape[1]
    cap = _check_cache(k_cache, v_cache, B, num_kv_heads, head_dim, q.dtype)
    q3, qs = _token_stride(q, B, S, num_heads * head_dim)
    k3, ks = _token_stride(k, B, S, num_kv_heads * head_dim)
    v3, vs = _token_stride(v, B, S, num_kv_heads * head_dim)
    c = cos_table.contiguous()
    s = sin_table.contiguous()
    if c.shape != s.shape or c.dim() != 2 or c.shape[1] != head_dim // 2:
        raise ValueError(f"RoPE tables must be [max_seq_len, {head_dim // 2}], got {tuple(c.shape)}")
    pos_ptr = None
    if position is not None:
        if position.dtype != torch.int32 or position.device != q.device or position.numel() < 1:
            raise TypeError("kv_attention: position must be an int32 tensor on q's device")
        pos_ptr = position.data_ptr()
        max_kv = cap
    else:
        start_pos = int(start_pos)
        if start_pos < 0 or start_pos + S > cap:
            raise ValueError(f"kv_attention: positions {start_pos}..{start_pos + S - 1} exceed the cache "
                             f"capacity {cap}")
        max_kv = start_pos + S
    out = torch.empty(B, S, num_heads * head_dim, dtype=q.dtype, device=q.device)
    if B == 0 or S == 0:
        return out
    need = kv_attention_workspace(B, num_heads, num_kv_heads, head_dim, S, max_kv)
    if need > 0:
        if workspace is None:
            workspace = torch.zeros(need, dtype=torch.uint8, device=q.device)
        elif workspace.numel() * workspace.element_size() < need or workspace.device != q.device:
            raise ValueError(f"kv_attention: workspace smaller than the {need} bytes needed")
    ws_ptr = workspace.data_ptr() if need > 0 else None
    with call_ctx(dev):
        _lib.check(_lib.lib().tk_kv_attention(
            q3.data_ptr(), qs, k3.data_ptr(), ks, v3.data_ptr(), vs, k_cache.data_ptr(), v_cache.data_ptr(), cap,
            c.data_ptr(), s.data_ptr(), c.shape[0], out.data_ptr(), num_heads * head_dim, B, S, num_heads,
            num_kv_heads, head_dim, start_pos if position is None else 0, pos_ptr, ws_ptr, need,
            _lib.dtype_code(q.dtype), _lib.stream_ptr(dev)), "tk_kv_attention", 1)
    return out


def kv_append(k, v, k_cache, v_cache, start_pos: int = 0) -> None:
    """Write k (already rotated) and v, [B, S, num_kv_heads * head_dim], into the cache at
    positions ``start_pos .. start_pos + S - 1``."""
    dev = _lib.require_cuda(k, v, k_cache, v_cache)
    if k.dtype not in (torch.float16, torch.bfloat16) or v.dtype != k.dtype:
        raise TypeError("kv_append: k and v must both be float16 or both bfloat16")
    B, S = k.shape[0], k.shape[1]
    hkv, D = k_cache.shape[1], k_cache.shape[3]
    cap = _check_cache(k_cache, v_cache, B, hkv, D, k.dtype)
    k3, ks = _token_stride(k, B, S, hkv * D)
    v3, vs = _token_stride(v, B, S, hkv * D)
    if start_pos < 0 or start_pos + S > cap:
        raise ValueError(f"kv_append: positions {start_pos}..{start_pos + S - 1} exceed the cache capacity {cap}")
    with call_ctx(dev):
        _lib.check(_lib.lib().tk_kv_append(
            k3.data_ptr(), ks, v3.data_ptr(), vs, k_cache.data_ptr(), v_cache.data_ptr(), cap, B, S, hkv, D,
            int(start_pos), _lib.dtype_code(k.dtype), _lib.stream_ptr(dev)), "tk_kv_append", 1 if B * S else 0)
