"""numpy restatement of the reference's eager kernels (test infrastructure only).

Every function cites the reference line range it restates (paths are relative
to the eb1386/TinKer project root). Arithmetic is done in float32 by default,
the precision of the reference's eager fallbacks, or in float64 when
``acc=np.float64`` is passed. Half-precision rounding points are reproduced with
:func:`round_to` so that the oracle can stand in for the reference's fp16/bf16
eager path as well as its fp32 one.
"""

from __future__ import annotations

import numpy as np

F16 = "float16"
BF16 = "bfloat16"
F32 = "float32"


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round an array to ``dtype`` and return it widened to float32.

    fp16 uses numpy's IEEE binary16 conversion (round to nearest even). bf16
    keeps the top 16 bits of the float32 pattern after round-to-nearest-even,
    the conversion ``Tensor.to(torch.bfloat16)`` performs. ``float32`` only
    narrows float64 input.
    """
    x = np.asarray(x)
    if dtype == F32:
        return x.astype(np.float32)
    if dtype == F16:
        return x.astype(np.float32).astype(np.float16).astype(np.float32)
    if dtype == BF16:
        u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
        nan = np.isnan(x)
        u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
        out = u.astype(np.uint32).view(np.float32).reshape(np.shape(x))
        return np.where(nan, np.float32(np.nan), out)
    raise ValueError(f"unknown dtype {dtype!r}")


def rope_tables(head_dim: int, max_seq_len: int, theta: float = 10000.0):
    """cos/sin tables ``[max_seq_len, head_dim // 2]`` in float32.

    Restates ``precompute_rope_tables`` (tinker/kernels/fused_attention.py:157-162):
    ``freqs[i] = 1 / theta ** (2i / head_dim)``, angles = outer(positions, freqs).
    """
    exps = np.arange(0, head_dim, 2, dtype=np.float32) / np.float32(head_dim)
    freqs = (np.float32(1.0) / np.power(np.float32(theta), exps, dtype=np.float32)).astype(np.float32)
    pos = np.arange(max_seq_len, dtype=np.float32)
    ang = np.outer(pos, freqs).astype(np.float32)
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def apply_rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray, start_pos: int = 0,
               out_dtype: str = F32, acc=np.float32) -> np.ndarray:
    """Interleaved RoPE on ``x[B, H, S, D]``.

    Restates ``_apply_rope_pytorch`` (tinker/kernels/fused_attention.py:165-173):
    pairs ``(x[2i], x[2i+1])`` rotate by ``(cos, sin)[start_pos + s, i]`` in float32,
    and the result is rounded back to the input dtype (``out_dtype``).
    """
    S = x.shape[2]
    c = cos[start_pos:start_pos + S].astype(acc)[None, None]
    s = sin[start_pos:start_pos + S].astype(acc)[None, None]
    xe = x[..., 0::2].astype(acc)
    xo = x[..., 1::2].astype(acc)
    ne = xe * c - xo * s
    no = xe * s + xo * c
    out = np.stack([ne, no], axis=-1).reshape(x.shape)
    return round_to(out, out_dtype) if out_dtype != F32 else out.astype(np.float32)


def attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, cos: np.ndarray, sin: np.ndarray,
              num_heads: int, num_kv_heads: int, head_dim: int, start_pos: int = 0,
              io_dtype: str = F32, acc=np.float64) -> np.ndarray:
    """RoPE + GQA causal attention, ``q[B,S,Hq*D]``, ``k/v[B,S,Hkv*D]`` -> ``[B,S,Hq*D]``.

    Restates ``_attention_pytorch`` (tinker/kernels/fused_attention.py:176-192):
    heads split from the hidden axis, RoPE applied to q and k (result rounded to
    the input dtype, :165-173), K/V heads repeated ``num_heads // num_kv_heads``
    times so query head ``h`` reads KV head ``h // groups`` (:186-188, the same
    mapping as the Triton kernel's ``kv_head = pid_h // num_kv_groups`` at :104),
    then ``scaled_dot_product_attention(is_causal=True)`` with scale
    ``1/sqrt(head_dim)`` (:191; :216 for the kernel). The softmax is computed in
    ``acc`` precision; the output is rounded to ``io_dtype``.
    """
    B, S, _ = q.shape
    groups = num_heads // num_kv_heads
    qh = q.reshape(B, S, num_heads, head_dim).transpose(0, 2, 1, 3)
    kh = k.reshape(B, S, num_kv_heads, head_dim).transpose(0, 2, 1, 3)
    vh = v.reshape(B, S, num_kv_heads, head_dim).transpose(0, 2, 1, 3)
    qh = apply_rope(qh, cos, sin, start_pos, out_dtype=io_dtype)
    kh = apply_rope(kh, cos, sin, start_pos, out_dtype=io_dtype)
    if groups > 1:
        kh = np.repeat(kh, groups, axis=1)
        vh = np.repeat(vh, groups, axis=1)
    qh = np.asarray(qh, dtype=acc)
    kh = np.asarray(kh, dtype=acc)
    vh = np.asarray(vh, dtype=acc)
    scale = 1.0 / np.sqrt(head_dim)
    scores = np.matmul(qh, kh.transpose(0, 1, 3, 2)) * scale
    mask = np.triu(np.ones((S, S), dtype=bool), k=1)
    scores = np.where(mask[None, None], -np.inf, scores)
    scores = scores - scores.max(axis=-1, keepdims=True)
    p = np.exp(scores)
    p = p / p.sum(axis=-1, keepdims=True)
    out = np.matmul(p, vh)
    out = out.transpose(0, 2, 1, 3).reshape(B, S, num_heads * head_dim)
    return round_to(out, io_dtype) if io_dtype != F32 else out.astype(np.float32)


def attention_rows(q: np.ndarray, k: np.ndarray, v: np.ndarray, cos: np.ndarray, sin: np.ndarray,
                   num_heads: int, num_kv_heads: int, head_dim: int, start_pos: int,
                   io_dtype: str = F32, acc=np.float64) -> np.ndarray:
    """Rows ``start_pos .. start_pos+S-1`` of :func:`attention` over a whole sequence.

    ``q[B,S,Hq*D]`` holds the queries of those positions only; ``k/v[B,start_pos+S,Hkv*D]`` all
    keys and values of the sequence (none rotated yet). The arithmetic is that of
    ``_attention_pytorch`` (tinker/kernels/fused_attention.py:176-192) with RoPE at absolute
    positions (:165-173) and the causal mask of ``is_causal=True`` (query at position p sees keys
    0..p, the kernel's ``q >= kv`` at :132), restricted to the last S query rows: what a decode
    step with a KV cache must return, which the reference (no cache) obtains by running the
    whole sequence.
    """
    B, S, _ = q.shape
    L = k.shape[1]
    if L != start_pos + S:
        raise ValueError("k/v must hold positions 0 .. start_pos + S - 1")
    groups = num_heads // num_kv_heads
    qh = q.reshape(B, S, num_heads, head_dim).transpose(0, 2, 1, 3)
    kh = k.reshape(B, L, num_kv_heads, head_dim).transpose(0, 2, 1, 3)
    vh = v.reshape(B, L, num_kv_heads, head_dim).transpose(0, 2, 1, 3)
    qh = apply_rope(qh, cos, sin, start_pos, out_dtype=io_dtype)
    kh = apply_rope(kh, cos, sin, 0, out_dtype=io_dtype)
    if groups > 1:
        kh = np.repeat(kh, groups, axis=1)
        vh = np.repeat(vh, groups, axis=1)
    qh = np.asarray(qh, dtype=acc)
    kh = np.asarray(kh, dtype=acc)
    vh = np.asarray(vh, dtype=acc)
    scale = 1.0 / np.sqrt(head_dim)
    scores = np.matmul(qh, kh.transpose(0, 1, 3, 2)) * scale
    mask = np.arange(L)[None, :] > (start_pos + np.arange(S))[:, None]
    scores = np.where(mask[None, None], -np.inf, scores)
    scores = scores - scores.max(axis=-1, keepdims=True)
    p = np.exp(scores)
    p = p / p.sum(axis=-1, keepdims=True)
    out = np.matmul(p, vh)
    out = out.transpose(0, 2, 1, 3).reshape(B, S, num_heads * head_dim)
    return round_to(out, io_dtype) if io_dtype != F32 else out.astype(np.float32)


def rmsnorm(x: np.ndarray, weight: np.ndarray, eps: float = 1e-6, out_dtype: str = F32,
            acc=np.float32) -> np.ndarray:
    """``y = x * rsqrt(mean(x^2) + eps) * w`` over the last axis.

    Restates ``_rmsnorm_pytorch`` (tinker/kernels/fused_rmsnorm.py:64-67), the
    same arithmetic the Triton kernel performs (:37-52): float32 accumulation,
    one rounding to the output dtype at the end.
    """
    xf = x.astype(acc)
    ms = np.mean(xf * xf, axis=-1, keepdims=True, dtype=acc)
    r = (1.0 / np.sqrt(ms + acc(eps))).astype(acc)
    y = xf * r * weight.astype(acc)
    return round_to(y, out_dtype) if out_dtype != F32 else y.astype(np.float32)


def add_rmsnorm(x: np.ndarray, residual: np.ndarray, weight: np.ndarray, eps: float = 1e-6,
                out_dtype: str = F32, acc=np.float32):
    """``s = x + residual`` (rounded to the model dtype) and ``rmsnorm(s)``.

    The residual stream update of the reference decoder block
    (benchmarks/bench_e2e.py:112-115: ``x = x + attn(...)`` in the model dtype)
    followed by the next block's RMSNorm. Returns ``(y, s)``.
    """
    s = x.astype(np.float32) + residual.astype(np.float32)
    s = round_to(s, out_dtype) if out_dtype != F32 else s
    return rmsnorm(s, weight, eps, out_dtype, acc), s


def swiglu(gate: np.ndarray, up: np.ndarray, out_dtype: str = F32, acc=np.float32) -> np.ndarray:
    """``silu(gate) * up``.

    Restates the arithmetic of ``_swiglu_kernel`` (tinker/kernels/fused_swiglu.py:37-44):
    ``gate * sigmoid(gate) * up`` in float32, one rounding to the output dtype.
    (The eager fallback ``F.silu(gate).mul_(up)`` at :57-58 rounds after the silu as
    well; the two agree to one half-precision ulp.)
    """
    g = gate.astype(acc)
    u = up.astype(acc)
    y = g / (acc(1.0) + np.exp(-g)) * u
    return round_to(y, out_dtype) if out_dtype != F32 else y.astype(np.float32)


def linear(x: np.ndarray, w: np.ndarray, out_dtype: str = F32, acc=np.float32) -> np.ndarray:
    """``x @ w.T`` as ``nn.Linear(bias=False)`` computes it (the projections of
    tinker/modules/attention.py:40-43 and tinker/modules/feed_forward.py:22-24)."""
    y = np.matmul(np.asarray(x, dtype=acc), np.asarray(w, dtype=acc).T)
    return round_to(y, out_dtype) if out_dtype != F32 else y.astype(np.float32)
