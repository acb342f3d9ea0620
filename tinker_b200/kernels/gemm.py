"""tcgen05 GEMMs for the projections (tinker_b200/csrc/gemm.cu).

The reference runs every projection through ``nn.Linear`` / cuBLAS
(eb1386/TinKer tinker/modules/attention.py:53-55,64 and
tinker/modules/feed_forward.py:27-30). Here they are hand-written sm_100a GEMMs:

* ``linear(x, w0, w1=None, w2=None, residual=None)`` - ``x @ cat(w0, w1, w2).T``
  without materialising the concatenation (the fused q|k|v projection), with an
  optional residual add in the epilogue.
* ``linear_rope(x, wq, wk, wv, cos, sin, head_dim, start_pos)`` - the q|k|v projection with
  RoPE applied to the q and k columns in the epilogue.
* ``row_sumsq(x)`` and the ``row_ssq_in`` / ``row_ssq_out`` options: an RMSNorm folded into the
  GEMM that consumes it (norm weight multiplied into the weights, 1/rms per row in the epilogue).
* ``gate_up_swiglu(x, w_gate, w_up)`` - ``silu(x @ w_gate.T) * (x @ w_up.T)`` as one
  GEMM with the SwiGLU applied to the fp32 accumulators.
* ``swiglu_ffn(x, w_gate, w_up, w_down, residual=None)`` - the whole FFN.
"""

from __future__ import annotations

import torch

from tinker_b200 import _lib
from tinker_b200.kernels._common import call_ctx, row_stride, rows_view, weights_are_stable


def _check_w(w: torch.Tensor, k: int, dtype) -> torch.Tensor:
    if w.dim() != 2 or w.shape[1] != k:
        raise ValueError(f"weight must be [n, {k}], got {tuple(w.shape)}")
    if w.dtype != dtype:
        raise TypeError(f"weight dtype {w.dtype} does not match input dtype {dtype}")
    return w if w.is_contiguous() else w.contiguous()


def _check_x(x: torch.Tensor) -> torch.Tensor:
    if x.dtype not in (torch.float16, torch.bfloat16):
        raise TypeError("tinker_b200 GEMMs take float16 or bfloat16 inputs")
    x2 = rows_view(x)
    if row_stride(x2) % 8 != 0 or x2.data_ptr() % 16 != 0:
        x2 = x2.contiguous()
    return x2


def _epilogue(residual=None, row_ssq_in=None, row_ssq_eps=1e-6, row_ssq_out=None, rope=None, l2_prefetch=None):
    """A ``tk_epilogue`` for the ``_ex`` entry points (None when only the plain store is needed)."""
    stable = weights_are_stable()
    pf = [t for t in (l2_prefetch or ()) if t is not None and t.is_cuda and t.is_contiguous() and t.numel()]
    if residual is None and row_ssq_in is None and row_ssq_out is None and rope is None and not stable and not pf:
        return None
    e = _lib.Epilogue()
    e.weights_prefetch = 1 if stable else 0
    for i, t in enumerate(pf[:len(e.l2_prefetch)]):
        e.l2_prefetch[i] = t.data_ptr()
        e.l2_prefetch_bytes[i] = t.numel() * t.element_size()
    e.residual = None if residual is None else residual.data_ptr()
    if row_ssq_in is not None:
        if row_ssq_in.dtype != torch.float32 or row_ssq_in.dim() != 2 or not row_ssq_in.is_contiguous():
            raise ValueError("row_ssq_in must be a contiguous float32 [parts, m] tensor")
        e.row_ssq_in = row_ssq_in.data_ptr()
        e.row_ssq_parts = row_ssq_in.shape[0]
        e.row_ssq_eps = float(row_ssq_eps)
    if row_ssq_out is not None:
        e.row_ssq_out = row_ssq_out.data_ptr()
    if rope is not None:
        cos, sin, head_dim, seq, start_pos = rope
        e.rope_cos, e.rope_sin = cos.data_ptr(), sin.data_ptr()
        e.rope_head_dim, e.rope_seq, e.rope_start = head_dim, seq, int(start_pos)
        e.rope_table_rows = cos.shape[0]
    return e


def _check_ssq(t: torch.Tensor | None, m: int, parts: int | None, what: str):
    if t is None:
        return
    if t.dtype != torch.float32 or t.dim() != 2 or t.shape[1] != m or not t.is_contiguous():
        raise ValueError(f"{what} must be a contiguous float32 [parts, {m}] tensor")
    if parts is not None and t.shape[0] != parts:
        raise ValueError(f"{what} must have {parts} partial sums per row")


def row_sumsq(x: torch.Tensor) -> torch.Tensor:
    """Per-32-column partial sums of squares of the rows of ``x`` [..., k]: float32 [k/32, rows],
    the ``row_ssq_in`` of a GEMM that consumes ``rmsnorm(x)`` with the norm weight folded in."""
    dev = _lib.require_cuda(x)
    x2 = _check_x(x)
    m, k = x2.shape
    parts = torch.empty((k + 31) // 32, m, dtype=torch.float32, device=x.device)
    with call_ctx(dev):
        _lib.check(_lib.lib().tk_row_sumsq(x2.data_ptr(), row_stride(x2), m, k, parts.data_ptr(),
                                           _lib.dtype_code(x.dtype), _lib.stream_ptr(dev)), "tk_row_sumsq", 1)
    return parts


def embedding_rows(tokens: torch.Tensor, table: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """``table[tokens]`` ([..., hidden], the gather of ``nn.Embedding`` without padding_idx / max_norm)
    and its per-32-column row sums of squares (float32 [hidden/32, rows], the ``row_ssq_in`` of a
    GEMM with the next RMSNorm folded in), in one launch. A token outside the table records device
    error 3 (``tinker_b200._lib.device_error``) and gives a zero row."""
    dev = _lib.require_cuda(tokens, table)
    if table.dtype not in (torch.float16, torch.bfloat16) or table.dim() != 2 or not table.is_contiguous():
        raise TypeError("embedding_rows: the table must be a contiguous float16 / bfloat16 [vocab, hidden] tensor")
    vocab, hidden = table.shape
    if hidden % 32:
        raise ValueError("embedding_rows: hidden must be a multiple of 32")
    ids = tokens.reshape(-1)
    if ids.dtype != torch.int64 or not ids.is_contiguous():
        ids = ids.to(torch.int64).contiguous()
    rows = ids.numel()
    out = torch.empty(*tokens.shape, hidden, dtype=table.dtype, device=table.device)
    parts = torch.empty(hidden // 32, rows, dtype=torch.float32, device=table.device)
    with call_ctx(dev):
        _lib.check(_lib.lib().tk_embedding_rows(ids.data_ptr(), table.data_ptr(), vocab, hidden, out.data_ptr(),
                                                parts.data_ptr(), rows, _lib.dtype_code(table.dtype),
                                                _lib.stream_ptr(dev)), "tk_embedding_rows", 1)
    return out, parts


def linear(x: torch.Tensor, w0: torch.Tensor, w1: torch.Tensor | None = None, w2: torch.Tensor | None = None,
           residual: torch.Tensor | None = None, out: torch.Tensor | None = None,
           row_ssq_in: torch.Tensor | None = None, row_ssq_eps: float = 1e-6,
           row_ssq_out: torch.Tensor | None = None, l2_prefetch=None) -> torch.Tensor:
    """``x @ cat([w0, w1, w2]).T (+ residual)``; x [..., k], w* [n*, k].

    ``row_ssq_in`` ([parts, m] float32, from ``row_sumsq`` or another GEMM's ``row_ssq_out``) scales
    each output row by ``1/sqrt(mean(x_row^2) + row_ssq_eps)``: with an RMSNorm weight folded into
    the weights this is ``rmsnorm(x) @ W.T``. ``row_ssq_out`` ([ceil(n/32), m] float32) receives the
    partial sums of squares of the stored rows for the next folded RMSNorm. ``l2_prefetch``: up to
    8 contiguous device tensors (the weights of the kernels that follow) that the launch pulls
    into L2 while it runs; they must stay alive until it has finished."""
    ws = [w for w in (w0, w1, w2) if w is not None]
    dev = _lib.require_cuda(x, *ws)
    x2 = _check_x(x)
    k = x2.shape[1]
    ws = [_check_w(w, k, x.dtype) for w in ws]
    n = sum(w.shape[0] for w in ws)
    m = x2.shape[0]
    lead = x.shape[:-1]
    if out is None:
        out = torch.empty(m, n, dtype=x.dtype, device=x.device)
    elif out.shape != (m, n) or not out.is_contiguous():
        raise ValueError("out must be a contiguous [m, n] tensor")
    r = None
    if residual is not None:
        r = residual.reshape(m, n)
        if not r.is_contiguous() or r.dtype != x.dtype:
            r = r.contiguous().to(x.dtype)
    _check_ssq(row_ssq_in, m, None, "row_ssq_in")
    _check_ssq(row_ssq_out, m, (n + 31) // 32, "row_ssq_out")
    ptrs = [w.data_ptr() for w in ws] + [None] * (3 - len(ws))
    rows = [w.shape[0] for w in ws] + [0] * (3 - len(ws))
    e = _epilogue(r, row_ssq_in, row_ssq_eps, row_ssq_out, l2_prefetch=l2_prefetch)
    with call_ctx(dev):
        if e is None:
            _lib.check(_lib.lib().tk_linear(x2.data_ptr(), row_stride(x2), ptrs[0], rows[0], ptrs[1], rows[1], ptrs[2],
                                            rows[2], out.data_ptr(), n, None, m, k,
                                            _lib.dtype_code(x.dtype), _lib.stream_ptr(dev)), "tk_linear", 1)
        else:
            _lib.check(_lib.lib().tk_linear_ex(x2.data_ptr(), row_stride(x2), ptrs[0], rows[0], ptrs[1], rows[1],
                                               ptrs[2], rows[2], out.data_ptr(), n, m, k, e,
                                               _lib.dtype_code(x.dtype), _lib.stream_ptr(dev)), "tk_linear_ex", 1)
    return out.reshape(*lead, n)


def linear_rope(x: torch.Tensor, wq: torch.Tensor, wk: torch.Tensor, wv: torch.Tensor, cos_table: torch.Tensor,
                sin_table: torch.Tensor, head_dim: int, start_pos: int = 0,
                row_ssq_in: torch.Tensor | None = None, row_ssq_eps: float = 1e-6,
                l2_prefetch=None) -> torch.Tensor:
    """``x @ cat([wq, wk, wv]).T`` for x [batch, seq, hidden] with RoPE applied to the q and k
    columns in the GEMM epilogue (each value rounded to the output dtype, then rotated in fp32 at
    position ``start_pos + s``): the q|k|v projection plus the RoPE of ``fused_attention``.
    ``row_ssq_in`` / ``row_ssq_eps`` / ``l2_prefetch`` as in ``linear`` (the attention RMSNorm
    folded in)."""
    dev = _lib.require_cuda(x, wq, wk, wv, cos_table, sin_table)
    if x.dim() != 3:
        raise ValueError("linear_rope: x must be [batch, seq, hidden]")
    if cos_table.dtype != torch.float32 or sin_table.dtype != torch.float32:
        raise TypeError("linear_rope: RoPE tables must be float32")
    B, S, k = x.shape
    x2 = _check_x(x)
    wq, wk, wv = (_check_w(w, k, x.dtype) for w in (wq, wk, wv))
    c, s_ = cos_table.contiguous(), sin_table.contiguous()
    if c.shape != s_.shape or c.dim() != 2 or c.shape[1] != head_dim // 2:
        raise ValueError(f"RoPE tables must be [max_seq_len, {head_dim // 2}], got {tuple(c.shape)}")
    n = wq.shape[0] + wk.shape[0] + wv.shape[0]
    m = x2.shape[0]
    _check_ssq(row_ssq_in, m, None, "row_ssq_in")
    out = torch.empty(m, n, dtype=x.dtype, device=x.device)
    with call_ctx(dev):
        if row_ssq_in is None and not weights_are_stable() and not l2_prefetch:
            _lib.check(_lib.lib().tk_linear_rope(
                x2.data_ptr(), row_stride(x2), wq.data_ptr(), wq.shape[0], wk.data_ptr(), wk.shape[0],
                wv.data_ptr(), wv.shape[0], out.data_ptr(), n, m, k, S, int(start_pos), head_dim, c.data_ptr(),
                s_.data_ptr(), c.shape[0], _lib.dtype_code(x.dtype), _lib.stream_ptr(dev)), "tk_linear_rope", 1)
        else:
            if wq.shape[0] % head_dim or wk.shape[0] % head_dim:
                raise ValueError("linear_rope: q and k widths must be multiples of head_dim")
            e = _epilogue(None, row_ssq_in, row_ssq_eps, None, (c, s_, head_dim, S, start_pos), l2_prefetch)
            _lib.check(_lib.lib().tk_linear_ex(
                x2.data_ptr(), row_stride(x2), wq.data_ptr(), wq.shape[0], wk.data_ptr(), wk.shape[0],
                wv.data_ptr(), wv.shape[0], out.data_ptr(), n, m, k, e, _lib.dtype_code(x.dtype),
                _lib.stream_ptr(dev)), "tk_linear_ex", 1)
    return out.reshape(B, S, n)


def gate_up_swiglu(x: torch.Tensor, w_gate: torch.Tensor, w_up: torch.Tensor,
                   row_ssq_in: torch.Tensor | None = None, row_ssq_eps: float = 1e-6,
                   l2_prefetch=None) -> torch.Tensor:
    """``silu(x @ w_gate.T) * (x @ w_up.T)`` as one GEMM with a SwiGLU epilogue; ``row_ssq_in`` /
    ``row_ssq_eps`` / ``l2_prefetch`` as in ``linear`` (the FFN RMSNorm folded into both weights)."""
    dev = _lib.require_cuda(x, w_gate, w_up)
    x2 = _check_x(x)
    k = x2.shape[1]
    wg, wu = _check_w(w_gate, k, x.dtype), _check_w(w_up, k, x.dtype)
    if wg.shape != wu.shape:
        raise ValueError("gate and up weights must have the same shape")
    f = wg.shape[0]
    m = x2.shape[0]
    _check_ssq(row_ssq_in, m, None, "row_ssq_in")
    h = torch.empty(m, f, dtype=x.dtype, device=x.device)
    e = _epilogue(None, row_ssq_in, row_ssq_eps, l2_prefetch=l2_prefetch)
    with call_ctx(dev):
        if e is None:
            _lib.check(_lib.lib().tk_gate_up_swiglu(x2.data_ptr(), row_stride(x2), wg.data_ptr(), wu.data_ptr(),
                                                    h.data_ptr(), m, k, f, _lib.dtype_code(x.dtype),
                                                    _lib.stream_ptr(dev)), "tk_gate_up_swiglu", 1)
        else:
            _lib.check(_lib.lib().tk_gate_up_swiglu_ex(x2.data_ptr(), row_stride(x2), wg.data_ptr(), wu.data_ptr(),
                                                       h.data_ptr(), m, k, f, e, _lib.dtype_code(x.dtype),
                                                       _lib.stream_ptr(dev)), "tk_gate_up_swiglu_ex", 1)
    return h.reshape(*x.shape[:-1], f)


def swiglu_ffn(x: torch.Tensor, w_gate: torch.Tensor, w_up: torch.Tensor, w_down: torch.Tensor,
               residual: torch.Tensor | None = None) -> torch.Tensor:
    """``down(silu(gate(x)) * up(x)) (+ residual)``: gate|up GEMM with SwiGLU epilogue, then down GEMM.

    The [m, f] activation between the two GEMMs is scratch memory allocated here
    from PyTorch's caching allocator.
    """
    dev = _lib.require_cuda(x, w_gate, w_up, w_down)
    x2 = _check_x(x)
    k = x2.shape[1]
    wg, wu = _check_w(w_gate, k, x.dtype), _check_w(w_up, k, x.dtype)
    f = wg.shape[0]
    wd = _check_w(w_down, f, x.dtype)
    if wd.shape[0] != k:
        raise ValueError("down projection must map back to the hidden size")
    m = x2.shape[0]
    h = torch.empty(m, f, dtype=x.dtype, device=x.device)
    out = torch.empty(m, k, dtype=x.dtype, device=x.device)
    r = None
    if residual is not None:
        r = residual.reshape(m, k).contiguous()
    with call_ctx(dev):
        _lib.check(_lib.lib().tk_swiglu_ffn(x2.data_ptr(), row_stride(x2), wg.data_ptr(), wu.data_ptr(),
                                            wd.data_ptr(), h.data_ptr(), out.data_ptr(),
                                            None if r is None else r.data_ptr(), m, k, f,
                                            _lib.dtype_code(x.dtype), _lib.stream_ptr(dev)), "tk_swiglu_ffn", 2)
    return out.reshape(*x.shape[:-1], k)
