"""Decoder-block fusion: the residual adds move into the GEMM epilogues.

The reference patches leaf modules only (tinker/patch.py:57-116), so each
pre-norm block still runs ``x = x + attn(norm1(x)); x = x + ffn(norm2(x))``
with two separate elementwise adds in user code. After leaf patching, a block
whose children are exactly a ``TinKerRMSNorm``, a ``TinKerAttention``, a
``TinKerRMSNorm`` and a ``TinKerSwiGLU`` (any attribute names, in that order)
and whose ``forward`` takes the hidden states alone is a candidate: its forward
is replaced by

    h = attn(norm1(x), residual=x)      # o_proj epilogue adds x
    y = ffn(norm2(h), residual=h)       # down_proj epilogue adds h

which is 7 kernels per block and no torch kernel in between. With ``fold_norms`` (the
default of ``optimize``) the two RMSNorms go into the GEMMs that consume them: their
weights are multiplied into the q|k|v and gate|up weights (folded copies, made once and
remade when a source weight changes in place), each consumer epilogue scales its rows by
1/rms, and the rms statistics come from the producing epilogues (o_proj writes those of
``h``, down_proj those of the block output, handed to the next block on the output
tensor; the first block computes them from its input) - 5 kernels per block:

    qkv = linear_rope(x, Wqkv * w1)  * 1/rms(x)        (RoPE epilogue)
    h   = o_proj(attention(qkv)) + x        -> rms statistics of h
    g   = swiglu(h (Wg|Wu * w2)) * 1/rms(h)
    y   = down(g) + h                       -> rms statistics of y

The result differs from norm-then-GEMM only by where the rounding to the model dtype
happens (the weight product instead of the normalised activations). The statistics handed
from one block to the next describe the output tensor as returned; a change made to it in
place before the next block is detected through the tensor's version counter, except for
inference tensors (``torch.inference_mode``), which have none - a model that rescales its
residual stream in place between blocks under inference mode needs ``fold_norms=False``. The replacement is
bound only after the block's own forward is shown to have exactly that
dataflow: forward hooks substitute large random tensors for the outputs of the
four children and record their inputs, and the block must feed ``x`` to norm1,
norm1's output to attn, ``x + attn`` to norm2, norm2's output to ffn, call each
once, and return ``x + attn + ffn``. Blocks with any other structure (parallel
attention/FFN, post-norm, scaled residuals) are left as they are.
"""

from __future__ import annotations

import inspect
import types
import weakref

import torch
import torch.nn as nn

from tinker_b200.kernels.fused_attention import causal_attention
from tinker_b200.kernels.gemm import gate_up_swiglu, linear, linear_rope, row_sumsq
from tinker_b200.modules.attention import TinKerAttention
from tinker_b200.modules.feed_forward import TinKerSwiGLU
from tinker_b200.modules.normalization import TinKerRMSNorm

_PATTERN = (TinKerRMSNorm, TinKerAttention, TinKerRMSNorm, TinKerSwiGLU)


def _block_parts(block: nn.Module):
    kids = list(block.named_children())
    if len(kids) != 4 or tuple(type(m) for _, m in kids) != _PATTERN:
        return None
    return tuple(n for n, _ in kids)


def _takes_hidden_states_only(block: nn.Module) -> bool:
    try:
        sig = inspect.signature(block.forward)
    except (TypeError, ValueError):
        return False
    required = [p for p in sig.parameters.values()
                if p.default is inspect.Parameter.empty
                and p.kind in (inspect.Parameter.POSITIONAL_ONLY, inspect.Parameter.POSITIONAL_OR_KEYWORD)]
    return len(required) == 1


def _fused_forward(self, x: torch.Tensor, kv_cache=None, start_pos: int = 0,
                   position: torch.Tensor | None = None) -> torch.Tensor:
    n1, at, n2, ff = self._tinker_block_parts
    h = getattr(self, at)(getattr(self, n1)(x), start_pos=start_pos, residual=x, kv_cache=kv_cache,
                          position=position)
    return getattr(self, ff)(getattr(self, n2)(h), residual=h)


def _fold_sources(block):
    n1, at, n2, ff = (getattr(block, n) for n in block._tinker_block_parts)
    return (n1.weight, n2.weight, at.q_proj.weight, at.k_proj.weight, at.v_proj.weight, ff.gate_proj.weight,
            ff.up_proj.weight)


def _folded_weights(block):
    """The norm weights multiplied into the weights of the GEMMs that consume the norms (made
    again whenever one of the source tensors was modified in place since)."""
    src = _fold_sources(block)
    key = tuple((t.data_ptr(), t._version) for t in src)
    cached = getattr(block, "_tinker_folded", None)
    if cached is not None and cached[0] == key:
        return cached[1]
    w1, w2, wq, wk, wv, wg, wu = src
    with torch.no_grad():
        def fold(w, nw):
            return (w.float() * nw.float()[None, :]).to(w.dtype).contiguous()
        folded = (fold(wq, w1), fold(wk, w1), fold(wv, w1), fold(wg, w2), fold(wu, w2))
    block._tinker_folded = (key, folded)
    return folded


def _version_of(t: torch.Tensor):
    return None if t.is_inference() else t._version


def _can_fold(block, x: torch.Tensor) -> bool:
    n1, at, n2, ff = (getattr(block, n) for n in block._tinker_block_parts)
    return (x.dim() == 3 and x.shape[-1] % 32 == 0 and at.cos_table.dtype == torch.float32
            and at.sin_table.dtype == torch.float32 and at.head_dim % 32 == 0)


def _folded_forward(self, x: torch.Tensor, kv_cache=None, start_pos: int = 0,
                    position: torch.Tensor | None = None) -> torch.Tensor:
    """The block's forward; with ``kv_cache`` (a ``KVCacheLayer``) x holds new tokens from
    ``start_pos`` (or the device ``position``) on that attend to, and are appended to, the cache."""
    if not _can_fold(self, x):
        return _fused_forward(self, x, kv_cache, start_pos, position)
    n1, at, n2, ff = (getattr(self, n) for n in self._tinker_block_parts)
    wq, wk, wv, wg, wu = _folded_weights(self)
    B, S, H = x.shape
    m = B * S
    stats = getattr(x, "_tinker_row_ssq", None)
    ssq_x = None
    if stats is not None:
        ssq, version = stats
        # valid only for the contents they were computed from: an in-place change since then
        # shows in the version counter (inference tensors have none; see the module docstring)
        if version == _version_of(x) and ssq.shape == (H // 32, m) and ssq.device == x.device:
            ssq_x = ssq
    if ssq_x is None:
        ssq_x = row_sumsq(x)
    hq, hkv = at.num_heads * at.head_dim, at.num_kv_heads * at.head_dim
    # the q|k|v launch pulls the block's other weights into L2, the o_proj launch those of whatever
    # runs next (see _ahead_weights); not at <= 8 rows, where the weight-streaming GEMV kernels read
    # each weight straight from HBM faster than after a prefetch (batch-1 decode: 0.421 ms per
    # token with the prefetch, 0.408 without)
    hint = m > 8
    later = (at.o_proj.weight, wg, wu, ff.down_proj.weight) if hint else None
    if kv_cache is not None:
        a = at.cached_attention(x, wq, wk, wv, kv_cache, start_pos, position, row_ssq_in=ssq_x,
                                row_ssq_eps=n1.eps, l2_prefetch=later)
    else:
        qkv = linear_rope(x, wq, wk, wv, at.cos_table, at.sin_table, at.head_dim, 0, row_ssq_in=ssq_x,
                          row_ssq_eps=n1.eps, l2_prefetch=later)
        a = causal_attention(qkv[..., :hq], qkv[..., hq:hq + hkv], qkv[..., hq + hkv:], at.num_heads,
                             at.num_kv_heads, at.head_dim)
    ssq_h = torch.empty(H // 32, m, dtype=torch.float32, device=x.device)
    h = linear(a, at.o_proj.weight, residual=x, row_ssq_out=ssq_h,
               l2_prefetch=_ahead_weights(self) if hint else None)
    g = gate_up_swiglu(h, wg, wu, row_ssq_in=ssq_h, row_ssq_eps=n2.eps)
    ssq_y = torch.empty(H // 32, m, dtype=torch.float32, device=x.device)
    y = linear(g, ff.down_proj.weight, residual=h, row_ssq_out=ssq_y)
    y._tinker_row_ssq = (ssq_y, _version_of(y))  # the next folded block reads the statistics from here
    return y


_AHEAD_MAX_BYTES = 80 << 20


def _ahead_weights(block) -> tuple:
    """The weights the launches after this block start with: the next fused block's folded
    q|k|v weights (when it has made them), or the LM head weight after the last block. The
    o_proj launch pulls them into L2 so that the next block's first GEMM (or the head) streams
    them from there; the q|k|v launch does the same for the rest of its own block. The launch
    chain of a forward at a few hundred rows leaves HBM mostly idle, so these reads come free."""
    ref = block.__dict__.get("_tinker_ahead")
    nxt = ref() if ref is not None else None
    if nxt is None:
        return ()
    if isinstance(nxt, nn.Linear):
        w = nxt.weight
        # a head far larger than a third of L2 (a tied 150k-token table) would not stay there
        return (w,) if w.numel() * w.element_size() <= _AHEAD_MAX_BYTES else ()
    cached = nxt.__dict__.get("_tinker_folded")
    return tuple(cached[1][:3]) if cached is not None else ()


def link_ahead(model: nn.Module) -> int:
    """Record for every fused block which module runs next (the next fused block in module
    order, and after the last one the model's ``output`` / ``lm_head`` Linear if it has one),
    for the L2 prefetch of ``_ahead_weights``. A wrong guess costs bandwidth, never results."""
    blocks = [m for m in model.modules() if getattr(m, "_tinker_block_parts", None) is not None]
    head = next((h for h in (getattr(model, n, None) for n in ("output", "lm_head")) if isinstance(h, nn.Linear)),
                None)
    for i, b in enumerate(blocks):
        nxt = blocks[i + 1] if i + 1 < len(blocks) else head
        b.__dict__["_tinker_ahead"] = weakref.ref(nxt) if nxt is not None else None
    return len(blocks)


def _dataflow_is_prenorm_residual(block: nn.Module, parts, x: torch.Tensor, gen) -> bool:
    """Run the block's own forward with its children's outputs replaced by known
    tensors and check the pre-norm residual dataflow (see the module docstring)."""
    mods = [getattr(block, n) for n in parts]
    subst = [torch.randn(x.shape, device=x.device, generator=gen).to(x.dtype) * 4.0 for _ in mods]
    seen = [[] for _ in mods]
    handles = []
    for i, m in enumerate(mods):
        handles.append(m.register_forward_pre_hook(lambda mod, args, i=i: seen[i].append(args[0] if args else None)))
        handles.append(m.register_forward_hook(lambda mod, args, out, i=i: subst[i]))
    try:
        with torch.inference_mode():
            out = block(x)
    finally:
        for h in handles:
            h.remove()
    if any(len(v) != 1 or v[0] is None for v in seen):
        return False
    n1, a, n2, f = subst
    h = x + a
    checks = [(seen[0][0], x), (seen[1][0], n1), (seen[2][0], h), (seen[3][0], n2), (out, h + f)]
    for got, want in checks:
        if not isinstance(got, torch.Tensor) or got.shape != want.shape:
            return False
        if not torch.allclose(got.float(), want.float(), rtol=1e-2, atol=1e-2):
            return False
    return True


def fuse_decoder_blocks(model: nn.Module, verbose: bool = False, probe_tokens: int = 16,
                        fold_norms: bool = True) -> int:
    """Give every qualifying pre-norm decoder block the fused forward (with the RMSNorms folded
    into the GEMMs when ``fold_norms``); returns how many."""
    fused = 0
    gen = None
    for name, block in model.named_modules():
        parts = _block_parts(block)
        if parts is None or getattr(block, "_tinker_block_parts", None) is not None:
            continue
        if not _takes_hidden_states_only(block):
            if verbose:
                print(f"  [tinker] block {name}: forward takes more than the hidden states, not fused")
            continue
        norm1 = getattr(block, parts[0])
        w = getattr(block, parts[1]).q_proj.weight
        if gen is None:
            gen = torch.Generator(device=w.device).manual_seed(1234)
        x = torch.randn(1, probe_tokens, norm1.weight.shape[0], device=w.device, generator=gen).to(w.dtype)
        try:
            ok = _dataflow_is_prenorm_residual(block, parts, x, gen)
        except Exception as e:  # a block whose forward cannot run on the probe keeps its own forward
            ok = False
            if verbose:
                print(f"  [tinker] block {name}: not fused ({e})")
        if not ok:
            if verbose:
                print(f"  [tinker] block {name}: not a pre-norm residual block, not fused")
            continue
        block._tinker_block_parts = parts
        block.forward = types.MethodType(_folded_forward if fold_norms else _fused_forward, block)
        fused += 1
        if verbose:
            print(f"  [tinker] fused decoder block {name}")
    if fused:
        link_ahead(model)
    return fused


def share_rope_tables(model: nn.Module) -> int:
    """Point every ``TinKerAttention`` with the same table shape, device and values at one
    cos/sin pair, so the attention kernels of all layers read one L2-resident copy.
    Returns the number of modules re-pointed."""
    shared: dict = {}
    n = 0
    for m in model.modules():
        if not isinstance(m, TinKerAttention):
            continue
        c, s_ = m.cos_table, m.sin_table
        key = (tuple(c.shape), c.dtype, c.device, float(m.rope_theta))
        if key not in shared:
            shared[key] = (c, s_)
            continue
        c0, s0 = shared[key]
        if c0 is c or not (torch.equal(c0, c) and torch.equal(s0, s_)):
            continue
        m.cos_table, m.sin_table = c0, s0
        n += 1
    return n

