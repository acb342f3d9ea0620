"""The whole decoder stack of a short prefill in one kernel (``tk_stack_forward``).

After ``optimize`` has fused every block of a decoder LM (``fusion.py``: RMSNorms folded
into the q|k|v and gate|up weights, residual adds in the GEMM epilogues), a forward over
at most 128 token rows (batch * seq) still launches 5 kernels per block. For such inputs
``install_stack_forward`` routes the model's forward through one persistent kernel that
runs the embedding, every block and the final RMSNorm (``csrc/stack.cu``), followed by
the model's own LM head. Larger inputs, inputs that are not int64 token ids, and models
whose forward is not exactly ``head(norm(blocks(embedding(tokens))))`` keep the
per-block path.

The top-level dataflow is checked once, at install time, by running the model's own
forward with the embedding, the blocks, the norm and the head replaced by stubs that
record their inputs and return marker tensors: the embedding must receive the tokens,
each block the previous block's output (the first: the embedding's), the norm the last
block's output, the head the norm's output, and the forward must return the head's.

Each token shape gets its own plan (``tk_stack_setup``: tile plan, tensor maps of every
weight, counters) on first use. Setting a plan up synchronises the device, so it cannot
happen during CUDA graph capture: a shape met for the first time while capturing takes
the per-block path (``optimize``'s capture runs three eager forwards first, which set
the plan up). The plan holds the folded weights as they were when it was made; it is
remade when a source weight was changed in place since (the same rule as the per-block
path), except inside a captured graph, which keeps what it was captured with.
"""

from __future__ import annotations

import types

import torch
import torch.nn as nn

from tinker_b200 import _lib
from tinker_b200.fusion import _folded_forward, _folded_weights, _version_of
from tinker_b200.kernels.gemm import embedding_rows
from tinker_b200.modules.attention import TinKerAttention
from tinker_b200.modules.normalization import TinKerRMSNorm

MAX_ROWS = 128


def _find(model: nn.Module, names):
    for n in names:
        m = getattr(model, n, None)
        if m is not None:
            return m
    return None


def _parts(model: nn.Module):
    emb = _find(model, ("embedding", "embed_tokens", "tok_embeddings"))
    layers = getattr(model, "layers", None)
    norm = getattr(model, "norm", None)
    head = _find(model, ("output", "lm_head"))
    if not isinstance(emb, nn.Embedding) or not isinstance(layers, (nn.ModuleList, list)) or not layers:
        return None
    if not isinstance(norm, TinKerRMSNorm) or not isinstance(head, nn.Linear) or head.bias is not None:
        return None
    return emb, list(layers), norm, head


def stack_blocker(model: nn.Module) -> str | None:
    """Why the one-kernel stack cannot run ``model`` (None: it can)."""
    parts = _parts(model)
    if parts is None:
        return "needs an nn.Embedding, a `layers` list, a TinKerRMSNorm `norm` and a bias-free Linear head"
    emb, layers, norm, head = parts
    w = emb.weight
    if not w.is_cuda or w.dtype not in (torch.float16, torch.bfloat16) or not w.is_contiguous():
        return "the embedding must be a contiguous float16 / bfloat16 CUDA tensor"
    if emb.padding_idx is not None or emb.max_norm is not None:
        return "embedding options (padding_idx, max_norm) are not supported"
    if norm.weight.dtype != w.dtype:
        return "the final norm weight must be in the model dtype"
    hidden = w.shape[1]
    a0 = None
    inter = None
    for i, block in enumerate(layers):
        if getattr(getattr(block, "forward", None), "__func__", None) is not _folded_forward:
            return f"layer {i} is not a fused block with folded norms (optimize(fold_norms=True))"
        n1, at, n2, ff = (getattr(block, n) for n in block._tinker_block_parts)
        if not isinstance(at, TinKerAttention):
            return f"layer {i}: attention is not a TinKerAttention"
        a0 = a0 or at
        if (at.num_heads, at.num_kv_heads, at.head_dim) != (a0.num_heads, a0.num_kv_heads, a0.head_dim):
            return "every layer must have the same attention shape"
        if at.head_dim != 64:
            return "head_dim must be 64"
        if at.cos_table.dtype != torch.float32 or not (at.cos_table is a0.cos_table or
                                                       torch.equal(at.cos_table, a0.cos_table)):
            return "every layer must use the same float32 RoPE tables"
        f = ff.gate_proj.weight.shape[0]
        inter = f if inter is None else inter
        if f != inter:
            return "every layer must have the same FFN width"
        if at.hidden_size != hidden or ff.hidden_size != hidden:
            return "layer widths must match the embedding width"
    if hidden % 64 or inter % 64:
        return "hidden and FFN widths must be multiples of 64"
    if head.weight.shape[1] != hidden:
        return "the LM head must read the hidden width"
    return None


def _dataflow_is_lm(model: nn.Module, orig_forward, emb, layers, norm, head, device) -> bool:
    """The model's own forward, with its parts replaced by recording stubs, computes
    head(norm(layer_n(... layer_1(embedding(tokens)))))."""
    gen = torch.Generator(device=device).manual_seed(4321)
    tokens = torch.randint(0, emb.num_embeddings, (1, 4), device=device, generator=gen)
    hidden = emb.weight.shape[1]
    mods = [emb, *layers, norm, head]
    dt = emb.weight.dtype
    outs = [torch.randn(1, 4, hidden, device=device, generator=gen).to(dt) for _ in range(len(mods) - 1)]
    outs.append(torch.randn(1, 4, head.weight.shape[0], device=device, generator=gen).to(dt))
    kept = [o.clone() for o in outs]  # an in-place change of a stub's output shows against these
    seen: list[list] = [[] for _ in mods]
    saved = []
    for i, m in enumerate(mods):
        saved.append(m.__dict__.get("forward"))

        def stub(self, *args, _i=i, **kwargs):
            seen[_i].append((args, kwargs))
            return outs[_i]

        m.forward = types.MethodType(stub, m)
    try:
        with torch.inference_mode():
            result = orig_forward(tokens)
    except Exception:
        return False
    finally:
        for m, f in zip(mods, saved):
            if f is None:
                del m.forward
            else:
                m.forward = f
    if any(len(s) != 1 or s[0][1] or len(s[0][0]) != 1 for s in seen):
        return False
    inputs = [s[0][0][0] for s in seen]
    if not (isinstance(inputs[0], torch.Tensor) and torch.equal(inputs[0], tokens)):
        return False
    for i in range(1, len(mods)):
        if inputs[i] is not outs[i - 1]:
            return False
    if not all(torch.equal(o, k) for o, k in zip(outs, kept)):
        return False
    return result is outs[-1]


class _StackPlan:
    """One token shape's plan: scratch, the layer table and the weights it points at."""

    def __init__(self, model, parts, batch: int, seq: int):
        emb, layers, norm, head = parts
        self.device = emb.weight.device
        self.dtype = emb.weight.dtype
        a0 = getattr(layers[0], layers[0]._tinker_block_parts[1])
        ff0 = getattr(layers[0], layers[0]._tinker_block_parts[3])
        self.hidden = emb.weight.shape[1]
        self.batch, self.seq = batch, seq
        table = (_lib.StackLayer * len(layers))()
        keep = []
        for i, block in enumerate(layers):
            n1, at, n2, ff = (getattr(block, n) for n in block._tinker_block_parts)
            wq, wk, wv, wg, wu = _folded_weights(block)
            keep += [wq, wk, wv, wg, wu]
            table[i] = _lib.StackLayer(wq.data_ptr(), wk.data_ptr(), wv.data_ptr(), at.o_proj.weight.data_ptr(),
                                       wg.data_ptr(), wu.data_ptr(), ff.down_proj.weight.data_ptr(),
                                       float(n1.eps), float(n2.eps))
        self.key = tuple(id(t) for t in keep)
        lib = _lib.lib()
        args = (len(layers), batch, seq, self.hidden, a0.num_heads, a0.num_kv_heads, a0.head_dim,
                ff0.gate_proj.weight.shape[0])
        with torch.cuda.device(self.device):
            nbytes = lib.tk_stack_scratch_bytes(*args)
            if nbytes <= 0:
                raise _lib.TinkerKernelError(f"tk_stack_scratch_bytes: {_lib.last_error()}")
            self.scratch = torch.empty(nbytes, dtype=torch.uint8, device=self.device)
            torch.cuda.synchronize(self.device)  # the set-up writes the scratch with synchronous copies
            _lib.check(lib.tk_stack_setup(table, *args, emb.weight.data_ptr(), emb.num_embeddings,
                                          a0.cos_table.data_ptr(), a0.sin_table.data_ptr(), a0.cos_table.shape[0], 0,
                                          norm.weight.data_ptr(), float(norm.eps),
                                          _lib.dtype_code(self.dtype), self.scratch.data_ptr(), nbytes),
                       "tk_stack_setup")
        self._keep = keep + [emb.weight, norm.weight, a0.cos_table, a0.sin_table]

    def plan(self) -> dict:
        """The tile plan the kernel runs: per projection (accumulator columns, tiles, k-splits, k-blocks)."""
        import ctypes
        out = (ctypes.c_int * 17)()
        _lib.check(_lib.lib().tk_stack_plan(self.scratch.data_ptr(), out, 17), "tk_stack_plan")
        names = ("qkv", "o_proj", "gate_up", "down")
        plan = {n: dict(zip(("bn", "tiles", "split", "k_blocks"), out[4 * i:4 * i + 4])) for i, n in enumerate(names)}
        plan["ctas"] = out[16]
        return plan

    def release(self) -> None:
        if self.scratch is not None:
            _lib.lib().tk_stack_release(self.scratch.data_ptr())
            self.scratch = None

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass

    def hidden_states(self, tokens: torch.Tensor) -> torch.Tensor:
        """The final RMSNorm of the last block's output, [batch, seq, hidden]."""
        y = torch.empty(self.batch * self.seq, self.hidden, dtype=self.dtype, device=self.device)
        _lib.check(_lib.lib().tk_stack_forward(tokens.data_ptr(), y.data_ptr(), self.scratch.data_ptr(),
                                               _lib.stream_ptr(self.device)), "tk_stack_forward", 1)
        return y.view(self.batch, self.seq, self.hidden)


def _stack_forward(self, tokens, *args, **kwargs):
    parts = self._tinker_stack_parts
    if (args or kwargs or not isinstance(tokens, torch.Tensor) or tokens.dim() != 2 or tokens.dtype != torch.long
            or tokens.numel() > MAX_ROWS or tokens.numel() == 0 or tokens.device != parts[0].weight.device):
        return self._tinker_stack_orig(tokens, *args, **kwargs)
    if not tokens.is_contiguous():
        tokens = tokens.contiguous()
    shape = (tokens.shape[0], tokens.shape[1])
    plans = self._tinker_stack_plans
    plan = plans.get(shape)
    capturing = torch.cuda.is_current_stream_capturing()
    if plan is not None and not capturing:
        layers = parts[1]
        key = tuple(id(t) for blk in layers for t in _folded_weights(blk))
        if key != plan.key:  # a weight was changed in place: fold again and make a new plan
            plan.release()
            plan = None
    if plan is None:
        if capturing:
            return self._tinker_stack_orig(tokens)
        plan = plans[shape] = _StackPlan(self, parts, *shape)
    # the model's LM head (torch's GEMM: measured faster than this library's at 128 rows)
    return parts[3](plan.hidden_states(tokens))


def _embedding_rows_forward(self, tokens: torch.Tensor) -> torch.Tensor:
    out, ssq = embedding_rows(tokens, self.weight)
    out._tinker_row_ssq = (ssq, _version_of(out))  # read by the first folded block
    return out


def install_embedding_rows(model: nn.Module, verbose: bool = False) -> bool:
    """Give the model's ``nn.Embedding`` a forward that gathers with ``tk_embedding_rows``, which also
    writes the row statistics of its output, so that the first folded block skips its row-statistics
    launch. Only for a forward that is exactly head(norm(blocks(embedding(tokens)))) (checked with
    stubs: an embedding output that the model scales or changes before the first block keeps the
    plain gather) whose first block is a folded block. Returns whether it was installed."""
    parts = _parts(model)
    if parts is None:
        return False
    emb, layers, norm, head = parts
    w = emb.weight
    if (emb.padding_idx is not None or emb.max_norm is not None or "forward" in emb.__dict__ or not w.is_cuda
            or w.dtype not in (torch.float16, torch.bfloat16) or not w.is_contiguous() or w.shape[1] % 32):
        return False
    if getattr(getattr(layers[0], "forward", None), "__func__", None) is not _folded_forward:
        return False
    if not _dataflow_is_lm(model, model.forward, emb, layers, norm, head, w.device):
        return False
    emb.forward = types.MethodType(_embedding_rows_forward, emb)
    if verbose:
        print("  [tinker] embedding gather with the first block's row statistics (one launch)")
    return True


def install_stack_forward(model: nn.Module, verbose: bool = False) -> bool:
    """Route ``model``'s forward over <= 128 token rows through ``tk_stack_forward`` when its
    blocks are fused with folded norms and its forward is embedding -> blocks -> norm -> head.
    Returns whether it was installed."""
    if getattr(model, "_tinker_stack_parts", None) is not None:
        return True
    reason = stack_blocker(model)
    parts = _parts(model)
    if reason is None and not _dataflow_is_lm(model, model.forward, *parts, parts[0].weight.device):
        reason = "the model's forward is not head(norm(blocks(embedding(tokens))))"
    if reason is not None:
        if verbose:
            print(f"  [tinker] one-kernel decoder stack not used: {reason}")
        return False
    model._tinker_stack_parts = parts
    model._tinker_stack_orig = model.forward
    model._tinker_stack_plans = {}
    model.forward = types.MethodType(_stack_forward, model)
    if verbose:
        print(f"  [tinker] one-kernel decoder stack for inputs of <= {MAX_ROWS} token rows")
    return True


def uninstall_stack_forward(model: nn.Module) -> None:
    """Give ``model`` back the per-block forward (releases every plan)."""
    if getattr(model, "_tinker_stack_parts", None) is None:
        return
    for plan in model._tinker_stack_plans.values():
        plan.release()
    model.forward = model._tinker_stack_orig
    del model._tinker_stack_parts, model._tinker_stack_orig, model._tinker_stack_plans
