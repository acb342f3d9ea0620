"""KV cache and cached decoding for patched Llama-style decoders.

The reference is inference-only without a KV cache (eb1386/TinKer README.md:97-103):
generating a token means a forward over the whole sequence so far. Here a
``KVCache`` keeps every layer's rotated keys and values, and ``CachedDecoder``
runs a prompt once (``prefill``) and then one token per step (``decode``), each
step attending to the cache through ``kv_attention``. The logits equal those of
the reference's full forward over the same tokens at the same positions, up to
the rounding of the half-precision intermediates.

A decode step is one CUDA graph replay: the token ids are copied into the
graph's input buffer, the attention kernels read the position from device
memory and the graph's last kernel advances it, so the same graph serves every
step and nothing but the token ids crosses from the host. Each block runs its
5 kernels; with ``fused_step=True`` the whole stack of blocks plus the final
RMSNorm runs as ONE persistent cooperative kernel per step instead
(``tk_decode_step``: grid barriers in place of the 5 launches per block), which
on B200 measures slower than the chained launches (0.63 vs 0.40 ms per token for
the 268M model at batch 1) and is kept as the alternative.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from tinker_b200 import _lib
from tinker_b200.fusion import _folded_forward, _folded_weights
from tinker_b200.kernels._common import call_ctx, stable_weights
from tinker_b200.kernels.kv_cache import kv_attention_workspace
from tinker_b200.modules.attention import TinKerAttention
from tinker_b200.modules.normalization import TinKerRMSNorm


class KVCacheLayer:
    """One layer's view of a ``KVCache``: ``k`` / ``v`` are ``[batch, num_kv_heads, capacity,
    head_dim]`` (keys after RoPE)."""

    def __init__(self, cache: "KVCache", index: int):
        self.cache = cache
        self.index = index
        self.k = cache.k[index]
        self.v = cache.v[index]

    def workspace(self, seq: int) -> torch.Tensor | None:
        return self.cache.workspace(seq)


class KVCache:
    """Keys and values of every layer, ``[num_layers, batch, num_kv_heads, capacity, head_dim]``.

    ``length`` is the number of positions filled (kept on the host by the caller that appends);
    ``position`` is a one-element int32 device tensor for CUDA graphs, whose kernels read the
    position when they run.
    """

    def __init__(self, num_layers: int, batch_size: int, num_heads: int, num_kv_heads: int, head_dim: int,
                 capacity: int, dtype: torch.dtype = torch.float16, device="cuda"):
        shape = (num_layers, batch_size, num_kv_heads, capacity, head_dim)
        self.k = torch.zeros(shape, dtype=dtype, device=device)
        self.v = torch.zeros(shape, dtype=dtype, device=device)
        self.num_heads = num_heads
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.batch_size = batch_size
        self.capacity = capacity
        self.length = 0
        self.position = torch.zeros(1, dtype=torch.int32, device=device)
        self._layers = [KVCacheLayer(self, i) for i in range(num_layers)]
        self._ws: dict = {}

    @property
    def num_layers(self) -> int:
        return len(self._layers)

    def layer(self, i: int) -> KVCacheLayer:
        return self._layers[i]

    def workspace(self, seq: int) -> torch.Tensor | None:
        """Zero-filled scratch for ``kv_attention`` with ``seq`` new tokens at any position up to
        the capacity (shared by the layers, whose kernels run one after another; the kernel
        returns it to zeros)."""
        need = kv_attention_workspace(self.batch_size, self.num_heads, self.num_kv_heads, self.head_dim, seq,
                                      self.capacity)
        if need == 0:
            return None
        ws = self._ws.get(seq)
        if ws is None or ws.numel() < need:
            ws = torch.zeros(need, dtype=torch.uint8, device=self.k.device)
            self._ws[seq] = ws
        return ws

    def reset(self) -> None:
        self.length = 0


def _find(model: nn.Module, names):
    for n in names:
        m = getattr(model, n, None)
        if m is not None:
            return m
    return None


class CachedDecoder:
    """Prefill + greedy token-by-token decoding of a patched decoder LM with a KV cache.

    ``model`` (or the model an ``optimize`` graph wrapper holds) needs a token embedding
    (``embedding`` / ``embed_tokens`` / ``tok_embeddings``), a ``layers`` list of pre-norm blocks
    that ``fuse_decoder_blocks`` fused (``optimize`` and ``patch_model`` + ``fuse_decoder_blocks``
    do that), a final ``norm`` and an LM head (``output`` / ``lm_head``). ``capacity`` defaults
    to the attention modules' RoPE table length. ``fused_step=True`` runs each decode step's
    blocks as one persistent kernel (``tk_decode_step``; raises when the model does not allow it);
    the default keeps the per-block kernels, which are faster on B200. The one-kernel step uses
    the folded weights as they are at its first step (like a captured graph).
    """

    def __init__(self, model: nn.Module, batch_size: int, capacity: int | None = None, cuda_graph: bool = True,
                 fused_step: bool = False):
        inner = getattr(model, "_model", None)
        if inner is not None and getattr(model, "_graph", None) is not None:
            model = inner  # an optimize() CUDA-graph wrapper: decode with its model
        self.model = model
        self.embedding = _find(model, ("embedding", "embed_tokens", "tok_embeddings"))
        self.layers = getattr(model, "layers", None)
        self.norm = getattr(model, "norm", None)
        self.head = _find(model, ("output", "lm_head"))
        if self.embedding is None or self.layers is None or self.norm is None or self.head is None:
            raise ValueError("CachedDecoder needs a model with an embedding, `layers`, `norm` and an LM head")
        attns = []
        for i, block in enumerate(self.layers):
            parts = getattr(block, "_tinker_block_parts", None)
            if parts is None:
                raise ValueError(f"layer {i} is not a fused decoder block (run optimize() or fuse_decoder_blocks)")
            attns.append(getattr(block, parts[1]))
        a0: TinKerAttention = attns[0]
        if capacity is None:
            capacity = a0.cos_table.shape[0]
        if capacity > a0.cos_table.shape[0]:
            raise ValueError(f"capacity {capacity} exceeds the RoPE table length {a0.cos_table.shape[0]}")
        w = self.embedding.weight
        self.device = w.device
        self.batch_size = batch_size
        self.cache = KVCache(len(attns), batch_size, a0.num_heads, a0.num_kv_heads, a0.head_dim, capacity,
                             dtype=w.dtype, device=w.device)
        self.cuda_graph = cuda_graph
        self._graph = None
        self._tokens = None
        self._logits = None
        self._position_stale = True  # cache.position must be set to cache.length before a replay
        self._attns = attns
        reason = self._fused_step_blocker()
        if fused_step and reason:
            raise ValueError(f"fused decode step unavailable: {reason}")
        self.fused_step = bool(fused_step)
        self._step_scratch = None

    @property
    def length(self) -> int:
        return self.cache.length

    def reset(self) -> None:
        self.cache.reset()
        self._position_stale = True

    def _fused_step_blocker(self) -> str | None:
        """Why the one-kernel decode step cannot run this model (None: it can)."""
        a0 = self._attns[0]
        w = self.embedding.weight
        if w.dtype not in (torch.float16, torch.bfloat16):
            return "the model dtype must be float16 or bfloat16"
        if self.batch_size > 8:
            return "more than 8 sequences"
        if a0.head_dim not in (64, 128) or a0.num_heads % a0.num_kv_heads or a0.num_heads // a0.num_kv_heads > 8:
            return "head_dim 64 or 128 and at most 8 query heads per kv head"
        if not isinstance(self.norm, TinKerRMSNorm) or self.norm.weight.dtype != w.dtype:
            return "the final norm must be a TinKerRMSNorm in the model dtype"
        hidden, inter = w.shape[1], None
        if hidden % 32:
            return "hidden size must be a multiple of 32"
        for block, at in zip(self.layers, self._attns):
            if getattr(block.forward, "__func__", None) is not _folded_forward:
                return "blocks must be fused with their RMSNorms folded (optimize(fold_norms=True))"
            n1, _, n2, ff = (getattr(block, n) for n in block._tinker_block_parts)
            if (at.num_heads, at.num_kv_heads, at.head_dim) != (a0.num_heads, a0.num_kv_heads, a0.head_dim):
                return "every layer must have the same attention shape"
            if at.cos_table.dtype != torch.float32 or not (at.cos_table is a0.cos_table or
                                                           torch.equal(at.cos_table, a0.cos_table)):
                return "every layer must use the same float32 RoPE tables"
            f = ff.gate_proj.weight.shape[0]
            inter = f if inter is None else inter
            if f != inter or f % 8:
                return "every layer must have the same FFN width, a multiple of 8"
            if n1.weight.dtype != w.dtype or n2.weight.dtype != w.dtype:
                return "norm weights must be in the model dtype"
        return None

    def _setup_step(self) -> None:
        """Upload the layer table of the one-kernel step (outside any graph capture)."""
        a0 = self._attns[0]
        L = len(self.layers)
        table = (_lib.StepLayer * L)()
        keep = []
        for i, block in enumerate(self.layers):
            n1, at, n2, ff = (getattr(block, n) for n in block._tinker_block_parts)
            wq, wk, wv, wg, wu = _folded_weights(block)
            keep += [wq, wk, wv, wg, wu]
            table[i] = _lib.StepLayer(wq.data_ptr(), wk.data_ptr(), wv.data_ptr(), at.o_proj.weight.data_ptr(),
                                      wg.data_ptr(), wu.data_ptr(), ff.down_proj.weight.data_ptr(),
                                      self.cache.k[i].data_ptr(), self.cache.v[i].data_ptr(), float(n1.eps),
                                      float(n2.eps))
        hidden = self.embedding.weight.shape[1]
        inter = self.layers[0].get_submodule(self.layers[0]._tinker_block_parts[3]).gate_proj.weight.shape[0]
        lib = _lib.lib()
        args = (L, self.batch_size, hidden, a0.num_heads, a0.num_kv_heads, a0.head_dim, inter, self.cache.capacity)
        nbytes = lib.tk_decode_step_scratch_bytes(*args)
        if nbytes <= 0:
            raise RuntimeError(f"tk_decode_step_scratch_bytes: {_lib.last_error()}")
        scratch = torch.empty(nbytes, dtype=torch.uint8, device=self.device)
        torch.cuda.synchronize(self.device)  # the set-up writes the scratch with synchronous copies
        with call_ctx(self.device):
            _lib.check(lib.tk_decode_step_setup(
                table, L, self.batch_size, hidden, a0.num_heads, a0.num_kv_heads, a0.head_dim, inter,
                a0.cos_table.data_ptr(), a0.sin_table.data_ptr(), a0.cos_table.shape[0], self.cache.capacity,
                self.cache.position.data_ptr(), self.norm.weight.data_ptr(), float(self.norm.eps),
                _lib.dtype_code(self.embedding.weight.dtype), scratch.data_ptr(), nbytes), "tk_decode_step_setup")
        self._step_scratch = scratch
        self._step_keep = keep

    def _fused_forward(self, tokens: torch.Tensor) -> torch.Tensor:
        """One new token per sequence through the one-kernel step; the position comes from
        cache.position. Returns the logits [batch, vocab]."""
        if self._step_scratch is None:
            self._setup_step()
        x = self.embedding(tokens).reshape(self.batch_size, -1)
        if not x.is_contiguous():
            x = x.contiguous()
        y = torch.empty_like(x)
        with call_ctx(self.device):
            _lib.check(_lib.lib().tk_decode_step(x.data_ptr(), y.data_ptr(), self._step_scratch.data_ptr(),
                                                 _lib.stream_ptr(self.device)), "tk_decode_step", 1)
        return self.head(y)

    def _forward(self, tokens: torch.Tensor, start_pos: int, position: torch.Tensor | None) -> torch.Tensor:
        if self.fused_step and tokens.shape[1] == 1 and position is not None:
            return self._fused_forward(tokens)
        x = self.embedding(tokens)
        for i, block in enumerate(self.layers):
            x = block.forward(x, kv_cache=self.cache.layer(i), start_pos=start_pos, position=position)
        return self.head(self.norm(x[:, -1:, :]))[:, 0, :]

    @torch.no_grad()
    def prefill(self, tokens: torch.Tensor) -> torch.Tensor:
        """Append ``tokens`` [batch, S] at the current length; returns the logits of the last
        position, [batch, vocab]."""
        tokens = tokens.to(self.device)
        if tokens.dim() != 2 or tokens.shape[0] != self.batch_size:
            raise ValueError(f"tokens must be [{self.batch_size}, S]")
        S = tokens.shape[1]
        if self.cache.length + S > self.cache.capacity:
            raise ValueError(f"{self.cache.length + S} positions exceed the cache capacity {self.cache.capacity}")
        logits = self._forward(tokens, self.cache.length, None)
        self.cache.length += S
        self._position_stale = True
        return logits

    def _capture(self) -> None:
        self._tokens = torch.zeros(self.batch_size, 1, dtype=torch.long, device=self.device)
        self.cache.position.fill_(self.cache.length)
        # eager warm-up on a side stream (workspace, folded weights, tensor maps); it writes the
        # cache row at the current length, which the first real step writes again
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            self._forward(self._tokens, 0, self.cache.position)
        torch.cuda.current_stream(self.device).wait_stream(side)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g), stable_weights():
            self._logits = self._forward(self._tokens, 0, self.cache.position)
            self.cache.position.add_(1)
        self._graph = g
        self._position_stale = False  # filled above; capturing ran nothing

    @torch.no_grad()
    def decode(self, tokens: torch.Tensor) -> torch.Tensor:
        """Append one token per sequence (``tokens`` [batch] or [batch, 1]); returns the logits of
        that position, [batch, vocab] (a buffer the next step overwrites when graphs are used)."""
        tokens = tokens.reshape(self.batch_size, 1)
        if self.cache.length + 1 > self.cache.capacity:
            raise ValueError(f"the cache is full ({self.cache.capacity} positions)")
        if not self.cuda_graph:
            if self.fused_step:  # the one-kernel step reads the position from device memory
                self.cache.position.fill_(self.cache.length)
                logits = self._forward(tokens.to(self.device), self.cache.length, self.cache.position)
            else:
                logits = self._forward(tokens.to(self.device), self.cache.length, None)
            self.cache.length += 1
            self._position_stale = True
            return logits
        if self._graph is None:
            self._capture()
        if self._position_stale:
            self.cache.position.fill_(self.cache.length)
            self._position_stale = False
        self._tokens.copy_(tokens, non_blocking=tokens.device.type == "cuda" or tokens.is_pinned())
        self._graph.replay()  # ends with position += 1
        self.cache.length += 1
        return self._logits

    @torch.no_grad()
    def generate(self, prompt: torch.Tensor, max_new_tokens: int) -> torch.Tensor:
        """Greedy decoding: prefill ``prompt`` [batch, S] into an empty cache, then
        ``max_new_tokens`` steps; returns the new token ids [batch, max_new_tokens] (CPU)."""
        self.reset()
        logits = self.prefill(prompt)
        out = []
        for _ in range(max_new_tokens):
            nxt = logits.argmax(-1)
            out.append(nxt.cpu())
            if len(out) == max_new_tokens:
                break
            logits = self.decode(nxt)
        return torch.stack(out, dim=1) if out else torch.empty(self.batch_size, 0, dtype=torch.long)

    def release(self) -> None:
        """Drop the captured graph (and its memory pool) and the one-kernel step's scratch."""
        self._graph = None
        self._logits = None
        if self._step_scratch is not None:
            _lib.lib().tk_decode_step_release(self._step_scratch.data_ptr())
            self._step_scratch = None

    def __del__(self):
        try:
            if getattr(self, "_step_scratch", None) is not None:
                _lib.lib().tk_decode_step_release(self._step_scratch.data_ptr())
        except Exception:
            pass
