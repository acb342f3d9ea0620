"""model optimizer - the main api (drop-in for eb1386/TinKer tinker/optimize.py:27-242).

``optimize`` applies, in the reference's order:
  1. module patching: RMSNorm / SwiGLU FFN / GQA attention -> ``TinKer*`` modules
     running the sm_100a kernels (the reference gates this on Triton being
     importable; here it needs the built kernel library and a B200)
  2. half precision (``dtype``), then decoder-block fusion (``fuse_blocks``)
  3. int8 dynamic quantization: not part of the B200 path (the reference's is a
     CPU-only ``quantize_dynamic``); reported and skipped
  4. ``compile=True``: ``torch.compile(model, mode=compile_mode)``; the patched modules
     call registered torch ops while being compiled (``tinker_b200.torch_ops``), so the
     kernels are single graph nodes, and block fusion / the one-kernel stack (Python-level
     rewrites that do not trace) are skipped. The default (None) does not compile: the
     hand-written kernels and the CUDA graph already remove what compiling would
  5. CUDA backend flags (TF32, cuDNN benchmark, flash SDPA) as in the reference
  6. optional CUDA graph capture of the whole forward (static shapes)
"""

import math
import statistics
import time

import torch
import torch.nn as nn

from tinker_b200 import _lib
from tinker_b200.fusion import fuse_decoder_blocks, share_rope_tables
from tinker_b200.kernels._common import stable_weights
from tinker_b200.patch import patch_model
from tinker_b200.stack import install_embedding_rows, install_stack_forward


def optimize(
    model: nn.Module,
    dtype: torch.dtype | None = None,
    compile: bool | None = None,
    compile_mode: str = "reduce-overhead",
    quantize: bool = False,
    replace_attention: bool = True,
    replace_ffn: bool = True,
    replace_norm: bool = True,
    rope_theta: float = 10000.0,
    max_seq_len: int = 2048,
    cuda_graph: bool = False,
    graph_input_shape: tuple | None = None,
    graph_vocab_size: int = 32000,
    verbose: bool = False,
    graph_clone_output: bool = True,
    fuse_blocks: bool = True,
    fold_norms: bool = True,
    stack_kernel: bool = False,
) -> nn.Module:
    """optimize a model for inference on a B200.

    Same arguments as the reference, plus three:
    ``graph_clone_output`` (default True, as in the reference) controls whether the
    CUDA-graph wrapper returns a clone of its static output or the static output
    itself; ``fuse_blocks`` (default True) gives qualifying pre-norm decoder blocks
    a forward whose residual adds run inside the GEMM epilogues
    (``tinker_b200.fusion``), after checking the block's dataflow; ``fold_norms``
    (default True) also folds those blocks' RMSNorms into the GEMMs after them;
    ``stack_kernel`` (default False) runs a forward over at most 128 token rows of a
    decoder LM whose blocks were fused and folded as one persistent kernel for the
    embedding, all blocks and the final norm (``tinker_b200.stack``), then the LM head.
    """
    model.eval()
    params = list(model.parameters())
    if not params or not params[0].is_cuda:
        raise RuntimeError("tinker_b200.optimize needs the model on a CUDA device (B200, sm_100a); "
                           "move it with model.to('cuda') first")
    _lib.require_cuda(params[0])

    if verbose:
        print("[tinker] patching modules (sm_100a fused kernels)...")
    model = patch_model(
        model,
        replace_attention=replace_attention,
        replace_ffn=replace_ffn,
        replace_norm=replace_norm,
        rope_theta=rope_theta,
        max_seq_len=max_seq_len,
        verbose=verbose,
    )

    if dtype is not None:
        if verbose:
            print(f"  [tinker] casting to {dtype}")
        model = model.to(dtype=dtype)

    if replace_attention:
        share_rope_tables(model)

    if compile and fuse_blocks and verbose:
        print("  [tinker] compile=True: decoder blocks left unfused (their Python-level fusion does not trace)")
    if fuse_blocks and not compile and replace_attention and replace_ffn and replace_norm:
        n = fuse_decoder_blocks(model, verbose=verbose, fold_norms=fold_norms)
        if verbose:
            print(f"  [tinker] fused {n} decoder blocks (residual adds in the GEMM epilogues)")
        if fold_norms and n:
            install_embedding_rows(model, verbose=verbose)
        if stack_kernel and fold_norms and n:
            install_stack_forward(model, verbose=verbose)

    if quantize and verbose:
        print("  [tinker] int8 quantization skipped: not part of the B200 kernel path")

    if compile:
        # the TinKer* modules call registered ops while compiled (tinker_b200.torch_ops), so the
        # patched model traces without graph breaks; a failure keeps the eager model, as in the
        # reference (tinker/optimize.py:77-88)
        if verbose:
            print(f"  [tinker] torch.compile (mode={compile_mode})")
        try:
            model = torch.compile(model, mode=compile_mode)
        except Exception as e:
            if verbose:
                print(f"  [tinker] compile failed: {e}")

    torch.backends.cudnn.benchmark = True
    torch.backends.cuda.matmul.allow_tf32 = True
    torch.backends.cudnn.allow_tf32 = True
    torch.set_float32_matmul_precision("high")
    torch.backends.cuda.enable_flash_sdp(True)
    torch.backends.cuda.enable_mem_efficient_sdp(True)
    if verbose:
        print("  [tinker] cuda: tf32 + cudnn benchmark + flash sdpa")

    for p in model.parameters():
        p.requires_grad_(False)
    if verbose:
        print("  [tinker] disabled gradients")

    if cuda_graph:
        if graph_input_shape is not None:
            model = _capture_cuda_graph(model, graph_input_shape, graph_vocab_size, verbose=verbose,
                                        clone_output=graph_clone_output)
        elif verbose:
            print("  [tinker] skipping cuda graph (no input shape)")

    if verbose:
        print(f"\n  [tinker] ready (sm_100a kernels + {torch.cuda.get_device_name(params[0].device)})")
    return model


class _CUDAGraphWrapper(nn.Module):
    """A model whose forward for one input shape is a CUDA graph replay.

    The graph reads its tokens from a static input buffer and writes its logits to a
    static output buffer (both owned by the graph's memory pool). A call with the
    captured shape copies the tokens in, replays the graph and returns the logits - a
    fresh copy by default, as the reference does (tinker/optimize.py:134-150), or, with
    ``clone_output=False``, the static buffer itself, which the next replay overwrites.
    Any other shape runs the wrapped model eagerly.
    """

    def __init__(self, model, static_input, static_output, graph, clone_output=True):
        super().__init__()
        self._model = model
        self._static_input = static_input
        self._static_output = static_output
        self._graph = graph
        self._clone_output = clone_output

    @property
    def _input_shape(self):
        return self._static_input.shape

    def forward(self, x):
        if x.shape != self._static_input.shape:
            return self._model(x)
        self._static_input.copy_(x, non_blocking=True)
        self._graph.replay()
        if self._clone_output:
            return self._static_output.clone()
        return self._static_output


def _capture_cuda_graph(model, input_shape, vocab_size, verbose=False, clone_output=True):
    """Capture ``model``'s forward on random token ids of ``input_shape`` in a CUDA graph.

    Three eager forwards come first (they build every kernel's launch state and the
    folded weights, which must not happen during capture), then one captured forward
    under ``stable_weights`` (no kernel of the forward writes a weight, so the GEMMs may
    stage weight tiles before their dependency wait). On any failure the model is
    returned unchanged and the reason reported when ``verbose``, as in the reference
    (tinker/optimize.py:153-173)."""
    device = next(model.parameters()).device
    tokens = torch.randint(0, vocab_size, tuple(input_shape), device=device)
    try:
        with torch.inference_mode():
            for _ in range(3):
                model(tokens)
            torch.cuda.synchronize(device)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph), stable_weights():
                logits = model(tokens)
    except Exception as e:  # capture is an optimisation: fall back to the eager model
        if verbose:
            print(f"  [tinker] cuda graph not captured ({type(e).__name__}: {e}); running eagerly")
        return model
    if verbose:
        print(f"  [tinker] cuda graph captured for inputs {tuple(input_shape)}")
    return _CUDAGraphWrapper(model, tokens, logits, graph, clone_output)


@torch.inference_mode()
def benchmark_model(
    model: nn.Module,
    input_shape: tuple = (1, 128),
    vocab_size: int = 32000,
    warmup: int = 10,
    runs: int = 100,
    device: str | None = None,
) -> dict:
    """Latency of ``model`` on random token ids of ``input_shape``.

    Each of ``runs`` timed calls is bracketed by device synchronisations and timed on
    the host clock, after ``warmup`` untimed calls; the result has the reference's keys
    (tinker/optimize.py:190-242): ``median_ms`` (the upper median of the sorted times),
    ``mean_ms``, ``min_ms``, ``tokens_per_sec`` at the median, ``device``, and on a GPU
    ``peak_memory_mb`` (since the timed calls started) and ``gpu``."""
    dev = torch.device(device if device is not None else ("cuda" if torch.cuda.is_available() else "cpu"))
    on_gpu = dev.type == "cuda"

    def settle():
        if on_gpu:
            torch.cuda.synchronize(dev)

    tokens = torch.randint(0, vocab_size, tuple(input_shape), device=dev)
    for _ in range(warmup):
        model(tokens)
    settle()
    if on_gpu:
        torch.cuda.reset_peak_memory_stats(dev)
    times_ms = []
    for _ in range(runs):
        settle()
        start = time.perf_counter()
        model(tokens)
        settle()
        times_ms.append((time.perf_counter() - start) * 1e3)
    ordered = sorted(times_ms)
    median = ordered[len(ordered) // 2]
    n_tokens = math.prod(input_shape)
    result = {
        "median_ms": round(median, 3),
        "mean_ms": round(statistics.fmean(times_ms), 3),
        "min_ms": round(ordered[0], 3),
        "tokens_per_sec": round(n_tokens / (median / 1e3)),
        "device": str(dev.type if device is None else device),
    }
    if on_gpu:
        result["peak_memory_mb"] = round(torch.cuda.max_memory_allocated(dev) / 2 ** 20, 1)
        result["gpu"] = torch.cuda.get_device_name(dev)
    return result
