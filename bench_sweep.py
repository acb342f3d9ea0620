"""Standalone kernel sweeps and the ~1B decoder, each against the reference's eager torch path
on the same GPU.

    python bench_sweep.py [--only rmsnorm,swiglu,ffn,attention,model268m,modelqwen,model1b]
                          [--dtypes fp16,bf16]

One JSON line per case on stdout. The cases are the standalone configurations the reference
benchmarks (benchmarks/bench_rmsnorm.py, bench_swiglu.py, bench_attention.py) at the sizes of the
measurement plan: RMSNorm rows {128, 4096, 65536} x hidden {1024, 2048, 4096}; the SwiGLU activation
alone at the reference's shapes and at 4096 / 16384 tokens; the SwiGLU FFN (gate|up GEMM with the
SwiGLU epilogue, then down) for tokens {128, 4096, 16384} at 1024 -> 2816 and 2048 -> 5632; causal
RoPE + GQA attention for batch {1, 8, 32} x seq {128, 512, 2048} x head_dim {64, 128} x heads 16/4,
16/16, 16/1; the 268M decoder at batch 1 x seq 128 (the headline workload) and the
Qwen2.5-0.5B-shaped decoder at batch 64 x seq 512 against the reference's own optimize() on the same
GPU; and the ~1B Llama-style decoder at batch {1, 16} x seq {128, 2048}. The eager comparison arm
restates the reference's eager fallbacks in torch (`_rmsnorm_pytorch`
tinker/kernels/fused_rmsnorm.py:64-67, `down(silu(gate(x)) * up(x))` of
tinker/modules/feed_forward.py:26-30 with `_swiglu_pytorch` fused_swiglu.py:57-58,
`_attention_pytorch` fused_attention.py:176-192), run on cuBLAS / SDPA. The Triton arm runs the
reference's own GPU path on the same inputs: its public kernel entries with Triton present
(`fused_rmsnorm` fused_rmsnorm.py:70-74 -> the kernel of :12-52; `fused_swiglu`
fused_swiglu.py:61-66 -> :13-44, between two cuBLAS projections as feed_forward.py:26-30 calls it;
`fused_attention` fused_attention.py:234-238 -> `_attention_triton` :195-231, the Triton RoPE and
attention kernels of :19-154), imported from the reference package installed under `baseline/_ref`;
without that package (or without Triton) the column is left out and the first line says why
(`--no-triton` skips it).

Timing: each call is captured 20+ times in a CUDA graph, rotating over enough copies of its
inputs that one replay touches more than twice the 126 MB L2 (so HBM figures are not L2 hits),
and the graph is replayed after warm-up; CUDA events around the replays give time per call.
Roofline denominators come from MEASURED_PEAKS.json (HBM copy GB/s, bf16 dense TF/s, burst).
"""

from __future__ import annotations

import argparse
import importlib
import json
import math
import os
import sys

import torch
import torch.nn.functional as F

ROOT = os.path.dirname(os.path.abspath(__file__))
L2_BYTES = 126 * 1024 * 1024
DTYPES = {"fp16": torch.float16, "bf16": torch.bfloat16}


def _peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "tflops": float(d["bf16_tflops"]), "note": "of measured"}
    return {"hbm_gbs": 6650.0, "tflops": 1590.0, "note": "of fallback"}


def _copies(bytes_per_call: int) -> int:
    """How many input copies one graph replay must rotate over to exceed twice the L2."""
    return max(1, min(64, math.ceil(2 * L2_BYTES / max(1, bytes_per_call))))


def _time_graph(fns, min_calls: int = 20) -> float:
    """Microseconds per call of the closures in ``fns`` (rotated), inside one CUDA graph."""
    calls = max(min_calls, len(fns))
    for fn in fns[:2]:
        fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(calls):
            fns[i % len(fns)]()
    for _ in range(2):
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 5
    e0.record()
    for _ in range(reps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    del g
    return e0.elapsed_time(e1) * 1e3 / (reps * calls)


# ---------------------------------------------------------------- reference eager arms (torch)

def _ref_rmsnorm(x, w, eps):
    xf = x.float()
    return (xf * xf.pow(2).mean(-1, keepdim=True).add(eps).rsqrt() * w.float()).to(x.dtype)


def _ref_ffn(x, wg, wu, wd):
    return F.linear(F.silu(F.linear(x, wg)).mul_(F.linear(x, wu)), wd)


def _ref_rope(x, cos, sin):  # x [B, H, S, D]
    S = x.shape[2]
    c, s = cos[:S][None, None], sin[:S][None, None]
    xe, xo = x[..., 0::2].float(), x[..., 1::2].float()
    return torch.stack([xe * c - xo * s, xe * s + xo * c], dim=-1).flatten(-2).to(x.dtype)


def _ref_attention(q, k, v, cos, sin, hq, hkv, d):
    B, S, _ = q.shape
    q = _ref_rope(q.view(B, S, hq, d).transpose(1, 2), cos, sin)
    k = _ref_rope(k.view(B, S, hkv, d).transpose(1, 2), cos, sin)
    v = v.view(B, S, hkv, d).transpose(1, 2)
    if hq != hkv:
        k = k.unsqueeze(2).expand(-1, -1, hq // hkv, -1, -1).reshape(B, hq, S, d)
        v = v.unsqueeze(2).expand(-1, -1, hq // hkv, -1, -1).reshape(B, hq, S, d)
    out = F.scaled_dot_product_attention(q, k, v, is_causal=True)
    return out.transpose(1, 2).contiguous().view(B, S, hq * d)


# ---------------------------------------------------------------- reference Triton arm

class _RefTriton:
    """The reference's kernel modules (tinker.kernels.fused_rmsnorm / fused_swiglu / fused_attention)
    and its ``tinker.optimize`` from its installed package, or ``None`` attributes and ``why``.

    This repository's own ``tinker`` package (the import-name alias of tinker_b200) may already be in
    ``sys.modules``; it is set aside while the reference is imported and put back afterwards, so the
    reference modules held here and the alias seen by everything else stay distinct."""

    def __init__(self, enabled: bool):
        self.rms = self.swiglu = self.attn = self.opt = None
        self.why = "skipped (--no-triton)"
        if not enabled:
            return
        path = os.path.join(ROOT, "baseline", "_ref")
        if not os.path.isdir(os.path.join(path, "tinker", "kernels")):
            self.why = "the reference package is not installed under baseline/_ref"
            return
        aside = {k: sys.modules.pop(k) for k in list(sys.modules) if k == "tinker" or k.startswith("tinker.")}
        sys.path.insert(0, path)
        try:
            mods = [importlib.import_module("tinker.kernels." + n)
                    for n in ("fused_rmsnorm", "fused_swiglu", "fused_attention")]
            opt = importlib.import_module("tinker.optimize")
        except Exception as e:  # the comparison arm is optional; ours is not
            self.why = f"importing the reference kernels failed: {type(e).__name__}: {e}"
            return
        finally:
            sys.path.remove(path)
            for k in [k for k in sys.modules if k == "tinker" or k.startswith("tinker.")]:
                del sys.modules[k]
            sys.modules.update(aside)
        if not all(os.path.abspath(m.__file__).startswith(os.path.abspath(path)) for m in mods + [opt]):
            self.why = "the imported tinker modules are not the installed reference's"
            return
        if not all(getattr(m, "HAS_TRITON", False) for m in mods):
            self.why = "Triton is not importable, so the reference takes its torch fallbacks"
            return
        self.rms, self.swiglu, self.attn = mods
        self.opt = opt
        self.why = None

    def time_or_none(self, fns):
        """Microseconds per call, or None when the arm is unavailable."""
        return None if self.why else _time_graph(fns)


def _with_triton(row: dict, key: str, tri_us, ours_us):
    if tri_us is not None:
        row[key] = round(tri_us, 2)
        row["speedup_vs_triton"] = round(tri_us / ours_us, 2)
    return row


# ---------------------------------------------------------------- sweeps

def sweep_rmsnorm(dtypes, peaks, emit, tri):
    from tinker_b200.kernels import fused_rmsnorm
    g = torch.Generator(device="cuda").manual_seed(0)
    for dt in dtypes:
        for rows in (128, 4096, 65536):
            for h in (1024, 2048, 4096):
                nbytes = rows * h * 4 + 2 * h
                n = _copies(nbytes)
                xs = [torch.randn(rows, h, device="cuda", generator=g).to(dt) for _ in range(n)]
                w = (1 + 0.1 * torch.randn(h, device="cuda", generator=g)).to(dt)
                ours = _time_graph([lambda x=x: fused_rmsnorm(x, w, 1e-6) for x in xs])
                ref = _time_graph([lambda x=x: _ref_rmsnorm(x, w, 1e-6) for x in xs])
                ref_tri = tri.time_or_none([lambda x=x: tri.rms.fused_rmsnorm(x, w, 1e-6) for x in xs])
                gbs = nbytes / ours * 1e-3
                emit(_with_triton({"kind": "rmsnorm", "case": f"rows {rows} x hidden {h}", "dtype": str(dt)[6:],
                      "ours_us": round(ours, 2), "ref_eager_us": round(ref, 2), "speedup": round(ref / ours, 2),
                      "bound": "hbm", "gbs": round(gbs, 1), "frac": round(gbs / peaks["hbm_gbs"], 3),
                      "peak": f"{peaks['hbm_gbs']} GB/s {peaks['note']}", "bytes": nbytes},
                     "ref_triton_us", ref_tri, ours))
                del xs


def sweep_swiglu(dtypes, peaks, emit, tri):
    """The activation alone, ``silu(gate) * up`` on [tokens, F]: the reference's own benchmark shapes
    (benchmarks/bench_swiglu.py:21-30: batch 1 and 4 x seq 128 at F 1376, 2816, 3584, 5504) plus 4096 and
    16384 tokens, where it is HBM-bound (bytes = 3 x tokens x F x 2)."""
    from tinker_b200.kernels import fused_swiglu
    g = torch.Generator(device="cuda").manual_seed(4)
    for dt in dtypes:
        for t, f in [(t, f) for f in (1376, 2816, 3584, 5504) for t in (128, 512)] + \
                    [(4096, 2816), (4096, 5504), (16384, 2816), (16384, 5504)]:
            nbytes = 3 * t * f * 2
            n = _copies(nbytes)
            gu = [(torch.randn(t, f, device="cuda", generator=g).to(dt),
                   torch.randn(t, f, device="cuda", generator=g).to(dt)) for _ in range(n)]
            ours = _time_graph([lambda p=p: fused_swiglu(*p) for p in gu])
            ref = _time_graph([lambda p=p: F.silu(p[0]) * p[1] for p in gu])
            ref_tri = tri.time_or_none([lambda p=p: tri.swiglu.fused_swiglu(*p) for p in gu])
            gbs = nbytes / ours * 1e-3
            emit(_with_triton({"kind": "swiglu", "case": f"tokens {t} x F {f}", "dtype": str(dt)[6:],
                               "ours_us": round(ours, 2), "ref_eager_us": round(ref, 2),
                               "speedup": round(ref / ours, 2), "bound": "hbm", "gbs": round(gbs, 1),
                               "frac": round(gbs / peaks["hbm_gbs"], 3),
                               "peak": f"{peaks['hbm_gbs']} GB/s {peaks['note']}", "bytes": nbytes},
                              "ref_triton_us", ref_tri, ours))
            del gu


def sweep_ffn(dtypes, peaks, emit, tri):
    from tinker_b200.kernels import swiglu_ffn
    g = torch.Generator(device="cuda").manual_seed(1)
    for dt in dtypes:
        for h, f in ((1024, 2816), (2048, 5632)):
            wg = (0.02 * torch.randn(f, h, device="cuda", generator=g)).to(dt)
            wu = (0.02 * torch.randn(f, h, device="cuda", generator=g)).to(dt)
            wd = (0.02 * torch.randn(h, f, device="cuda", generator=g)).to(dt)
            for t in (128, 4096, 16384):
                flops = 6 * t * h * f
                nbytes = 2 * (3 * h * f + 2 * t * h) + 2 * 2 * t * f
                n = _copies(2 * t * h) if t <= 4096 else 1
                xs = [torch.randn(t, h, device="cuda", generator=g).to(dt) for _ in range(n)]
                ours = _time_graph([lambda x=x: swiglu_ffn(x, wg, wu, wd) for x in xs])
                ref = _time_graph([lambda x=x: _ref_ffn(x, wg, wu, wd) for x in xs])
                ref_tri = tri.time_or_none(
                    [lambda x=x: F.linear(tri.swiglu.fused_swiglu(F.linear(x, wg), F.linear(x, wu)), wd) for x in xs])
                tf = flops / ours * 1e-6
                gbs = nbytes / ours * 1e-3
                bound = "hbm" if t <= 128 else "tensor"
                frac = gbs / peaks["hbm_gbs"] if bound == "hbm" else tf / peaks["tflops"]
                emit(_with_triton({"kind": "swiglu_ffn", "case": f"tokens {t}, {h} -> {f}", "dtype": str(dt)[6:],
                      "ours_us": round(ours, 2), "ref_eager_us": round(ref, 2), "speedup": round(ref / ours, 2),
                      "bound": bound, "tflops": round(tf, 1), "gbs": round(gbs, 1), "frac": round(frac, 3),
                      "peak": (f"{peaks['hbm_gbs']} GB/s" if bound == "hbm" else f"{peaks['tflops']} TF/s")
                      + f" {peaks['note']}", "flops": flops, "bytes": nbytes},
                     "ref_triton_us", ref_tri, ours))
                del xs


def sweep_attention(dtypes, peaks, emit, tri):
    from tinker_b200.kernels import causal_attention, fused_attention, precompute_rope_tables
    g = torch.Generator(device="cuda").manual_seed(2)
    for dt in dtypes:
        for d in (64, 128):
            cos, sin = precompute_rope_tables(d, 2048, 10000.0, device="cuda")
            for b in (1, 8, 32):
                for s in (128, 512, 2048):
                    for hq, hkv in ((16, 4), (16, 16), (16, 1)):
                        flops = 2 * 2 * b * hq * d * s * s // 2  # causal convention: half of the dense S x S
                        nbytes = 2 * b * s * d * (2 * hq + 2 * hkv)
                        n = _copies(nbytes)
                        qkv = [(torch.randn(b, s, hq * d, device="cuda", generator=g).to(dt),
                                torch.randn(b, s, hkv * d, device="cuda", generator=g).to(dt),
                                torch.randn(b, s, hkv * d, device="cuda", generator=g).to(dt)) for _ in range(n)]
                        rope = _time_graph([lambda t=t: fused_attention(*t, cos, sin, hq, hkv, d) for t in qkv])
                        plain = _time_graph([lambda t=t: causal_attention(*t, hq, hkv, d) for t in qkv])
                        ref = _time_graph([lambda t=t: _ref_attention(*t, cos, sin, hq, hkv, d) for t in qkv])
                        ref_tri = tri.time_or_none(
                            [lambda t=t: tri.attn.fused_attention(*t, cos, sin, hq, hkv, d) for t in qkv])
                        tf_rope, tf_plain = flops / rope * 1e-6, flops / plain * 1e-6
                        emit(_with_triton({"kind": "attention", "case": f"B {b} S {s} D {d} heads {hq}/{hkv}",
                              "dtype": str(dt)[6:], "ours_rope_us": round(rope, 2), "ours_prerotated_us": round(plain, 2),
                              "ref_eager_us": round(ref, 2), "speedup": round(ref / rope, 2),
                              "bound": "latency" if s <= 128 else "tensor", "tflops_rope": round(tf_rope, 1),
                              "tflops_prerotated": round(tf_plain, 1), "frac_rope": round(tf_rope / peaks["tflops"], 3),
                              "frac_prerotated": round(tf_plain / peaks["tflops"], 3),
                              "peak": f"{peaks['tflops']} TF/s {peaks['note']}", "flops": flops, "bytes": nbytes},
                             "ref_triton_us", ref_tri, rope))
                        del qkv


def _time_replays(graph, reps: int) -> float:
    for _ in range(2):
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) * 1e3 / reps


def _time_calls(fn, reps: int) -> float:
    """Microseconds per call of ``fn`` issued back to back (CUDA events around ``reps`` calls)."""
    with torch.inference_mode():
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
    return e0.elapsed_time(e1) * 1e3 / reps


def sweep_model1b(peaks, emit):
    import tinker_b200
    from bench_model import LLAMA_1B, build_model, make_tokens
    cfg = LLAMA_1B
    ref_model = build_model(cfg, seed=0).to("cuda", torch.float16).eval()
    params = sum(p.numel() for p in ref_model.parameters())
    for b, s in ((1, 128), (16, 2048)):
        reps = 20 if b * s <= 128 else 3
        tok = make_tokens(cfg, b, s, seed=1).cuda()
        with torch.inference_mode():
            ref = _time_graph([lambda: ref_model(tok)], min_calls=reps)
        torch.cuda.empty_cache()
        m = tinker_b200.optimize(build_model(cfg, seed=0).cuda(), dtype=torch.float16, cuda_graph=True,
                                 graph_input_shape=(b, s), graph_vocab_size=cfg.vocab_size, graph_clone_output=False)
        m._static_input.copy_(tok)
        ours = _time_replays(m._graph, reps)
        flops = 2 * b * s * (params - cfg.vocab_size * cfg.hidden_size)  # embedding rows are a gather
        flops += 2 * 2 * b * cfg.num_layers * cfg.num_heads * cfg.head_dim * s * s // 2
        wbytes = 2 * (params - cfg.vocab_size * cfg.hidden_size)
        bound = "hbm" if b * s <= 128 else "tensor"
        tf = flops / ours * 1e-6
        gbs = (wbytes + 2 * b * s * cfg.vocab_size) / ours * 1e-3
        emit({"kind": "model_1b", "case": f"batch {b} x seq {s}", "dtype": "float16", "params": params,
              "ours_us": round(ours, 1), "ref_eager_us": round(ref, 1), "speedup": round(ref / ours, 2),
              "tokens_per_s": round(b * s / ours * 1e6), "bound": bound, "tflops": round(tf, 1), "gbs": round(gbs, 1),
              "frac": round(gbs / peaks["hbm_gbs"] if bound == "hbm" else tf / peaks["tflops"], 3),
              "note": "reference arm: the unpatched fp16 model (cuBLAS + SDPA) captured in a CUDA graph"})
        del m
        torch.cuda.empty_cache()


def _model_arms(emit, tri, kind, cfg, b, s, dtype, reps, compiled_arm):
    """One decoder workload inside CUDA graphs, in up to four arms on this GPU: this library's
    ``optimize``; the reference's own ``optimize`` (tinker/optimize.py:27-117: ``patch_model`` onto its
    Triton modules, the dtype cast, graph capture by ``_capture_cuda_graph`` :153-171; ``compile=False``);
    optionally the same with its default ``compile`` (torch.compile first); the unpatched model captured
    in a graph. Graph replays are timed with CUDA events; every arm runs the same model and tokens."""
    import tinker_b200
    from bench_model import build_model, make_tokens
    tok = make_tokens(cfg, b, s, seed=1).cuda()
    row = {"kind": kind, "case": f"batch {b} x seq {s}", "dtype": str(dtype)[6:], "replays": reps}
    base = build_model(cfg, seed=0).to("cuda", dtype).eval()
    with torch.inference_mode():
        row["ref_eager_graph_us"] = round(_time_graph([lambda: base(tok)], min_calls=reps), 1)
    del base
    torch.cuda.empty_cache()
    m = tinker_b200.optimize(build_model(cfg, seed=0).cuda(), dtype=dtype, cuda_graph=True,
                             graph_input_shape=(b, s), graph_vocab_size=cfg.vocab_size, graph_clone_output=False)
    m._static_input.copy_(tok)
    ours = _time_replays(m._graph, reps)
    row["ours_us"] = round(ours, 1)
    row["speedup_vs_eager_graph"] = round(row["ref_eager_graph_us"] / ours, 2)
    if tri.why is None:
        ref_opt = tri.opt
        rm = ref_opt.optimize(build_model(cfg, seed=0).cuda(), dtype=dtype, compile=False, cuda_graph=True,
                              graph_input_shape=(b, s), graph_vocab_size=cfg.vocab_size)
        if hasattr(rm, "_graph"):
            rm._static_input.copy_(tok)
            ref_us = _time_replays(rm._graph, reps)
            row["ref_triton_graph_us"] = round(ref_us, 1)
            row["speedup_vs_triton"] = round(ref_us / ours, 2)
            # both graphs ran on the same tokens (first and last sequence compared): the same forward
            row["max_abs_logits_vs_ours"] = max(
                float((rm._static_output[i].float() - m._static_output[i].float()).abs().max()) for i in (0, b - 1))
        else:
            row["ref_triton_graph_us"] = None
            row["note"] = "the reference's graph capture failed, so its optimize returned the eager model"
        del rm
        torch.cuda.empty_cache()
        if compiled_arm:
            # the reference's default: compile=None means torch.compile(mode="reduce-overhead") when
            # Triton is importable (tinker/optimize.py:77-85), then its graph capture of the compiled model
            try:
                rc = ref_opt.optimize(build_model(cfg, seed=0).cuda(), dtype=dtype, cuda_graph=True,
                                      graph_input_shape=(b, s), graph_vocab_size=cfg.vocab_size)
                if hasattr(rc, "_graph"):
                    rc._static_input.copy_(tok)
                    ref_c = _time_replays(rc._graph, reps)
                    row["ref_triton_compiled_note"] = "compiled model captured by the reference's graph wrapper"
                else:
                    ref_c = _time_calls(lambda: rc(tok), reps)
                    row["ref_triton_compiled_note"] = ("the reference's graph capture of the compiled model failed, "
                                                       "so its optimize returned the compiled model: timed per call")
                row["ref_triton_compiled_us"] = round(ref_c, 1)
                row["speedup_vs_triton_compiled"] = round(ref_c / ours, 2)
                del rc
            except Exception as e:  # a comparison arm; ours was measured above
                msg = " ".join(str(e).split())
                row["ref_triton_compiled_note"] = f"failed: {type(e).__name__}: {msg[:120]} ... {msg[-400:]}"
    emit(row)
    del m
    torch.cuda.empty_cache()


def sweep_model268m(peaks, emit, tri):
    """The headline workload: the 268M decoder at batch 1 x seq 128, fp16, 200 replays per arm."""
    from bench_model import LLAMA_268M
    _model_arms(emit, tri, "model_268m", LLAMA_268M, 1, 128, torch.float16, 200, compiled_arm=True)


def sweep_model_qwen(peaks, emit, tri):
    """The batched workload: the Qwen2.5-0.5B-shaped decoder at batch 64 x seq 512, bf16, 3 replays per
    arm (the reference's compiled path is left out: it fails in inductor, as at the 268M shape)."""
    from bench_model import QWEN25_05B_SHAPED
    _model_arms(emit, tri, "model_qwen_b64s512", QWEN25_05B_SHAPED, 64, 512, torch.bfloat16, 3, compiled_arm=False)


def run_case(spec: str, reps: int = 3):
    """One configuration, eager, ``reps`` calls inside an NVTX range ``timed`` (for profilers):
    ``rmsnorm:ROWS,H`` | ``ffn:T,H,F`` | ``attention:B,S,D,HQ,HKV`` (pre-rotated kernel) |
    ``rope_attention:B,S,D,HQ,HKV`` (the drop-in entry), all bf16."""
    from tinker_b200.kernels import causal_attention, fused_attention, fused_rmsnorm, precompute_rope_tables, swiglu_ffn
    kind, _, args = spec.partition(":")
    v = [int(a) for a in args.split(",")]
    dt = torch.bfloat16
    g = torch.Generator(device="cuda").manual_seed(3)
    if kind == "rmsnorm":
        x = torch.randn(v[0], v[1], device="cuda", generator=g).to(dt)
        w = (1 + 0.1 * torch.randn(v[1], device="cuda", generator=g)).to(dt)
        fn = lambda: fused_rmsnorm(x, w, 1e-6)
    elif kind == "ffn":
        t, h, f = v
        x = torch.randn(t, h, device="cuda", generator=g).to(dt)
        ws = [(0.02 * torch.randn(*sh, device="cuda", generator=g)).to(dt) for sh in ((f, h), (f, h), (h, f))]
        fn = lambda: swiglu_ffn(x, *ws)
    elif kind in ("attention", "rope_attention"):
        b, s, d, hq, hkv = v
        q = torch.randn(b, s, hq * d, device="cuda", generator=g).to(dt)
        k = torch.randn(b, s, hkv * d, device="cuda", generator=g).to(dt)
        vv = torch.randn(b, s, hkv * d, device="cuda", generator=g).to(dt)
        cos, sin = precompute_rope_tables(d, s, device="cuda")
        if kind == "attention":
            fn = lambda: causal_attention(q, k, vv, hq, hkv, d)
        else:
            fn = lambda: fused_attention(q, k, vv, cos, sin, hq, hkv, d)
    else:
        raise ValueError(f"unknown case {spec}")
    fn()
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_push("timed")
    for _ in range(reps):
        fn()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default="rmsnorm,swiglu,ffn,attention,model268m,modelqwen,model1b")
    ap.add_argument("--dtypes", default="fp16,bf16")
    ap.add_argument("--case", default=None, help="run one configuration for a profiler (see run_case)")
    ap.add_argument("--no-triton", action="store_true", help="leave out the reference's Triton arm")
    args = ap.parse_args(argv)
    torch.cuda.set_device(0)
    if args.case:
        with torch.inference_mode():
            run_case(args.case)
        return
    peaks = _peaks()
    dtypes = [DTYPES[d] for d in args.dtypes.split(",")]

    def emit(d):
        print(json.dumps(d), flush=True)

    kinds = args.only.split(",")
    arms = ("rmsnorm", "swiglu", "ffn", "attention", "model268m", "modelqwen")
    tri = _RefTriton(not args.no_triton and any(k in kinds for k in arms))
    if tri.why and not args.no_triton:
        emit({"kind": "note", "ref_triton": f"unavailable: {tri.why}"})
    with torch.inference_mode():
        if "rmsnorm" in kinds:
            sweep_rmsnorm(dtypes, peaks, emit, tri)
        if "swiglu" in kinds:
            sweep_swiglu(dtypes, peaks, emit, tri)
        if "ffn" in kinds:
            sweep_ffn(dtypes, peaks, emit, tri)
        if "attention" in kinds:
            sweep_attention(dtypes, peaks, emit, tri)
    if "model268m" in kinds:
        sweep_model268m(peaks, emit, tri)
    if "modelqwen" in kinds:
        sweep_model_qwen(peaks, emit, tri)
    if "model1b" in kinds:
        sweep_model1b(peaks, emit)


if __name__ == "__main__":
    main()
