#!/usr/bin/env python
"""Benchmark of the B200 fused-kernel path behind tinker_b200.optimize().

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline (``value``): forward latency of the 268M Llama-style decoder
(vocab 32000, hidden 1024, 18 layers, 16/4 heads, head_dim 64, FFN 2816,
fp16, seeded N(0, 0.02) weights) at batch 1 x seq 128, captured in a CUDA
graph by ``optimize(cuda_graph=True)``; inputs resident in HBM, time per graph
replay from CUDA events. With N GPUs (torchrun, one process per GPU) every rank
runs an independent replica - the path has no collective - and ``value`` is the
max over ranks. ``e2e`` times the same forward through the public call with
the token ids copied from pinned host memory and the logits copied back.

Also reported: ``batched`` - Qwen2.5-0.5B-shaped bf16 prefill of batch 64 x
seq 512, the 64 sequences split into contiguous blocks of 64/N per rank
(aggregate tokens/s); ``decode`` - cached greedy decoding of the 268M decoder
(KV cache, one CUDA graph per token) at batch 1 and 64 after a 128-token
prompt, and the KV-cache attention kernel alone at batch 64 x 2048 cached
positions; ``roofline`` for the kernel with the largest share of the
forward; ``cpu_baseline`` - the numpy oracle's fp32 forward on the host cores.

``--impl reference`` times the reference's CPU path (the numpy restatement of
its fp32 eager forward, oracle/) on this host instead, rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "fwd ms @268M b1 s128 (CUDA graph)"
PUBLISHED_MS = 2.11  # reference README.md:13, RTX 5080, "TinKer fp16 + CUDA graph"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def _args():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batched-steps", type=int, default=10)
    ap.add_argument("--no-batched", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--only", choices=["forward", "stack", "lm_head", "gate_up_swiglu", "down_proj", "qkv_rope_proj",
                                       "o_proj", "causal_attention", "rmsnorm", "row_sumsq", "qwen_forward",
                                       "decode", "kv_attention"],
                    help="profiling helper: time only the graph replay or one kernel kind (268M shapes), "
                         "the Qwen-shaped batched forward (--qwen-batch sequences of 512), cached decoding "
                         "(decode) or the KV-cache attention kernel alone (kv_attention)")
    ap.add_argument("--no-decode", action="store_true")
    ap.add_argument("--qwen-batch", type=int, default=64)
    ap.add_argument("--sweep", default=None, metavar="KINDS",
                    help="run the standalone sweeps instead (comma list of rmsnorm, ffn, attention, model1b; "
                         "bench_sweep.py), one JSON line per case")
    return ap.parse_args()


def _peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "of measured"
    return dict(FALLBACK_PEAKS), "of fallback"


# ------------------------------------------------------------------------------------
# CPU side: the reference's own fp32 eager forward (its blocks, carried in oracle/torch_model.py)
# timed on the host cores; its logits are also the parity reference for the timed graph
# ------------------------------------------------------------------------------------
def _blas_threads() -> int:
    try:
        from threadpoolctl import threadpool_info
        n = [d.get("num_threads", 0) for d in threadpool_info() if d.get("user_api") == "blas"]
        if n:
            return max(n)
    except Exception:
        pass
    return os.cpu_count() or 1


def _use_all_host_threads() -> int:
    """torchrun exports OMP_NUM_THREADS=1; the CPU baseline uses every core of the host."""
    import torch
    n = os.cpu_count() or 1
    torch.set_num_threads(n)
    try:
        from threadpoolctl import threadpool_limits
        threadpool_limits(limits=n, user_api="blas")
    except Exception:
        pass
    return torch.get_num_threads()


def _reference_cpu_model(cfg, seed=0):
    """The reference's unpatched fp32 eager model (oracle/torch_model.py) with the seeded weights."""
    from oracle.torch_model import build_model as build_reference
    return build_reference(cfg, seed=seed)


def _reference_forward(model, tokens, layers=None):
    """The reference model's forward, optionally over its first ``layers`` blocks only (a bounded
    CPU sample; embedding, final norm and head always run)."""
    x = model.embedding(tokens)
    for blk in model.layers[:layers]:
        x = blk(x)
    return model.output(model.norm(x))


def cpu_reference_timer(cfg, tokens, budget_s: float = 20.0, min_runs: int = 10, warmup: int = 3):
    """Median ms of the reference's fp32 eager forward on all host threads (warm-up, then
    min_runs..as many as fit in budget_s), its logits, and the thread count."""
    import torch
    threads = _use_all_host_threads()
    model = _reference_cpu_model(cfg)
    with torch.inference_mode():
        for _ in range(warmup):
            logits = _reference_forward(model, tokens)
        times = []
        t_end = time.perf_counter() + budget_s
        while len(times) < min_runs or (time.perf_counter() < t_end and len(times) < 100):
            t = time.perf_counter()
            _reference_forward(model, tokens)
            times.append((time.perf_counter() - t) * 1e3)
    return statistics.median(times), len(times), logits.float().numpy(), threads


def numpy_port_timer(cfg, tokens, runs: int = 5):
    """Secondary CPU figure: median ms of the numpy restatement (oracle/) of the same forward."""
    import oracle
    _use_all_host_threads()
    from bench_model import build_model
    w = {k: v.detach().float().numpy() for k, v in build_model(cfg, seed=0).state_dict().items()}
    ocfg = oracle.ModelConfig(**{f: getattr(cfg, f) for f in oracle.ModelConfig.__dataclass_fields__})
    tok = tokens.numpy()
    oracle.forward_logits(w, tok, ocfg)
    times = []
    for _ in range(runs):
        t = time.perf_counter()
        oracle.forward_logits(w, tok, ocfg)
        times.append((time.perf_counter() - t) * 1e3)
    return statistics.median(times)


def logits_parity(ours, ref) -> dict:
    """Max-abs error of half-precision logits against the fp32 reference, raw top-1 agreement,
    and top-1 agreement over the positions whose fp32 top-1/top-2 gap exceeds twice the max-abs
    error (random weights give near-ties that no half-precision forward resolves)."""
    import numpy as np
    ours = np.asarray(ours, dtype=np.float64).reshape(-1, ref.shape[-1])
    ref = np.asarray(ref, dtype=np.float64).reshape(-1, ref.shape[-1])
    err = np.abs(ours - ref)
    top2 = np.sort(ref, axis=-1)[:, -2:]
    gap = top2[:, 1] - top2[:, 0]
    agree = ours.argmax(-1) == ref.argmax(-1)
    clear = gap > 2 * err.max()
    return {"max_abs": float(f"{err.max():.4g}"), "mean_abs": float(f"{err.mean():.4g}"),
            "top1": round(float(agree.mean()), 5),
            "top1_clear_margin": round(float(agree[clear].mean()), 5) if clear.any() else 1.0,
            "positions": int(ref.shape[0]), "clear_positions": int(clear.sum())}


def run_reference(args):
    """``--impl reference``: the reference's CPU path - its unpatched fp32 eager forward - timed on
    this host's cores, rank 0 only; each step one forward of the 268M decoder at batch 1 x seq 128
    (fewer blocks, scaled, if a full forward would not fit the step budget)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return  # the CPU reference runs once, on rank 0
    import torch
    from bench_model import LLAMA_268M, make_tokens
    cfg = LLAMA_268M
    tokens = make_tokens(cfg, 1, 128, seed=1)
    threads = _use_all_host_threads()
    model = _reference_cpu_model(cfg)
    with torch.inference_mode():
        t = time.perf_counter()
        _reference_forward(model, tokens)
        full_s = time.perf_counter() - t
        budget = 180.0 / max(1, args.steps + args.warmup)  # the whole run within ~3 minutes
        layers = cfg.num_layers
        if full_s > budget:
            layers = max(1, int(cfg.num_layers * budget / full_s))
        for _ in range(args.warmup):
            _reference_forward(model, tokens, layers)
        times = []
        for _ in range(args.steps):
            t = time.perf_counter()
            _reference_forward(model, tokens, layers)
            times.append((time.perf_counter() - t) * 1e3 * cfg.num_layers / layers)
    ms = statistics.median(times)
    what = ("the reference's unpatched fp32 eager forward (benchmarks/bench_e2e.py blocks + embedding/head, "
            "torch CPU ops), 268M decoder, batch 1 x seq 128")
    sample = what if layers == cfg.num_layers else \
        f"{layers} of 18 blocks + embedding/head per step, scaled x{cfg.num_layers / layers:.2f}: {what}"
    line = {
        "impl": "reference", "metric": METRIC, "value": round(ms, 3), "unit": "ms", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": False,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic: seeded N(0,0.02) weights, uniform token ids",
        "config": {"workload": "llama268m-b1s128", "global_batch": 1, "seq_len": 128, "parallelism": "cpu"},
        "cpu_baseline": {"value": round(ms, 3), "unit": "ms", "cores": threads, "kind": "reference",
                         "sample": sample},
        "e2e": {"value": round(ms, 3), "unit": "ms", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------
# GPU side
# ------------------------------------------------------------------------------------
class ClockSampler:
    """nvidia-smi clock / throttle-reason samples of one GPU while the GPU is busy."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.proc = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", gpu_id, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        mhz, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 8:
                continue
            try:
                mhz.append(float(f[0]))
                mx = float(f[1])
            except ValueError:
                continue
            for n, v in zip(names, f[4:8]):
                if v.lower() == "active":
                    reasons.add(n)
        if not mhz:
            return None
        return {"sm_mhz": statistics.median(mhz), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(mhz)}


def _gpu_id(dev) -> str:
    import torch
    try:
        return "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        return str(dev.index)


def _dist_init(args):
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=dev)
    return rank, world, dev


def _barrier(world):
    import torch
    import torch.distributed as dist
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()


def _max_over_ranks(x: float, world: int, dev) -> float:
    import torch
    import torch.distributed as dist
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _time_replays(graph, steps: int):
    import torch
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    evs[0].record()
    for i in range(steps):
        graph.replay()
        evs[i + 1].record()
    torch.cuda.synchronize()
    per = [evs[i].elapsed_time(evs[i + 1]) for i in range(steps)]
    return evs[0].elapsed_time(evs[-1]) / steps, statistics.median(per)


def _kernel_cases(model, cfg, dev, tokens_per_fwd: int):
    """For each kernel kind of the forward: (one closure per layer launching it on that
    layer's weights, algorithmic bytes per launch, flops per launch, launches per forward).
    The kinds are those of the fused, norm-folded decoder block: q|k|v with RoPE and the
    attention RMSNorm in its epilogue, attention, o_proj + residual writing the row
    statistics, gate|up + SwiGLU with the FFN RMSNorm in its epilogue, down + residual
    writing the row statistics; plus the final RMSNorm and the first block's row statistics."""
    import torch
    from tinker_b200.kernels import causal_attention, fused_rmsnorm, gate_up_swiglu, linear, linear_rope, row_sumsq
    base = model._model if hasattr(model, "_model") else model
    layers = list(base.layers)
    M, H = tokens_per_fwd, cfg.hidden_size
    F, D, hq, hkv = cfg.intermediate_size, cfg.head_dim, cfg.num_heads, cfg.num_kv_heads
    dt = next(base.parameters()).dtype
    es = 2
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn(M, H, device=dev, generator=g).to(dt)
    hbuf = torch.randn(M, F, device=dev, generator=g).to(dt)
    a = torch.randn(M, hq * D, device=dev, generator=g).to(dt)
    qkv = torch.randn(1, M, (hq + 2 * hkv) * D, device=dev, generator=g).to(dt)
    x3 = x.view(1, M, H)
    ssq_in = row_sumsq(x)
    ssq_out = torch.empty(H // 32, M, dtype=torch.float32, device=dev)
    ssq_b = 4 * M * (H // 32)
    S = M
    L = len(layers)
    return {
        "gate_up_swiglu": ([lambda l=l: gate_up_swiglu(x, l.ffn.gate_proj.weight, l.ffn.up_proj.weight,
                                                       row_ssq_in=ssq_in, row_ssq_eps=cfg.eps) for l in layers],
                           2 * F * H * es + M * H * es + M * F * es + ssq_b, 2 * M * H * 2 * F, L),
        "down_proj": ([lambda l=l: linear(hbuf, l.ffn.down_proj.weight, residual=x, row_ssq_out=ssq_out)
                       for l in layers], H * F * es + M * F * es + 2 * M * H * es + ssq_b, 2 * M * F * H, L),
        "qkv_rope_proj": ([lambda l=l: linear_rope(x3, l.attn.q_proj.weight, l.attn.k_proj.weight,
                                                   l.attn.v_proj.weight, l.attn.cos_table, l.attn.sin_table, D,
                                                   row_ssq_in=ssq_in, row_ssq_eps=cfg.eps)
                           for l in layers],
                          (hq + 2 * hkv) * D * H * es + M * H * es + M * (hq + 2 * hkv) * D * es + 2 * S * (D // 2) * 4
                          + ssq_b, 2 * M * H * (hq + 2 * hkv) * D, L),
        "o_proj": ([lambda l=l: linear(a, l.attn.o_proj.weight, residual=x, row_ssq_out=ssq_out) for l in layers],
                   H * hq * D * es + M * hq * D * es + 2 * M * H * es + ssq_b, 2 * M * hq * D * H, L),
        "causal_attention": ([lambda: causal_attention(qkv[..., :hq * D], qkv[..., hq * D:(hq + hkv) * D],
                                                       qkv[..., (hq + hkv) * D:], hq, hkv, D) for _ in layers],
                             2 * S * D * (2 * hq + 2 * hkv), 2 * 2 * hq * D * S * S // 2, L),
        "rmsnorm": ([lambda: fused_rmsnorm(x, base.norm.weight, cfg.eps)], M * H * 2 * es + H * es, 4 * M * H, 1),
        "row_sumsq": ([lambda: row_sumsq(x)], M * H * es + ssq_b, 2 * M * H, 1),
    }


def _stack_launch(model, tokens):
    """(closure launching the one-kernel decoder stack on the model's plan for these tokens,
    closure launching the LM head GEMM on its output, algorithmic HBM bytes per stack launch)."""
    import torch
    base = model._model if hasattr(model, "_model") else model
    plan = base._tinker_stack_plans[tuple(tokens.shape)]
    emb, layers, norm, head = base._tinker_stack_parts
    y = plan.hidden_states(tokens)
    weights = 0
    for blk in layers:
        n1, at, n2, ff = (getattr(blk, n) for n in blk._tinker_block_parts)
        for w in (at.q_proj.weight, at.k_proj.weight, at.v_proj.weight, at.o_proj.weight, ff.gate_proj.weight,
                  ff.up_proj.weight, ff.down_proj.weight):
            weights += w.numel() * w.element_size()
    m, hidden = tokens.numel(), emb.weight.shape[1]
    # every layer's (folded) weights once, the embedding rows in, the final norm's rows out, its weight
    nbytes = weights + 2 * m * hidden * 2 + hidden * 2
    return (lambda: plan.hidden_states(tokens)), (lambda: head(y)), nbytes


def _time_launches(fn, steps: int, warmup: int = 3):
    """Mean ms of ``fn`` launched back to back ``steps`` times (CUDA events on the current stream)."""
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def _stack_roofline(model, tokens, peaks, peak_note, steps: int = 200):
    """Roofline of the forward's dominant kernel, the one-kernel decoder stack: its algorithmic
    bytes (all layer weights streamed once, embedding rows in, normalised rows out) over its
    mean launch time, CUDA events around back-to-back launches on the launching stream (each
    launch streams ~406 MB of weights, more than the 126 MB L2, so no flush is needed)."""
    stack, head, nbytes = _stack_launch(model, tokens)
    t_stack = _time_launches(stack, steps) * 1e-3
    t_head = _time_launches(head, steps) * 1e-3
    achieved = nbytes / t_stack / 1e9
    traffic = None
    tp = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tp):
        with open(tp) as f:
            traffic = json.load(f).get("llama268m-b1s128/stack")
    return {"kernel": "stack_kernel (embedding + 18 decoder blocks + final RMSNorm, one launch)", "bound": "hbm",
            "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
            "frac": round(achieved / peaks["hbm_gbs"], 3), "traffic": traffic, "bytes_per_launch": nbytes,
            "us_per_launch": round(t_stack * 1e6, 2), "lm_head_us": round(t_head * 1e6, 2),
            "note": f"peak {peak_note} (burst copy); launch time from CUDA events over {steps} launches"}


def _kernel_rooflines(model, cfg, dev, peaks, peak_note, tokens_per_fwd: int):
    """Time each kernel kind on the model's own weights inside a CUDA graph, cold: graph
    A = [L2 flush, launch] per layer, graph B = [L2 flush] per layer; the kernel's time is
    (A - B) / layers, CUDA events around the replays. The flush reads a buffer larger than
    L2. Returns (per-kind table, roofline of the kind with the largest share of the forward)."""
    import torch
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=dev)  # 256 MB > 126 MB L2
    flush.zero_()
    sink = torch.empty((), dtype=torch.float32, device=dev)

    def graph_of(fns):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for fn in fns:
                torch.sum(flush, dim=0, out=sink)
                if fn is not None:
                    fn()
        return g

    def time_graph(g, reps=5):
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps * 1e-3  # seconds

    kinds = {}
    cases = _kernel_cases(model, cfg, dev, tokens_per_fwd)
    for name, (fns, nbytes, flops, per_fwd) in cases.items():
        for fn in fns[:2]:
            fn()  # first-launch set-up (kernel attributes, tensor maps) outside the capture
        torch.cuda.synchronize()
        ga, gb = graph_of(fns), graph_of([None] * len(fns))
        t = max(1e-9, (time_graph(ga) - time_graph(gb)) / len(fns))
        del ga, gb
        kinds[name] = dict(t=t, bytes=nbytes, flops=flops, per_fwd=per_fwd)
    table = {}
    for k, v in kinds.items():
        table[k] = {"us": round(v["t"] * 1e6, 2), "launches_per_fwd": v["per_fwd"],
                    "share_us": round(v["t"] * 1e6 * v["per_fwd"], 1),
                    "hbm_gbs": round(v["bytes"] / v["t"] / 1e9, 1),
                    "frac_hbm": round(v["bytes"] / v["t"] / 1e9 / peaks["hbm_gbs"], 3)}
    top = max(kinds, key=lambda k: kinds[k]["t"] * kinds[k]["per_fwd"])
    v = kinds[top]
    achieved = v["bytes"] / v["t"] / 1e9
    traffic = None
    tp = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tp):
        with open(tp) as f:
            traffic = json.load(f).get(f"llama268m-b1s128/{top}")
    roof = {"kernel": top, "bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"],
            "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 3), "traffic": traffic,
            "bytes_per_launch": v["bytes"],
            "note": f"peak {peak_note} (burst copy); per launch in a CUDA graph after an L2 flush (cold)"}
    return table, roof


DECODE_PROMPT, DECODE_NEW = 128, 128


def _decode_bench(dev, peaks, peak_note, batch: int, prompt: int = DECODE_PROMPT, new: int = DECODE_NEW):
    """Cached greedy decoding of the 268M decoder: a ``prompt``-token prefill, then ``new`` steps,
    each one CUDA graph replay fed the previous step's argmax. ``value``: device-resident steps
    (the argmax stays on the GPU); ``e2e``: every step copies its token ids from pinned host memory
    and the chosen ids back."""
    import torch
    import tinker_b200
    from tinker_b200 import _lib
    from bench_model import LLAMA_268M, build_model, make_tokens
    cfg = LLAMA_268M
    model = tinker_b200.optimize(build_model(cfg, seed=0).to(dev), dtype=torch.float16, cuda_graph=False)
    dec = tinker_b200.CachedDecoder(model, batch_size=batch, capacity=prompt + new + 1)
    ids = make_tokens(cfg, batch, prompt, seed=1).to(dev)
    with torch.inference_mode():
        probe = tinker_b200.CachedDecoder(model, batch_size=batch, capacity=4, cuda_graph=False)
        probe.prefill(ids[:, :1])
        n0 = _lib.launch_counter[0]
        probe.decode(ids[:, 1])
        launches = _lib.launch_counter[0] - n0
        del probe
        for _ in range(2):  # warm-up, captures the step graph
            dec.reset()
            lg = dec.prefill(ids)
            for _ in range(8):
                lg = dec.decode(lg.argmax(-1))
        dec.reset()
        lg = dec.prefill(ids)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.nvtx.range_push("timed")  # profilers select the decode steps with an NVTX filter
        e0.record()
        for _ in range(new):
            lg = dec.decode(lg.argmax(-1))
        e1.record()
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / new
        dec.reset()
        lg = dec.prefill(ids)
        tok_host = lg.argmax(-1).cpu().pin_memory()
        ids_host = torch.empty_like(tok_host).pin_memory()
        torch.cuda.synchronize()
        per = []
        for _ in range(new):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            lg = dec.decode(tok_host.to(dev, non_blocking=True))
            ids_host.copy_(lg.argmax(-1), non_blocking=True)
            b.record()
            b.synchronize()
            per.append(a.elapsed_time(b))
            tok_host.copy_(ids_host)
    e2e_ms = statistics.mean(per)
    kv_len = prompt + new // 2  # mean cache length over the timed steps
    weights = sum(p.numel() * p.element_size() for p in model.parameters()) \
        - model.embedding.weight.numel() * model.embedding.weight.element_size()
    kv_bytes = cfg.num_layers * 2 * batch * cfg.num_kv_heads * kv_len * cfg.head_dim * 2
    step_bytes = weights + kv_bytes
    gbs = step_bytes / (ms * 1e-3) / 1e9
    out = {"metric": f"decode tokens/s @268M b{batch} (KV cache, {prompt}-token prompt, {new} new tokens, "
                     "CUDA graph per step)",
           "value": round(batch / (ms * 1e-3)), "unit": "tokens/s", "ms_per_step": round(ms, 4), "batch": batch,
           "e2e": {"value": round(batch / (e2e_ms * 1e-3)), "unit": "tokens/s", "ms_per_step": round(e2e_ms, 4),
                   "h2d_bytes_per_step": batch * 8, "d2h_bytes_per_step": batch * 8},
           "roofline": {"bound": "hbm", "bytes_per_step": step_bytes, "achieved": round(gbs, 1),
                        "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": round(gbs / peaks["hbm_gbs"], 3),
                        "note": f"weights (without the embedding) + K/V cache at the mean length {kv_len}, "
                                f"{peak_note}"},
           "gpu_launches_per_step": launches}
    del dec, model
    torch.cuda.empty_cache()
    return out


def _kv_attention_bench(dev, peaks, peak_note, steps: int = 50, batch: int = 64, kv_len: int = 2048):
    """The KV-cache attention kernel alone on a bandwidth-sized decode step: ``batch`` sequences of
    the 268M heads (16 q / 4 kv, head_dim 64) with ``kv_len - 1`` cached positions and one new
    token; caches rotated so that the inputs exceed L2 between launches."""
    import torch
    from tinker_b200.kernels.kv_cache import kv_attention, kv_attention_workspace
    from tinker_b200.kernels.fused_attention import precompute_rope_tables
    hq, hkv, d = 16, 4, 64
    g = torch.Generator(device=dev).manual_seed(3)
    n_sets = 3  # 3 x 134 MB of cache > L2
    caches = [(torch.randn(batch, hkv, kv_len, d, device=dev, generator=g).half(),
               torch.randn(batch, hkv, kv_len, d, device=dev, generator=g).half()) for _ in range(n_sets)]
    qkv = torch.randn(batch, 1, (hq + 2 * hkv) * d, device=dev, generator=g).half()
    q, k, v = qkv[..., :hq * d], qkv[..., hq * d:(hq + hkv) * d], qkv[..., (hq + hkv) * d:]
    cos, sin = precompute_rope_tables(d, kv_len, device=dev)
    ws = torch.zeros(kv_attention_workspace(batch, hq, hkv, d, 1, kv_len), dtype=torch.uint8, device=dev)
    start = kv_len - 1

    def call(i):
        kc, vc = caches[i % n_sets]
        kv_attention(q, k, v, cos, sin, kc, vc, hq, hkv, d, start_pos=start, workspace=ws)

    for i in range(5):
        call(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("timed")
    e0.record()
    for i in range(steps):
        call(i)
    e1.record()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) / steps * 1e3
    nbytes = 2 * batch * hkv * kv_len * d * 2 + qkv.numel() * 2 + batch * hq * d * 2
    gbs = nbytes / (us * 1e-6) / 1e9
    del caches
    torch.cuda.empty_cache()
    return {"kernel": "kv_attention", "case": f"b{batch} kv_len {kv_len} 16q/4kv d64 fp16, 1 new token",
            "us": round(us, 2), "bytes": nbytes, "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"],
            "unit": "GB/s", "frac": round(gbs / peaks["hbm_gbs"], 3), "note": peak_note}


def run_only(args):
    """Profiling helper: run just one forward replay loop, or one kernel kind, on the 268M
    shapes (``--only forward`` / ``--only gate_up_swiglu`` ...) and print its mean time."""
    import torch
    import tinker_b200
    from bench_model import LLAMA_268M, build_model, make_tokens
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    if args.only in ("decode", "kv_attention"):
        peaks, peak_note = _peaks()
        if args.only == "decode":
            for b in (1, 64):
                print(json.dumps({"only": "decode", **_decode_bench(dev, peaks, peak_note, b)}), flush=True)
        else:
            print(json.dumps({"only": "kv_attention", **_kv_attention_bench(dev, peaks, peak_note, args.steps)}),
                  flush=True)
        return
    if args.only == "qwen_forward":
        from bench_model import QWEN25_05B_SHAPED
        qcfg = QWEN25_05B_SHAPED
        qtok = make_tokens(qcfg, args.qwen_batch, 512, seed=7)
        qm = tinker_b200.optimize(build_model(qcfg, seed=0).to(dev), dtype=torch.bfloat16, cuda_graph=True,
                                  graph_input_shape=tuple(qtok.shape), graph_vocab_size=qcfg.vocab_size,
                                  graph_clone_output=False)
        qm._static_input.copy_(qtok.to(dev))
        for _ in range(args.warmup):
            qm._graph.replay()
        ms, _ = _time_replays(qm._graph, args.steps)
        print(json.dumps({"only": args.only, "batch": args.qwen_batch, "steps": args.steps, "ms_mean": round(ms, 4),
                          "tokens_per_s": round(args.qwen_batch * 512 / (ms * 1e-3))}), flush=True)
        return
    cfg = LLAMA_268M
    tokens = make_tokens(cfg, 1, 128, seed=1)
    if args.only in ("stack", "lm_head"):
        model = tinker_b200.optimize(build_model(cfg, seed=0).to(dev), dtype=torch.float16, stack_kernel=True)
        tok = tokens.to(dev)
        with torch.inference_mode():
            model(tok)  # makes the plan for this shape
            stack, head, _ = _stack_launch(model, tok)
            fn = stack if args.only == "stack" else head
            for _ in range(args.warmup):
                fn()
            torch.cuda.synchronize()
            torch.cuda.nvtx.range_push("timed")
            ms = _time_launches(fn, args.steps, warmup=0)
            torch.cuda.nvtx.range_pop()
        print(json.dumps({"only": args.only, "steps": args.steps, "ms_mean": round(ms, 5)}), flush=True)
        return
    graph = args.only == "forward"
    model = tinker_b200.optimize(build_model(cfg, seed=0).to(dev), dtype=torch.float16, cuda_graph=graph,
                                 graph_input_shape=(1, 128), graph_vocab_size=cfg.vocab_size)
    if graph:
        model._static_input.copy_(tokens.to(dev))
        for _ in range(args.warmup):
            model._graph.replay()
        torch.cuda.nvtx.range_push("timed")
        ms, _ = _time_replays(model._graph, args.steps)
        torch.cuda.nvtx.range_pop()
    else:
        fns = _kernel_cases(model, cfg, dev, 128)[args.only][0]
        for i in range(args.warmup):
            fns[i % len(fns)]()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.nvtx.range_push("timed")  # profilers select these launches with an NVTX filter
        e0.record()
        for i in range(args.steps):
            fns[i % len(fns)]()
        e1.record()
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / args.steps
    print(json.dumps({"only": args.only, "steps": args.steps, "ms_mean": round(ms, 5)}), flush=True)


def run_ours(args):
    import torch
    import tinker_b200
    from tinker_b200 import _lib
    from bench_model import LLAMA_268M, QWEN25_05B_SHAPED, build_model, make_tokens

    rank, world, dev = _dist_init(args)
    peaks, peak_note = _peaks()
    cfg = LLAMA_268M
    tokens = make_tokens(cfg, 1, 128, seed=1)

    # ---- build + capture ---------------------------------------------------------------
    cpu_model = build_model(cfg, seed=0)
    model = tinker_b200.optimize(cpu_model.to(dev), dtype=torch.float16, cuda_graph=True,
                                 graph_input_shape=(1, 128), graph_vocab_size=cfg.vocab_size)
    if type(model).__name__ != "_CUDAGraphWrapper":
        raise RuntimeError("CUDA graph capture failed")
    with torch.inference_mode():  # count this library's kernels in one forward (the graph holds the same)
        n0 = _lib.launch_counter[0]
        model._model(tokens.to(dev))
        launches_per_fwd = _lib.launch_counter[0] - n0
    model._static_input.copy_(tokens.to(dev))
    graph = model._graph
    sampler = ClockSampler(_gpu_id(dev))

    # ---- device-resident timing ---------------------------------------------------------------
    # warm-up; then at least ~1.5 s of replays so that the clock samples see the GPU under load
    for _ in range(max(3, args.warmup)):
        graph.replay()
    torch.cuda.synchronize()
    t_end = time.perf_counter() + 1.5
    while time.perf_counter() < t_end:
        for _ in range(200):
            graph.replay()
        torch.cuda.synchronize()
    _barrier(world)
    ms_mean, ms_median = _time_replays(graph, args.steps)
    _barrier(world)
    ms = _max_over_ranks(ms_mean, world, dev)
    graph_logits = model._static_output.float().cpu().numpy()  # the timed replays' own output

    # ---- end to end through the public call -----------------------------------------------------
    tok_host = tokens.pin_memory()
    out_host = torch.empty((1, 128, cfg.vocab_size), dtype=torch.float16, pin_memory=True)
    with torch.inference_mode():
        for _ in range(max(3, args.warmup)):
            out_host.copy_(model(tok_host.to(dev, non_blocking=True)), non_blocking=True)
        _barrier(world)
        e2e = []
        for _ in range(args.steps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            logits = model(tok_host.to(dev, non_blocking=True))
            out_host.copy_(logits, non_blocking=True)
            e1.record()
            e1.synchronize()
            e2e.append(e0.elapsed_time(e1))
    _barrier(world)
    e2e_ms = _max_over_ranks(statistics.mean(e2e), world, dev)
    clocks = sampler.stop()

    # ---- per-kernel rooflines (rank 0 view; every rank runs the same work) ------------------------
    if getattr(model._model, "_tinker_stack_parts", None) is not None:  # the one-kernel stack is the forward
        with torch.inference_mode():
            roof = _stack_roofline(model, tokens.to(dev), peaks, peak_note)
        table, _ = _kernel_rooflines(model, cfg, dev, peaks, peak_note, 128)
    else:
        table, roof = _kernel_rooflines(model, cfg, dev, peaks, peak_note, 128)
    weight_bytes = sum(p.numel() * p.element_size() for p in model._model.parameters())
    emb = model._model.embedding.weight
    fwd_bytes = (weight_bytes - emb.numel() * emb.element_size() + 128 * cfg.hidden_size * 2
                 + 128 * cfg.vocab_size * 2)
    roof_fwd = {"bound": "hbm", "bytes_per_fwd": fwd_bytes, "achieved": round(fwd_bytes / (ms * 1e-3) / 1e9, 1),
                "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": round(fwd_bytes / (ms * 1e-3) / 1e9 / peaks["hbm_gbs"], 3),
                "note": f"whole forward: weights + embedding rows + logits over the replay time, {peak_note}"}
    del model, graph, cpu_model
    torch.cuda.empty_cache()

    # ---- batched Qwen-shaped prefill, sequences split across ranks ---------------------------------
    batched = None
    batched_rows = None  # (tokens, logits) of the first and last sequence of the timed graph, for parity
    if not args.no_batched:
        qcfg = QWEN25_05B_SHAPED
        per_rank = 64 // world
        qtok = make_tokens(qcfg, 64, 512, seed=7)[rank * per_rank:(rank + 1) * per_rank]
        qm = tinker_b200.optimize(build_model(qcfg, seed=0).to(dev), dtype=torch.bfloat16, cuda_graph=True,
                                  graph_input_shape=(per_rank, 512), graph_vocab_size=qcfg.vocab_size,
                                  graph_clone_output=False)
        if type(qm).__name__ != "_CUDAGraphWrapper":
            raise RuntimeError("CUDA graph capture failed (batched)")
        qm._static_input.copy_(qtok.to(dev))
        for _ in range(3):
            qm._graph.replay()
        _barrier(world)
        qms, _ = _time_replays(qm._graph, args.batched_steps)
        _barrier(world)
        qms = _max_over_ranks(qms, world, dev)
        pick = [0, per_rank - 1]
        batched_rows = (qtok[pick], qm._static_output[pick].float().cpu().numpy())
        flops = 2 * 64 * 512 * (qcfg.num_params() - qcfg.vocab_size * qcfg.hidden_size) \
            + 2 * 64 * 512 * qcfg.vocab_size * qcfg.hidden_size \
            + qcfg.num_layers * 2 * 2 * 64 * qcfg.num_heads * qcfg.head_dim * 512 * 512 // 2
        batched = {"metric": "tokens/s Qwen2.5-0.5B-shaped bf16 prefill b64 s512 (CUDA graph)",
                   "value": round(64 * 512 / (qms * 1e-3)), "unit": "tokens/s", "ms_per_step": round(qms, 3),
                   "seqs_per_rank": per_rank, "scaling": "strong",
                   "tflops": round(flops / (qms * 1e-3) / world / 1e12, 1),
                   "frac_tensor_per_gpu": round(flops / (qms * 1e-3) / world / 1e12 / peaks["bf16_tflops_sustained"], 3),
                   "note": f"per-GPU TFLOP/s vs the sustained bf16 peak {peak_note}; LM head via cuBLAS"}
        del qm
        torch.cuda.empty_cache()

    # ---- cached decoding (each rank its own replica) ---------------------------------------------
    decode = None
    if not args.no_decode:
        decode = [_decode_bench(dev, peaks, peak_note, b) for b in (1, 64)]
        for d_ in decode:  # whole job: every replica's tokens over the slowest replica's step time
            d_["ms_per_step"] = round(_max_over_ranks(d_["ms_per_step"], world, dev), 4)
            d_["value"] = round(world * d_["batch"] / (d_["ms_per_step"] * 1e-3))
            d_["n_gpus"] = world
        decode.append(_kv_attention_bench(dev, peaks, peak_note))

    # ---- CPU baseline (rank 0 at N=1): the reference's fp32 eager forward; its logits are the
    # parity reference for the timed graph's own output ---------------------------------------------
    cpu = None
    parity = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu_ms, runs, ref_logits, threads = cpu_reference_timer(cfg, tokens)
        port_ms = numpy_port_timer(cfg, tokens)
        cpu = {"value": round(cpu_ms, 3), "unit": "ms", "cores": threads, "kind": "reference",
               "sample": f"median of {runs} full 268M fp32 forwards (b1 s128) of the reference's unpatched eager "
                         "model (its benchmarks/bench_e2e.py blocks + embedding/head, torch CPU ops) after 3 warm-ups",
               "numpy_port_ms": round(port_ms, 3)}
        parity = {"llama268m_b1s128_fp16_graph": {**logits_parity(graph_logits, ref_logits),
                                                  "vs": "reference fp32 eager forward (CPU), same weights/tokens"}}
        if batched_rows is not None:
            qcfg = QWEN25_05B_SHAPED
            with torch.inference_mode():
                qref = _reference_forward(_reference_cpu_model(qcfg), batched_rows[0])
            parity["qwen_shaped_b64s512_bf16_graph"] = {
                **logits_parity(batched_rows[1], qref.float().numpy()),
                "vs": "reference fp32 eager forward (CPU) of the first and last of the 64 sequences"}
            del qref

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(ms, 4), "unit": "ms", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": False, "scaling": "weak",
            "vs_baseline": round(ms / PUBLISHED_MS, 4), "dtype": "fp16",
            "data": "synthetic: seeded N(0,0.02) random weights, uniform token ids",
            "config": {"workload": "llama268m-b1s128", "model": "Llama-style 268M (vocab 32000, hidden 1024, 18 layers, "
                       "16q/4kv heads, head_dim 64, FFN 2816, untied head)", "global_batch": world, "seq_len": 128,
                       "parallelism": f"replicas x{world} (no collective)",
                       "l2": "no flush: each forward streams 471 MB of weights, more than the 126 MB L2"},
            "median_step_ms": round(ms_median, 4),
            "tokens_per_s": round(world * 128 / (ms * 1e-3)),
            "vs_baseline_ref": f"{PUBLISHED_MS} ms, reference README.md:13 (RTX 5080)",
            "e2e": {"value": round(e2e_ms, 4), "unit": "ms", "h2d_bytes_per_step": 128 * 8,
                    "d2h_bytes_per_step": 128 * cfg.vocab_size * 2},
            "roofline": roof, "roofline_forward": roof_fwd, "kernels": table,
            "gpu_launches": launches_per_fwd * args.steps, "gpu_launches_per_fwd": launches_per_fwd,
            "clocks": clocks, "cpu_baseline": cpu, "parity": parity, "batched": batched, "decode": decode,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def main():
    args = _args()
    if args.sweep:
        import bench_sweep as sweep
        sweep.main(["--only", args.sweep])
    elif args.impl == "reference":
        run_reference(args)
    elif args.only:
        run_only(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
