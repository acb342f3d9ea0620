"""Generate the golden vectors that pin the numpy oracle to the reference.

Run in a container that has the reference checkout (eb1386/TinKer) on disk:

    python tests/golden/make_golden.py --reference /path/to/TinKer

It imports the reference's own eager code paths (``tinker/kernels/*.py`` and the
model blocks of ``benchmarks/bench_e2e.py``), runs them on seeded inputs on the
CPU, and writes compressed ``.npz`` fixtures next to this script. The tests only
read the fixtures; nothing at test time needs the reference checkout.
"""

from __future__ import annotations

import argparse
import importlib.util
import os
import sys

import numpy as np
import torch
import torch.nn as nn

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from bench_model import LLAMA_268M, TINY, init_weights, make_tokens  # noqa: E402


def _f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().to(torch.float32).cpu().numpy()


def _load_reference(ref: str):
    sys.path.insert(0, ref)
    import tinker  # noqa: F401  (the reference package)
    # the kernel package re-exports functions under the submodule names, so
    # fetch the submodules themselves from sys.modules
    fa = importlib.import_module("tinker.kernels.fused_attention")
    fr = importlib.import_module("tinker.kernels.fused_rmsnorm")
    fs = importlib.import_module("tinker.kernels.fused_swiglu")
    spec = importlib.util.spec_from_file_location("ref_bench_e2e",
                                                  os.path.join(ref, "benchmarks", "bench_e2e.py"))
    be = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(be)
    return tinker, fa, fr, fs, be


def _ref_lm(be, cfg):
    """The reference's SimpleTransformer blocks with an embedding and an untied head."""

    class RefLM(nn.Module):
        def __init__(self):
            super().__init__()
            st = be.SimpleTransformer(cfg.num_layers, cfg.hidden_size, cfg.num_heads,
                                      cfg.num_kv_heads, cfg.head_dim, cfg.intermediate_size)
            self.embedding = nn.Embedding(cfg.vocab_size, cfg.hidden_size)
            self.layers = st.layers
            self.norm = st.norm
            self.output = nn.Linear(cfg.hidden_size, cfg.vocab_size, bias=False)

        def forward(self, tokens):
            x = self.embedding(tokens)
            for layer in self.layers:
                x = layer(x)
            return self.output(self.norm(x))

    return RefLM()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("TINKER_REFERENCE"),
                    help="path of the eb1386/TinKer checkout (or set TINKER_REFERENCE)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give the reference checkout with --reference PATH or the TINKER_REFERENCE variable")
    tinker, fa, fr, fs, be = _load_reference(args.reference)
    dt = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}

    # 1. RoPE tables (fused_attention.py:157-162)
    out = {}
    for d, t, theta in [(4, 16, 1e4), (64, 64, 1e4), (64, 64, 1e6), (128, 64, 1e4)]:
        c, s = fa.precompute_rope_tables(d, t, theta)
        out[f"cos_d{d}_t{t}_th{int(theta)}"] = _f32(c)
        out[f"sin_d{d}_t{t}_th{int(theta)}"] = _f32(s)
    np.savez_compressed(os.path.join(HERE, "rope_tables.npz"), **out)

    # 2. interleaved RoPE on [B,H,S,D] (fused_attention.py:165-173)
    g = torch.Generator().manual_seed(11)
    out = {}
    c, s = fa.precompute_rope_tables(64, 64, 1e4)
    for i, (start, dtn) in enumerate([(0, "float32"), (3, "float32"), (0, "bfloat16")]):
        x = torch.randn(1, 2, 5, 64, generator=g).to(dt[dtn])
        y = fa._apply_rope_pytorch(x, c, s, start_pos=start)
        out[f"x{i}"], out[f"y{i}"] = _f32(x), _f32(y)
        out[f"meta{i}"] = np.array([start, ["float32", "bfloat16"].index(dtn)])
    np.savez_compressed(os.path.join(HERE, "rope_apply.npz"), **out)

    # 3. RoPE + GQA causal attention (fused_attention.py:176-192)
    g = torch.Generator().manual_seed(12)
    out = {}
    cases = [(1, 33, 4, 2, 64, 0, "float32"), (2, 17, 4, 4, 64, 0, "float32"),
             (1, 20, 4, 1, 64, 3, "float32"), (1, 16, 2, 1, 128, 0, "float32"),
             (1, 24, 4, 2, 64, 0, "bfloat16"), (1, 1, 4, 2, 64, 0, "float32")]
    for i, (B, S, hq, hkv, d, start, dtn) in enumerate(cases):
        c, s = fa.precompute_rope_tables(d, 64, 1e4)
        q = torch.randn(B, S, hq * d, generator=g).to(dt[dtn])
        k = torch.randn(B, S, hkv * d, generator=g).to(dt[dtn])
        v = torch.randn(B, S, hkv * d, generator=g).to(dt[dtn])
        o = fa._attention_pytorch(q, k, v, c, s, hq, hkv, d, start_pos=start)
        out[f"q{i}"], out[f"k{i}"], out[f"v{i}"], out[f"o{i}"] = _f32(q), _f32(k), _f32(v), _f32(o)
        out[f"meta{i}"] = np.array([B, S, hq, hkv, d, start, ["float32", "bfloat16"].index(dtn)])
    np.savez_compressed(os.path.join(HERE, "attention.npz"), **out)

    # 4. RMSNorm (fused_rmsnorm.py:64-67)
    g = torch.Generator().manual_seed(13)
    out = {}
    cases = [(3, 256, 1e-6, "float32"), (4, 1280, 1e-6, "bfloat16"), (2, 1024, 1e-5, "float16"),
             (5, 4096, 1e-6, "float32")]
    for i, (rows, dim, eps, dtn) in enumerate(cases):
        x = torch.randn(rows, dim, generator=g).to(dt[dtn])
        w = (1.0 + 0.1 * torch.randn(dim, generator=g)).to(dt[dtn])
        y = fr._rmsnorm_pytorch(x, w, eps)
        out[f"x{i}"], out[f"w{i}"], out[f"y{i}"] = _f32(x), _f32(w), _f32(y)
        out[f"meta{i}"] = np.array([rows, dim, eps, ["float32", "bfloat16", "float16"].index(dtn)])
    np.savez_compressed(os.path.join(HERE, "rmsnorm.npz"), **out)

    # 5. SwiGLU activation (fused_swiglu.py:57-58)
    g = torch.Generator().manual_seed(14)
    out = {}
    cases = [(5, 1376, "float32"), (3, 2816, "bfloat16"), (2, 512, "float16")]
    for i, (rows, n, dtn) in enumerate(cases):
        a = torch.randn(rows, n, generator=g).to(dt[dtn])
        b = torch.randn(rows, n, generator=g).to(dt[dtn])
        y = fs._swiglu_pytorch(a.clone(), b)
        out[f"g{i}"], out[f"u{i}"], out[f"y{i}"] = _f32(a), _f32(b), _f32(y)
        out[f"meta{i}"] = np.array([rows, n, ["float32", "bfloat16", "float16"].index(dtn)])
    np.savez_compressed(os.path.join(HERE, "swiglu.npz"), **out)

    # 6. tiny decoder, fp32 logits; also checks the reference's patched CPU model matches.
    torch.manual_seed(0)
    m = _ref_lm(be, TINY)
    init_weights(m, seed=5)
    m.eval()
    tok = make_tokens(TINY, 2, 16, seed=6)
    with torch.inference_mode():
        logits = m(tok)
    patched = tinker.patch_model(_ref_lm(be, TINY))
    patched.load_state_dict(m.state_dict())
    patched.eval()
    with torch.inference_mode():
        assert torch.equal(patched(tok), logits), "reference patched CPU path differs from eager"
    np.savez_compressed(os.path.join(HERE, "tiny_model.npz"), tokens=tok.numpy(),
                        logits=_f32(logits), weight_seed=np.array(5), token_seed=np.array(6))

    # 7. the 268M decoder (batch 1 x seq 128), fp32 logits summary
    m = _ref_lm(be, LLAMA_268M)
    init_weights(m, seed=0)
    m.eval()
    tok = make_tokens(LLAMA_268M, 1, 128, seed=1)
    with torch.inference_mode():
        logits = m(tok)[0].double()
    top2 = torch.topk(logits, 2, dim=-1).values
    np.savez_compressed(os.path.join(HERE, "llama268m_b1s128.npz"), tokens=tok.numpy(),
                        slice=_f32(logits[:, :64]), argmax=logits.argmax(-1).numpy(),
                        maxval=top2[:, 0].numpy(), gap=(top2[:, 0] - top2[:, 1]).numpy(),
                        rowsum=logits.sum(-1).numpy(), rowsumsq=(logits * logits).sum(-1).numpy(),
                        weight_seed=np.array(0), token_seed=np.array(1))
    print("wrote fixtures to", HERE)


if __name__ == "__main__":
    main()
