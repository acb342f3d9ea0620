"""End-to-end parity of the patched, graph-captured decoder against the fp32 oracle.

The 268M Llama-style model (vocab 32000, hidden 1024, 18 layers, 16/4 heads,
head_dim 64, FFN 2816) at batch 1 x seq 128 is built with seeded N(0, 0.02)
weights, optimised with ``optimize(dtype=float16, cuda_graph=True)`` and compared
with the numpy oracle's float32 forward on the same (unrounded) weights - the
reference's fp32 eager path. Reported: max-abs logits error, top-1 agreement,
and top-1 agreement over positions whose fp32 top-1/top-2 margin exceeds the
observed error (random weights give near-ties, so raw top-1 cannot reach 100%
even for the reference's own fp16 eager model). Bars: max-abs <= 2e-2 (fp16),
margin-aware top-1 = 100%, and no worse than 2x the reference's own fp16 eager
error on the same GPU.
"""

import numpy as np
import pytest
import torch

import oracle
from tests._util import np32, require_b200

pytestmark = pytest.mark.gpu


def _oracle_logits(model, tokens, cfg):
    w = {k: v.detach().float().cpu().numpy() for k, v in model.state_dict().items()}
    ocfg = oracle.ModelConfig(**{f: getattr(cfg, f) for f in oracle.ModelConfig.__dataclass_fields__})
    return oracle.forward_logits(w, tokens.numpy(), ocfg)


def _stats(logits, ref):
    err = np.abs(logits.astype(np.float64) - ref)
    s = np.sort(ref, axis=-1)
    gap = s[..., -1] - s[..., -2]
    agree = logits.argmax(-1) == ref.argmax(-1)
    clear = gap > 2 * err.max()
    return float(err.max()), float(agree.mean()), float(agree[clear].mean()) if clear.any() else 1.0


def test_llama268m_b1s128_fp16_graph():
    require_b200()
    import tinker_b200
    from bench_model import LLAMA_268M, build_model, make_tokens
    cfg = LLAMA_268M
    tokens = make_tokens(cfg, 1, 128, seed=1)
    cpu_model = build_model(cfg, seed=0)
    ref = _oracle_logits(cpu_model, tokens, cfg).astype(np.float64)

    from oracle.torch_model import build_model as build_reference
    eager16 = build_reference(cfg, seed=0, device="cuda", dtype=torch.float16)  # the reference's fp16 eager path
    with torch.inference_mode():
        base = np32(eager16(tokens.cuda()))
    base_err, base_top1, _ = _stats(base, ref)

    model = cpu_model.to("cuda")
    model = tinker_b200.optimize(model, dtype=torch.float16, cuda_graph=True, graph_input_shape=(1, 128),
                                 graph_vocab_size=cfg.vocab_size)
    assert type(model).__name__ == "_CUDAGraphWrapper", "graph capture failed"
    with torch.inference_mode():
        out = np32(model(tokens.cuda()))
        out2 = np32(model(tokens.cuda()))
    np.testing.assert_array_equal(out, out2)  # replay is deterministic
    err, top1, top1_clear = _stats(out, ref)
    print(f"\n268M fp16 graph: max-abs {err:.3e} top1 {top1:.4f} top1(clear margin) {top1_clear:.4f}; "
          f"reference fp16 eager: max-abs {base_err:.3e} top1 {base_top1:.4f}")
    assert err <= 2e-2
    assert top1_clear == 1.0
    assert err <= 2 * base_err + 1e-3


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_tiny_model_patched_eager(dtype):
    require_b200()
    import tinker_b200
    from bench_model import TINY, build_model, make_tokens
    tokens = make_tokens(TINY, 3, 40, seed=2)
    cpu_model = build_model(TINY, seed=3)
    ref = _oracle_logits(cpu_model, tokens, TINY).astype(np.float64)
    model = tinker_b200.optimize(cpu_model.to("cuda"), dtype=dtype)
    kinds = {type(m).__name__ for m in model.modules()}
    assert {"TinKerAttention", "TinKerSwiGLU", "TinKerRMSNorm"} <= kinds
    with torch.inference_mode():
        out = np32(model(tokens.cuda()))
    err = np.abs(out - ref).max() / np.abs(ref).max()
    assert err <= (1e-2 if dtype == torch.float16 else 4e-2)


def test_qwen_shaped_two_layers_bf16():
    """Qwen2.5-0.5B shapes (hidden 896, 14/2 heads, FFN 4864, theta 1e6, tied head), 2 layers, bf16."""
    require_b200()
    import tinker_b200
    from bench_model import QWEN25_05B_SHAPED, build_model, make_tokens
    cfg = QWEN25_05B_SHAPED.with_(num_layers=2, vocab_size=4096)
    tokens = make_tokens(cfg, 2, 512, seed=4)
    cpu_model = build_model(cfg, seed=5)
    ref = _oracle_logits(cpu_model, tokens, cfg).astype(np.float64)
    model = tinker_b200.optimize(cpu_model.to("cuda"), dtype=torch.bfloat16)
    with torch.inference_mode():
        out = np32(model(tokens.cuda()))
    rel = np.linalg.norm(out - ref) / np.linalg.norm(ref)
    assert rel <= 2e-2


def test_block_fusion_matches_unfused_and_skips_other_structures():
    """Fused blocks (residual adds in the GEMM epilogues) equal the leaf-patched blocks;
    a block with another structure (parallel attention + FFN) is not fused."""
    require_b200()
    import torch.nn as nn
    import tinker_b200
    from bench_model import TINY, build_model, make_tokens
    from tinker_b200.fusion import fuse_decoder_blocks
    cfg = TINY.with_(num_layers=3)
    tokens = make_tokens(cfg, 2, 64, seed=9).cuda()
    a = tinker_b200.optimize(build_model(cfg, seed=4).cuda(), dtype=torch.float16, fuse_blocks=False)
    b = tinker_b200.optimize(build_model(cfg, seed=4).cuda(), dtype=torch.float16, fuse_blocks=True)
    assert all(getattr(l, "_tinker_block_parts", None) for l in b.layers)
    assert not any(getattr(l, "_tinker_block_parts", None) for l in a.layers)
    with torch.inference_mode():
        ya, yb = a(tokens).float(), b(tokens).float()
    assert ((ya - yb).norm() / ya.norm()).item() < 5e-3

    class Parallel(nn.Module):  # x + attn(n1(x)) + ffn(n2(x)): same children, different math
        def __init__(self, blk):
            super().__init__()
            self.attn_norm, self.attn, self.ffn_norm, self.ffn = blk.attn_norm, blk.attn, blk.ffn_norm, blk.ffn

        def forward(self, x):
            return x + self.attn(self.attn_norm(x)) + self.ffn(self.ffn_norm(x))

    wrapper = nn.Module()
    wrapper.blk = Parallel(a.layers[0])
    assert fuse_decoder_blocks(wrapper) == 0


def test_folded_norms_match_unfolded_and_follow_weight_updates():
    """RMSNorms folded into the q|k|v and gate|up GEMMs (5 launches per block) give the same
    logits as norm-then-GEMM blocks, and a norm weight changed in place is folded again."""
    require_b200()
    import tinker_b200
    from tinker_b200 import _lib
    from bench_model import TINY, build_model, make_tokens
    cfg = TINY.with_(num_layers=3)
    tokens = make_tokens(cfg, 2, 96, seed=5).cuda()
    a = tinker_b200.optimize(build_model(cfg, seed=8).cuda(), dtype=torch.float16, fold_norms=False)
    b = tinker_b200.optimize(build_model(cfg, seed=8).cuda(), dtype=torch.float16, fold_norms=True)
    with torch.inference_mode():
        ya = a(tokens).float()
        n0 = _lib.launch_counter[0]
        yb = b(tokens).float()
        launches = _lib.launch_counter[0] - n0
    assert ((ya - yb).norm() / ya.norm()).item() < 5e-3
    # 5 per block + row statistics of the first block's input + final norm
    assert launches == 5 * cfg.num_layers + 2
    with torch.no_grad():
        for m in (a, b):
            m.layers[1].ffn_norm.weight.mul_(1.5)
    with torch.inference_mode():
        ya2, yb2 = a(tokens).float(), b(tokens).float()
    assert ((ya2 - ya).norm() / ya.norm()).item() > 1e-2
    assert ((ya2 - yb2).norm() / ya2.norm()).item() < 5e-3


def test_folded_norm_statistics_follow_in_place_changes():
    """The row statistics a folded block hands to the next one are recomputed when the hidden
    states were changed in place in between (a model that scales the residual stream), which
    the tensor's version counter shows outside inference mode."""
    require_b200()
    import torch.nn as nn
    import tinker_b200
    from bench_model import TINY, build_model, make_tokens

    class Scaled(nn.Module):  # x = block(x); x *= 1.5 (in place) between blocks
        def __init__(self, lm):
            super().__init__()
            self.lm = lm

        def forward(self, tokens):
            x = self.lm.embedding(tokens)
            for layer in self.lm.layers:
                x = layer(x)
                x.mul_(1.5)
            return self.lm.output(self.lm.norm(x))

    cfg = TINY.with_(num_layers=3)
    tokens = make_tokens(cfg, 2, 64, seed=3).cuda()
    a = Scaled(tinker_b200.optimize(build_model(cfg, seed=6).cuda(), dtype=torch.float16, fold_norms=False))
    b = Scaled(tinker_b200.optimize(build_model(cfg, seed=6).cuda(), dtype=torch.float16, fold_norms=True))
    with torch.no_grad():  # version counters exist outside inference mode
        ya, yb = a(tokens).float(), b(tokens).float()
    assert ((ya - yb).norm() / ya.norm()).item() < 5e-3


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_embedding_rows_is_the_gather_with_row_statistics(dtype):
    """tk_embedding_rows: the rows of nn.Embedding bit for bit, the per-32-column sums of squares of
    tk_row_sumsq, and a token outside the table as device error 3 with a zero row; optimize() gives a
    plain decoder's embedding this forward and its first folded block then skips its statistics."""
    require_b200()
    import tinker_b200
    from tinker_b200 import _lib
    from tinker_b200.kernels.gemm import embedding_rows, row_sumsq
    from bench_model import TINY, build_model, make_tokens
    g = torch.Generator(device="cuda").manual_seed(2)
    table = torch.randn(1000, 256, device="cuda", generator=g).to(dtype)
    ids = torch.randint(0, 1000, (3, 37), device="cuda", generator=g)
    out, parts = embedding_rows(ids, table)
    torch.cuda.synchronize()
    assert torch.equal(out, table[ids])
    np.testing.assert_allclose(np32(parts), np32(row_sumsq(out)), rtol=1e-6, atol=1e-6)
    _lib.device_error(clear=True)
    bad = ids.clone()
    bad[1, 5] = 1000
    out2, _ = embedding_rows(bad, table)
    torch.cuda.synchronize()
    assert _lib.device_error(clear=True) == 3
    assert torch.count_nonzero(out2[1, 5]) == 0 and torch.equal(out2[0], out[0])
    model = tinker_b200.optimize(build_model(TINY, seed=3).cuda(), dtype=dtype)
    assert "forward" in model.embedding.__dict__
    tokens = make_tokens(TINY, 2, 24, seed=4).cuda()
    with torch.inference_mode():
        n0 = _lib.launch_counter[0]
        model(tokens)
        assert _lib.launch_counter[0] - n0 == 5 * TINY.num_layers + 2  # embedding + blocks + final norm
