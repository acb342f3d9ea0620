"""Host logic of the drop-in API on the CPU: module detection and replacement,
from_module inference, state_dict compatibility, and the loud failures of the
no-fallback design (CPU tensors, CPU models)."""

import pytest
import torch
import torch.nn as nn

import tinker_b200
from bench_model import TINY, LLAMA_268M, DecoderLM, build_model
from tinker_b200.modules import TinKerAttention, TinKerRMSNorm, TinKerSwiGLU
from tinker_b200.patch import _is_gqa_attention, _is_rmsnorm, _is_swiglu


def test_detectors_follow_the_reference_rules():
    m = build_model(TINY)
    blk = m.layers[0]
    assert _is_rmsnorm(blk.attn_norm) and _is_rmsnorm(m.norm)
    assert _is_swiglu(blk.ffn) and not _is_swiglu(blk.attn)
    assert _is_gqa_attention(blk.attn) and not _is_gqa_attention(blk.ffn)
    assert not _is_rmsnorm(nn.LayerNorm(8))  # has a bias
    assert not _is_rmsnorm(m.embedding)
    hf_norm = nn.Module()
    hf_norm.weight = nn.Parameter(torch.ones(4))
    hf_norm.variance_epsilon = 1e-5
    assert _is_rmsnorm(hf_norm)


def test_patch_model_replaces_every_block_module_and_keeps_state_dict():
    m = build_model(TINY)
    sd = {k: v.clone() for k, v in m.state_dict().items()}
    tinker_b200.patch_model(m, verbose=True)
    kinds = [type(x).__name__ for x in m.modules()]
    assert kinds.count("TinKerAttention") == TINY.num_layers
    assert kinds.count("TinKerSwiGLU") == TINY.num_layers
    assert kinds.count("TinKerRMSNorm") == 2 * TINY.num_layers + 1
    sd2 = m.state_dict()
    assert set(sd) == set(sd2)
    for k in sd:
        assert torch.equal(sd[k], sd2[k]), k


def test_patch_flags_select_module_kinds():
    m = build_model(TINY)
    tinker_b200.patch_model(m, replace_attention=False, replace_ffn=False)
    kinds = {type(x).__name__ for x in m.modules()}
    assert "TinKerRMSNorm" in kinds and "TinKerAttention" not in kinds and "TinKerSwiGLU" not in kinds


def test_attention_from_module_infers_heads_and_theta():
    cfg = LLAMA_268M.with_(num_layers=1, vocab_size=16, rope_theta=1e6)
    m = DecoderLM(cfg)
    att = TinKerAttention.from_module(m.layers[0].attn, rope_theta=1e4, max_seq_len=512)
    assert (att.num_heads, att.num_kv_heads, att.head_dim) == (16, 4, 64)
    assert att.rope_theta == 1e6  # taken from the source module (attention.py:95-97)
    assert att.cos_table.shape == (512, 32)

    class NoHeadDim(nn.Module):
        def __init__(self):
            super().__init__()
            self.wq = nn.Linear(256, 256, bias=False)
            self.wk = nn.Linear(256, 128, bias=False)
            self.wv = nn.Linear(256, 128, bias=False)
            self.wo = nn.Linear(256, 256, bias=False)

    att = TinKerAttention.from_module(NoHeadDim())
    assert (att.num_heads, att.num_kv_heads, att.head_dim) == (4, 2, 64)


def test_rope_tables_stay_float32_when_cast():
    att = TinKerAttention(256, 4, 2, 64).to(torch.float16)
    assert att.q_proj.weight.dtype == torch.float16
    assert att.cos_table.dtype == torch.float32 and att.sin_table.dtype == torch.float32


def test_swiglu_and_norm_from_module():
    m = build_model(TINY)
    f = TinKerSwiGLU.from_module(m.layers[0].ffn)
    assert (f.hidden_size, f.intermediate_size) == (TINY.hidden_size, TINY.intermediate_size)
    assert torch.equal(f.down_proj.weight, m.layers[0].ffn.down_proj.weight)
    src = nn.Module()
    src.weight = nn.Parameter(torch.randn(8))
    src.variance_epsilon = 1e-5
    n = TinKerRMSNorm.from_module(src)
    assert n.eps == 1e-5 and torch.equal(n.weight, src.weight)
    with pytest.raises(ValueError, match="SwiGLU"):
        TinKerSwiGLU.from_module(nn.Linear(2, 2))


def test_no_cpu_fallback():
    m = build_model(TINY)
    with pytest.raises(RuntimeError, match="CUDA"):
        tinker_b200.optimize(m)
    tinker_b200.patch_model(m)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        m(torch.zeros(1, 4, dtype=torch.long))


def test_param_count_of_the_268m_config():
    assert LLAMA_268M.num_params() == 268_473_344


def test_block_fusion_candidates_and_signature_rule():
    from tinker_b200.fusion import _block_parts, _takes_hidden_states_only
    m = build_model(TINY)
    tinker_b200.patch_model(m)
    blk = m.layers[0]
    assert _block_parts(blk) == ("attn_norm", "attn", "ffn_norm", "ffn")
    assert _takes_hidden_states_only(blk)
    assert _block_parts(m) is None

    class TwoArgs(nn.Module):
        def forward(self, x, mask):
            return x

    assert not _takes_hidden_states_only(TwoArgs())


def test_block_dataflow_check_accepts_prenorm_and_rejects_other_structures():
    from tinker_b200.fusion import _dataflow_is_prenorm_residual

    class N(nn.Module):
        def __init__(self):
            super().__init__()
            self.weight = nn.Parameter(torch.ones(8))

        def forward(self, x):
            return x * 1.0

    class L(nn.Module):
        def forward(self, x):
            return x * 0.5

    class PreNorm(nn.Module):
        def __init__(self):
            super().__init__()
            self.n1, self.a, self.n2, self.f = N(), L(), N(), L()

        def forward(self, x):
            x = x + self.a(self.n1(x))
            return x + self.f(self.n2(x))

    class Parallel(PreNorm):
        def forward(self, x):
            return x + self.a(self.n1(x)) + self.f(self.n2(x))

    class PostNorm(PreNorm):
        def forward(self, x):
            x = self.n1(x + self.a(x))
            return self.n2(x + self.f(x))

    class Scaled(PreNorm):
        def forward(self, x):
            x = x + 0.5 * self.a(self.n1(x))
            return x + self.f(self.n2(x))

    parts = ("n1", "a", "n2", "f")
    g = torch.Generator().manual_seed(0)
    x = torch.randn(1, 4, 8)
    assert _dataflow_is_prenorm_residual(PreNorm(), parts, x, g)
    for cls in (Parallel, PostNorm, Scaled):
        assert not _dataflow_is_prenorm_residual(cls(), parts, x, g), cls.__name__


def test_rope_tables_are_shared_across_layers():
    from tinker_b200.fusion import share_rope_tables
    m = build_model(TINY.with_(num_layers=3))
    tinker_b200.patch_model(m)
    assert share_rope_tables(m) == 2
    assert m.layers[0].attn.cos_table is m.layers[2].attn.cos_table
    m.to(torch.float16)
    assert m.layers[1].attn.sin_table.dtype == torch.float32


# ---- decisions pinned to the reference's patch_model ------------------------------------------
def _zoo():
    import importlib
    import os
    import sys
    here = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
    if here not in sys.path:
        sys.path.insert(0, here)
    return importlib.import_module("patch_zoo")


@pytest.mark.parametrize("flags", ["all", "no_norm", "no_ffn", "no_attention", "theta_arg"])
def test_patch_decisions_match_the_reference(flags):
    """The reference's own patch_model, run over the module zoo of tests/golden/patch_zoo.py by
    make_patch_golden.py, replaced exactly these children with exactly these sizes."""
    import json
    import os
    zoo = _zoo()
    with open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "patch_decisions.json")) as f:
        want = json.load(f)[flags]
    got = zoo.describe(tinker_b200.patch_model(zoo.zoo(), **zoo.FLAG_SETS[flags]))
    assert got == want


def test_reference_dummy_modules_from_module():
    """The source modules of the reference's from_module tests (tests/test_attention.py:171-180,
    tests/test_rmsnorm.py:71-77, tests/test_swiglu.py:77-87): sizes, epsilon and weights carry over."""
    torch.manual_seed(0)
    src = nn.Module()
    src.head_dim = 64
    src.q_proj, src.k_proj = nn.Linear(512, 512, bias=False), nn.Linear(512, 128, bias=False)
    src.v_proj, src.o_proj = nn.Linear(512, 128, bias=False), nn.Linear(512, 512, bias=False)
    att = TinKerAttention.from_module(src.to(torch.bfloat16))
    assert (att.num_heads, att.num_kv_heads, att.head_dim) == (8, 2, 64)
    for n in ("q_proj", "k_proj", "v_proj", "o_proj"):
        assert torch.equal(getattr(att, n).weight.to(torch.bfloat16), getattr(src, n).weight)

    norm = nn.Module()
    norm.eps = 1e-5
    norm.weight = nn.Parameter(torch.randn(512))
    tn = TinKerRMSNorm.from_module(norm)
    assert tn.eps == 1e-5 and torch.equal(tn.weight, norm.weight)

    ffn = nn.Module()
    ffn.gate_proj, ffn.up_proj = nn.Linear(512, 1376, bias=False), nn.Linear(512, 1376, bias=False)
    ffn.down_proj = nn.Linear(1376, 512, bias=False)
    tf = TinKerSwiGLU.from_module(ffn)
    assert (tf.hidden_size, tf.intermediate_size) == (512, 1376)
    for n in ("gate_proj", "up_proj", "down_proj"):
        assert torch.equal(getattr(tf, n).weight, getattr(ffn, n).weight)


def test_benchmark_model_reports_the_reference_keys():
    """benchmark_model on a CPU model: the reference's result keys, a consistent median/min/mean
    and tokens/s at the median."""
    from tinker_b200 import benchmark_model

    class Toy(nn.Module):
        def __init__(self):
            super().__init__()
            self.emb = nn.Embedding(50, 8)

        def forward(self, t):
            return self.emb(t).sum(-1)

    r = benchmark_model(Toy(), input_shape=(2, 16), vocab_size=50, warmup=2, runs=9, device="cpu")
    assert set(r) == {"median_ms", "mean_ms", "min_ms", "tokens_per_sec", "device"}
    assert r["device"] == "cpu"
    assert 0 <= r["min_ms"] <= r["median_ms"]
    assert r["tokens_per_sec"] == pytest.approx(32 / (r["median_ms"] / 1e3), rel=0.05, abs=1)


def test_reference_import_paths_resolve_to_this_package():
    """Code written against the reference imports `tinker` and its submodules by path."""
    import tinker
    from tinker.kernels import fused_attention, fused_rmsnorm, fused_swiglu, precompute_rope_tables  # noqa: F401
    from tinker.kernels.fused_rmsnorm import fused_rmsnorm as fr
    from tinker.modules import TinKerAttention as TA
    from tinker.modules.feed_forward import TinKerSwiGLU as TS
    from tinker.patch import patch_model as pm
    from tinker.optimize import benchmark_model as bm
    assert tinker.optimize is tinker_b200.optimize and pm is tinker_b200.patch_model
    assert fr is fused_rmsnorm and TA is TinKerAttention and TS is TinKerSwiGLU and bm is tinker_b200.benchmark_model


def test_prefetch_chain_links_blocks_in_order_and_caps_the_head():
    """``link_ahead`` points every fused block at the next one and the last at the LM head;
    ``_ahead_weights`` names the next block's folded q|k|v weights once they exist, the head
    weight unless it is larger than the cap (a tied 150k-token table would not stay in L2)."""
    from tinker_b200 import fusion
    m = build_model(TINY.with_(num_layers=3))
    tinker_b200.patch_model(m)
    for blk in m.layers:  # what fuse_decoder_blocks records once a block passed its checks
        blk._tinker_block_parts = fusion._block_parts(blk)
    assert fusion.link_ahead(m) == 3
    b0, b1, b2 = m.layers
    assert b0._tinker_ahead() is b1 and b1._tinker_ahead() is b2 and b2._tinker_ahead() is m.output
    assert fusion._ahead_weights(b0) == ()  # the next block has not folded its weights yet
    folded = tuple(torch.zeros(2, 2) for _ in range(5))
    b1._tinker_folded = (None, folded)
    assert fusion._ahead_weights(b0) == folded[:3]
    assert fusion._ahead_weights(b2) == (m.output.weight,)
    big = nn.Linear(8, (fusion._AHEAD_MAX_BYTES // 32) + 1, bias=False)  # just above the cap in fp32
    m.output = big
    fusion.link_ahead(m)
    assert fusion._ahead_weights(b2) == ()
    assert "_tinker_ahead" not in dict(m.named_modules())  # plain attributes, not submodules
