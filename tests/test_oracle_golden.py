"""Pin the numpy oracle to vectors produced by the reference implementation itself.

The fixtures under tests/golden/ were written by tests/golden/make_golden.py,
which imports the reference's eager code (tinker/kernels/*.py and the model
blocks of benchmarks/bench_e2e.py). Runs on the CPU.
"""

import os

import numpy as np
import pytest
import torch

import oracle
from oracle import ops

GOLD = os.path.join(os.path.dirname(__file__), "golden")
DT = ["float32", "bfloat16", "float16"]


def _load(name):
    return np.load(os.path.join(GOLD, name))


def test_rope_tables_match_reference():
    z = _load("rope_tables.npz")
    for key in z.files:
        if not key.startswith("cos_"):
            continue
        d, t, th = key[4:].split("_")
        c, s = ops.rope_tables(int(d[1:]), int(t[1:]), float(th[2:]))
        np.testing.assert_allclose(c, z[key], atol=2e-6, rtol=0)
        np.testing.assert_allclose(s, z["sin_" + key[4:]], atol=2e-6, rtol=0)


def test_rope_apply_matches_reference():
    z = _load("rope_apply.npz")
    c, s = ops.rope_tables(64, 64, 1e4)
    for i in range(3):
        start, dti = z[f"meta{i}"]
        dtn = ["float32", "bfloat16"][int(dti)]
        y = ops.apply_rope(z[f"x{i}"], c, s, int(start), out_dtype=dtn)
        tol = 1e-6 if dtn == "float32" else 2 ** -7  # one bf16 ulp at |y| < 2
        np.testing.assert_allclose(y, z[f"y{i}"], atol=tol, rtol=tol)


def test_attention_matches_reference():
    z = _load("attention.npz")
    i = 0
    while f"meta{i}" in z.files:
        B, S, hq, hkv, d, start, dti = (int(v) for v in z[f"meta{i}"])
        dtn = ["float32", "bfloat16"][dti]
        c, s = ops.rope_tables(d, 64, 1e4)
        o = ops.attention(z[f"q{i}"], z[f"k{i}"], z[f"v{i}"], c, s, hq, hkv, d, start, io_dtype=dtn)
        ref = z[f"o{i}"]
        assert o.shape == ref.shape == (B, S, hq * d)
        tol = 2e-5 if dtn == "float32" else 1.6e-2
        np.testing.assert_allclose(o, ref, atol=tol, rtol=tol)
        i += 1
    assert i == 6


def test_rmsnorm_matches_reference():
    z = _load("rmsnorm.npz")
    for i in range(4):
        rows, dim, eps, dti = z[f"meta{i}"]
        dtn = DT[int(dti)]
        y = ops.rmsnorm(z[f"x{i}"], z[f"w{i}"], float(eps), out_dtype=dtn)
        ref = z[f"y{i}"]
        if dtn == "float32":
            np.testing.assert_allclose(y, ref, atol=1e-5, rtol=1e-5)
        else:
            # same float32 math, one rounding: identical except at rounding ties
            assert np.mean(y == ref) > 0.999
            ulp = 2 ** -7 if dtn == "bfloat16" else 2 ** -10
            np.testing.assert_allclose(y, ref, rtol=ulp, atol=1e-6)


def test_swiglu_matches_reference():
    z = _load("swiglu.npz")
    for i in range(3):
        rows, n, dti = z[f"meta{i}"]
        dtn = DT[int(dti)]
        y = ops.swiglu(z[f"g{i}"], z[f"u{i}"], out_dtype=dtn)
        ref = z[f"y{i}"]
        # the reference's eager path rounds after silu and again after the product;
        # the oracle (like the Triton kernel) rounds once: within two ulps
        tol = {"float32": 1e-6, "bfloat16": 2 * 2 ** -8, "float16": 2 * 2 ** -11}[dtn]
        np.testing.assert_allclose(y, ref, rtol=tol, atol=tol)


def _weights_np(model):
    return {k: v.detach().float().numpy() for k, v in model.state_dict().items()}


def test_tiny_model_matches_reference():
    from bench_model import TINY, build_model
    z = _load("tiny_model.npz")
    m = build_model(TINY, seed=int(z["weight_seed"]))
    cfg = oracle.ModelConfig(**{f: getattr(TINY, f) for f in oracle.ModelConfig.__dataclass_fields__})
    logits = oracle.forward_logits(_weights_np(m), z["tokens"], cfg)
    np.testing.assert_allclose(logits, z["logits"], atol=2e-5, rtol=1e-4)
    # both eager torch models give the reference's logits: the copy of the reference's own
    # blocks (oracle/torch_model.py, the CPU baseline) and the bench's user model
    # (bench_model.py, written independently), from the same seeded weights
    from oracle.torch_model import build_model as build_reference
    ref_model = build_reference(TINY, seed=int(z["weight_seed"]))
    assert ref_model.state_dict().keys() == m.state_dict().keys()
    tok = torch.from_numpy(z["tokens"])
    with torch.inference_mode():
        for model in (ref_model, m):
            np.testing.assert_allclose(model(tok).numpy(), z["logits"], atol=1e-5, rtol=1e-5)


@pytest.mark.slow
def test_llama268m_logits_match_reference():
    from bench_model import LLAMA_268M, build_model
    z = _load("llama268m_b1s128.npz")
    m = build_model(LLAMA_268M, seed=int(z["weight_seed"]))
    cfg = oracle.ModelConfig(**{f: getattr(LLAMA_268M, f) for f in oracle.ModelConfig.__dataclass_fields__})
    logits = oracle.forward_logits(_weights_np(m), z["tokens"], cfg)[0].astype(np.float64)
    np.testing.assert_allclose(logits[:, :64], z["slice"], atol=2e-4, rtol=0)
    np.testing.assert_allclose(logits.sum(-1), z["rowsum"], atol=5e-2, rtol=1e-5)
    np.testing.assert_allclose((logits * logits).sum(-1), z["rowsumsq"], rtol=1e-5)
    am = logits.argmax(-1)
    # top-1 may only differ where the reference's own top-1/top-2 gap is below fp32 noise
    diff = am != z["argmax"]
    assert np.all(z["gap"][diff] < 1e-4)
