"""SwiGLU parity: the elementwise kernel (fused_swiglu) and the fused FFN (TinKerSwiGLU).

fused_swiglu vs the oracle (float32 math, one rounding): equal to one ulp.
The FFN (gate|up GEMM with SwiGLU epilogue, then down GEMM) vs float64 numpy
on the same half inputs: norm-wise relative error <= 1e-3 for fp16; for bf16
the rounding of the intermediate activation alone is ~2^-9/sqrt(3) relative,
so the bar is 4e-3, and the kernel must also be no worse than the reference's
own eager bf16 path (gate and up rounded, silu rounded, product rounded).
"""

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import oracle
from tests._util import DTYPES, NP_NAME, np32, rel_err, require_b200, ulp

pytestmark = pytest.mark.gpu

REF_CONFIGS = [(688, 1376, 64, 1), (1024, 2816, 64, 1), (1280, 3584, 64, 1), (1024, 4096, 64, 1),
               (512, 1376, 1, 1), (1024, 2816, 32, 8)]


@pytest.mark.parametrize("hidden, inter, seq, batch", REF_CONFIGS)
@pytest.mark.parametrize("dt", ["bf16", "fp16", "fp32"])
def test_fused_swiglu_kernel(hidden, inter, seq, batch, dt):
    require_b200()
    from tinker_b200.kernels.fused_swiglu import fused_swiglu
    torch.manual_seed(42)
    dtype = DTYPES[dt]
    gate = torch.randn(batch, seq, inter, device="cuda", dtype=dtype)
    up = torch.randn(batch, seq, inter, device="cuda", dtype=dtype)
    out = fused_swiglu(gate, up)
    ref = oracle.swiglu(np32(gate), np32(up), out_dtype=NP_NAME[dtype])
    np.testing.assert_allclose(np32(out), ref, rtol=ulp(dtype) if dtype != torch.float32 else 1e-6,
                               atol=1e-6)


def test_fused_swiglu_shape_assert_and_odd_sizes():
    require_b200()
    from tinker_b200.kernels.fused_swiglu import fused_swiglu
    a = torch.randn(3, 5, device="cuda", dtype=torch.float16)
    with pytest.raises(AssertionError):
        fused_swiglu(a, torch.randn(3, 6, device="cuda", dtype=torch.float16))
    b = torch.randn(3, 5, device="cuda", dtype=torch.float16)
    np.testing.assert_allclose(np32(fused_swiglu(a, b)), oracle.swiglu(np32(a), np32(b), out_dtype="float16"),
                               rtol=ulp(torch.float16), atol=1e-6)


@pytest.mark.parametrize("dt", ["fp16", "bf16"])
@pytest.mark.parametrize("rows, inter", [(4099, 2816), (1, 8), (37, 1376)])
def test_fused_swiglu_contiguous_sizes_and_strided_rows(rows, inter, dt):
    """Contiguous inputs run as one flat array of 16-byte vectors (four per thread from a few thousand
    rows on, with a ragged last block at 4099 rows); gate and up taken as the two halves of one
    [rows, 2F] tensor (row stride 2F) run the strided kernel. Both equal the oracle to one ulp."""
    require_b200()
    from tinker_b200.kernels.fused_swiglu import fused_swiglu
    torch.manual_seed(7)
    dtype = DTYPES[dt]
    gate = torch.randn(rows, inter, device="cuda", dtype=dtype)
    up = torch.randn(rows, inter, device="cuda", dtype=dtype)
    ref = oracle.swiglu(np32(gate), np32(up), out_dtype=NP_NAME[dtype])
    np.testing.assert_allclose(np32(fused_swiglu(gate, up)), ref, rtol=ulp(dtype), atol=1e-6)
    both = torch.cat([gate, up], dim=1)
    g2, u2 = both[:, :inter], both[:, inter:]
    assert g2.stride(0) == 2 * inter
    np.testing.assert_allclose(np32(fused_swiglu(g2, u2)), ref, rtol=ulp(dtype), atol=1e-6)


def _ffn_ref(x, wg, wu, wd):
    xx = np32(x).astype(np.float64).reshape(-1, x.shape[-1])
    a = xx @ np32(wg).astype(np.float64).T
    b = xx @ np32(wu).astype(np.float64).T
    return (a / (1 + np.exp(-a)) * b) @ np32(wd).astype(np.float64).T


@pytest.mark.parametrize("dt", ["fp16", "bf16"])
@pytest.mark.parametrize("tokens", [128, 4096, 16384])
@pytest.mark.parametrize("hidden, inter", [(1024, 2816), (2048, 5632)])
def test_ffn_sweep(dt, tokens, hidden, inter):
    require_b200()
    from tinker_b200.modules import TinKerSwiGLU
    dtype = DTYPES[dt]
    torch.manual_seed(tokens + hidden)
    mod = TinKerSwiGLU(hidden, inter)
    for lin in (mod.gate_proj, mod.up_proj, mod.down_proj):
        torch.nn.init.normal_(lin.weight, 0.0, 0.02)
    mod = mod.to("cuda", dtype)
    x = torch.randn(tokens, hidden, device="cuda", dtype=dtype)
    out = mod(x)
    # the float64 host reference runs on a row sample (<= ~384 rows) to bound host time
    idx = torch.arange(0, tokens, max(1, tokens // 384), device="cuda")
    out, x = out[idx], x[idx]
    ref = _ffn_ref(x, mod.gate_proj.weight, mod.up_proj.weight, mod.down_proj.weight)
    err = rel_err(np32(out), ref)
    eager = mod.down_proj(F.silu(mod.gate_proj(x)) * mod.up_proj(x))  # the reference's eager arithmetic
    err_eager = rel_err(np32(eager), ref)
    assert err <= (1e-3 if dtype == torch.float16 else 4e-3)
    assert err <= max(err_eager * 1.05, 2e-4)


def test_module_from_module_and_residual():
    """tests/test_swiglu.py:177-216 of the reference, plus the residual epilogue."""
    require_b200()
    from tinker_b200.modules import TinKerSwiGLU

    class _DummySwiGLU(torch.nn.Module):
        def __init__(self, h, f):
            super().__init__()
            self.gate_proj = torch.nn.Linear(h, f, bias=False)
            self.up_proj = torch.nn.Linear(h, f, bias=False)
            self.down_proj = torch.nn.Linear(f, h, bias=False)

        def forward(self, x):
            return self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))

    torch.manual_seed(0)
    src = _DummySwiGLU(512, 1376).to("cuda", torch.bfloat16)
    mod = TinKerSwiGLU.from_module(src).to(device="cuda", dtype=torch.bfloat16)
    assert (mod.hidden_size, mod.intermediate_size) == (512, 1376)
    x = torch.randn(1, 16, 512, device="cuda", dtype=torch.bfloat16)
    torch.testing.assert_close(mod(x), src(x), atol=1e-2, rtol=1e-2)
    r = torch.randn(1, 16, 512, device="cuda", dtype=torch.bfloat16)
    ref = _ffn_ref(x, src.gate_proj.weight, src.up_proj.weight, src.down_proj.weight) + np32(r).reshape(16, 512)
    assert rel_err(np32(mod(x, residual=r)).reshape(16, 512), ref) <= 4e-3
