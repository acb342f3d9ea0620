"""GEMM parity (through the C ABI) against float64 numpy: the tcgen05 kernels, and the
weight-streaming kernel the same entry points use for at most 8 rows.

y = x . w^T with fp32 accumulation and one rounding: the result must match the
exactly computed product of the same half-precision inputs to within the
output dtype's rounding (norm-wise relative error <= 1e-3 for fp16 and
<= 4e-3 for bf16, whose unit roundoff is 2^-9), and every element to within a
few ulps plus accumulation noise.
"""

import numpy as np
import pytest
import torch

from tests._util import DTYPES, np32, rel_err, require_b200

pytestmark = pytest.mark.gpu

TOL = {torch.float16: 1e-3, torch.bfloat16: 4e-3}


def _ref(x, ws, residual=None):
    w = np.concatenate([np32(t).astype(np.float64) for t in ws], axis=0)
    y = np32(x).astype(np.float64).reshape(-1, w.shape[1]) @ w.T
    if residual is not None:
        y = y + np32(residual).astype(np.float64).reshape(y.shape)
    return y


SHAPES = [
    (128, 1536, 1024),   # 268M q|k|v at batch 1 x seq 128
    (128, 1024, 1024),   # o_proj
    (128, 1024, 2816),   # down_proj
    (1, 256, 64),        # single row
    (200, 96, 40),       # ragged m, n tail, k tail (k < one k-block)
    (4096, 896, 896),    # large m (Qwen-shaped o_proj, 8 sequences of 512)
    (1000, 4864, 896),   # many tiles, ragged m
    (384, 2048, 5632),   # 1B down_proj, deep k
    (3, 1536, 1024),     # decode rows: the weight-streaming path (m <= 8)
    (8, 1024, 2816),
    (5, 96, 40),
]


@pytest.mark.parametrize("dt", ["fp16", "bf16"])
@pytest.mark.parametrize("m, n, k", SHAPES)
def test_linear(dt, m, n, k):
    require_b200()
    from tinker_b200.kernels import linear
    dtype = DTYPES[dt]
    g = torch.Generator(device="cuda").manual_seed(m * 7 + n + k)
    x = torch.randn(m, k, device="cuda", generator=g).to(dtype)
    w = (0.02 * torch.randn(n, k, device="cuda", generator=g)).to(dtype)
    y = linear(x, w)
    assert y.shape == (m, n) and y.dtype == dtype
    ref = _ref(x, [w])
    assert rel_err(np32(y), ref) <= TOL[dtype]
    np.testing.assert_allclose(np32(y), ref, rtol=4 * TOL[dtype], atol=4 * TOL[dtype] * np.abs(ref).max())


@pytest.mark.parametrize("dt", ["fp16", "bf16"])
@pytest.mark.parametrize("hq, hkv", [(1024, 256), (896, 128), (512, 512), (512, 64)])
@pytest.mark.parametrize("m", [2, 8, 128, 1030])
def test_linear_three_weight_blocks(dt, hq, hkv, m):
    """q|k|v projection as one GEMM over three separate weights."""
    require_b200()
    from tinker_b200.kernels import linear
    dtype = DTYPES[dt]
    torch.manual_seed(hq + hkv + m)
    k = 1024
    x = torch.randn(m, k, device="cuda").to(dtype)
    wq = (0.02 * torch.randn(hq, k, device="cuda")).to(dtype)
    wk = (0.02 * torch.randn(hkv, k, device="cuda")).to(dtype)
    wv = (0.02 * torch.randn(hkv, k, device="cuda")).to(dtype)
    y = linear(x, wq, wk, wv)
    assert y.shape == (m, hq + 2 * hkv)
    assert rel_err(np32(y), _ref(x, [wq, wk, wv])) <= TOL[dtype]


@pytest.mark.parametrize("dt", ["fp16", "bf16"])
@pytest.mark.parametrize("m", [300, 4])
def test_linear_residual_epilogue(dt, m):
    require_b200()
    from tinker_b200.kernels import linear
    dtype = DTYPES[dt]
    torch.manual_seed(1)
    x = torch.randn(m, 2816, device="cuda").to(dtype)
    w = (0.02 * torch.randn(1024, 2816, device="cuda")).to(dtype)
    r = torch.randn(m, 1024, device="cuda").to(dtype)
    y = linear(x, w, residual=r)
    assert rel_err(np32(y), _ref(x, [w], r)) <= TOL[dtype]


@pytest.mark.parametrize("dt", ["fp16", "bf16"])
@pytest.mark.parametrize("m, hidden, f", [(128, 1024, 2816), (4096, 2048, 5632), (77, 896, 4864), (1, 512, 1376),
                                          (8, 1024, 2816), (3, 896, 4864),
                                          (640, 256, 40)])
def test_gate_up_swiglu(dt, m, hidden, f):
    require_b200()
    from tinker_b200.kernels import gate_up_swiglu
    dtype = DTYPES[dt]
    g = torch.Generator(device="cuda").manual_seed(m + hidden + f)
    x = torch.randn(m, hidden, device="cuda", generator=g).to(dtype)
    wg = (0.02 * torch.randn(f, hidden, device="cuda", generator=g)).to(dtype)
    wu = (0.02 * torch.randn(f, hidden, device="cuda", generator=g)).to(dtype)
    h = gate_up_swiglu(x, wg, wu)
    a = _ref(x, [wg])
    b = _ref(x, [wu])
    ref = a / (1 + np.exp(-a)) * b
    assert h.shape == (m, f)
    assert rel_err(np32(h), ref) <= TOL[dtype]


def test_linear_rejects_bad_arguments():
    require_b200()
    from tinker_b200 import _lib
    from tinker_b200.kernels import linear
    x = torch.randn(4, 12, device="cuda", dtype=torch.float16)  # k = 12 is not a multiple of 8
    w = torch.randn(32, 12, device="cuda", dtype=torch.float16)
    with pytest.raises(_lib.TinkerKernelError, match="multiples of 8"):
        linear(x, w)
    with pytest.raises(TypeError):
        linear(x.float(), w.float())


@pytest.mark.parametrize("dt", ["fp16", "bf16"])
@pytest.mark.parametrize("hq, hkv", [(896, 128), (1024, 256)])
def test_pair_tiles_three_weight_blocks(dt, hq, hkv):
    """Large M runs 256-row tiles on CTA pairs (tcgen05 cta_group::2)."""
    require_b200()
    from tinker_b200.kernels import linear
    dtype = DTYPES[dt]
    torch.manual_seed(hq + hkv)
    m, k = 4096, 896
    x = torch.randn(m, k, device="cuda").to(dtype)
    wq = (0.02 * torch.randn(hq, k, device="cuda")).to(dtype)
    wk = (0.02 * torch.randn(hkv, k, device="cuda")).to(dtype)
    wv = (0.02 * torch.randn(hkv, k, device="cuda")).to(dtype)
    y = linear(x, wq, wk, wv)
    idx = torch.arange(0, m, 5, device="cuda")  # float64 host reference on a row sample
    assert rel_err(np32(y[idx]), _ref(x[idx], [wq, wk, wv])) <= TOL[dtype]


@pytest.mark.parametrize("dt", ["fp16", "bf16"])
def test_pair_tiles_residual_and_ragged_m(dt):
    require_b200()
    from tinker_b200.kernels import linear
    dtype = DTYPES[dt]
    torch.manual_seed(3)
    m, n, k = 8000, 1024, 2816  # 8000 rows: the last 256-row tile is partial
    x = torch.randn(m, k, device="cuda").to(dtype)
    w = (0.02 * torch.randn(n, k, device="cuda")).to(dtype)
    r = torch.randn(m, n, device="cuda").to(dtype)
    y = linear(x, w, residual=r)
    idx = torch.cat([torch.arange(0, m, 37, device="cuda"), torch.arange(m - 70, m, device="cuda")])
    assert rel_err(np32(y[idx]), _ref(x[idx], [w], r[idx])) <= TOL[dtype]


@pytest.mark.parametrize("dt", ["fp16", "bf16"])
def test_pair_tiles_swiglu(dt):
    require_b200()
    from tinker_b200.kernels import gate_up_swiglu
    dtype = DTYPES[dt]
    torch.manual_seed(4)
    m, hidden, f = 4608, 896, 4864
    x = torch.randn(m, hidden, device="cuda").to(dtype)
    wg = (0.02 * torch.randn(f, hidden, device="cuda")).to(dtype)
    wu = (0.02 * torch.randn(f, hidden, device="cuda")).to(dtype)
    h = gate_up_swiglu(x, wg, wu)
    idx = torch.arange(0, m, 11, device="cuda")
    a, b = _ref(x[idx], [wg]), _ref(x[idx], [wu])
    assert rel_err(np32(h[idx]), a / (1 + np.exp(-a)) * b) <= TOL[dtype]


# ---- RMSNorm folded into the GEMM (row_ssq_in) and row statistics out (row_ssq_out) ----

def _rms_ref(x, w_norm, eps):
    """The reference's RMSNorm in float64 on the half input, rounded like its kernel's output."""
    xf = np32(x).astype(np.float64)
    y = xf / np.sqrt((xf ** 2).mean(-1, keepdims=True) + eps) * np32(w_norm).astype(np.float64)
    return y


@pytest.mark.parametrize("dt", ["fp16", "bf16"])
@pytest.mark.parametrize("m, n, k", [(128, 1024, 1024), (128, 5632, 1024), (300, 896, 896), (4096, 1152, 896),
                                     (1, 1024, 1024), (8, 1536, 1024)])
def test_row_sumsq_and_folded_norm_linear(dt, m, n, k):
    """row_sumsq gives the per-32-column sums of squares; linear with row_ssq_in and the norm weight
    folded into w equals rmsnorm(x) @ w.T (tinker/modules/normalization.py:29-31 then nn.Linear)."""
    require_b200()
    from tinker_b200.kernels import linear, row_sumsq
    dtype = DTYPES[dt]
    g = torch.Generator(device="cuda").manual_seed(m + n + k)
    x = torch.randn(m, k, device="cuda", generator=g).to(dtype)
    wn = (1 + 0.1 * torch.randn(k, device="cuda", generator=g)).to(dtype)
    w = (0.02 * torch.randn(n, k, device="cuda", generator=g)).to(dtype)
    parts = row_sumsq(x)
    assert parts.shape == (k // 32, m)
    exp = (np32(x).astype(np.float64).reshape(m, k // 32, 32) ** 2).sum(-1).T
    np.testing.assert_allclose(np32(parts), exp, rtol=1e-5, atol=1e-5)
    wf = (w.float() * wn.float()[None, :]).to(dtype)
    y = linear(x, wf, row_ssq_in=parts, row_ssq_eps=1e-6)
    ref = _rms_ref(x, wn, 1e-6) @ np32(w).astype(np.float64).T
    assert rel_err(np32(y), ref) <= 2 * TOL[dtype]


@pytest.mark.parametrize("dt", ["fp16", "bf16"])
@pytest.mark.parametrize("m, n, k", [(128, 1024, 1024), (128, 1024, 2816), (1000, 896, 4864), (130, 96, 64),
                                     (1, 1024, 1024), (4, 1024, 2816), (7, 96, 64)])
def test_row_ssq_out_of_residual_linear(dt, m, n, k):
    """row_ssq_out holds, per 32 output columns, the sum of squares of the stored (rounded) rows."""
    require_b200()
    from tinker_b200.kernels import linear
    dtype = DTYPES[dt]
    g = torch.Generator(device="cuda").manual_seed(3 * m + n + k)
    x = torch.randn(m, k, device="cuda", generator=g).to(dtype)
    w = (0.02 * torch.randn(n, k, device="cuda", generator=g)).to(dtype)
    r = torch.randn(m, n, device="cuda", generator=g).to(dtype)
    ssq = torch.full(((n + 31) // 32, m), float("nan"), device="cuda")
    y = linear(x, w, residual=r, row_ssq_out=ssq)
    assert rel_err(np32(y), _ref(x, [w], r)) <= TOL[dtype]
    yf = np32(y).astype(np.float64)
    pad = (-n) % 32
    exp = (np.pad(yf, ((0, 0), (0, pad))).reshape(m, -1, 32) ** 2).sum(-1).T
    np.testing.assert_allclose(np32(ssq), exp, rtol=1e-5, atol=1e-4)


@pytest.mark.parametrize("dt", ["fp16", "bf16"])
@pytest.mark.parametrize("m, hidden, f", [(128, 1024, 2816), (4096, 896, 4864), (256, 512, 1376), (1, 1024, 2816),
                                          (6, 896, 4864)])
def test_folded_norm_gate_up_swiglu(dt, m, hidden, f):
    require_b200()
    from tinker_b200.kernels import gate_up_swiglu, row_sumsq
    dtype = DTYPES[dt]
    g = torch.Generator(device="cuda").manual_seed(m + f)
    x = torch.randn(m, hidden, device="cuda", generator=g).to(dtype)
    wn = (1 + 0.1 * torch.randn(hidden, device="cuda", generator=g)).to(dtype)
    wg = (0.03 * torch.randn(f, hidden, device="cuda", generator=g)).to(dtype)
    wu = (0.03 * torch.randn(f, hidden, device="cuda", generator=g)).to(dtype)
    fold = lambda w: (w.float() * wn.float()[None, :]).to(dtype)
    h = gate_up_swiglu(x, fold(wg), fold(wu), row_ssq_in=row_sumsq(x), row_ssq_eps=1e-5)
    xn = _rms_ref(x, wn, 1e-5)
    a = xn @ np32(wg).astype(np.float64).T
    b = xn @ np32(wu).astype(np.float64).T
    assert rel_err(np32(h), a / (1 + np.exp(-a)) * b) <= 2 * TOL[dtype]


def test_folded_norm_arguments_rejected():
    require_b200()
    from tinker_b200 import _lib
    from tinker_b200.kernels import gate_up_swiglu, linear
    x = torch.randn(128, 256, device="cuda", dtype=torch.float16)
    w = torch.randn(64, 256, device="cuda", dtype=torch.float16)
    with pytest.raises(ValueError, match="row_ssq_in"):
        linear(x, w, row_ssq_in=torch.zeros(8, 100, device="cuda"))
    with pytest.raises(ValueError, match="row_ssq_out"):
        linear(x, w, row_ssq_out=torch.zeros(3, 128, device="cuda"))
    # the SwiGLU epilogue stores h, not the rows a next RMSNorm would read
    e = _lib.Epilogue()
    e.row_ssq_out = torch.zeros(4, 128, device="cuda").data_ptr()
    h = torch.empty(128, 64, device="cuda", dtype=torch.float16)
    rc = _lib.lib().tk_gate_up_swiglu_ex(x.data_ptr(), 256, w.data_ptr(), w.data_ptr(), h.data_ptr(), 128, 256, 64, e,
                                         0, _lib.stream_ptr(x.device))
    assert rc == _lib.TK_ERR_INVALID


@pytest.mark.parametrize("m, n, k", [(128, 1024, 1024), (128, 1024, 2816), (300, 896, 896), (4, 1024, 1024)])
def test_l2_prefetch_hints_change_no_result(m, n, k):
    """tk_epilogue.l2_prefetch only pulls ranges into L2: the products with hints (aligned and
    unaligned ranges, more ranges than slots, an empty tensor, the output itself) are bitwise those
    without, for the split-K, plain and weight-streaming kernels."""
    require_b200()
    from tinker_b200.kernels.gemm import gate_up_swiglu, linear
    g = torch.Generator(device="cuda").manual_seed(m + n)
    x = torch.randn(m, k, device="cuda", generator=g).half()
    w = (torch.randn(n, k, device="cuda", generator=g) / k ** 0.5).half()
    r = torch.randn(m, n, device="cuda", generator=g).half()
    other = torch.randn(3 << 20, device="cuda", generator=g).half()
    hints = (other[1:], w, other[5:1000], torch.empty(0, device="cuda"), r, x, other, w[:, 3:].contiguous(), x[1:])
    y0 = linear(x, w, residual=r)
    y1 = linear(x, w, residual=r, l2_prefetch=hints)
    h0 = gate_up_swiglu(x, w, w)
    h1 = gate_up_swiglu(x, w, w, l2_prefetch=hints[:3])
    torch.cuda.synchronize()
    assert torch.equal(y0, y1)
    assert torch.equal(h0, h1)
    assert rel_err(np32(y1), _ref(x, [w], r)) <= TOL[torch.float16]
