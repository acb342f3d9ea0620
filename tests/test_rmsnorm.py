"""RMSNorm parity: CUDA kernel (through the C ABI) vs the numpy oracle.

Cases: the reference's own test shapes (tests/test_rmsnorm.py:21-28 of
eb1386/TinKer), the kernel sweep rows {128, 4096, 65536} x hidden {1024, 2048, 4096}
in fp16 and bf16, fp32, odd and unaligned dims, strided rows and the fused
residual variant. Bar: the kernel output equals the oracle's (float32 math,
one rounding) to within one ulp of the output dtype everywhere, and the
norm-wise relative error against the float32 result is <= 1e-3.
"""

import numpy as np
import pytest
import torch

import oracle
from tests._util import DTYPES, NP_NAME, np32, rel_err, require_b200, ulp

pytestmark = pytest.mark.gpu

REF_CONFIGS = [(256, 32, 1), (1024, 128, 1), (1280, 128, 1), (512, 64, 1), (1024, 1, 1), (1024, 64, 8)]


def _check(y, x, w, eps, dtype):
    ref = oracle.rmsnorm(np32(x), np32(w), eps, out_dtype=NP_NAME[dtype])
    exact = oracle.rmsnorm(np32(x), np32(w), eps)
    yy = np32(y)
    np.testing.assert_allclose(yy, ref, rtol=ulp(dtype), atol=1e-6 if dtype == torch.float32 else ulp(dtype) * 1e-2)
    # <= 1e-3 relative to the float32 result; a bf16 output cannot do better than its own
    # rounding (~1.6e-3 for these values), so there the bar is correct rounding (+1%)
    assert rel_err(yy, exact) <= max(1e-3, 1.01 * rel_err(ref, exact))


@pytest.mark.parametrize("dim, seq, batch", REF_CONFIGS)
def test_reference_shapes_bf16(dim, seq, batch):
    require_b200()
    from tinker_b200.kernels.fused_rmsnorm import fused_rmsnorm
    torch.manual_seed(42)
    x = torch.randn(batch, seq, dim, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(dim, device="cuda", dtype=torch.bfloat16)
    _check(fused_rmsnorm(x, w), x, w, 1e-6, torch.bfloat16)


@pytest.mark.parametrize("dt", ["fp16", "bf16"])
@pytest.mark.parametrize("rows", [128, 4096, 65536])
@pytest.mark.parametrize("hidden", [1024, 2048, 4096])
def test_sweep(dt, rows, hidden):
    require_b200()
    from tinker_b200.kernels import fused_rmsnorm
    g = torch.Generator(device="cuda").manual_seed(rows + hidden)
    dtype = DTYPES[dt]
    x = torch.randn(rows, hidden, device="cuda", generator=g).to(dtype)
    w = (1 + 0.1 * torch.randn(hidden, device="cuda", generator=g)).to(dtype)
    _check(fused_rmsnorm(x, w, 1e-6), x, w, 1e-6, dtype)


@pytest.mark.parametrize("dim", [1000, 8192, 20000, 7])
@pytest.mark.parametrize("dt", ["fp16", "fp32"])
def test_odd_and_wide_dims(dim, dt):
    require_b200()
    from tinker_b200.kernels import fused_rmsnorm
    torch.manual_seed(dim)
    dtype = DTYPES[dt]
    x = torch.randn(33, dim, device="cuda").to(dtype)
    w = torch.randn(dim, device="cuda").to(dtype)
    _check(fused_rmsnorm(x, w, 1e-5), x, w, 1e-5, dtype)


def test_strided_rows_and_fp32_weight():
    require_b200()
    from tinker_b200.kernels import fused_rmsnorm
    torch.manual_seed(3)
    big = torch.randn(64, 3072, device="cuda", dtype=torch.float16)
    x = big[:, 1024:2048]  # row stride 3072
    w = torch.randn(1024, device="cuda", dtype=torch.float32)
    y = fused_rmsnorm(x, w)
    ref = oracle.rmsnorm(np32(x), np32(w), 1e-6, out_dtype="float16")
    np.testing.assert_allclose(np32(y), ref, rtol=ulp(torch.float16), atol=1e-5)


@pytest.mark.parametrize("dt", ["fp16", "bf16"])
def test_add_rmsnorm(dt):
    require_b200()
    from tinker_b200.kernels import fused_add_rmsnorm
    torch.manual_seed(5)
    dtype = DTYPES[dt]
    x = torch.randn(257, 1024, device="cuda").to(dtype)
    r = torch.randn(257, 1024, device="cuda").to(dtype)
    w = (1 + 0.1 * torch.randn(1024, device="cuda")).to(dtype)
    y, s = fused_add_rmsnorm(x, r, w, 1e-6)
    y_ref, s_ref = oracle.add_rmsnorm(np32(x), np32(r), np32(w), 1e-6, out_dtype=NP_NAME[dtype])
    np.testing.assert_array_equal(np32(s), s_ref)
    np.testing.assert_allclose(np32(y), y_ref, rtol=ulp(dtype), atol=ulp(dtype) * 1e-2)


def test_module_and_from_module():
    """tests/test_rmsnorm.py:51-101 of the reference: module output and eps propagation."""
    require_b200()
    from tinker_b200.modules import TinKerRMSNorm

    class _DummyRMSNorm(torch.nn.Module):
        def __init__(self, dim, eps=1e-6):
            super().__init__()
            self.eps = eps
            self.weight = torch.nn.Parameter(torch.ones(dim))

    torch.manual_seed(0)
    src = _DummyRMSNorm(512, eps=1e-5).to("cuda", torch.bfloat16)
    torch.nn.init.normal_(src.weight)
    mod = TinKerRMSNorm.from_module(src).to(device="cuda", dtype=torch.bfloat16)
    assert mod.eps == src.eps
    torch.testing.assert_close(mod.weight.data, src.weight.data)
    x = torch.randn(1, 32, 512, device="cuda", dtype=torch.bfloat16)
    _check(mod(x), x, src.weight, 1e-5, torch.bfloat16)


def test_rows_zero_is_a_no_op():
    require_b200()
    from tinker_b200.kernels import fused_rmsnorm
    x = torch.empty(0, 1024, device="cuda", dtype=torch.float16)
    w = torch.ones(1024, device="cuda", dtype=torch.float16)
    assert fused_rmsnorm(x, w).shape == (0, 1024)
