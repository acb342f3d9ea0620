"""RoPE + GQA causal attention parity (tcgen05 kernel through the C ABI) vs the numpy oracle.

The oracle restates the reference's eager path (fused_attention.py:176-192):
RoPE in float32 rounded to the input dtype, K/V heads repeated per group,
causal softmax(q k^T / sqrt(d)) v, here computed in float64. Bar (from the
spec): norm-wise relative error <= 5e-3 per call. Cases: the reference's test
configurations (tests/test_attention.py:84-95: tiny-gqa, plasma1.0, plasma1.1,
MHA, MQA, seq 1, seq 128), the standalone sweep (batch x seq x head_dim x
head layout, fp16 and bf16), ragged sequence lengths, start_pos > 0, q/k/v as
column slices of one fused projection, and all three RoPE table dtypes.
"""

import numpy as np
import pytest
import torch

import oracle
from tests._util import DTYPES, NP_NAME, np32, rel_err, require_b200

pytestmark = pytest.mark.gpu
TOL = 5e-3


def _run(B, S, hq, hkv, d, dtype, start_pos=0, theta=1e4, table_dtype=torch.float32, seed=42, fused=False,
         check=None):
    """Kernel output and oracle output; with ``check`` (batch indices) the kernel runs on the
    whole batch and both are returned for those sequences only (sequences are independent)."""
    from tinker_b200.kernels.fused_attention import fused_attention, precompute_rope_tables
    g = torch.Generator(device="cuda").manual_seed(seed)
    if fused:
        qkv = torch.randn(B, S, (hq + 2 * hkv) * d, device="cuda", generator=g).to(dtype)
        q, k, v = qkv[..., :hq * d], qkv[..., hq * d:(hq + hkv) * d], qkv[..., (hq + hkv) * d:]
    else:
        q = torch.randn(B, S, hq * d, device="cuda", generator=g).to(dtype)
        k = torch.randn(B, S, hkv * d, device="cuda", generator=g).to(dtype)
        v = torch.randn(B, S, hkv * d, device="cuda", generator=g).to(dtype)
    cos, sin = precompute_rope_tables(d, max(S + start_pos, 256), theta, device="cuda", dtype=table_dtype)
    out = fused_attention(q, k, v, cos, sin, hq, hkv, d, start_pos=start_pos)
    if check is not None:
        out, q, k, v = out[check], q[check], k[check], v[check]
    ref = oracle.attention(np32(q), np32(k), np32(v), np32(cos), np32(sin), hq, hkv, d, start_pos,
                           io_dtype=NP_NAME[dtype])
    return out, ref


REF_CONFIGS = [
    (256, 4, 2, 64, 32, 1), (1024, 16, 4, 64, 64, 1), (1280, 20, 4, 64, 64, 1), (512, 8, 8, 64, 64, 1),
    (512, 8, 1, 64, 64, 1), (256, 4, 2, 64, 1, 1), (256, 4, 2, 64, 128, 1),
]


@pytest.mark.parametrize("hidden, hq, hkv, d, S, B", REF_CONFIGS)
def test_reference_configs_bf16(hidden, hq, hkv, d, S, B):
    require_b200()
    out, ref = _run(B, S, hq, hkv, d, torch.bfloat16)
    assert out.shape == (B, S, hq * d)
    assert rel_err(np32(out), ref) <= TOL


@pytest.mark.parametrize("dt", ["fp16", "bf16"])
@pytest.mark.parametrize("B, S", [(1, 128), (8, 512), (2, 2048)])
@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("hq, hkv", [(16, 4), (16, 16), (16, 1)])
def test_sweep(dt, B, S, d, hq, hkv):
    require_b200()
    out, ref = _run(B, S, hq, hkv, d, DTYPES[dt], seed=B * S + d + hkv)
    assert rel_err(np32(out), ref) <= TOL


# the sweep's batch-32 and long-sequence shapes (the reference benchmarks them,
# tinker/kernels/fused_attention.py:195-231 on these sizes): the kernel runs on the whole
# batch, the oracle checks the first and the last sequence
LARGE = [(32, 128, 64, 16, 4), (32, 512, 64, 16, 4), (32, 512, 128, 16, 4), (32, 512, 64, 16, 1),
         (8, 2048, 64, 16, 4), (8, 2048, 128, 16, 4), (8, 2048, 64, 16, 16), (8, 2048, 128, 16, 1),
         (32, 2048, 64, 16, 4)]


@pytest.mark.parametrize("dt", ["fp16", "bf16"])
@pytest.mark.parametrize("B, S, d, hq, hkv", LARGE)
def test_sweep_large(dt, B, S, d, hq, hkv):
    require_b200()
    out, ref = _run(B, S, hq, hkv, d, DTYPES[dt], seed=B * S + d + hkv + 1, check=[0, B - 1])
    assert rel_err(np32(out), ref) <= TOL


@pytest.mark.parametrize("S", [1, 7, 127, 129, 300])
def test_ragged_seq(S):
    require_b200()
    out, ref = _run(3, S, 8, 2, 64, torch.float16, seed=S)
    assert rel_err(np32(out), ref) <= TOL


@pytest.mark.parametrize("table_dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_start_pos_theta_and_table_dtypes(table_dtype):
    require_b200()
    out, ref = _run(2, 96, 14, 2, 64, torch.bfloat16, start_pos=37, theta=1e6, table_dtype=table_dtype)
    assert rel_err(np32(out), ref) <= TOL


@pytest.mark.parametrize("d", [64, 128])
def test_fused_qkv_views(d):
    require_b200()
    out, ref = _run(2, 200, 8, 2, d, torch.float16, fused=True)
    assert rel_err(np32(out), ref) <= TOL


def test_single_token_returns_v():
    """tests/test_numerical.py:88-119 of the reference: with S=1 the output is the GQA-expanded V."""
    require_b200()
    from tinker_b200.kernels.fused_attention import fused_attention, precompute_rope_tables
    torch.manual_seed(7)
    d, hq, hkv = 64, 4, 2
    cos, sin = precompute_rope_tables(d, 16, device="cuda")
    q = torch.randn(1, 1, hq * d, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(1, 1, hkv * d, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(1, 1, hkv * d, device="cuda", dtype=torch.bfloat16)
    out = fused_attention(q, k, v, cos, sin, hq, hkv, d)
    exp = v.view(1, 1, hkv, d).repeat_interleave(hq // hkv, dim=2).reshape(1, 1, hq * d)
    torch.testing.assert_close(out, exp, atol=1e-2, rtol=1e-2)


def test_uniform_values_return_v():
    """tests/test_numerical.py:122-156 of the reference: constant V over positions gives V."""
    require_b200()
    from tinker_b200.kernels.fused_attention import fused_attention, precompute_rope_tables
    torch.manual_seed(99)
    d, hq, hkv, S = 64, 4, 2, 16
    cos, sin = precompute_rope_tables(d, 64, device="cuda")
    q = torch.randn(1, S, hq * d, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(1, S, hkv * d, device="cuda", dtype=torch.bfloat16)
    v1 = torch.randn(1, 1, hkv * d, device="cuda", dtype=torch.bfloat16)
    v = v1.expand(1, S, -1).contiguous()
    out = fused_attention(q, k, v, cos, sin, hq, hkv, d)
    exp = v1.view(1, 1, hkv, d).repeat_interleave(hq // hkv, dim=2).reshape(1, 1, hq * d).expand(1, S, -1)
    torch.testing.assert_close(out, exp, atol=1e-2, rtol=1e-2)


def test_rejects_unsupported_and_out_of_table():
    require_b200()
    from tinker_b200 import _lib
    from tinker_b200.kernels.fused_attention import fused_attention, precompute_rope_tables
    q = torch.randn(1, 8, 4 * 32, device="cuda", dtype=torch.float16)
    kv = torch.randn(1, 8, 2 * 32, device="cuda", dtype=torch.float16)
    cos, sin = precompute_rope_tables(32, 16, device="cuda")
    with pytest.raises(_lib.TinkerKernelError, match="head_dim"):
        fused_attention(q, kv, kv, cos, sin, 4, 2, 32)
    q = torch.randn(1, 8, 4 * 64, device="cuda", dtype=torch.float16)
    kv = torch.randn(1, 8, 2 * 64, device="cuda", dtype=torch.float16)
    cos, sin = precompute_rope_tables(64, 16, device="cuda")
    with pytest.raises(_lib.TinkerKernelError, match="table"):
        fused_attention(q, kv, kv, cos, sin, 4, 2, 64, start_pos=10)


def test_module_matches_oracle():
    """TinKerAttention = q|k|v GEMM + fused attention + o_proj GEMM (tests/test_attention.py:132-166)."""
    require_b200()
    from tinker_b200.modules import TinKerAttention
    torch.manual_seed(42)
    mod = TinKerAttention(1024, 16, 4, 64, max_seq_len=256).to("cuda").to(torch.bfloat16)
    assert mod.cos_table.dtype == torch.float32
    x = torch.randn(2, 64, 1024, device="cuda", dtype=torch.bfloat16)
    out = mod(x)
    xn = np32(x)
    q = oracle.linear(xn, np32(mod.q_proj.weight), out_dtype="bfloat16")
    k = oracle.linear(xn, np32(mod.k_proj.weight), out_dtype="bfloat16")
    v = oracle.linear(xn, np32(mod.v_proj.weight), out_dtype="bfloat16")
    a = oracle.attention(q, k, v, np32(mod.cos_table), np32(mod.sin_table), 16, 4, 64, io_dtype="bfloat16")
    ref = oracle.linear(a, np32(mod.o_proj.weight), acc=np.float64)
    assert rel_err(np32(out), ref) <= 1e-2


def test_from_module():
    """tests/test_attention.py:171-204 of the reference."""
    require_b200()
    from tinker_b200.modules import TinKerAttention

    class _DummyAttention(torch.nn.Module):
        def __init__(self, hidden, hq, hkv, d):
            super().__init__()
            self.head_dim = d
            self.q_proj = torch.nn.Linear(hidden, hq * d, bias=False)
            self.k_proj = torch.nn.Linear(hidden, hkv * d, bias=False)
            self.v_proj = torch.nn.Linear(hidden, hkv * d, bias=False)
            self.o_proj = torch.nn.Linear(hq * d, hidden, bias=False)

    src = _DummyAttention(512, 8, 2, 64).to("cuda", torch.bfloat16)
    mod = TinKerAttention.from_module(src).to(device="cuda", dtype=torch.bfloat16)
    assert (mod.num_heads, mod.num_kv_heads, mod.head_dim) == (8, 2, 64)
    for n in ("q_proj", "k_proj", "v_proj", "o_proj"):
        torch.testing.assert_close(getattr(mod, n).weight.data, getattr(src, n).weight.data)


def _qkv_rope_case(B, S, hidden, hq, hkv, d, dtype, start_pos, seed):
    """x, q|k|v weights and RoPE tables for the projection-with-RoPE path."""
    from tinker_b200.kernels.fused_attention import precompute_rope_tables
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(B, S, hidden, device="cuda", generator=g).to(dtype)
    ws = [(torch.randn(n * d, hidden, device="cuda", generator=g) * hidden ** -0.5).to(dtype)
          for n in (hq, hkv, hkv)]
    cos, sin = precompute_rope_tables(d, S + start_pos + 5, 1e4, device="cuda")
    return x, ws, cos, sin


@pytest.mark.parametrize("dt", ["fp16", "bf16"])
@pytest.mark.parametrize("B, S, hidden, hq, hkv, d, start_pos",
                         [(1, 128, 1024, 16, 4, 64, 0), (2, 200, 512, 8, 2, 64, 3), (3, 77, 896, 14, 2, 64, 0),
                          (2, 160, 1024, 8, 2, 128, 11), (8, 512, 896, 14, 2, 64, 0)])
def test_linear_rope_columns(dt, B, S, hidden, hq, hkv, d, start_pos):
    """q|k|v projection with RoPE in the epilogue = linear, rounding, then the reference's RoPE
    (tinker/kernels/fused_attention.py:53-69, :203-214) on the q and k heads; v unrotated."""
    require_b200()
    from tinker_b200.kernels.gemm import linear_rope
    dtype = DTYPES[dt]
    x, ws, cos, sin = _qkv_rope_case(B, S, hidden, hq, hkv, d, dtype, start_pos, seed=S + d)
    y = linear_rope(x, *ws, cos, sin, d, start_pos)
    assert y.shape == (B, S, (hq + 2 * hkv) * d)
    xn = np32(x).reshape(B * S, hidden)
    parts = [oracle.linear(xn, np32(w), out_dtype=NP_NAME[dtype]).reshape(B, S, -1) for w in ws]
    ref = []
    for i, (part, heads) in enumerate(zip(parts, (hq, hkv, hkv))):
        if i < 2:
            bhsd = part.reshape(B, S, heads, d).transpose(0, 2, 1, 3)
            part = oracle.apply_rope(bhsd, np32(cos), np32(sin), start_pos, out_dtype=NP_NAME[dtype])
            part = part.transpose(0, 2, 1, 3).reshape(B, S, heads * d)
        ref.append(part)
    ref = np.concatenate(ref, axis=-1)
    tol = {torch.float16: 2e-3, torch.bfloat16: 8e-3}[dtype]
    assert rel_err(np32(y), ref) <= tol
    # the v columns carry no rotation
    assert rel_err(np32(y[..., (hq + hkv) * d:]), parts[2]) <= tol


@pytest.mark.parametrize("dt", ["fp16", "bf16"])
@pytest.mark.parametrize("B, S, hq, hkv, d, start_pos",
                         [(1, 128, 16, 4, 64, 0), (2, 300, 8, 2, 64, 5), (4, 512, 14, 2, 64, 0),
                          (2, 256, 8, 8, 128, 0), (1, 1, 4, 1, 64, 9), (2, 1000, 16, 4, 128, 0)])
def test_rotated_projection_then_causal_attention(dt, B, S, hq, hkv, d, start_pos):
    """linear_rope + causal_attention (the module path) = q|k|v projection + fused_attention of
    the oracle, on the same inputs."""
    require_b200()
    from tinker_b200.kernels.fused_attention import causal_attention
    from tinker_b200.kernels.gemm import linear_rope
    dtype = DTYPES[dt]
    hidden = 512
    x, ws, cos, sin = _qkv_rope_case(B, S, hidden, hq, hkv, d, dtype, start_pos, seed=7 * S + hq)
    qkv = linear_rope(x, *ws, cos, sin, d, start_pos)
    hqd, hkvd = hq * d, hkv * d
    out = causal_attention(qkv[..., :hqd], qkv[..., hqd:hqd + hkvd], qkv[..., hqd + hkvd:], hq, hkv, d)
    xn = np32(x).reshape(B * S, hidden)
    q, k, v = (oracle.linear(xn, np32(w), out_dtype=NP_NAME[dtype]).reshape(B, S, -1) for w in ws)
    ref = oracle.attention(q, k, v, np32(cos), np32(sin), hq, hkv, d, start_pos, io_dtype=NP_NAME[dtype])
    assert out.shape == (B, S, hqd)
    assert rel_err(np32(out), ref) <= TOL


def test_causal_attention_equals_rope_attention_on_rotated_inputs():
    """The no-RoPE kernel on q, k rotated by the RoPE kernel's own arithmetic gives the same
    result as the RoPE kernel on the raw inputs (one kernel, two entry points)."""
    require_b200()
    from tinker_b200.kernels.fused_attention import causal_attention, fused_attention, precompute_rope_tables
    B, S, hq, hkv, d = 2, 384, 8, 2, 64
    g = torch.Generator(device="cuda").manual_seed(3)
    q = torch.randn(B, S, hq * d, device="cuda", generator=g).to(torch.float16)
    k = torch.randn(B, S, hkv * d, device="cuda", generator=g).to(torch.float16)
    v = torch.randn(B, S, hkv * d, device="cuda", generator=g).to(torch.float16)
    cos, sin = precompute_rope_tables(d, S, device="cuda")

    def rot(t, heads):
        x = t.float().view(B, S, heads, d // 2, 2)
        c, s = cos[:S].view(1, S, 1, d // 2), sin[:S].view(1, S, 1, d // 2)
        e, o = x[..., 0], x[..., 1]
        return torch.stack([e * c - o * s, e * s + o * c], -1).reshape(B, S, heads * d).to(t.dtype)

    a = fused_attention(q, k, v, cos, sin, hq, hkv, d)
    b = causal_attention(rot(q, hq), rot(k, hkv), v, hq, hkv, d)
    torch.testing.assert_close(a, b, atol=2e-3, rtol=2e-3)


def test_linear_rope_rejects_bad_arguments():
    require_b200()
    from tinker_b200 import _lib
    from tinker_b200.kernels.gemm import linear_rope
    from tinker_b200.kernels.fused_attention import precompute_rope_tables
    x = torch.randn(1, 8, 256, device="cuda", dtype=torch.float16)
    w = torch.randn(128, 256, device="cuda", dtype=torch.float16)
    cos, sin = precompute_rope_tables(64, 8, device="cuda")
    with pytest.raises(_lib.TinkerKernelError, match="table"):
        linear_rope(x, w, w, w, cos, sin, 64, start_pos=1)
    with pytest.raises(TypeError, match="float32"):
        linear_rope(x, w, w, w, cos.half(), sin.half(), 64)


def _rope_attention_direct(q, k, v, cos, sin, hq, hkv, d, start_pos=0):
    """tk_rope_attention itself (RoPE on load), whatever fused_attention picks for this length."""
    from tinker_b200 import _lib
    B, S, _ = q.shape
    out = torch.empty(B, S, hq * d, dtype=q.dtype, device=q.device)
    _lib.check(_lib.lib().tk_rope_attention(
        q.data_ptr(), q.stride(1), k.data_ptr(), k.stride(1), v.data_ptr(), v.stride(1), cos.data_ptr(),
        sin.data_ptr(), _lib.dtype_code(cos.dtype), cos.shape[0], out.data_ptr(), hq * d, B, S, hq, hkv, d,
        start_pos, _lib.dtype_code(q.dtype), _lib.stream_ptr(q.device)), "tk_rope_attention", 1)
    return out


@pytest.mark.parametrize("dt", ["fp16", "bf16"])
@pytest.mark.parametrize("B, S, hq, hkv, d, start_pos", [(2, 1000, 16, 4, 64, 3), (1, 2048, 8, 8, 128, 0),
                                                          (3, 384, 14, 2, 64, 0)])
def test_rope_on_load_kernel_long_sequences(dt, B, S, hq, hkv, d, start_pos):
    """The RoPE-on-load kernel at lengths where fused_attention uses the separate RoPE pass."""
    require_b200()
    from tinker_b200.kernels.fused_attention import precompute_rope_tables
    dtype = DTYPES[dt]
    g = torch.Generator(device="cuda").manual_seed(S + d)
    q = torch.randn(B, S, hq * d, device="cuda", generator=g).to(dtype)
    k = torch.randn(B, S, hkv * d, device="cuda", generator=g).to(dtype)
    v = torch.randn(B, S, hkv * d, device="cuda", generator=g).to(dtype)
    cos, sin = precompute_rope_tables(d, S + start_pos, device="cuda")
    out = _rope_attention_direct(q, k, v, cos, sin, hq, hkv, d, start_pos)
    ref = oracle.attention(np32(q), np32(k), np32(v), np32(cos), np32(sin), hq, hkv, d, start_pos,
                           io_dtype=NP_NAME[dtype])
    assert rel_err(np32(out), ref) <= TOL


@pytest.mark.parametrize("table_dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("dt", ["fp16", "bf16"])
def test_rope_qk_pass_matches_oracle_rope(dt, table_dtype):
    """tk_rope_qk = the reference's RoPE (fused_attention.py:165-173 arithmetic) on q and k heads."""
    require_b200()
    from tinker_b200 import _lib
    from tinker_b200.kernels.fused_attention import precompute_rope_tables
    dtype = DTYPES[dt]
    B, S, hq, hkv, d, start = 2, 300, 8, 2, 64, 7
    g = torch.Generator(device="cuda").manual_seed(11)
    qkv = torch.randn(B, S, (hq + 2 * hkv) * d, device="cuda", generator=g).to(dtype)
    q, k = qkv[..., :hq * d], qkv[..., hq * d:(hq + hkv) * d]
    cos, sin = precompute_rope_tables(d, S + start, device="cuda", dtype=table_dtype)
    out = torch.empty(B, S, (hq + hkv) * d, dtype=dtype, device="cuda")
    _lib.check(_lib.lib().tk_rope_qk(q.data_ptr(), qkv.stride(1), k.data_ptr(), qkv.stride(1), cos.data_ptr(),
                                     sin.data_ptr(), _lib.dtype_code(table_dtype), cos.shape[0], out.data_ptr(),
                                     (hq + hkv) * d, B, S, hq, hkv, d, start, _lib.dtype_code(dtype),
                                     _lib.stream_ptr(qkv.device)), "tk_rope_qk", 1)
    for heads, src, lo in ((hq, q, 0), (hkv, k, hq * d)):
        x = np32(src).reshape(B, S, heads, d).transpose(0, 2, 1, 3)
        ref = oracle.apply_rope(x, np32(cos), np32(sin), start, out_dtype=NP_NAME[dtype])
        got = np32(out[..., lo:lo + heads * d]).reshape(B, S, heads, d).transpose(0, 2, 1, 3)
        # same fp32 arithmetic, one rounding: equal up to one ulp where an FMA contraction differs
        np.testing.assert_allclose(got, ref, rtol=2.0 ** -7 if dtype == torch.bfloat16 else 2.0 ** -10, atol=1e-6)


@pytest.mark.parametrize("entry", ["causal", "rope"])
@pytest.mark.parametrize("d", [64, 128])
def test_repeated_calls_are_bitwise_identical(entry, d):
    """Every tile waits for the operands it reads: repeated calls on the same inputs give the same
    bits (a tile computed from smem that TMA had not yet filled shows up as run-to-run noise)."""
    require_b200()
    from tinker_b200.kernels.fused_attention import causal_attention, precompute_rope_tables
    B, S, hq, hkv = 4, 1024, 16, 4
    g = torch.Generator(device="cuda").manual_seed(d)
    q = torch.randn(B, S, hq * d, device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn(B, S, hkv * d, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(B, S, hkv * d, device="cuda", generator=g).to(torch.bfloat16)
    cos, sin = precompute_rope_tables(d, S, device="cuda")
    if entry == "causal":
        outs = [causal_attention(q, k, v, hq, hkv, d) for _ in range(8)]
    else:
        outs = [_rope_attention_direct(q, k, v, cos, sin, hq, hkv, d) for _ in range(8)]
    torch.cuda.synchronize()
    assert all(torch.equal(outs[0], o) for o in outs[1:])
