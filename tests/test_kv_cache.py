"""KV-cache attention and cached decoding vs the numpy oracle.

The reference has no KV cache (README.md:102): a new token's output is a row of
the causal RoPE attention over the whole sequence (fused_attention.py:176-192).
``oracle.attention_rows`` computes exactly those rows (pinned here to
``oracle.attention``, itself pinned to the reference's golden vectors); the
kernel (``kv_attention``: RoPE of the new rows, cache append, split-K attention
over the cache) must match it within the attention bar of 5e-3 norm-wise. The
cache contents must be the oracle's rotated keys (to one rounding) and the
values bit for bit. Model level: prefill + per-step decode logits of a patched
decoder equal the full forward over the same tokens (our own forward, and the
fp32 oracle for the last positions).
"""

import numpy as np
import pytest
import torch

import oracle
from tests._util import DTYPES, NP_NAME, np32, rel_err, require_b200

TOL = 5e-3


def test_oracle_rows_equal_full_attention():
    rng = np.random.default_rng(0)
    B, L, hq, hkv, d, start = 2, 37, 8, 2, 64, 29
    q = rng.standard_normal((B, L, hq * d)).astype(np.float32)
    k = rng.standard_normal((B, L, hkv * d)).astype(np.float32)
    v = rng.standard_normal((B, L, hkv * d)).astype(np.float32)
    cos, sin = oracle.rope_tables(d, 64)
    full = oracle.attention(q, k, v, cos, sin, hq, hkv, d)
    rows = oracle.attention_rows(q[:, start:], k, v, cos, sin, hq, hkv, d, start)
    np.testing.assert_allclose(rows, full[:, start:], rtol=1e-6, atol=1e-6)


def test_wrappers_refuse_cpu_tensors():
    from tinker_b200.kernels.kv_cache import kv_append, kv_attention
    q = torch.zeros(1, 1, 4 * 64, dtype=torch.float16)
    kv = torch.zeros(1, 1, 2 * 64, dtype=torch.float16)
    cache = torch.zeros(1, 2, 8, 64, dtype=torch.float16)
    cos = torch.zeros(8, 32)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        kv_attention(q, kv, kv, cos, cos, cache, cache, 4, 2, 64, start_pos=3)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        kv_append(kv, kv, cache, cache, 0)


# ---------------------------------------------------------------------------- GPU


def _case(B, hq, hkv, d, start, S, cap, dtype, seed):
    """Unrotated q (new rows) and k/v for all positions, the cache filled with the oracle's
    rotated keys and the values of positions < start, and the oracle's rows."""
    from tinker_b200.kernels.fused_attention import precompute_rope_tables
    g = torch.Generator(device="cuda").manual_seed(seed)
    L = start + S
    q = torch.randn(B, S, hq * d, device="cuda", generator=g).to(dtype)
    k = torch.randn(B, L, hkv * d, device="cuda", generator=g).to(dtype)
    v = torch.randn(B, L, hkv * d, device="cuda", generator=g).to(dtype)
    cos, sin = precompute_rope_tables(d, cap + 3, 1e4, device="cuda")
    kh = np32(k).reshape(B, L, hkv, d).transpose(0, 2, 1, 3)
    k_rot = oracle.apply_rope(kh, np32(cos), np32(sin), 0, out_dtype=NP_NAME[dtype])  # [B, hkv, L, d]
    k_cache = torch.zeros(B, hkv, cap, d, dtype=dtype, device="cuda")
    v_cache = torch.zeros_like(k_cache)
    k_cache[:, :, :start] = torch.from_numpy(np.ascontiguousarray(k_rot[:, :, :start])).to("cuda", dtype)
    v_cache[:, :, :start] = v[:, :start].reshape(B, start, hkv, d).transpose(1, 2)
    ref = oracle.attention_rows(np32(q), np32(k), np32(v), np32(cos), np32(sin), hq, hkv, d, start,
                                io_dtype=NP_NAME[dtype])
    return q, k[:, start:].contiguous(), v[:, start:].contiguous(), cos, sin, k_cache, v_cache, k_rot, v, ref


CASES = [  # dt, B, hq, hkv, d, start, S, cap
    ("fp16", 1, 16, 4, 64, 127, 1, 2048),    # 268M decode step after a 127-token prompt
    ("bf16", 2, 14, 2, 64, 300, 1, 512),     # Qwen-shaped heads
    ("fp16", 3, 8, 2, 128, 1000, 3, 1100),   # head_dim 128, a 3-token chunk
    ("bf16", 1, 32, 8, 64, 0, 1, 64),        # the first token (nothing cached)
    ("fp16", 2, 16, 4, 64, 50, 16, 128),     # 64 query rows per kv head: 4 row blocks
    ("bf16", 1, 16, 16, 128, 33, 5, 64),     # MHA
    ("fp16", 1, 16, 1, 64, 2047, 1, 2048),   # MQA, the last slot of the cache
    ("fp16", 4, 14, 2, 64, 4095, 1, 4096),   # long context
    ("bf16", 2, 8, 2, 64, 10, 40, 64),       # a 40-token chunk: 160 rows per kv head
]


@pytest.mark.gpu
@pytest.mark.parametrize("dt, B, hq, hkv, d, start, S, cap", CASES)
def test_kv_attention_matches_oracle_and_appends(dt, B, hq, hkv, d, start, S, cap):
    require_b200()
    from tinker_b200.kernels.kv_cache import kv_attention
    dtype = DTYPES[dt]
    q, kn, vn, cos, sin, kc, vc, k_rot, v_all, ref = _case(B, hq, hkv, d, start, S, cap, dtype, seed=start + S)
    before = kc.clone(), vc.clone()
    out = kv_attention(q, kn, vn, cos, sin, kc, vc, hq, hkv, d, start_pos=start)
    assert out.shape == (B, S, hq * d)
    assert rel_err(np32(out), ref) <= TOL
    L = start + S
    # the new rows: keys rotated (one rounding of the same fp32 rotation), values copied
    got_k = np32(kc[:, :, start:L])
    want_k = k_rot[:, :, start:L]
    assert np.max(np.abs(got_k - want_k)) <= 2 * float(np.max(np.abs(want_k))) * 2.0 ** -8
    assert torch.equal(vc[:, :, start:L], v_all[:, start:L].reshape(B, S, hkv, d).transpose(1, 2))
    # nothing else changed
    assert torch.equal(kc[:, :, :start], before[0][:, :, :start]) and torch.equal(kc[:, :, L:], before[0][:, :, L:])
    assert torch.equal(vc[:, :, :start], before[1][:, :, :start]) and torch.equal(vc[:, :, L:], before[1][:, :, L:])


@pytest.mark.gpu
@pytest.mark.parametrize("S", [1, 4])
def test_device_position_and_repeat(S):
    """The position read from device memory gives the oracle's rows; calling again with the same
    inputs (the workspace counters were returned to zero) gives bit-identical results."""
    require_b200()
    from tinker_b200 import _lib
    from tinker_b200.kernels.kv_cache import kv_attention, kv_attention_workspace
    B, hq, hkv, d, start, cap = 2, 16, 4, 64, 200, 1024
    q, kn, vn, cos, sin, kc, vc, _, _, ref = _case(B, hq, hkv, d, start, S, cap, torch.float16, seed=5)
    pos = torch.tensor([start], dtype=torch.int32, device="cuda")
    ws = torch.zeros(kv_attention_workspace(B, hq, hkv, d, S, cap), dtype=torch.uint8, device="cuda")
    assert ws.numel() > 0
    _lib.device_error(clear=True)
    out1 = kv_attention(q, kn, vn, cos, sin, kc, vc, hq, hkv, d, position=pos, workspace=ws)
    out2 = kv_attention(q, kn, vn, cos, sin, kc, vc, hq, hkv, d, position=pos, workspace=ws)
    torch.cuda.synchronize()
    assert _lib.device_error(clear=True) == 0
    assert rel_err(np32(out1), ref) <= TOL
    assert torch.equal(out1, out2)
    assert int(ws[:256].view(torch.int32).abs().sum()) == 0  # counters back to zero


@pytest.mark.gpu
def test_device_position_past_the_cache_records_error():
    """A device-side position with start + S beyond the cache: the kernel checks it, records
    device error 2 and touches neither the cache nor the output (no memory access out of range)."""
    require_b200()
    from tinker_b200 import _lib
    from tinker_b200.kernels.kv_cache import kv_attention
    B, hq, hkv, d, cap = 1, 8, 2, 64, 64
    q, kn, vn, cos, sin, kc, vc, _, _, _ = _case(B, hq, hkv, d, 10, 1, cap, torch.float16, seed=9)
    before = kc.clone()
    _lib.device_error(clear=True)
    pos = torch.tensor([cap], dtype=torch.int32, device="cuda")
    kv_attention(q, kn, vn, cos, sin, kc, vc, hq, hkv, d, position=pos)
    torch.cuda.synchronize()
    assert _lib.device_error(clear=True) == 2
    assert torch.equal(kc, before)
    assert _lib.device_error(clear=True) == 0


@pytest.mark.gpu
def test_kv_append_and_rejects():
    require_b200()
    from tinker_b200.kernels.kv_cache import kv_append, kv_attention
    B, hkv, d, cap, S, start = 2, 4, 64, 32, 5, 7
    qkv = torch.randn(B, S, (8 + 2 * hkv) * d, device="cuda", dtype=torch.bfloat16)
    k, v = qkv[..., 8 * d:(8 + hkv) * d], qkv[..., (8 + hkv) * d:]
    kc = torch.zeros(B, hkv, cap, d, device="cuda", dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    kv_append(k, v, kc, vc, start)
    assert torch.equal(kc[:, :, start:start + S], k.reshape(B, S, hkv, d).transpose(1, 2))
    assert torch.equal(vc[:, :, start:start + S], v.reshape(B, S, hkv, d).transpose(1, 2))
    assert kc[:, :, :start].abs().sum() == 0 and kc[:, :, start + S:].abs().sum() == 0
    with pytest.raises(ValueError, match="capacity"):
        kv_append(k, v, kc, vc, cap - 2)
    cos = torch.zeros(cap, d // 2, device="cuda")
    q = qkv[..., :8 * d]
    with pytest.raises(ValueError, match="capacity"):
        kv_attention(q, k, v, cos, cos, kc, vc, 8, hkv, d, start_pos=cap - 1)
    with pytest.raises(TypeError, match="float32"):
        kv_attention(q, k, v, cos.half(), cos.half(), kc, vc, 8, hkv, d, start_pos=0)
    big_k = torch.zeros(B, hkv, 1024, d, device="cuda", dtype=torch.bfloat16)
    big_cos = torch.zeros(1024, d // 2, device="cuda")
    with pytest.raises(ValueError, match="workspace"):  # 905 keys: split over chunks, scratch needed
        kv_attention(q, k, v, big_cos, big_cos, big_k, big_k.clone(), 8, hkv, d, start_pos=900,
                     workspace=torch.zeros(16, dtype=torch.uint8, device="cuda"))


def _decoder(num_layers, dtype=torch.float16, seed=0, base=None):
    """A decoder with the 268M shapes (or ``base``'s) and fewer layers: (config, fp32 weights as
    numpy, optimised model without a forward graph)."""
    import tinker_b200
    from bench_model import LLAMA_268M, build_model
    cfg = (base or LLAMA_268M).with_(num_layers=num_layers, max_seq_len=512)
    cpu = build_model(cfg, seed=seed)
    weights = {k: v.detach().float().numpy().copy() for k, v in cpu.state_dict().items()}
    model = tinker_b200.optimize(cpu.to("cuda"), dtype=dtype, cuda_graph=False)
    return cfg, weights, model


@pytest.mark.gpu
@pytest.mark.parametrize("fused_step", [True, False])
@pytest.mark.parametrize("prompt_len", [100, 8])
def test_cached_decoder_matches_full_forward(prompt_len, fused_step):
    """Prefill (tensor-core prompt path at 100 tokens, the kv_attention path at 8) then 16 decode
    steps through the CUDA graph, with the one-kernel step or the per-block kernels: every step's
    logits equal the last row of the full forward of the same model over all tokens so far."""
    require_b200()
    import tinker_b200
    from bench_model import make_tokens
    cfg, _, model = _decoder(4)
    B, steps = 2, 16
    tokens = make_tokens(cfg, B, prompt_len + steps, seed=3).cuda()
    dec = tinker_b200.CachedDecoder(model, batch_size=B, capacity=256, cuda_graph=True, fused_step=fused_step)
    assert dec.fused_step == fused_step
    with torch.inference_mode():
        got = [dec.prefill(tokens[:, :prompt_len]).float().clone()]
        for t in range(prompt_len, prompt_len + steps):
            got.append(dec.decode(tokens[:, t]).float().clone())
        full = model(tokens).float()
    assert dec.length == prompt_len + steps
    for i, lg in enumerate(got):
        want = full[:, prompt_len - 1 + i]
        err = (lg - want).abs().max().item()
        assert err <= 2e-2, f"step {i}: max |logits - full forward| = {err}"


@pytest.mark.gpu
def test_cached_decoder_matches_oracle_and_eager_steps():
    """Logits of the last decode step vs the fp32 oracle's full forward (the reference's eager
    algorithm over the whole sequence), and the graph steps vs eager (no graph) steps."""
    require_b200()
    import tinker_b200
    from bench_model import make_tokens
    cfg, w, model = _decoder(3)
    B, P, steps = 1, 40, 6
    tokens = make_tokens(cfg, B, P + steps, seed=4)
    ocfg = oracle.ModelConfig(**{f: getattr(cfg, f) for f in oracle.ModelConfig.__dataclass_fields__})
    ref = oracle.forward_logits(w, tokens.numpy(), ocfg)[:, -1]
    outs = []
    for graph in (True, False):
        dec = tinker_b200.CachedDecoder(model, batch_size=B, capacity=128, cuda_graph=graph)
        with torch.inference_mode():
            lg = dec.prefill(tokens[:, :P].cuda())
            for t in range(P, P + steps):
                lg = dec.decode(tokens[:, t].cuda())
            outs.append(np32(lg))
    assert np.max(np.abs(outs[0] - ref)) <= 2e-2
    assert np.max(np.abs(outs[0] - outs[1])) <= 5e-3


@pytest.mark.gpu
def test_generate_greedy_matches_recompute():
    """Greedy generation with the cache picks, at every step where the choice is clear, the token
    the full forward over the sequence so far picks (random weights give near-ties)."""
    require_b200()
    import tinker_b200
    from bench_model import make_tokens
    cfg, _, model = _decoder(2)
    B, P, n = 2, 24, 12
    prompt = make_tokens(cfg, B, P, seed=6).cuda()
    dec = tinker_b200.CachedDecoder(model, batch_size=B, capacity=64)
    with torch.inference_mode():
        ids = dec.generate(prompt, n).cuda()
        seq = torch.cat([prompt, ids], dim=1)
        full = model(seq).float()[:, P - 1:P - 1 + n]
    top2 = full.topk(2, dim=-1).values
    clear = (top2[..., 0] - top2[..., 1]) > 5e-2
    assert torch.equal(full.argmax(-1)[clear], ids[clear])


def _shape(name):
    from bench_model import LLAMA_268M, QWEN25_05B_SHAPED
    return {"llama268m": LLAMA_268M, "qwen-shaped": QWEN25_05B_SHAPED,
            "head_dim128": LLAMA_268M.with_(num_heads=8, num_kv_heads=4, head_dim=128)}[name]


@pytest.mark.gpu
@pytest.mark.parametrize("shape, dt, tol", [("llama268m", "fp16", 2e-2), ("qwen-shaped", "bf16", 6e-2),
                                            ("head_dim128", "fp16", 2e-2)])
def test_chunked_prefill_then_decode(shape, dt, tol):
    """A prompt in two chunks (the second at position 40 goes through kv_attention: 30 new tokens,
    up to 210 query rows per kv head), then decode steps; each result equals the matching row of
    the full forward over all tokens so far. Covers 8-row CTAs (7 query heads per kv head, bf16,
    tied embeddings) and head_dim 128."""
    require_b200()
    import tinker_b200
    from bench_model import make_tokens
    cfg, _, model = _decoder(2, DTYPES[dt], base=_shape(shape))
    B, steps = 2, 4
    tokens = make_tokens(cfg, B, 70 + steps, seed=8).cuda()
    dec = tinker_b200.CachedDecoder(model, batch_size=B, capacity=128)
    with torch.inference_mode():
        got = [dec.prefill(tokens[:, :40]).float().clone(), dec.prefill(tokens[:, 40:70]).float().clone()]
        for t in range(70, 70 + steps):
            got.append(dec.decode(tokens[:, t]).float().clone())
        full = model(tokens).float()
    want = [full[:, 39], full[:, 69]] + [full[:, t] for t in range(70, 70 + steps)]
    for i, (a, b) in enumerate(zip(got, want)):
        err = (a - b).abs().max().item()
        assert err <= tol * max(1.0, b.abs().max().item()), f"result {i}: max |logits - full forward| = {err}"


@pytest.mark.gpu
@pytest.mark.parametrize("shape, dt, B", [("llama268m", "fp16", 1), ("llama268m", "bf16", 3), ("qwen-shaped", "bf16", 8),
                                          ("head_dim128", "fp16", 5)])
def test_fused_step_matches_per_block_step(shape, dt, B):
    """The one-kernel decode step (grid barriers between the phases) against the per-block kernels
    on the same model, cache contents and tokens: logits and the cache rows it appends agree to
    the rounding of the fp32 sums (different summation order and row-statistics parts)."""
    require_b200()
    import tinker_b200
    from bench_model import make_tokens
    cfg, _, model = _decoder(3, DTYPES[dt], base=_shape(shape))
    P, steps = 30, 5
    tokens = make_tokens(cfg, B, P + steps, seed=11).cuda()
    outs, caches = [], []
    for fused in (True, False):
        dec = tinker_b200.CachedDecoder(model, batch_size=B, capacity=64, fused_step=fused)
        with torch.inference_mode():
            dec.prefill(tokens[:, :P])
            steps_out = [dec.decode(tokens[:, t]).float().clone() for t in range(P, P + steps)]
        outs.append(torch.stack(steps_out))
        caches.append((dec.cache.k[:, :, :, :P + steps].float().clone(), dec.cache.v[:, :, :, :P + steps].float().clone()))
        dec.release()
    scale = outs[1].abs().max().item()
    assert (outs[0] - outs[1]).abs().max().item() <= 2e-2 * max(1.0, scale)
    for a, b in zip(caches[0], caches[1]):
        assert (a - b).abs().max().item() <= 5e-2 * max(1.0, b.abs().max().item())


@pytest.mark.gpu
def test_fused_step_stops_on_device_error():
    """A position past the cache: the attention phase records device error 2 and every CTA leaves
    at the next grid barrier (no wait runs out); the decoder is usable again after clearing it."""
    require_b200()
    import tinker_b200
    from tinker_b200 import _lib
    from bench_model import make_tokens
    cfg, _, model = _decoder(2)
    tokens = make_tokens(cfg, 1, 12, seed=12).cuda()
    dec = tinker_b200.CachedDecoder(model, batch_size=1, capacity=16, cuda_graph=False, fused_step=True)
    _lib.device_error(clear=True)
    with torch.inference_mode():
        dec.prefill(tokens[:, :10])
        dec._setup_step()
        dec.cache.position.fill_(16)  # start + 1 > capacity
        dec._fused_forward(tokens[:, 10:11])
        torch.cuda.synchronize()
        assert _lib.device_error(clear=True) == 2
        lg = dec.decode(tokens[:, 10])  # position 10 again, now in range
        torch.cuda.synchronize()
    assert _lib.device_error(clear=True) == 0
    assert torch.isfinite(lg.float()).all()


@pytest.mark.gpu
def test_fused_step_bounded_wait_runs_out_and_recovers():
    """A grid-barrier wait that nothing completes: with the test hook one CTA of the one-kernel
    step withholds its arrival at the first barrier, so every CTA's wait there runs out after
    the 2 s limit. The launch returns, device error 1 (timeout) is recorded, and after clearing
    it the next step on the same decoder is finite and equals the per-block step."""
    require_b200()
    import time
    import tinker_b200
    from tinker_b200 import _lib
    from bench_model import make_tokens
    cfg, _, model = _decoder(2)
    tokens = make_tokens(cfg, 1, 12, seed=13).cuda()
    ref = tinker_b200.CachedDecoder(model, batch_size=1, capacity=16, cuda_graph=False, fused_step=False)
    dec = tinker_b200.CachedDecoder(model, batch_size=1, capacity=16, cuda_graph=False, fused_step=True)
    _lib.device_error(clear=True)
    lib = _lib.lib()
    with torch.inference_mode():
        ref.prefill(tokens[:, :10])
        want = ref.decode(tokens[:, 10]).float()
        dec.prefill(tokens[:, :10])
        dec._setup_step()
        dec.cache.position.fill_(10)
        scratch = dec._step_scratch.data_ptr()
        _lib.check(lib.tk_decode_step_withhold_arrival(scratch, 3), "tk_decode_step_withhold_arrival")
        t0 = time.perf_counter()
        dec._fused_forward(tokens[:, 10:11])
        torch.cuda.synchronize()
        waited = time.perf_counter() - t0
        assert _lib.device_error(clear=True) == 1  # TK_DEVERR_TIMEOUT
        assert 1.5 < waited < 30, waited
        _lib.check(lib.tk_decode_step_withhold_arrival(scratch, -1), "tk_decode_step_withhold_arrival")
        got = dec.decode(tokens[:, 10]).float()  # position 10 again (the failed step wrote no cache row)
        torch.cuda.synchronize()
    assert _lib.device_error(clear=True) == 0
    assert torch.isfinite(got).all()
    assert (got - want).abs().max().item() <= 2e-2 * max(1.0, want.abs().max().item())
    with pytest.raises(RuntimeError):
        _lib.check(lib.tk_decode_step_withhold_arrival(scratch, -2), "tk_decode_step_withhold_arrival")
