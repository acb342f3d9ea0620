"""The one-kernel decoder stack (``tk_stack_forward``, ``tinker_b200.stack``).

GPU parity: the stack kernel against the per-block path of the same optimised model (the
same arithmetic, only the summation order of the k-splits differs: <= 5e-3 norm-wise and
<= 2e-2 max-abs on the logits), and against the fp32 oracle (the reference's eager
forward restated, tests/test_oracle_golden.py pins it) with the bars of the 268M test;
batches of several sequences (attention must not cross sequences); repeat calls give
identical bits; one library launch per forward; in-place weight changes are followed;
a token id outside the table records device error 3 without faulting and the next
forward is correct. CPU: the top-level dataflow check accepts the LM structure and
rejects forwards that do anything else.
"""

import numpy as np
import pytest
import torch
import torch.nn as nn

import oracle
from tests._util import np32, rel_err, require_b200


def _oracle_logits(model, tokens, cfg):
    w = {k: v.detach().float().cpu().numpy() for k, v in model.state_dict().items()}
    ocfg = oracle.ModelConfig(**{f: getattr(cfg, f) for f in oracle.ModelConfig.__dataclass_fields__})
    return oracle.forward_logits(w, tokens.numpy(), ocfg)


def _pair(cfg, seed, dtype=torch.float16):
    import tinker_b200
    from bench_model import build_model
    a = tinker_b200.optimize(build_model(cfg, seed=seed).cuda(), dtype=dtype, stack_kernel=True)
    b = tinker_b200.optimize(build_model(cfg, seed=seed).cuda(), dtype=dtype, stack_kernel=False)
    assert getattr(a, "_tinker_stack_parts", None) is not None, "stack forward not installed"
    assert getattr(b, "_tinker_stack_parts", None) is None
    return a, b


@pytest.mark.gpu
@pytest.mark.parametrize("batch, seq", [(1, 128), (2, 48), (4, 32), (1, 1), (3, 7)])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_stack_matches_per_block_path(batch, seq, dtype):
    require_b200()
    from bench_model import LLAMA_268M, make_tokens
    cfg = LLAMA_268M.with_(num_layers=3, vocab_size=4096)
    a, b = _pair(cfg, seed=batch * 100 + seq, dtype=dtype)
    tokens = make_tokens(cfg, batch, seq, seed=seq).cuda()
    with torch.inference_mode():
        ya, yb = np32(a(tokens)), np32(b(tokens))
    assert np.isfinite(ya).all()
    tol = 5e-3 if dtype == torch.float16 else 2e-2
    assert rel_err(ya, yb) <= tol
    assert np.abs(ya - yb).max() <= (2e-2 if dtype == torch.float16 else 1e-1)


@pytest.mark.gpu
def test_stack_268m_against_oracle_and_launches():
    """The full 268M decoder at b1 s128 through the stack kernel, eagerly: the oracle bars of
    the graph test, one library launch per forward (the LM head is the model's own), identical
    bits on repeat calls."""
    require_b200()
    import tinker_b200
    from tinker_b200 import _lib
    from bench_model import LLAMA_268M, build_model, make_tokens
    cfg = LLAMA_268M
    tokens = make_tokens(cfg, 1, 128, seed=1)
    cpu_model = build_model(cfg, seed=0)
    ref = _oracle_logits(cpu_model, tokens, cfg).astype(np.float64)
    model = tinker_b200.optimize(cpu_model.to("cuda"), dtype=torch.float16, stack_kernel=True)
    with torch.inference_mode():
        out = np32(model(tokens.cuda()))
        n0 = _lib.launch_counter[0]
        out2 = np32(model(tokens.cuda()))
        launches = _lib.launch_counter[0] - n0
    np.testing.assert_array_equal(out, out2)
    assert launches == 1
    plan = next(iter(model._tinker_stack_plans.values())).plan()
    assert plan["ctas"] == torch.cuda.get_device_properties(0).multi_processor_count
    err = np.abs(out - ref)
    s = np.sort(ref, axis=-1)
    clear = (s[..., -1] - s[..., -2]) > 2 * err.max()
    top1 = (out.argmax(-1) == ref.argmax(-1))[clear].mean()
    msg = f"max-abs {err.max():.3e}, top-1 (clear margin, {int(clear.sum())} positions) {top1:.4f}, plan {plan}"
    print("\n" + msg)
    assert err.max() <= 2e-2, msg
    assert top1 == 1.0, msg
    assert _lib.device_error(clear=True) == 0


@pytest.mark.gpu
def test_stack_follows_in_place_weight_changes():
    require_b200()
    from bench_model import TINY, make_tokens
    cfg = TINY.with_(num_layers=3)
    a, b = _pair(cfg, seed=21)
    tokens = make_tokens(cfg, 2, 40, seed=4).cuda()
    with torch.inference_mode():
        ya0 = a(tokens).float()
    with torch.no_grad():
        for m in (a, b):
            m.layers[1].ffn_norm.weight.mul_(1.5)
            m.layers[2].attn.o_proj.weight.mul_(0.5)
    with torch.inference_mode():
        ya, yb = a(tokens).float(), b(tokens).float()
    assert ((ya - ya0).norm() / ya0.norm()).item() > 1e-2
    assert ((ya - yb).norm() / yb.norm()).item() < 5e-3


@pytest.mark.gpu
def test_stack_bad_token_records_error_and_recovers():
    require_b200()
    from tinker_b200 import _lib
    from bench_model import TINY, make_tokens
    a, b = _pair(TINY, seed=5)
    tokens = make_tokens(TINY, 1, 16, seed=6).cuda()
    _lib.device_error(clear=True)
    bad = tokens.clone()
    bad[0, 3] = TINY.vocab_size + 7
    with torch.inference_mode():
        a(bad)
        torch.cuda.synchronize()
        assert _lib.device_error(clear=True) == 3
        ya, yb = a(tokens).float(), b(tokens).float()
        torch.cuda.synchronize()
    assert _lib.device_error(clear=True) == 0
    assert ((ya - yb).norm() / yb.norm()).item() < 5e-3


@pytest.mark.gpu
def test_stack_in_cuda_graph_and_larger_inputs_fall_back():
    """optimize(cuda_graph=True) captures the stack kernel (its plan made by the warm-up
    forwards); an input of more than 128 rows takes the per-block path."""
    require_b200()
    import tinker_b200
    from tinker_b200 import _lib
    from bench_model import TINY, build_model, make_tokens
    cfg = TINY.with_(num_layers=2)
    tokens = make_tokens(cfg, 2, 64, seed=8).cuda()
    g = tinker_b200.optimize(build_model(cfg, seed=9).cuda(), dtype=torch.float16, cuda_graph=True,
                             graph_input_shape=(2, 64), graph_vocab_size=cfg.vocab_size, stack_kernel=True)
    ref = tinker_b200.optimize(build_model(cfg, seed=9).cuda(), dtype=torch.float16, stack_kernel=False)
    assert type(g).__name__ == "_CUDAGraphWrapper" and (2, 64) in g._model._tinker_stack_plans
    big = make_tokens(cfg, 3, 50, seed=9).cuda()
    with torch.inference_mode():
        np.testing.assert_allclose(np32(g(tokens)), np32(ref(tokens)), rtol=0, atol=2e-2)
        n0 = _lib.launch_counter[0]
        yb = g(big)  # 150 rows: not the captured shape, and beyond the stack kernel
        assert _lib.launch_counter[0] - n0 == 5 * cfg.num_layers + 2
        assert rel_err(np32(yb), np32(ref(big))) <= 5e-3


def test_dataflow_check_accepts_lm_and_rejects_other_forwards():
    from tinker_b200.stack import _dataflow_is_lm
    from bench_model import TINY, build_model

    m = build_model(TINY)
    parts = (m.embedding, list(m.layers), m.norm, m.output)
    assert _dataflow_is_lm(m, m.forward, *parts, "cpu")

    class Scaled(nn.Module):
        def __init__(self, lm):
            super().__init__()
            self.embedding, self.layers, self.norm, self.output = lm.embedding, lm.layers, lm.norm, lm.output

        def forward(self, tokens):
            x = self.embedding(tokens) * 2.0  # an embedding scale the stack kernel does not apply
            for layer in self.layers:
                x = layer(x)
            return self.output(self.norm(x))

    class Skip(Scaled):
        def forward(self, tokens):
            x = self.embedding(tokens)
            for layer in self.layers[:-1]:
                x = layer(x)
            return self.output(self.norm(x))

    class Soft(Scaled):
        def forward(self, tokens):
            x = self.embedding(tokens)
            for layer in self.layers:
                x = layer(x)
            return torch.softmax(self.output(self.norm(x)), dim=-1)

    class InPlace(Scaled):
        def forward(self, tokens):
            x = self.embedding(tokens)
            x.mul_(2.0)  # the same tensor goes on, with other values
            for layer in self.layers:
                x = layer(x)
            return self.output(self.norm(x))

    for cls in (Scaled, Skip, Soft, InPlace):
        w = cls(m)
        assert not _dataflow_is_lm(w, w.forward, *parts, "cpu"), cls.__name__
    # the stubs are gone again
    assert "forward" not in m.embedding.__dict__ and "forward" not in m.layers[0].__dict__
