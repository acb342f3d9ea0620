"""torch.compile over patched models: the kernel calls are registered ops (tinker_b200.torch_ops).

CPU: every op is registered and its fake implementation gives the real output shape.
GPU: a patched model traces end to end (``fullgraph=True``, no graph break at any kernel)
and gives the eager model's logits; ``optimize(compile=True)`` compiles as the reference
does (tinker/optimize.py:77-88) and gives the same logits.
"""

import pytest
import torch

from tests._util import require_b200


def test_ops_are_registered_with_fake_shapes():
    import tinker_b200  # noqa: F401  (registers torch.ops.tinker.*)
    from torch._subclasses.fake_tensor import FakeTensorMode
    with FakeTensorMode():
        x = torch.empty(2, 5, 128, dtype=torch.float16)
        w = torch.empty(128, dtype=torch.float16)
        assert torch.ops.tinker.rmsnorm(x, w, 1e-6).shape == (2, 5, 128)
        assert torch.ops.tinker.swiglu(x, x).shape == (2, 5, 128)
        wg, wd = torch.empty(256, 128, dtype=torch.float16), torch.empty(128, 256, dtype=torch.float16)
        assert torch.ops.tinker.swiglu_ffn(x, wg, wg, wd, None).shape == (2, 5, 128)
        q = torch.empty(2, 5, 4 * 64, dtype=torch.float16)
        kv = torch.empty(2, 5, 2 * 64, dtype=torch.float16)
        cs = torch.empty(16, 32)
        assert torch.ops.tinker.fused_attention(q, kv, kv, cs, cs, 4, 2, 64, 0).shape == (2, 5, 256)
        wq, wk, wo = (torch.empty(256, 128, dtype=torch.float16), torch.empty(128, 128, dtype=torch.float16),
                      torch.empty(128, 256, dtype=torch.float16))
        assert torch.ops.tinker.attention(x, wq, wk, wk, wo, cs, cs, 4, 2, 64, 0, None).shape == (2, 5, 128)


@pytest.mark.gpu
def test_patched_model_compiles_fullgraph():
    require_b200()
    import tinker_b200
    from bench_model import TINY, build_model, make_tokens
    torch._dynamo.reset()
    model = tinker_b200.optimize(build_model(TINY, seed=3).cuda(), dtype=torch.float16, fuse_blocks=False)
    tokens = make_tokens(TINY, 2, 32, seed=4).cuda()
    compiled = torch.compile(model, backend="aot_eager", fullgraph=True)
    with torch.inference_mode():
        want = model(tokens).float()
        got = compiled(tokens).float()
    assert ((got - want).norm() / want.norm()).item() < 1e-3


@pytest.mark.gpu
def test_optimize_compile_true():
    require_b200()
    import tinker_b200
    from bench_model import TINY, build_model, make_tokens
    torch._dynamo.reset()
    tokens = make_tokens(TINY, 2, 32, seed=5).cuda()
    ref = tinker_b200.optimize(build_model(TINY, seed=6).cuda(), dtype=torch.float16)
    model = tinker_b200.optimize(build_model(TINY, seed=6).cuda(), dtype=torch.float16, compile=True,
                                 compile_mode="default")
    assert type(model).__name__ == "OptimizedModule"
    with torch.inference_mode():
        want = ref(tokens).float()
        got = model(tokens).float()
    assert ((got - want).norm() / want.norm()).item() < 5e-3
