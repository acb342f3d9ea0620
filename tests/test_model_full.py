"""Full-size parity of the two other decoder configs against the fp32 oracle.

* Qwen2.5-0.5B-shaped decoder, bf16: vocab 151936 with the LM head tied to the
  embedding, hidden 896, all 24 layers, 14 query / 2 KV heads, head_dim 64, FFN 4864,
  RoPE theta 1e6; batch 2 x seq 512, all 1024 positions checked.
* ~1B Llama-style decoder, fp16 (vocab 32000, hidden 2048, 16 layers, 32/8 heads, FFN
  5632, eps 1e-5): batch 1 x seq 128 through the CUDA graph, all positions; and the
  batch 16 x seq 2048 graph that the throughput figure times, with its first and last
  sequences (4096 positions) checked.

Weights are seeded N(0, 0.02) as for the benchmarks; the oracle is the numpy restatement
of the reference's fp32 eager forward (benchmarks/bench_e2e.py:97-138 blocks with the
embedding / head of examples/patch_any_model.py:95-108), pinned to the reference by
tests/test_oracle_golden.py. Reported in each assertion message and checked:

* max-abs logits error against fp32, and no more than twice the error of the reference's
  own eager forward in the same half precision on the same GPU (oracle/torch_model.py,
  the reference's blocks run with torch's CUDA ops) - plus <= 2e-2 for the fp16 cases;
* top-1 agreement over the positions whose fp32 top-1/top-2 gap exceeds twice the
  observed max-abs error: 100 %. (Raw top-1 is reported: on random weights near-ties
  make it < 100 % even for the reference's own half-precision eager model.)
"""

import numpy as np
import pytest
import torch

import oracle
from tests._util import np32, require_b200

pytestmark = pytest.mark.gpu


def _weights(model):
    return {k: v.detach().float().cpu().numpy() for k, v in model.state_dict().items()}


def _ocfg(cfg):
    return oracle.ModelConfig(**{f: getattr(cfg, f) for f in oracle.ModelConfig.__dataclass_fields__})


def _stats(ours, ref):
    ours = np.asarray(ours, dtype=np.float64).reshape(-1, ref.shape[-1])
    ref = np.asarray(ref, dtype=np.float64).reshape(-1, ref.shape[-1])
    err = np.abs(ours - ref).max()
    top2 = np.sort(ref, axis=-1)[:, -2:]
    agree = ours.argmax(-1) == ref.argmax(-1)
    clear = (top2[:, 1] - top2[:, 0]) > 2 * err
    return float(err), float(agree.mean()), float(agree[clear].mean()) if clear.any() else 1.0, int(clear.sum())


def _reference_eager_error(cfg, dtype, tokens, ref, rows=None):
    """Max-abs error of the reference's own eager forward in ``dtype`` on this GPU."""
    from oracle.torch_model import build_model as build_reference
    m = build_reference(cfg, seed=0, device="cuda", dtype=dtype)
    with torch.inference_mode():
        out = m(tokens.cuda())
        out = np32(out if rows is None else out[rows])
    del m
    torch.cuda.empty_cache()
    return _stats(out, ref)


def _check(name, ours, ref, base, half_bar=None):
    err, top1, top1_clear, n_clear = _stats(ours, ref)
    msg = (f"{name}: max-abs {err:.4g}, top-1 {top1:.4f}, top-1 over {n_clear} clear-margin positions "
           f"{top1_clear:.4f}; reference eager in the same dtype: max-abs {base[0]:.4g}, top-1 {base[1]:.4f}")
    print("\n" + msg)
    assert top1_clear == 1.0, msg
    assert err <= 2 * base[0] + 1e-3, msg
    if half_bar is not None:
        assert err <= half_bar, msg


def test_qwen_shaped_full_model_bf16_b2s512():
    require_b200()
    import tinker_b200
    from bench_model import QWEN25_05B_SHAPED, build_model, make_tokens
    cfg = QWEN25_05B_SHAPED
    tokens = make_tokens(cfg, 2, 512, seed=4)
    cpu_model = build_model(cfg, seed=0)
    ref = oracle.forward_logits(_weights(cpu_model), tokens.numpy(), _ocfg(cfg))
    base = _reference_eager_error(cfg, torch.bfloat16, tokens, ref)
    model = tinker_b200.optimize(cpu_model.to("cuda"), dtype=torch.bfloat16)
    assert model.output.weight is model.embedding.weight  # the tied head stays tied
    with torch.inference_mode():
        ours = np32(model(tokens.cuda()))
    _check("Qwen-shaped bf16 b2 s512, 24 layers, tied 151936 head", ours, ref, base)


def test_llama1b_fp16_b1s128_graph():
    require_b200()
    import tinker_b200
    from bench_model import LLAMA_1B, build_model, make_tokens
    cfg = LLAMA_1B
    tokens = make_tokens(cfg, 1, 128, seed=1)
    cpu_model = build_model(cfg, seed=0)
    ref = oracle.forward_logits(_weights(cpu_model), tokens.numpy(), _ocfg(cfg))
    base = _reference_eager_error(cfg, torch.float16, tokens, ref)
    model = tinker_b200.optimize(cpu_model.to("cuda"), dtype=torch.float16, cuda_graph=True,
                                 graph_input_shape=(1, 128), graph_vocab_size=cfg.vocab_size)
    assert type(model).__name__ == "_CUDAGraphWrapper"
    with torch.inference_mode():
        ours = np32(model(tokens.cuda()))
    _check("~1B fp16 b1 s128 graph", ours, ref, base, half_bar=2e-2)


def test_llama1b_fp16_b16s2048_graph_first_and_last_sequence():
    require_b200()
    import tinker_b200
    from bench_model import LLAMA_1B, build_model, make_tokens
    cfg = LLAMA_1B
    tokens = make_tokens(cfg, 16, 2048, seed=1)
    rows = [0, 15]
    cpu_model = build_model(cfg, seed=0)
    # sequences are independent: the oracle runs only the two that are checked
    ref = oracle.forward_logits(_weights(cpu_model), tokens[rows].numpy(), _ocfg(cfg))
    base = _reference_eager_error(cfg, torch.float16, tokens[rows], ref)
    model = tinker_b200.optimize(cpu_model.to("cuda"), dtype=torch.float16, cuda_graph=True,
                                 graph_input_shape=(16, 2048), graph_vocab_size=cfg.vocab_size,
                                 graph_clone_output=False)
    assert type(model).__name__ == "_CUDAGraphWrapper"
    with torch.inference_mode():
        ours = np32(model(tokens.cuda())[rows])
    _check("~1B fp16 b16 s2048 graph, sequences 0 and 15", ours, ref, base, half_bar=2e-2)
