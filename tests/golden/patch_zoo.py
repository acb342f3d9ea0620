"""A zoo of user modules for pinning ``patch_model``'s decisions to the reference's.

``zoo()`` returns one container whose children (some nested, one shared by two
parents) are the module shapes a user model may present to the patcher: RMSNorms
under both epsilon names, norms that must not match (biased, buffer weight, 2-D
weight), SwiGLU FFNs under each naming scheme (layers or bare tensors), attention
modules under each naming scheme with and without ``head_dim`` / ``rope_theta``, and
modules missing one projection. ``make_patch_golden.py`` runs the reference's
``patch_model`` over it and records what replaced each child; the tests run this
repository's ``patch_model`` over the same zoo and compare.
"""

import torch
import torch.nn as nn


class EpsNorm(nn.Module):
    def __init__(self, dim, eps=1e-6):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))


class HFNorm(nn.Module):
    def __init__(self, dim, eps=1e-5):
        super().__init__()
        self.variance_epsilon = eps
        self.weight = nn.Parameter(torch.ones(dim))


class BufferNorm(nn.Module):
    def __init__(self, dim):
        super().__init__()
        self.eps = 1e-6
        self.register_buffer("weight", torch.ones(dim))


class MatrixNorm(nn.Module):
    def __init__(self, dim):
        super().__init__()
        self.eps = 1e-6
        self.weight = nn.Parameter(torch.ones(dim, dim))


class LinearNames(nn.Module):
    """Linear layers under given attribute names (in, out) and optional plain attributes."""

    def __init__(self, layers, **attrs):
        super().__init__()
        for name, (n_in, n_out) in layers.items():
            setattr(self, name, nn.Linear(n_in, n_out, bias=False))
        for k, v in attrs.items():
            setattr(self, k, v)


class TensorFFN(nn.Module):
    def __init__(self, hidden, inner):
        super().__init__()
        self.gate = nn.Parameter(torch.randn(inner, hidden) * 0.02)
        self.up = nn.Parameter(torch.randn(inner, hidden) * 0.02)
        self.down = nn.Parameter(torch.randn(hidden, inner) * 0.02)


class NormAndFFN(EpsNorm):
    """Matches both the norm rule and the FFN rule; the norm rule comes first."""

    def __init__(self, dim, inner):
        super().__init__(dim)
        self.gate_proj = nn.Linear(dim, inner, bias=False)
        self.up_proj = nn.Linear(dim, inner, bias=False)
        self.down_proj = nn.Linear(inner, dim, bias=False)


def zoo() -> nn.Module:
    torch.manual_seed(0)
    root = nn.Module()
    root.norm_eps = EpsNorm(64, 1e-6)
    root.norm_hf = HFNorm(64, 1e-5)
    root.layernorm = nn.LayerNorm(64)
    root.layernorm_nobias = nn.LayerNorm(64, bias=False)
    root.norm_buffer = BufferNorm(64)
    root.norm_matrix = MatrixNorm(8)
    root.ffn_llama = LinearNames({"gate_proj": (64, 96), "up_proj": (64, 96), "down_proj": (96, 64)})
    root.ffn_w123 = LinearNames({"w1": (64, 160), "w3": (64, 160), "w2": (160, 64)})
    root.ffn_tensors = TensorFFN(64, 128)
    root.ffn_no_down = LinearNames({"gate_proj": (64, 96), "up_proj": (64, 96)})
    root.norm_and_ffn = NormAndFFN(64, 96)
    root.attn_llama = LinearNames({"q_proj": (512, 512), "k_proj": (512, 128), "v_proj": (512, 128),
                                   "o_proj": (512, 512)}, head_dim=64)
    root.attn_gpt = LinearNames({"query": (256, 256), "key": (256, 128), "value": (256, 128), "output": (256, 256)})
    root.attn_wq_128 = LinearNames({"wq": (1024, 1024), "wk": (1024, 256), "wv": (1024, 256), "wo": (1024, 1024)},
                                   head_dim=128)
    root.attn_odd_width = LinearNames({"q": (96, 96), "k": (96, 32), "v": (96, 32), "out_proj": (96, 96)})
    root.attn_theta = LinearNames({"q_proj": (256, 256), "k_proj": (256, 64), "v_proj": (256, 64),
                                   "o_proj": (256, 256)}, rope_theta=1e6)
    root.attn_no_o = LinearNames({"q_proj": (256, 256), "k_proj": (256, 64), "v_proj": (256, 64)})
    block = nn.Module()
    block.inner = nn.Module()
    block.inner.norm = EpsNorm(32, 1e-5)
    block.inner.mlp = LinearNames({"gate_proj": (32, 48), "up_proj": (32, 48), "down_proj": (48, 32)})
    root.block = block
    shared = EpsNorm(16, 1e-6)
    root.left = nn.Module()
    root.right = nn.Module()
    root.left.norm = shared
    root.right.norm = shared
    return root


FLAG_SETS = {
    "all": {},
    "no_norm": {"replace_norm": False},
    "no_ffn": {"replace_ffn": False},
    "no_attention": {"replace_attention": False},
    "theta_arg": {"rope_theta": 5e5, "max_seq_len": 512},
}


def describe(model: nn.Module) -> dict:
    """path -> what sits there after patching: the replacement's class and its inferred
    sizes, or "kept" for the zoo's original modules."""
    out = {}
    for path, m in model.named_modules():
        if not path or path.count(".") > 2:
            continue
        name = type(m).__name__
        if name == "TinKerRMSNorm":
            out[path] = {"type": name, "dim": int(m.weight.shape[0]), "eps": float(m.eps)}
        elif name == "TinKerSwiGLU":
            out[path] = {"type": name, "hidden": int(m.hidden_size), "inner": int(m.intermediate_size)}
        elif name == "TinKerAttention":
            out[path] = {"type": name, "heads": int(m.num_heads), "kv_heads": int(m.num_kv_heads),
                         "head_dim": int(m.head_dim), "theta": float(m.rope_theta),
                         "table_rows": int(m.cos_table.shape[0])}
        elif not name.startswith("TinKer") and "." not in path or path.startswith("block") or \
                path.startswith(("left", "right")):
            out[path] = {"type": "kept"}
    return out
