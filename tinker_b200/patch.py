"""Module patcher: the drop-in for eb1386/TinKer's ``patch_model`` (tinker/patch.py:43-123).

The patcher is a table of rules, tried in order on every child of every module of the
model; the first enabled rule whose predicate accepts the child builds its
replacement. The rules and their order are the reference's (tinker/patch.py:10-40,
:57-116), so the same user modules are replaced:

* ``norm`` - a 1-D ``nn.Parameter`` named ``weight``, an ``eps`` or
  ``variance_epsilon`` attribute and no bias -> ``TinKerRMSNorm``;
* ``ffn`` - gate / up / down projections found by name -> ``TinKerSwiGLU``;
* ``attention`` - q / k / v / o projection layers found by name -> ``TinKerAttention``.

Every replacement takes the device and dtype of one source weight: the norm's
``weight``, or the ``weight`` of the first gate (FFN) / q (attention) attribute the
source has, as the reference does (tinker/patch.py:76-80, :95-99) - so an FFN whose
projections are bare tensors is recognised but left unpatched there too. Replacements
are swapped in only after the whole walk, so the walk sees the original model; a
child whose replacement cannot be built stays as it is (reported when ``verbose``).
"""

from __future__ import annotations

from collections import Counter
from dataclasses import dataclass
from typing import Callable

import torch
import torch.nn as nn

from tinker_b200.modules._roles import (ATTENTION_ROLES, SWIGLU_ROLES, attention_projections, first_present,
                                       plays_roles, swiglu_weights)
from tinker_b200.modules.attention import TinKerAttention
from tinker_b200.modules.feed_forward import TinKerSwiGLU
from tinker_b200.modules.normalization import TinKerRMSNorm


def _is_rmsnorm(module: nn.Module) -> bool:
    """An RMSNorm by structure: 1-D weight parameter, an epsilon attribute, no bias."""
    weight = getattr(module, "weight", None)
    has_eps = hasattr(module, "eps") or hasattr(module, "variance_epsilon")
    no_bias = getattr(module, "bias", None) is None
    return isinstance(weight, nn.Parameter) and weight.dim() == 1 and has_eps and no_bias


def _is_swiglu(module: nn.Module) -> bool:
    return plays_roles(swiglu_weights, module)


def _is_gqa_attention(module: nn.Module) -> bool:
    return plays_roles(attention_projections, module)


@dataclass(frozen=True)
class _Rule:
    kind: str  # the patch_model flag that enables it: replace_<kind>
    label: str
    accepts: Callable[[nn.Module], bool]
    build: Callable[[nn.Module, float, int], nn.Module]
    weight_of: Callable[[nn.Module], torch.Tensor]  # its device and dtype are the replacement's


_RULES = (
    _Rule("norm", "rmsnorm", _is_rmsnorm,
          lambda src, theta, seq: TinKerRMSNorm.from_module(src),
          lambda src: src.weight),
    _Rule("ffn", "swiglu", _is_swiglu,
          lambda src, theta, seq: TinKerSwiGLU.from_module(src),
          lambda src: first_present(src, SWIGLU_ROLES, "gate").weight),
    _Rule("attention", "attention", _is_gqa_attention,
          lambda src, theta, seq: TinKerAttention.from_module(src, rope_theta=theta, max_seq_len=seq),
          lambda src: first_present(src, ATTENTION_ROLES, "q").weight),
)


def patch_model(
    model: nn.Module,
    replace_attention: bool = True,
    replace_ffn: bool = True,
    replace_norm: bool = True,
    rope_theta: float = 10000.0,
    max_seq_len: int = 2048,
    verbose: bool = False,
) -> nn.Module:
    """Replace the RMSNorm, SwiGLU FFN and GQA attention submodules of ``model`` in place
    with the fused-kernel modules; returns ``model``."""
    enabled = {"norm": replace_norm, "ffn": replace_ffn, "attention": replace_attention}
    rules = [r for r in _RULES if enabled[r.kind]]
    swaps: list[tuple[nn.Module, str, nn.Module]] = []
    done: Counter = Counter()
    for parent_path, parent in model.named_modules():
        for attr, child in parent.named_children():
            rule = next((r for r in rules if r.accepts(child)), None)
            if rule is None:
                continue
            path = f"{parent_path}.{attr}" if parent_path else attr
            try:
                w = rule.weight_of(child)
                new = rule.build(child, rope_theta, max_seq_len).to(device=w.device, dtype=w.dtype)
            except Exception as e:  # leave this child alone, keep patching the rest
                if verbose:
                    print(f"  [tinker] {path}: {rule.label} not replaced ({e})")
                continue
            swaps.append((parent, attr, new))
            done[rule.kind] += 1
            if verbose:
                print(f"  [tinker] {path}: {rule.label} -> {type(new).__name__}")
    for parent, attr, new in swaps:
        setattr(parent, attr, new)
    if verbose:
        print(f"\n  [tinker] replaced {sum(done.values())} modules "
              f"(attention {done['attention']}, ffn {done['ffn']}, norm {done['norm']})")
    return model
