"""Finding the projections of a user's attention / FFN module by attribute name.

A source module plays a role ("q", "gate", ...) through the first attribute, from a
fixed list of candidate names, that is set on it. The candidate lists are the ones
the reference accepts (tinker/modules/attention.py:127-153 for attention,
tinker/modules/feed_forward.py:50-76 for the SwiGLU FFN), in the same order, so that
the same user modules are recognised and the same attributes are taken.

What counts as "set" differs per kind, as in the reference: an attention role takes
the first candidate that exists and has a ``weight`` (the projection layer itself is
returned); an FFN role stops at the first candidate that exists and either has a
``weight`` (its weight is returned) or is itself a tensor (returned as is).
"""

from __future__ import annotations

import torch
import torch.nn as nn

ATTENTION_ROLES = (
    ("q", ("q_proj", "query", "wq", "q")),
    ("k", ("k_proj", "key", "wk", "k")),
    ("v", ("v_proj", "value", "wv", "v")),
    ("o", ("o_proj", "output", "wo", "out_proj", "o")),
)
SWIGLU_ROLES = (
    ("gate", ("gate_proj", "w1", "gate")),
    ("up", ("up_proj", "w3", "up")),
    ("down", ("down_proj", "w2", "down")),
)

_SKIP = object()  # "this candidate does not play the role; try the next name"


def _layer_with_weight(obj):
    return obj if hasattr(obj, "weight") else _SKIP


def _weight_or_tensor(obj):
    if hasattr(obj, "weight"):
        return obj.weight
    if isinstance(obj, torch.Tensor):
        return obj
    return _SKIP


def _resolve(module: nn.Module, roles, take, what: str) -> dict:
    found = {}
    for role, names in roles:
        found[role] = None
        for name in names:
            obj = getattr(module, name, None)
            if obj is None:
                continue
            got = take(obj)
            if got is not _SKIP:
                found[role] = got
                break
    missing = [role for role, got in found.items() if got is None]
    if missing:
        expected = ", ".join("/".join(names) for _, names in roles)
        raise ValueError(f"{type(module).__name__} is not a {what} module: nothing plays the "
                         f"{', '.join(missing)} role (expected attributes named {expected})")
    return found


def attention_projections(module: nn.Module) -> dict:
    """{"q", "k", "v", "o"} -> the source module's projection layers; ValueError if one is missing."""
    return _resolve(module, ATTENTION_ROLES, _layer_with_weight, "GQA attention")


def swiglu_weights(module: nn.Module) -> dict:
    """{"gate", "up", "down"} -> the source module's projection weights; ValueError if one is missing."""
    return _resolve(module, SWIGLU_ROLES, _weight_or_tensor, "SwiGLU FFN")


def first_present(module: nn.Module, roles, role: str):
    """The first candidate attribute of ``role`` that ``module`` has at all (no other test)."""
    names = dict(roles)[role]
    return getattr(module, next(n for n in names if hasattr(module, n)))


def plays_roles(finder, module: nn.Module) -> bool:
    try:
        finder(module)
    except (ValueError, AttributeError):
        return False
    return True
