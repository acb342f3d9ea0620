"""Helpers shared by the kernel wrappers: device/stream plumbing around the C ABI."""

from __future__ import annotations

import contextlib
import threading

import torch

from tinker_b200 import _lib


def call_ctx(dev: torch.device):
    """Make `dev` current for the duration of a library call if it is not already."""
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    if idx == torch.cuda.current_device():
        return contextlib.nullcontext()
    return torch.cuda.device(idx)


def rows_view(x: torch.Tensor) -> torch.Tensor:
    """2-D [rows, last] view whose last dim is contiguous (copies only if it must)."""
    x2 = x.reshape(-1, x.shape[-1])
    if x2.shape[-1] > 1 and x2.stride(-1) != 1:
        x2 = x2.contiguous()
    return x2


def row_stride(x2: torch.Tensor) -> int:
    return x2.stride(0) if x2.shape[0] > 1 else x2.shape[1]


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


_graph_state = threading.local()


@contextlib.contextmanager
def stable_weights():
    """Inside this block the GEMMs may load their first weight tiles into shared memory before
    the previous kernel has finished (programmatic dependent launch). Only valid where no kernel
    enqueued since the stream last waited for all earlier work writes any weight: ``optimize``
    wraps its CUDA-graph capture in it (no kernel of the captured forward writes a weight, and the
    graph's first kernel is an ordinary launch)."""
    prev = getattr(_graph_state, "stable", False)
    _graph_state.stable = True
    try:
        yield
    finally:
        _graph_state.stable = prev


def weights_are_stable() -> bool:
    return getattr(_graph_state, "stable", False)


__all__ = ["call_ctx", "rows_view", "row_stride", "ptr", "_lib", "stable_weights", "weights_are_stable"]
