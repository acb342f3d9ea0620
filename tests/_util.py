"""Shared helpers for the parity tests."""

import numpy as np
import pytest
import torch

DTYPES = {"fp16": torch.float16, "bf16": torch.bfloat16, "fp32": torch.float32}
NP_NAME = {torch.float16: "float16", torch.bfloat16: "bfloat16", torch.float32: "float32"}


def has_b200() -> bool:
    if not torch.cuda.is_available():
        return False
    major, minor = torch.cuda.get_device_capability(0)
    return (major, minor) == (10, 0)


def require_b200():
    if not has_b200():
        pytest.fail("this GPU test needs a B200 (sm_100); none is visible")


def np32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def rel_err(actual, expected) -> float:
    """Norm-wise relative error ||a - e||_2 / ||e||_2 (the parity metric of these tests)."""
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    den = np.linalg.norm(e.ravel())
    return float(np.linalg.norm((a - e).ravel()) / (den if den > 0 else 1.0))


def ulp(dtype: torch.dtype) -> float:
    """Spacing of the dtype at 1.0."""
    return {torch.float16: 2.0 ** -10, torch.bfloat16: 2.0 ** -7, torch.float32: 2.0 ** -23}[dtype]
