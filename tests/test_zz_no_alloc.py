"""tk_swiglu_ffn_noalloc: the SwiGLU FFN for callers that cannot allocate device memory.

Some callers of this library cannot hand it a scratch buffer: a host that owns
all device memory and passes only inputs and outputs, or a serving loop that
must not call cudaMalloc/cudaFree (they can synchronise the device and take
milliseconds). For them tk_swiglu_ffn_noalloc keeps the [m, f] activation in a
fixed 8 MiB array inside the library. This test calls it through the C ABI,
twice in a row with different inputs (the array keeps the previous call's
contents), and checks each result against tk_swiglu_ffn with a caller-provided
scratch buffer and against the float64 FFN on the host, within the FFN tolerance
of the other tests (<= 1e-3 norm-wise relative for fp16), at the 268M decoder's
shape, at a 4-row batch (the few-row kernels) and at m * f * 2 exactly equal to
the array's 8 MiB. It also checks that sizes beyond the array are rejected.
The file is named to be collected last.
"""

import numpy as np
import pytest
import torch

from tests._util import np32, rel_err, require_b200

pytestmark = pytest.mark.gpu


def _call(fn, *args):
    from tinker_b200 import _lib
    rc = fn(*args)
    if rc != _lib.TK_OK:
        raise RuntimeError(_lib.last_error())


def _ffn_oracle(x, wg, wu, wd):
    """The FFN in float64 on the host: down(silu(x gate^T) * (x up^T)) (oracle.swiglu's arithmetic)."""
    xx = np32(x).astype(np.float64)
    a = xx @ np32(wg).astype(np.float64).T
    b = xx @ np32(wu).astype(np.float64).T
    return (a / (1.0 + np.exp(-a)) * b) @ np32(wd).astype(np.float64).T


# (m, hidden, f): the 268M decoder's FFN at batch 1 x seq 128; a decode-sized batch that takes
# the few-row (GEMV) kernels; and m * f * 2 exactly the 8 MiB of the array
CASES = [(128, 1024, 2816), (4, 1024, 2816), (1024, 1024, 4096)]


@pytest.mark.parametrize("m, hidden, f", CASES)
def test_noalloc_ffn_matches_scratch_ffn_twice(m, hidden, f):
    require_b200()
    from tinker_b200 import _lib
    lib = _lib.lib()
    torch.manual_seed(11 + m)
    dev = torch.device("cuda", 0)
    wg = (0.02 * torch.randn(f, hidden, device=dev)).half()
    wu = (0.02 * torch.randn(f, hidden, device=dev)).half()
    wd = (0.02 * torch.randn(hidden, f, device=dev)).half()
    stream = torch.cuda.current_stream(dev).cuda_stream
    for call in range(2):
        x = torch.randn(m, hidden, device=dev).half()
        h = torch.empty(m, f, device=dev, dtype=torch.float16)
        ref = torch.empty(m, hidden, device=dev, dtype=torch.float16)
        out = torch.full((m, hidden), float("nan"), device=dev, dtype=torch.float16)
        _call(lib.tk_swiglu_ffn, x.data_ptr(), hidden, wg.data_ptr(), wu.data_ptr(), wd.data_ptr(),
              h.data_ptr(), ref.data_ptr(), None, m, hidden, f, _lib.TK_F16, stream)
        _call(lib.tk_swiglu_ffn_noalloc, x.data_ptr(), hidden, wg.data_ptr(), wu.data_ptr(), wd.data_ptr(),
              out.data_ptr(), None, m, hidden, f, _lib.TK_F16, stream)
        torch.cuda.synchronize()
        o, r = np32(out), np32(ref)
        assert np.isfinite(o).all(), f"call {call}: non-finite output"
        # same result as the entry point with a caller-provided buffer ...
        assert rel_err(o, r) <= 1e-3, f"call {call}"
        np.testing.assert_allclose(o, r, rtol=2e-3, atol=2e-3 * np.abs(r).max())
        # ... and as the float64 FFN (the FFN bar of the other tests: <= 1e-3 for fp16)
        assert rel_err(o, _ffn_oracle(x, wg, wu, wd)) <= 1e-3, f"call {call}"


def test_noalloc_ffn_rejects_sizes_beyond_its_array():
    require_b200()
    from tinker_b200 import _lib
    lib = _lib.lib()
    m, hidden, f = 1024, 1024, 5632  # m * f * 2 = 11.5 MB > 8 MiB
    rc = lib.tk_swiglu_ffn_noalloc(16, hidden, 16, 16, 16, 16, None, m, hidden, f, _lib.TK_F16, None)
    assert rc == _lib.TK_ERR_INVALID
    assert "scratch" in _lib.last_error()
