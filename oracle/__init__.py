"""CPU oracle for the TinKer fused-kernel path.

TEST INFRASTRUCTURE ONLY. This package restates, in numpy, the reference's
eager PyTorch algorithm for every function on the hot path (RoPE tables,
interleaved RoPE, causal GQA attention, RMSNorm, SwiGLU and the Llama-style
decoder forward the reference benchmarks), plus the rows of that attention a
KV-cache decode step returns (``attention_rows``, pinned to ``attention``). It is the checker that the CUDA
path is compared against, and the CPU baseline that ``bench.py`` times. Only
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs may import
it; the product package ``tinker_b200`` never does.

Parity pinning: ``tests/golden/`` holds vectors produced by importing the
reference implementation itself (eb1386/TinKer, ``tinker/kernels/*.py`` and
``benchmarks/bench_e2e.py``) together with the script that made them, and
``tests/test_oracle_golden.py`` checks this oracle against every one of them.
"""

from oracle.ops import (  # noqa: F401
    round_to,
    rope_tables,
    apply_rope,
    attention,
    attention_rows,
    rmsnorm,
    add_rmsnorm,
    swiglu,
    linear,
)
from oracle.model import ModelConfig, forward_logits  # noqa: F401
