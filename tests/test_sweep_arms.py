"""The standalone sweep's comparison arm that runs the reference's own Triton kernels: it loads the
reference package installed under baseline/_ref (not this repository's ``tinker`` alias), leaves the
alias in place for everything else, and says why when it cannot run."""

import os
import sys

import pytest

import bench_sweep


def test_disabled_and_missing_reference_say_why(monkeypatch, tmp_path):
    assert bench_sweep._RefTriton(False).why.startswith("skipped")
    monkeypatch.setattr(bench_sweep, "ROOT", str(tmp_path))
    t = bench_sweep._RefTriton(True)
    assert t.rms is None and "not installed" in t.why


def test_reference_arm_loads_the_installed_reference_not_the_alias():
    ref = os.path.join(bench_sweep.ROOT, "baseline", "_ref", "tinker")
    if not os.path.isdir(ref):
        pytest.skip("the reference is not installed under baseline/_ref")
    pytest.importorskip("triton")
    import tinker  # this repository's alias of tinker_b200, imported first on purpose
    alias = sys.modules["tinker"]
    t = bench_sweep._RefTriton(True)
    assert t.why is None
    for m in (t.rms, t.swiglu, t.attn, t.opt):
        assert os.path.abspath(m.__file__).startswith(os.path.abspath(ref))
    assert sys.modules["tinker"] is alias and tinker.optimize is sys.modules["tinker_b200"].optimize
