"""The plan selector through the C ABI, on the cases of the reference's own unit test
(tests/selection_test.cpp:3-21 of sfFFT), and the compiled reference test itself when present."""
import math
import os
import subprocess

import pytest

import sffft_b200 as sf

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
nan, inf = float("nan"), float("inf")


def cands():
    C = sf.Candidate
    return [C("strict", "fp32", "p0", 2.0, 0.0004), C("relaxed", "fp32", "p1", 1.0, 0.003),
            C("bf16", "bf16", "p2", 0.5, 0.006), C("nan_error", "fp32", "p3", 0.01, nan),
            C("inf_error", "fp32", "p4", 0.01, inf), C("nan_time", "fp32", "p5", nan, 0),
            C("zero_time", "fp32", "p6", 0, 0), C("negative_error", "fp32", "p7", 0.01, -1)]


def test_selection_cases():
    c = cands()
    s = sf.select_candidate
    assert s(c, 0.001, "fp32") == 0
    assert s(c, 0.01, "fp32") == 1
    assert s(c, 0.01, "bf16") == 2
    assert s(c, 0.01, "any") == 2
    assert s(c, 0.0004, "fp32") == 0
    assert s(c, 0.0001, "fp32") is None
    assert s(c, 0.001, "bf16") is None
    for bad in (nan, inf, -1, 0):
        assert s(c, bad, "fp32") is None
    assert s(c, 0.01, "unknown") is None
    assert s([], 0.01, "fp32") is None
    c.append(sf.Candidate("tie", "fp32", "p8", 1.0, 0.002))
    assert s(c, 0.01, "fp32") == len(c) - 1


def test_relative_l2():
    assert sf.relative_l2(0, 0) == 0
    assert math.isinf(sf.relative_l2(1, 0))
    assert sf.relative_l2(1, 100) == 0.1


def test_reference_selection_test_binary():
    exe = os.path.join(ROOT, "oracle", "_ref", "selection_test")
    if not os.path.exists(exe):
        pytest.skip("reference selection_test not built here (needs the reference tree: make -C oracle ref)")
    out = subprocess.run([exe], capture_output=True, text=True)
    assert out.returncode == 0 and "PASS" in out.stdout
