"""The oracle pinned to the reference itself: the reference benchmark (src/sffft.cu, compiled in place for
sm_100a into oracle/_ref/ref_harness by oracle/Makefile) and this repository's CLI run the same calibration
on the same device.  Both draw their inputs from the reference generator (src/sffft.cu:308-310,339-341) and
score the cuFFT fp32 pipeline (:365-371) against an fp64 direct convolution (:376-378), so identical
`cufft_pipeline_fp32` errors mean the generator, the fp64 oracle and the error metric here reproduce the
reference's to the printed digits.  The fused rows of both programs must meet the reference's own smoke-test
bounds (tests/precision_smoke.sh:62,73) and cover the same (method, plan) candidates."""
import os
import subprocess

import pytest

import sffft_b200 as sf

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "oracle", "_ref", "ref_harness")


def rows(cmd):
    p = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
    assert p.returncode == 0, p.stdout[-2000:] + p.stderr[-2000:]
    return [l.split(",") for l in p.stdout.splitlines() if l.startswith("RESULT,")]


@pytest.mark.skipif(not os.path.exists(REF), reason="reference binary not built (make -C oracle ref)")
@pytest.mark.parametrize("L", [128, 1024, 8192])
def test_cufft_rows_equal_the_reference_binary(L):
    B, H = 2, 3
    ours = rows([sf.CLI_PATH, str(B), str(H), str(L)])
    ref = rows([REF, "run", str(B), str(H), str(L)])
    for method in ("cufft_pipeline_fp32", "cufft_core_fp32"):
        a = [r[5] for r in ours if r[2] == method]
        b = [r[5] for r in ref if r[2] == method]
        assert a and a == b, (method, a, b)
    # the same candidates (method, plan/warps) are calibrated by both programs
    key = lambda r: (r[2], "/".join(r[3].split("/")[:2]))
    assert sorted(key(r) for r in ours if r[2].startswith("fused")) == \
        sorted(key(r) for r in ref if r[2].startswith("fused"))
    for r in ours:
        if r[2].startswith("fused"):
            assert float(r[5]) <= (6e-3 if "bf16io" in r[2] else 2e-3), r
