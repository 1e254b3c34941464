"""The sffft CLI against the reference's behavioural contract (sfFFT tests/precision_smoke.sh): exit codes,
unattainable budgets, I/O isolation, seeds, fp16 overflow rejection, allocator modes and the 112 + 112
RESULT rows of --kernel auto.  The exit-code-1 cases need no GPU and live in test_cli_args.py."""
import os
import subprocess

import pytest

import sffft_b200 as sf

pytestmark = pytest.mark.gpu


def run(*args, timeout=900):
    p = subprocess.run([sf.CLI_PATH] + [str(a) for a in args], capture_output=True, text=True, timeout=timeout)
    return p.returncode, p.stdout


def rows(out, kind):
    return [l.split(",") for l in out.splitlines() if l.split(",")[0] == kind]


def fval(s):
    return float(s)


def test_unattainable_budgets_exit_2():
    rc, out = run(1, 1, 128, "--max-error", "1e-8", "--io", "fp32")
    assert rc == 2 and any(r[1] == "128" and r[2] == "fp32" for r in rows(out, "NO_MATCH"))
    rc, out = run(1, 1, 128, "--max-error", "1e-3", "--io", "bf16")
    assert rc == 2 and any(r[1] == "128" and r[2] == "bf16" for r in rows(out, "NO_MATCH"))


@pytest.mark.parametrize("seed", [42, 12345])
def test_seeds_select_every_length(seed):
    rc, out = run(1, 1, "--max-error", "1e-3", "--io", "fp32", "--seed", seed)
    sel = rows(out, "SELECT")
    assert rc == 0 and len(sel) == 7
    assert all(fval(r[5]) <= fval(r[6]) and r[7] == "fp32" for r in sel)


def test_fp16_overflow_rejected():
    rc, out = run(1, 1, 128, "--max-error", "1e-3", "--io", "fp32", "--input-scale", "15000")
    rejected = [r for r in rows(out, "RESULT") if "fp16acc" in r[2] and ("nan" in r[5] or "inf" in r[5])]
    sel = rows(out, "SELECT")
    assert rc == 0 and rejected and len(sel) == 1
    assert sel[0][2] == "fused_fp32io" and fval(sel[0][5]) <= fval(sel[0][6])
    rc, out = run(1, 1, 128, "--max-error", "1e-3", "--io", "fp32", "--input-scale", "25000")
    assert rc == 2 and any(r[1] == "128" and r[2] == "fp32" for r in rows(out, "NO_MATCH"))


@pytest.mark.parametrize("allocator", ["device", "managed", "mapped", "hybrid"])
def test_allocators_with_cached_kernels(allocator):
    rc, out = run(1, 1, "--max-error", "1e-3", "--io", "fp32", "--allocator", allocator, "--kernel", "cached")
    assert rc == 0
    for r in rows(out, "RESULT"):
        if r[2].startswith("fused"):
            assert "nan" not in r[5] and "inf" not in r[5]
            assert fval(r[5]) <= (6e-3 if "bf16io" in r[2] else 2e-3)
    sel = rows(out, "SELECT")
    assert len(sel) == 7 and all(fval(r[5]) <= fval(r[6]) and r[7] == "fp32" and "kernel_cached" in r[3] for r in sel)
    mem = rows(out, "MEMORY")
    assert len(mem) == 7
    for m in mem:
        assert m[2] == allocator
        if allocator != "device":
            assert int(m[7]) == 0 and int(m[4]) == 0          # no downloads, no persistent host shadows
        if allocator in ("managed", "mapped"):
            assert int(m[6]) == 0                             # no explicit uploads


@pytest.mark.parametrize("seed", [42, 12345])
def test_auto_kernel_row_counts(seed):
    rc, out = run(1, 1, "--max-error", "1e-3", "--io", "fp32", "--kernel", "auto", "--seed", seed)
    res = rows(out, "RESULT")
    fused = [r for r in res if r[2].startswith("fused")]
    assert all("nan" not in r[5] and fval(r[5]) <= (6e-3 if "bf16io" in r[2] else 2e-3) for r in fused)
    assert sum("kernel_cached" in r[3] for r in res) == 112
    assert sum("kernel_legacy" in r[3] for r in res) == 112
    sel = rows(out, "SELECT")
    assert rc == 0 and len(sel) == 7 and all(fval(r[5]) <= fval(r[6]) and r[7] == "fp32" for r in sel)


def test_cached_overflow_rejected():
    rc, out = run(1, 1, 128, "--max-error", "1e-3", "--io", "fp32", "--kernel", "cached", "--input-scale", "15000")
    assert rc == 0
    assert any("fp16acc" in r[2] and ("nan" in r[5] or "inf" in r[5]) for r in rows(out, "RESULT"))
    sel = rows(out, "SELECT")
    assert len(sel) == 1 and sel[0][2] == "fused_fp32io"


def test_long_length_and_headers():
    rc, out = run(2, 2, 16384)
    assert rc == 0
    assert out.startswith("# MEMORY_CAPS,")
    res = rows(out, "RESULT")
    assert {r[1] for r in res} == {"16384"}
    assert any(r[2] == "cufft_pipeline_fp32" for r in res)
    assert all(fval(r[5]) <= (6e-3 if "bf16io" in r[2] else 2e-3) for r in res if r[2].startswith("fused"))


def test_cufft_rows_match_reference_generator(oracle):
    # the calibration inputs are the reference's: the cuFFT-vs-fp64 error of the first sampled sequences
    # is reproduced by the oracle on the same seeded inputs
    rc, out = run(1, 1, 256, "--seed", 42)
    res = [r for r in rows(out, "RESULT") if r[2] == "cufft_pipeline_fp32"]
    assert rc == 0 and len(res) == 1 and fval(res[0][5]) < 1e-6
