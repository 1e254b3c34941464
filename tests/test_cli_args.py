"""CLI argument validation (exit codes of sfFFT tests/precision_smoke.sh:20-35); these paths exit before any
CUDA call, so they run without a GPU."""
import subprocess

import pytest

import sffft_b200 as sf


def code(*args):
    return subprocess.run([sf.CLI_PATH] + [str(a) for a in args], capture_output=True, text=True).returncode


def test_help():
    assert code("--help") == 0
    assert code("-h") == 0


@pytest.mark.parametrize("args", [
    ["--max-error", v] for v in ("nan", "inf", "0", "-1", "1e-999", "garbage")] + [
    ["--max-error"], ["--io", "unknown"], ["--seed", "0"], ["--seed", "-1"], ["--input-scale", "inf"],
    ["--input-scale", "0"], ["--allocator", "unknown"], ["--allocator"], ["--kernel", "unknown"], ["--kernel"],
    ["0", "1", "128"], ["1", "0", "128"], ["1", "1", "129"], ["2147483647", "2", "128"], ["1", "1", "32768"],
    ["1", "2", "3", "4"], ["x"]])
def test_invalid_arguments_exit_1(args):
    assert code(*args) == 1
