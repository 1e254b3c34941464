"""Test configuration.  `-m gpu` tests need a B200 and the built native library; everything else runs
on CPU (the oracle, the host logic, the C-ABI surface, the CPU emulator of the kernel)."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU and the built CUDA library")


@pytest.fixture(scope="session")
def oracle():
    from tests.oracle_py import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a visible CUDA device")
    return torch.device("cuda:0")


def rel_l2(a, b):
    cplx = np.iscomplexobj(a) or np.iscomplexobj(b)
    a = np.asarray(a, dtype=np.complex128 if cplx else np.float64)
    b = np.asarray(b, dtype=np.complex128 if cplx else np.float64)
    d = float(np.sum(np.abs(a - b) ** 2))
    r = float(np.sum(np.abs(b) ** 2))
    if r > 0:
        return (d / r) ** 0.5
    return 0.0 if d == 0 else float("inf")
