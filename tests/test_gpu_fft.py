"""Standalone real FFTs (sffft_rfft / sffft_irfft) against numpy's fp64 FFT, on one plan per length.

The reference exposes no standalone FFT (README.md:174 lists forward and inverse FFTs as not yet
exposed), so the definition is numpy.fft.rfft / irfft in fp64.  The transforms run in fp32 with exact
twiddles; the bound is 3e-6 relative L2 (fp32 rounding of two or three direct DFT digits of up to 64
terms and their twiddles; the filter-spectrum prep on the same stages holds 2e-6)."""
import numpy as np
import pytest
import torch

import sffft_b200 as sf
from tests.conftest import rel_l2
from tests.oracle_py import to_bf16

pytestmark = pytest.mark.gpu
TOL = 3e-6
PLANS = ["16x16/w4", "32x16/w8", "32x32/w8", "64x32/w8", "64x64/w8", "32x16x16/w8", "32x32x16/w8", "32x32x32/w8"]


def plan_for(name):
    R = [int(x) for x in name.split("/")[0].split("x")]
    return sf.Plan(int(np.prod(R)) // 2, io="fp32", config=name)


@pytest.mark.parametrize("name", PLANS)
def test_rfft_irfft_match_numpy(cuda_device, name):
    plan = plan_for(name)
    N = plan.N
    rng = np.random.default_rng(N)
    x = rng.standard_normal((3, N)).astype(np.float32)
    X = plan.rfft(torch.from_numpy(x).to(cuda_device))
    Xn = np.fft.rfft(x.astype(np.float64), axis=-1)
    assert rel_l2(X.cpu().numpy(), Xn) <= TOL
    # inverse of an arbitrary half spectrum (not only of a real signal's)
    Z = (rng.standard_normal((2, 4, N // 2 + 1)) + 1j * rng.standard_normal((2, 4, N // 2 + 1))).astype(np.complex64)
    z = plan.irfft(torch.from_numpy(Z).to(cuda_device))
    assert z.shape == (2, 4, N)
    assert rel_l2(z.cpu().numpy(), np.fft.irfft(Z.astype(np.complex128), n=N, axis=-1)) <= TOL
    # round trip
    xr = plan.irfft(X)
    assert rel_l2(xr.cpu().numpy(), x) <= TOL
    plan.close()


@pytest.mark.parametrize("name", ["16x16/w4", "64x32/w8", "32x16x16/w8"])
def test_rfft_bf16_input(cuda_device, name):
    plan = plan_for(name)
    N = plan.N
    x = to_bf16(np.random.default_rng(1).standard_normal((5, N)).astype(np.float32))
    X = plan.rfft(torch.from_numpy(x).to(cuda_device).to(torch.bfloat16))
    assert rel_l2(X.cpu().numpy(), np.fft.rfft(x.astype(np.float64), axis=-1)) <= TOL
    plan.close()


def test_irfft_ignores_imaginary_parts_of_dc_and_nyquist(cuda_device):
    plan = plan_for("64x32/w8")
    N = plan.N
    rng = np.random.default_rng(2)
    Z = (rng.standard_normal((3, N // 2 + 1)) + 1j * rng.standard_normal((3, N // 2 + 1))).astype(np.complex64)
    Z0 = Z.copy()
    Z0[:, 0] = Z0[:, 0].real
    Z0[:, -1] = Z0[:, -1].real
    a = plan.irfft(torch.from_numpy(Z).to(cuda_device))
    b = plan.irfft(torch.from_numpy(Z0).to(cuda_device))
    assert torch.equal(a, b)
    plan.close()


def test_fft_arguments_are_checked(cuda_device):
    plan = plan_for("16x16/w4")
    with pytest.raises(ValueError):
        plan.rfft(torch.zeros((2, 128), device=cuda_device))           # N = 256 samples per row
    with pytest.raises(ValueError):
        plan.irfft(torch.zeros((2, 129), dtype=torch.complex64, device=cuda_device)[:, :128])
    with pytest.raises(ValueError):
        plan.rfft(torch.zeros((2, 256), device=cuda_device), work=torch.empty(16, device=cuda_device))
    lib = sf.lib()
    x = torch.zeros((2, 256), device=cuda_device)
    X = torch.empty((2, 129), dtype=torch.complex64, device=cuda_device)
    w = torch.empty((2, 256, 2), device=cuda_device)
    assert lib.sffft_rfft(plan._h, x.data_ptr(), 7, 2, X.data_ptr(), w.data_ptr(), None) == sf.ERR_INVALID_ARGUMENT
    assert lib.sffft_rfft(plan._h, x.data_ptr(), 0, 2, X.data_ptr(), None, None) == sf.ERR_INVALID_ARGUMENT
    assert lib.sffft_irfft(plan._h, X.data_ptr(), 0, x.data_ptr(), w.data_ptr(), None) == sf.ERR_INVALID_ARGUMENT
    plan.close()
