"""Filter-spectrum prep kernel vs the fp64 digit-order restatement of cufftExecC2C + permuteK."""
import numpy as np
import pytest
import torch

import sffft_b200 as sf
from tests.oracle_py import spectrum_digit_order, to_bf16

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", ["16x16/w4", "32x16/w4", "16x64/w4", "64x32/w4", "64x64/w4", "16x16x16/w4",
                                  "32x16x16/w4", "16x32x32/w4", "16x16x64/w8", "32x32x32/w4"])
def test_spectrum_digit_order(oracle, cuda_device, name):
    R = [int(x) for x in name.split("/")[0].split("x")]
    L = int(np.prod(R)) // 2
    _, k = oracle.gen_profile(1, 3, L, seed=3)
    plan = sf.Plan(L, config=name)
    Kf = plan.filter_spectrum(torch.from_numpy(k).to(cuda_device)).cpu().numpy()
    ref = spectrum_digit_order(k, R)
    got = Kf[..., 0] + 1j * Kf[..., 1]
    assert np.linalg.norm(got - ref) / np.linalg.norm(ref) < 2e-6


def test_spectrum_from_bf16_filter(oracle, cuda_device):
    _, k = oracle.gen_profile(1, 2, 1024, seed=4)
    kb = to_bf16(k)
    plan = sf.Plan(1024, io="bf16", config="64x32/w4")
    Kf = plan.filter_spectrum(torch.from_numpy(k).to(cuda_device).to(torch.bfloat16)).cpu().numpy()
    ref = spectrum_digit_order(kb, [64, 32])
    got = Kf[..., 0] + 1j * Kf[..., 1]
    assert np.linalg.norm(got - ref) / np.linalg.norm(ref) < 2e-6
