"""The cuFFT baseline pipeline (the reference's run-time oracle) against the fp64 direct convolution."""
import numpy as np
import pytest
import torch

import sffft_b200 as sf
from tests.conftest import rel_l2

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("L", [128, 1024, 8192])
def test_cufft_pipeline(oracle, cuda_device, L):
    B, H = 2, 3
    u, k = oracle.gen_reference(B, H, L, seed=9)
    ut = torch.from_numpy(u).to(cuda_device)
    kt = torch.from_numpy(k).to(cuda_device)
    bl = sf.Baseline(L, B, H, kt)
    y = torch.empty_like(ut)
    bl.run(ut, y, full=True)
    torch.cuda.synchronize()
    assert rel_l2(y.cpu().numpy(), oracle.direct_conv(u, k)) < 2e-6
    bl.close()
