"""Per-row accuracy when the two batch rows that share one complex transform differ greatly in size.

The reference transforms every (b, h) row alone (sfFFT src/sffft.cu:249); here rows 2j and 2j+1 of a channel
share one transform, so each row is scaled by a power of two before the fp16 stages (the kernel measures the
rows' energies while converting them) and unscaled in the output epilogue.  Every single row must meet the
tolerance of its I/O and accumulation mode against the fp64 direct convolution (relative L2: fp32 I/O 5e-4,
bf16 I/O 3e-3 with fp32 accumulation; 1e-3 / 4e-3 with fp16 accumulation), including rows 1e3 and 1e4 below
their partner, an all-zero row beside a full-scale one (whose output must be exactly zero) and a pair of
tiny rows (rms 1e-5)."""
import numpy as np
import pytest
import torch

import sffft_b200 as sf
from tests.oracle_py import PAIR_SCALES, per_row_rel_l2, scaled_pair_inputs

pytestmark = pytest.mark.gpu
TOL = {("fp32", "fp32"): 5e-4, ("bf16", "fp32"): 3e-3, ("fp32", "fp16"): 1e-3, ("bf16", "fp16"): 4e-3}


@pytest.mark.parametrize("name", ["64x32/w8", "16x16/w4", "32x16x16/w8", "32x32x16/w8"])
@pytest.mark.parametrize("io,acc", [("fp32", "fp32"), ("bf16", "fp32"), ("fp32", "fp16"), ("bf16", "fp16")])
def test_every_row_within_tolerance(oracle, cuda_device, name, io, acc):
    R = [int(x) for x in name.split("/")[0].split("x")]
    L = int(np.prod(R)) // 2
    H = 3
    u, k = scaled_pair_inputs(oracle, H, L, io, seed=31)
    plan = sf.Plan(L, io=io, acc=acc, config=name)
    dt = torch.bfloat16 if io == "bf16" else torch.float32
    Kf = plan.filter_spectrum(torch.from_numpy(k).to(cuda_device))
    y = plan.conv(torch.from_numpy(u).to(cuda_device).to(dt), Kf)
    plan.check()
    plan.close()
    y = y.float().cpu().numpy()
    errs = per_row_rel_l2(y, oracle.direct_conv(u, k))
    assert errs.shape == (len(PAIR_SCALES), H)
    assert np.all(errs <= TOL[(io, acc)]), f"per-row relative L2 (rows x channels):\n{errs}"
    zero_rows = [b for b, s in enumerate(PAIR_SCALES) if s == 0.0]
    assert zero_rows and not y[zero_rows].any()


def test_balanced_batches_are_unchanged_by_a_scaled_neighbour(oracle, cuda_device):
    # a pair's scaling is decided per pair: rescaling one pair of a group leaves the other pairs' outputs
    # bit-identical
    L, B, H = 1024, 8, 2
    u, k = oracle.gen_profile(B, H, L, seed=41)
    plan = sf.Plan(L, config="64x32/w8")
    Kf = plan.filter_spectrum(torch.from_numpy(k).to(cuda_device))
    y1 = plan.conv(torch.from_numpy(u).to(cuda_device), Kf).cpu()
    u2 = u.copy()
    u2[1] *= 1e-3                                      # pair (0, 1) now needs rescaling
    y2 = plan.conv(torch.from_numpy(u2).to(cuda_device), Kf).cpu()
    plan.check()
    plan.close()
    assert torch.equal(y1[2:], y2[2:])
