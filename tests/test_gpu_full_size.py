"""Parity at the benchmark configurations' full sizes, with the plan each configuration names.

Every output is compared with the cuFFT fp32 pipeline on the device (the reference's own run-time oracle,
src/sffft.cu:365-371), and sampled sequences with the fp64 direct convolution (src/sffft.cu:376-378).
Inputs follow the configurations' distributions (oracle.gen_profile: u ~ N(0,1), k = N(0,1) exp(-d n/L),
divided by sqrt(L) where the configuration says so); bf16 configurations round u and k to bf16 and give
both references the rounded values.  Tolerances (relative L2): fp32 I/O 5e-4, bf16 I/O 3e-3, bf16 I/O with
fp16 accumulation 4e-3 (the separately stated bound).  A size-independent property closes each case: the
convolution is linear, so y(2u) / 2 matches y(u) to within the fp16 rounding of the smallest (subnormal)
intermediates, far inside the tolerance."""
import numpy as np
import pytest
import torch

import sffft_b200 as sf
from tests.conftest import rel_l2
from tests.oracle_py import to_bf16

pytestmark = pytest.mark.gpu

# (B, H, L, io, acc, plan, decay, sqrt_norm, tolerance)
CONFIGS = {
    "configs0": (1, 1, 128, "fp32", "fp32", "16x16/w4", 4.0, False, 5e-4),
    "configs1": (8, 768, 1024, "fp32", "fp32", "64x32/w8", 4.0, True, 5e-4),
    "configs2": (8, 768, 4096, "bf16", "fp32", "32x16x16/w8", 4.0, True, 3e-3),
    "configs3": (8, 768, 8192, "bf16", "fp16", "32x32x16/w8", 4.0, True, 4e-3),
    "configs4": (16, 1024, 16384, "fp32", "fp32", "32x32x32/w8", 8.0, True, 5e-4),
}


@pytest.mark.parametrize("name", list(CONFIGS))
def test_baseline_config_full_size(oracle, cuda_device, name):
    B, H, L, io, acc, plan_name, decay, sqrt_norm, tol = CONFIGS[name]
    u, k = oracle.gen_profile(B, H, L, decay=decay, sqrt_norm=sqrt_norm, seed=21)
    if io == "bf16":
        u, k = to_bf16(u), to_bf16(k)
    dt = torch.bfloat16 if io == "bf16" else torch.float32
    ut32 = torch.from_numpy(u).to(cuda_device)
    kt32 = torch.from_numpy(k).to(cuda_device)
    plan = sf.Plan(L, io=io, acc=acc, config=plan_name)
    Kf = plan.filter_spectrum(kt32.to(dt))
    y = plan.conv(ut32.to(dt), Kf)
    plan.check()
    y32 = y.float()
    # all outputs against the cuFFT fp32 pipeline
    bl = sf.Baseline(L, B, H, kt32)
    yc = torch.empty_like(ut32)
    bl.run(ut32, yc, full=True)
    torch.cuda.synchronize()
    bl.close()
    err_cufft = (torch.linalg.norm((y32 - yc).double()) / torch.linalg.norm(yc.double())).item()
    assert err_cufft <= tol, f"vs cuFFT pipeline: {err_cufft:.3e}"
    # sampled sequences against the fp64 direct convolution
    total = B * H
    seqs = np.unique(np.linspace(0, total - 1, min(total, 12)).astype(np.int64))
    ref = oracle.direct_conv_seqs(u, k, seqs)
    got = y32.reshape(total, L)[torch.from_numpy(seqs).to(cuda_device)].double().cpu().numpy()
    assert rel_l2(got, ref) <= tol, f"vs fp64 on {len(seqs)} sequences: {rel_l2(got, ref):.3e}"
    # linearity: doubling the input doubles every output up to the rounding of subnormal fp16 intermediates
    y2 = plan.conv((2 * ut32).to(dt), Kf).float()
    plan.check()
    err_lin = (torch.linalg.norm((y2 / 2 - y32).double()) / torch.linalg.norm(y32.double())).item()
    assert err_lin <= tol / 10, f"linearity: {err_lin:.3e}"
    plan.close()
