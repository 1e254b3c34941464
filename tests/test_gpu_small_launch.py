"""Small launches (channel shards of a multi-GPU run): with at most one or two groups per SM the default plans
run their 1- or 2-slot variants (one or two teams of 16 or 8 warps instead of four teams of four).  Both
variants of every default plan against the fp64 oracle on sampled sequences; tolerances as in the parity
tests (fp32 I/O 5e-4, bf16 I/O 3e-3, fp32 accumulation)."""
import numpy as np
import pytest
import torch

import sffft_b200 as sf

pytestmark = pytest.mark.gpu

# (L, pairs per group G) of the default plans up to 8192
DEFAULTS = [(128, 8), (256, 8), (512, 4), (1024, 4), (2048, 2), (4096, 1), (8192, 1)]


def sample_err(oracle, u, k, y, nseq=12):
    B, H, L = u.shape
    seqs = np.unique(np.linspace(0, B * H - 1, nseq).astype(np.int64))
    ref = oracle.direct_conv_seqs(u, k, seqs)
    got = y.reshape(B * H, L)[seqs].astype(np.float64)
    return float(np.sqrt(np.sum((got - ref) ** 2) / np.sum(ref ** 2)))


@pytest.mark.parametrize("L,G", DEFAULTS)
@pytest.mark.parametrize("per_sm", [1, 2])
@pytest.mark.parametrize("io", ["fp32", "bf16"])
def test_small_launch_variants(oracle, cuda_device, L, G, per_sm, io):
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    B = 8
    H = max(1, (per_sm * sms - (sms // 2 if per_sm == 2 else 0)) * G // 4)   # groups = 4H / G
    u, k = oracle.gen_profile(B, H, L, seed=L + per_sm)
    dt = torch.bfloat16 if io == "bf16" else torch.float32
    if io == "bf16":
        from tests.oracle_py import to_bf16
        u, k = to_bf16(u), to_bf16(k)
    plan = sf.Plan(L, io=io)
    Kf = plan.filter_spectrum(torch.from_numpy(k).to(cuda_device))
    y = plan.conv(torch.from_numpy(u).to(cuda_device).to(dt), Kf)
    plan.check()
    plan.close()
    err = sample_err(oracle, u, k, y.float().cpu().numpy())
    assert err <= (3e-3 if io == "bf16" else 5e-4), err
