"""Non-causal (two-sided) and circular convolution: the same fused kernel with the spectrum of the filter
laid out over the N = 2L taps (sffft_filter_spectrum_ex), checked against the oracle's fp64 direct sums.

The reference exposes only the causal form and lists these two as not yet exposed (README.md:174), so
parity here is against the fp64 definition, with the causal path's tolerances (relative L2): fp32 I/O
5e-4, bf16 I/O 3e-3 (u and k rounded to bf16 and given to the oracle rounded), fp16 accumulation 4e-3 for
bf16 I/O.  Two exact properties close it: a two-sided filter whose negative lags are zero has the causal
filter's spectrum bit for bit, and a circular filter that is an impulse at lag s rotates the input by s."""
import numpy as np
import pytest
import torch

import sffft_b200 as sf
from tests.conftest import rel_l2
from tests.oracle_py import to_bf16

pytestmark = pytest.mark.gpu
TOL = {("fp32", "fp32"): 5e-4, ("bf16", "fp32"): 3e-3, ("bf16", "fp16"): 4e-3}

# one plan per length, two- and three-stage, both warp counts
PLANS = ["16x16/w4", "32x16/w8", "32x32/w4", "64x32/w8", "64x64/w8", "16x16x16/w4", "32x16x16/w8",
         "32x32x16/w8", "32x32x32/w8"]


def filters(H, L, layout, seed):
    rng = np.random.default_rng(seed)
    if layout == "two_sided":
        lag = np.abs(np.arange(2 * L - 1) - (L - 1))
        return (rng.standard_normal((H, 2 * L - 1)) * np.exp(-4.0 * lag / L) / np.sqrt(L)).astype(np.float32)
    return (rng.standard_normal((H, L)) * np.exp(-4.0 * np.arange(L) / L) / np.sqrt(L)).astype(np.float32)


def run(plan, u, k, layout, dev):
    dt = torch.bfloat16 if plan.io == "bf16" else torch.float32
    Kf = plan.filter_spectrum(torch.from_numpy(k).to(dev), layout=layout)
    y = plan.conv(torch.from_numpy(u).to(dev).to(dt), Kf)
    plan.check()
    return y.float().cpu().numpy()


@pytest.mark.parametrize("layout", ["two_sided", "circular"])
@pytest.mark.parametrize("name", PLANS)
@pytest.mark.parametrize("io,acc", [("fp32", "fp32"), ("bf16", "fp32"), ("bf16", "fp16")])
def test_layout_matches_fp64(oracle, cuda_device, name, layout, io, acc):
    R = [int(x) for x in name.split("/")[0].split("x")]
    L = int(np.prod(R)) // 2
    B, H = 3, 5                      # odd B: the last batch row has no partner
    rng = np.random.default_rng(L)
    u = rng.standard_normal((B, H, L)).astype(np.float32)
    k = filters(H, L, layout, seed=L + 1)
    if io == "bf16":
        u, k = to_bf16(u), to_bf16(k)
    plan = sf.Plan(L, io=io, acc=acc, config=name)
    y = run(plan, u, k, layout, cuda_device).reshape(B * H, L)
    plan.close()
    seqs = np.arange(B * H) if L <= 4096 else np.array([0, 7, 14])
    ref = oracle.direct_conv_layout_seqs(u, k, layout, seqs)
    err = rel_l2(y[seqs], ref)
    assert err <= TOL[(io, acc)], f"{name} {layout} {io}/{acc}: {err:.3e}"


@pytest.mark.parametrize("name", ["16x16/w8", "64x32/w8", "32x16x16/w8"])
def test_two_sided_with_zero_negative_lags_is_causal(cuda_device, name):
    R = [int(x) for x in name.split("/")[0].split("x")]
    L = int(np.prod(R)) // 2
    H = 4
    k = filters(H, L, "circular", seed=5)          # a one-sided decaying filter
    k2 = np.concatenate([np.zeros((H, L - 1), np.float32), k], axis=1)
    plan = sf.Plan(L, io="fp32", config=name)
    Kc = plan.filter_spectrum(torch.from_numpy(k).to(cuda_device))
    K2 = plan.filter_spectrum(torch.from_numpy(k2).to(cuda_device), layout="two_sided")
    torch.cuda.synchronize()
    plan.close()
    assert torch.equal(Kc, K2)


@pytest.mark.parametrize("name", ["16x16/w4", "64x32/w8", "32x16x16/w8"])
def test_circular_impulse_rotates(cuda_device, name):
    R = [int(x) for x in name.split("/")[0].split("x")]
    L = int(np.prod(R)) // 2
    B, H = 2, 3
    shifts = [1, L // 3, L - 1]
    k = np.zeros((H, L), np.float32)
    for h, s in enumerate(shifts):
        k[h, s] = 1.0
    u = np.random.default_rng(9).standard_normal((B, H, L)).astype(np.float32)
    plan = sf.Plan(L, io="fp32", config=name)
    y = run(plan, u, k, "circular", cuda_device)
    plan.close()
    for h, s in enumerate(shifts):
        ref = np.roll(u[:, h, :], s, axis=1)
        assert rel_l2(y[:, h, :], ref) <= 5e-4, f"shift {s}"


def test_layout_arguments_are_checked(cuda_device):
    plan = sf.Plan(128, io="fp32", config="16x16/w4")
    with pytest.raises(ValueError):
        plan.filter_spectrum(torch.zeros((2, 128), device=cuda_device), layout="two_sided")   # needs 255 taps
    with pytest.raises(ValueError):
        plan.filter_spectrum(torch.zeros((2, 255), device=cuda_device), layout="circular")
    with pytest.raises(ValueError):
        plan.filter_spectrum(torch.zeros((2, 128), device=cuda_device), layout="acausal")
    lib = sf.lib()
    k = torch.zeros((2, 128), device=cuda_device)
    Kf = torch.empty((2, 256, 2), device=cuda_device)
    assert lib.sffft_filter_spectrum_ex(plan._h, k.data_ptr(), 0, 3, 2, Kf.data_ptr(), None) == sf.ERR_INVALID_ARGUMENT
    plan.close()
