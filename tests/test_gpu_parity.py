"""Parity of the fused B200 kernel (through the C ABI) with the fp64 oracle on seeded inputs.

Tolerances (relative L2 over all outputs), those of the benchmark configurations: fp32 I/O <= 5e-4 and bf16 I/O <= 3e-3 with
fp32 accumulation; the fp16-accumulation mode is held to 1e-3 (fp32 I/O) and 4e-3 (bf16 I/O).  bf16 cases
round u and k to bf16 and give the oracle those rounded values."""
import numpy as np
import pytest
import torch

import sffft_b200 as sf
from tests.conftest import rel_l2
from tests.oracle_py import spectrum_digit_order, to_bf16

pytestmark = pytest.mark.gpu
TOL = {("fp32", "fp32"): 5e-4, ("bf16", "fp32"): 3e-3, ("fp32", "fp16"): 1e-3, ("bf16", "fp16"): 4e-3}


def run_gpu(plan, u, k, dev):
    dt = torch.bfloat16 if plan.io == "bf16" else torch.float32
    ut = torch.from_numpy(u).to(dev).to(dt)
    kt = torch.from_numpy(k).to(dev)
    Kf = plan.filter_spectrum(kt)
    y = plan.conv(ut, Kf)
    plan.check()
    return y.float().cpu().numpy(), Kf


def case(oracle, dev, name, B, H, io="fp32", acc="fp32", kernel="cached", seed=0):
    R = [int(x) for x in name.split("/")[0].split("x")]
    L = int(np.prod(R)) // 2
    u, k = oracle.gen_profile(B, H, L, decay=4.0, sqrt_norm=True, seed=seed + 11)
    if io == "bf16":
        u, k = to_bf16(u), to_bf16(k)
    plan = sf.Plan(L, io=io, acc=acc, config=name, kernel=kernel)
    y, _ = run_gpu(plan, u, k, dev)
    plan.close()
    return rel_l2(y, oracle.direct_conv(u, k))


CATALOG = [n for L, n in sf.catalog()] if True else []


@pytest.mark.parametrize("name", CATALOG)
@pytest.mark.parametrize("io,acc", [("fp32", "fp32"), ("bf16", "fp32"), ("fp32", "fp16"), ("bf16", "fp16")])
def test_every_plan(oracle, cuda_device, name, io, acc):
    N = int(np.prod([int(x) for x in name.split("/")[0].split("x")]))
    B, H = (4, 3) if N <= 4096 else (2, 2)
    assert case(oracle, cuda_device, name, B, H, io, acc) <= TOL[(io, acc)]


@pytest.mark.parametrize("name", ["16x16/w4", "64x32/w8", "32x16x16/w4", "16x16x64/w8"])
def test_legacy_matrices_match(oracle, cuda_device, name):
    # in-kernel DFT matrices ("legacy", sincospif) and the cached table give the same accuracy
    a = case(oracle, cuda_device, name, 2, 2, kernel="legacy")
    b = case(oracle, cuda_device, name, 2, 2, kernel="cached")
    assert a <= 5e-4 and b <= 5e-4 and abs(a - b) < 1e-4


@pytest.mark.parametrize("B,H", [(1, 1), (5, 3), (7, 9), (2, 33)])
def test_ragged_batches(oracle, cuda_device, B, H):
    # odd B (unpaired last sequence), partial last CTA, several channels per CTA
    for name in ["16x16/w4", "32x32/w4", "64x32/w4"]:
        assert case(oracle, cuda_device, name, B, H) <= 5e-4


def test_results_do_not_depend_on_neighbours(oracle, cuda_device):
    # a sequence's output is the same whatever its pair partner and CTA neighbours hold
    L = 1024
    u, k = oracle.gen_profile(4, 2, L, seed=5)
    plan = sf.Plan(L, config="64x32/w4")
    y1, _ = run_gpu(plan, u, k, cuda_device)
    u2 = u.copy()
    u2[1] *= 0.0
    u2[3] = np.random.default_rng(1).standard_normal(u2[3].shape).astype(np.float32)
    y2, _ = run_gpu(plan, u2, k, cuda_device)
    # b=0 and b=2 unchanged: outputs within fp16-pipeline noise of each other
    for b in (0, 2):
        assert rel_l2(y2[b], y1[b]) < 1e-3
    assert np.abs(y2[1]).max() < 1e-2 * np.abs(y1[1]).max()


def test_zero_input_gives_zero(cuda_device):
    plan = sf.Plan(256, config="32x16/w4")
    u = torch.zeros((2, 3, 256), device=cuda_device)
    k = torch.randn((3, 256), device=cuda_device)
    y = plan.conv(u, plan.filter_spectrum(k))
    plan.check()
    assert torch.count_nonzero(y).item() == 0


def test_invalid_calls_fail_cleanly(cuda_device):
    plan = sf.Plan(128)
    u = torch.zeros((2, 1, 128), device=cuda_device)
    Kf = torch.zeros((1, 256, 2), device=cuda_device)
    lib = sf.lib()
    assert lib.sffft_conv(plan._h, u.data_ptr() + 4, Kf.data_ptr(), u.data_ptr(), 2, 1, None) == sf.ERR_INVALID_ARGUMENT
    assert lib.sffft_conv(plan._h, u.data_ptr(), Kf.data_ptr(), u.data_ptr(), 0, 1, None) == sf.ERR_INVALID_ARGUMENT
    with pytest.raises(sf.SffftError):
        sf.Plan(128, config="64x32/w4")
    plan.check()


@pytest.mark.parametrize("L", [1024, 4096])
def test_back_to_back_calls_on_one_stream(cuda_device, L):
    # each fused launch may start its prologue while the stream's previous kernel finishes, but reads its input only
    # after that kernel has completed: a chain y3 = conv(conv(conv(u))), with torch kernels in between that rewrite
    # the next input, issued without synchronisation, equals the same calls made one at a time
    B, H = 8, 96
    g = torch.Generator(device=cuda_device).manual_seed(L)
    u = torch.randn((B, H, L), device=cuda_device, generator=g)
    k = torch.randn((H, L), device=cuda_device, generator=g) / L ** 0.5
    plan = sf.Plan(L)
    Kf = plan.filter_spectrum(k)
    stream = torch.cuda.current_stream(cuda_device)
    ys = [torch.empty_like(u) for _ in range(3)]
    x = u
    for i in range(3):
        plan.conv(x, Kf, ys[i], stream=stream)
        x = ys[i] * 0.5 + 1.0          # a torch kernel producing the next input on the same stream
    torch.cuda.synchronize()
    plan.check()
    x = u
    for i in range(3):
        torch.cuda.synchronize()
        y = plan.conv(x.clone(), Kf)
        torch.cuda.synchronize()
        assert torch.equal(y, ys[i])
        x = y * 0.5 + 1.0
    # fused launches straight after each other, the second reading the first's output
    a, b = torch.empty_like(u), torch.empty_like(u)
    plan.conv(u, Kf, a, stream=stream)
    plan.conv(a, Kf, b, stream=stream)
    torch.cuda.synchronize()
    plan.check()
    assert torch.equal(b, plan.conv(a.clone(), Kf))
    plan.close()
