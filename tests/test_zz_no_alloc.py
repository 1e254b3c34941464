"""The allocation-free entry point, sffft_conv_noalloc, for callers that cannot allocate device memory while
they run (for example a plugin whose execute step must not allocate).  It is called through the C ABI on two
calls in a row with different inputs, since every call reuses the same fixed scratch, and its output must be
bit-identical to the regular path -- sffft_filter_spectrum + sffft_conv on a plan with in-kernel DFT
matrices, the same kernel with the same spectrum -- and within the mode's tolerance of the fp64 direct
convolution.  This file is named so that pytest collects it last."""
import ctypes

import numpy as np
import pytest
import torch

import sffft_b200 as sf

pytestmark = pytest.mark.gpu

TOL = {("fp32", "fp32"): 5e-4, ("bf16", "fp32"): 3e-3, ("fp32", "fp16"): 1e-3, ("bf16", "fp16"): 4e-3}


def noalloc():
    fn = sf.lib().sffft_conv_noalloc
    V, I = ctypes.c_void_p, ctypes.c_int
    fn.argtypes = [I, I, I, V, V, I, V, I, I, V, I]
    fn.restype = I
    return fn


def inputs(B, H, L, seed, io):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    u = torch.randn((B, H, L), device="cuda", generator=g)
    n = torch.arange(L, device="cuda", dtype=torch.float32)
    k = torch.randn((H, L), device="cuda", generator=g) * torch.exp(-4.0 * n / L) / L ** 0.5
    if io == "bf16":
        u, k = u.to(torch.bfloat16), k.to(torch.bfloat16)
    return u, k


def regular(L, io, acc, u, k):
    plan = sf.Plan(L, io=io, acc=acc, kernel="legacy")
    y = plan.conv(u, plan.filter_spectrum(k))
    plan.check()
    plan.close()
    return y


@pytest.mark.parametrize("L,B,H,io,acc", [(1024, 4, 3, "fp32", "fp32"), (128, 5, 7, "bf16", "fp32"),
                                          (4096, 2, 2, "fp32", "fp16")])
def test_matches_regular_path_on_two_calls(oracle, L, B, H, io, acc):
    fn = noalloc()
    kd = sf.IO[io]
    for call, seed in enumerate((11, 12)):
        u, k = inputs(B, H, L, seed, io)
        y = torch.full_like(u, float("nan"))
        st = fn(L, sf.IO[io], sf.ACC[acc], u.data_ptr(), k.data_ptr(), kd, y.data_ptr(), B, H, None, 1)
        assert st == sf.OK, sf.status_string(st)
        ref = regular(L, io, acc, u, k)
        assert torch.equal(y, ref), f"call {call}: differs from the regular path"
        fp64 = oracle.direct_conv(u.float().cpu().numpy(), k.float().cpu().numpy())
        got = y.float().cpu().numpy().astype(np.float64)
        err = float(np.linalg.norm(got - fp64) / np.linalg.norm(fp64))
        assert err <= TOL[(io, acc)], f"call {call}: rel L2 {err:.3e} against the fp64 oracle"


def test_rejects_problems_beyond_the_scratch():
    fn = noalloc()
    L, H = 8192, 129                       # 129 * 16384 * 8 bytes > 16 MiB of spectrum scratch
    u = torch.zeros((1, H, L), device="cuda")
    k = torch.zeros((H, L), device="cuda")
    y = torch.zeros_like(u)
    st = fn(L, 0, 0, u.data_ptr(), k.data_ptr(), 0, y.data_ptr(), 1, H, None, 1)
    assert st == 8                         # SFFFT_ERR_SCRATCH_LIMIT
    assert "scratch" in sf.status_string(st)
    assert torch.count_nonzero(y).item() == 0
    # the largest admitted spectrum for this length is accepted
    u = torch.randn((1, 128, L), device="cuda")
    k = torch.randn((128, L), device="cuda")
    y = torch.empty_like(u)
    assert fn(L, 0, 0, u.data_ptr(), k.data_ptr(), 0, y.data_ptr(), 1, 128, None, 1) == sf.OK
