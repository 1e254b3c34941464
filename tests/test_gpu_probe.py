"""tcgen05 operand layouts on B200: one MMA through the fused kernel's own layout writers and
descriptors (sffft_debug_umma_probe) against a host GEMM, for every operand form the kernel uses."""
import numpy as np
import pytest

import sffft_b200 as sf

pytestmark = pytest.mark.gpu


def small_int_halves(shape, rng):
    v = rng.integers(-4, 5, size=shape).astype(np.float16)
    return v, v.view(np.uint16)


CASES = (
    [(0, s, 128, b, 128) for s in range(4) for b in range(4)] +      # MN-major SW128 A; K-major SW128 B
    [(128, s, 64, b, 64) for s in range(4) for b in range(2)] +      # K-major SW128 A; SW64 B
    [(64, s, 32, 0, 32) for s in range(2)] +                         # K-major SW64 A; SW32 B
    [(32, 0, 128, 1, 16), (0, 1, 64, 1, 32), (0, 2, 32, 0, 16)]
)


@pytest.mark.parametrize("a_kind,a_slice,b_pitch,b_slice,n", CASES)
def test_umma_layouts_fp32_accumulator(a_kind, a_slice, b_pitch, b_slice, n):
    rng = np.random.default_rng(a_kind * 100 + a_slice * 10 + b_slice + n)
    A, Ab = small_int_halves((128, 16), rng)
    Bm, Bb = small_int_halves((n, 16), rng)
    D = sf.umma_probe(a_kind, a_slice, b_pitch, b_slice, Ab, Bb)
    ref = A.astype(np.float32) @ Bm.astype(np.float32).T
    np.testing.assert_array_equal(D.view(np.float32), ref)


def test_umma_fp16_accumulator_format():
    # fp16 accumulators occupy one 32-bit TMEM column each, value in the low 16 bits
    rng = np.random.default_rng(5)
    A, Ab = small_int_halves((128, 16), rng)
    Bm, Bb = small_int_halves((32, 16), rng)
    D = sf.umma_probe(0, 0, 128, 0, Ab, Bb, acc16=True)
    ref = (A.astype(np.float32) @ Bm.astype(np.float32).T).astype(np.float16)
    np.testing.assert_array_equal((D & 0xFFFF).astype(np.uint16).view(np.float16), ref)


def test_bounded_wait_reports_timeout_and_context_survives():
    assert sf.lib().sffft_debug_wait_timeout(2000) == sf.ERR_TIMEOUT
    # the context is still usable afterwards
    rng = np.random.default_rng(0)
    A, Ab = small_int_halves((128, 16), rng)
    Bm, Bb = small_int_halves((16, 16), rng)
    D = sf.umma_probe(0, 0, 128, 0, Ab, Bb)
    np.testing.assert_array_equal(D.view(np.float32), A.astype(np.float32) @ Bm.astype(np.float32).T)


@pytest.mark.parametrize("name,B,H", [("64x32/w8", 2, 1), ("32x16x16/w8", 8, 4), ("16x16/w4", 8, 40)])
def test_fused_kernel_timeout_path(oracle, cuda_device, name, B, H):
    # One warp of the fused kernel withholds its arrival on a stage barrier, so that group's MMAs are never
    # issued; with every wait limited to 2 ms the kernel's roles see the abort flag, wait for the MMAs in
    # flight, free their TMEM and return, and the plan's status word reads SFFFT_ERR_TIMEOUT.  A regular launch
    # on the same context then passes parity (a CTA that kept its TMEM would block every later allocation on
    # its SM).  Other CTAs of the launch (H = 4, 40) finish their groups normally.
    import torch

    from tests.conftest import rel_l2
    R = [int(x) for x in name.split("/")[0].split("x")]
    L = int(np.prod(R)) // 2
    u, k = oracle.gen_profile(B, H, L, seed=7)
    plan = sf.Plan(L, config=name)
    ut = torch.from_numpy(u).to(cuda_device)
    Kf = plan.filter_spectrum(torch.from_numpy(k).to(cuda_device))
    y = torch.zeros_like(ut)
    st = sf.lib().sffft_debug_conv_timeout(plan._h, ut.data_ptr(), Kf.data_ptr(), y.data_ptr(), B, H, 2000, None)
    assert st == sf.OK
    assert sf.lib().sffft_plan_check(plan._h) == sf.ERR_TIMEOUT
    assert sf.lib().sffft_plan_check(plan._h) == sf.OK          # the check cleared the status word
    y2 = plan.conv(ut, Kf)
    plan.check()
    assert rel_l2(y2.cpu().numpy(), oracle.direct_conv(u, k)) <= 5e-4
    plan.close()
