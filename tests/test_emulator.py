"""The fused kernel's stage code run on the CPU with an emulated tcgen05 backend (sffft_b200/csrc/emu.cpp),
against the fp64 oracle.  This checks every plan's shared-memory layouts, UMMA descriptors, pairing,
twiddles and digit order without a GPU; the GPU parity tests check the same code on B200."""
import numpy as np
import pytest

import sffft_b200 as sf
from tests.conftest import rel_l2
from tests.oracle_py import (bf16_bits, bf16_from_bits, per_row_rel_l2, scaled_pair_inputs, segment_spectra_digit_order,
                             spectrum_digit_order, to_bf16)

TOL = {("fp32", "fp32"): 5e-4, ("bf16", "fp32"): 3e-3, ("fp32", "fp16"): 1e-3, ("bf16", "fp16"): 4e-3}


def radices(name):
    return [int(x) for x in name.split("@")[0].split("/")[0].split("x")]


def run_case(oracle, name, B, H, io="fp32", acc="fp32", seed=0):
    R = radices(name)
    L = int(np.prod(R)) // 2
    u, k = oracle.gen_profile(B, H, L, decay=4.0, sqrt_norm=True, seed=seed + 1)
    if io == "bf16":
        u, k = to_bf16(u), to_bf16(k)
    Kc = spectrum_digit_order(k, R)
    Kf = np.stack([Kc.real, Kc.imag], -1).astype(np.float32)
    if io == "bf16":
        y = bf16_from_bits(sf.emu_conv(name, bf16_bits(u), Kf, io="bf16", acc=acc)).reshape(u.shape)
    else:
        y = sf.emu_conv(name, u, Kf, io="fp32", acc=acc)
    ref = oracle.direct_conv(u, k)
    return rel_l2(y, ref)


CATALOG = [n for L, n in sf.catalog()]


@pytest.mark.parametrize("name", [n for n in CATALOG if int(np.prod(radices(n))) <= 8192])
def test_every_plan_fp32(oracle, name):
    N = int(np.prod(radices(name)))
    B, H = (3, 2) if N <= 4096 else (2, 1)
    assert run_case(oracle, name, B, H) <= TOL[("fp32", "fp32")]


def test_largest_plan(oracle):
    assert run_case(oracle, "32x32x32/w4", 1, 1) <= TOL[("fp32", "fp32")]


@pytest.mark.parametrize("name", ["16x16/w4", "64x32/w4", "32x16x16/w4"])
@pytest.mark.parametrize("io,acc", [("bf16", "fp32"), ("fp32", "fp16"), ("bf16", "fp16")])
def test_io_and_accumulation_modes(oracle, name, io, acc):
    assert run_case(oracle, name, 2, 1, io=io, acc=acc) <= TOL[(io, acc)]


def test_odd_batch_and_partial_ctas(oracle):
    # B=5 leaves one unpaired sequence per channel; H=3 with G=8 pairs per CTA leaves a partial CTA
    assert run_case(oracle, "16x16/w4", 5, 3) <= 5e-4
    assert run_case(oracle, "32x32/w4", 1, 5) <= 5e-4


def test_zero_and_impulse_inputs():
    L = 128
    u = np.zeros((2, 1, L), np.float32)
    Kf = np.zeros((1, 2 * L, 2), np.float32)
    assert not sf.emu_conv("16x16/w4", u, Kf).any()
    # impulse filter k = delta: Kf = 1 everywhere -> y = u (to fp16-pipeline accuracy)
    rng = np.random.default_rng(3)
    u = rng.standard_normal((2, 1, L)).astype(np.float32)
    Kf[..., 0] = 1.0
    assert rel_l2(sf.emu_conv("16x16/w4", u, Kf), u) < 5e-4


@pytest.mark.parametrize("name", ["16x16/w4", "32x32/w4", "64x32/w4", "32x64/w8", "64x64/w4", "16x16x16/w4"])
def test_staged_spectrum_path(oracle, name):
    # B = 8 puts one channel in each group, so the spectrum epilogue reads staged spectrum rows
    assert run_case(oracle, name, 8, 2) <= TOL[("fp32", "fp32")]


def test_staged_spectrum_partial_groups(oracle):
    # B = 2: one channel per pair; H = 33 leaves the last group with a single pair (empty slots must not
    # read outside the staged spectrum rows)
    for name in ["16x16/w4", "32x32/w4"]:
        assert run_case(oracle, name, 2, 33) <= TOL[("fp32", "fp32")]


@pytest.mark.parametrize("name", ["16x16/w4", "16x16x16/w4"])
@pytest.mark.parametrize("io,acc", [("fp32", "fp32"), ("bf16", "fp32"), ("fp32", "fp16"), ("bf16", "fp16")])
def test_pairs_of_very_different_scale(oracle, name, io, acc):
    # every single row within the tolerance, including rows 1e3 / 1e4 below their pair partner, an all-zero
    # row beside a full-scale one (exactly zero output), and a pair of tiny rows
    from tests.oracle_py import PAIR_SCALES, per_row_rel_l2, scaled_pair_inputs
    R = radices(name)
    L = int(np.prod(R)) // 2
    u, k = scaled_pair_inputs(oracle, 2, L, io, seed=21)
    Kc = spectrum_digit_order(k, R)
    Kf = np.stack([Kc.real, Kc.imag], -1).astype(np.float32)
    if io == "bf16":
        y = bf16_from_bits(sf.emu_conv(name, bf16_bits(u), Kf, io="bf16", acc=acc)).reshape(u.shape)
    else:
        y = sf.emu_conv(name, u, Kf, io="fp32", acc=acc)
    errs = per_row_rel_l2(y, oracle.direct_conv(u, k))
    assert errs.shape == (len(PAIR_SCALES), 2)
    assert np.all(errs <= TOL[(io, acc)]), errs
    assert not y[4].any()


@pytest.mark.parametrize("name,io", [("64x32/w8", "fp32"), ("32x16x16/w8", "bf16")])
def test_pairs_of_very_different_scale_eight_warp_plans(oracle, name, io):
    # the 8-warp plans' output stage: a thread's units cover several chunks and tiles, so the pair whose output
    # scales it applies changes from unit to unit (the bench plan, and configs[2]'s plan in its bf16-I/O form)
    from tests.oracle_py import PAIR_SCALES, per_row_rel_l2, scaled_pair_inputs
    R = radices(name)
    L = int(np.prod(R)) // 2
    u, k = scaled_pair_inputs(oracle, 2, L, io, seed=23)
    Kc = spectrum_digit_order(k, R)
    Kf = np.stack([Kc.real, Kc.imag], -1).astype(np.float32)
    if io == "bf16":
        y = bf16_from_bits(sf.emu_conv(name, bf16_bits(u), Kf, io="bf16", acc="fp32")).reshape(u.shape)
    else:
        y = sf.emu_conv(name, u, Kf, io="fp32", acc="fp32")
    errs = per_row_rel_l2(y, oracle.direct_conv(u, k))
    assert errs.shape == (len(PAIR_SCALES), 2)
    assert np.all(errs <= TOL[(io, "fp32")]), errs
    assert not y[4].any()


SMALL_VARIANTS = [f"{n}@{v}" for n in ["16x16/w8", "32x16/w8", "32x32/w8", "64x32/w8", "64x64/w8", "32x16x16/w8"]
                  for v in (1, 2) if not (n == "16x16/w8" and v == 1)]


@pytest.mark.parametrize("name", SMALL_VARIANTS)
def test_small_launch_variants(oracle, name):
    # the 1- and 2-slot variants of the default plans (wider teams), used for launches with at most one or two
    # groups per SM
    assert run_case(oracle, name, 4, 3) <= TOL[("fp32", "fp32")]
    assert run_case(oracle, name, 2, 1, io="bf16", acc="fp16") <= TOL[("bf16", "fp16")]


# Composite plans' partitioned convolution (row energies, forward launch storing pair spectra, inverse launch
# summing them against the filter-segment spectra), every sequence against the fp64 oracle.
@pytest.mark.parametrize("name,P,B,H,io,acc", [("16x16/w4", 2, 3, 2, "fp32", "fp32"), ("16x16/w4", 4, 2, 1, "bf16", "fp32"),
                                               ("32x16/w8", 2, 3, 1, "fp32", "fp16"),
                                               ("32x16x16/w8", 2, 2, 1, "fp32", "fp32")])
def test_composite_partitioned_convolution(oracle, name, P, B, H, io, acc):
    R = radices(name)
    L = P * int(np.prod(R)) // 2
    u, k = oracle.gen_profile(B, H, L, decay=4.0, sqrt_norm=True, seed=P + B)
    if io == "bf16":
        u, k = to_bf16(u), to_bf16(k)
    Kc = segment_spectra_digit_order(k, P, R)
    Kf = np.stack([Kc.real, Kc.imag], -1).astype(np.float32)
    if io == "bf16":
        y = bf16_from_bits(sf.emu_conv_composite(name, P, bf16_bits(u), Kf, io=io, acc=acc)).reshape(u.shape)
    else:
        y = sf.emu_conv_composite(name, P, u, Kf, io=io, acc=acc)
    assert rel_l2(y, oracle.direct_conv(u, k)) <= TOL[(io, acc)]


def test_composite_pairs_of_very_different_scale(oracle):
    # rows scaled 1, 1e-3, 1e-4, 0, 1e-5 ... next to their partners: each row's scale comes from its energy over
    # the whole row, shared by its blocks, so every row keeps its own relative accuracy
    P, name = 2, "16x16/w4"
    L = P * 128
    u, k = scaled_pair_inputs(oracle, 1, L, "fp32", seed=11)
    Kc = segment_spectra_digit_order(k, P, radices(name))
    Kf = np.stack([Kc.real, Kc.imag], -1).astype(np.float32)
    y = sf.emu_conv_composite(name, P, u, Kf)
    errs = per_row_rel_l2(y, oracle.direct_conv(u, k))
    assert np.all(errs <= TOL[("fp32", "fp32")]), errs


def test_composite_without_block_kernels_is_rejected():
    u = np.zeros((2, 1, 512), np.float32)
    with pytest.raises(ValueError):
        sf.emu_conv_composite("32x32/w4", 2, u, np.zeros((2, 1, 1024, 2), np.float32))
