"""Composite plans: lengths past the largest single-kernel plan as partitioned convolutions on a block plan
(sffft_plan_create with "<P>x[<plan>]", the default for L > 16384): one forward launch over every input block,
one inverse launch summing the block spectra against the filter-segment spectra, in a caller-owned workspace.

The reference stops at L = 8192 and lists multi-pass plans as missing (README.md:175), so parity is with
the oracle's fp64 direct causal convolution (the reference's own check, src/sffft.cu:376-378), at the
causal path's tolerances: fp32 I/O 5e-4, bf16 I/O 3e-3, bf16 I/O with fp16 accumulation 4e-3.  Small
composites of small block plans are checked on every sequence; the default plans for L = 32768 and
65536 on sampled sequences.  A size-independent property closes it: the convolution is linear."""
import numpy as np
import pytest
import torch

import sffft_b200 as sf
from tests.conftest import rel_l2
from tests.oracle_py import per_row_rel_l2, scaled_pair_inputs, to_bf16

pytestmark = pytest.mark.gpu
TOL = {("fp32", "fp32"): 5e-4, ("bf16", "fp32"): 3e-3, ("bf16", "fp16"): 4e-3}


def run(plan, u, k, dev):
    dt = torch.bfloat16 if plan.io == "bf16" else torch.float32
    Kf = plan.filter_spectrum(torch.from_numpy(k).to(dev).to(dt))
    y = plan.conv(torch.from_numpy(u).to(dev).to(dt), Kf)
    plan.check()
    return y.float().cpu().numpy(), Kf


@pytest.mark.parametrize("config,L", [("2x[16x16/w4]", 256), ("4x[16x16/w8]", 512), ("8x[32x16/w8]", 2048),
                                      ("2x[64x32/w8]", 2048), ("2x[32x16x16/w8]", 8192)])
@pytest.mark.parametrize("io,acc", [("fp32", "fp32"), ("bf16", "fp32"), ("bf16", "fp16")])
def test_small_composites_match_fp64(oracle, cuda_device, config, L, io, acc):
    B, H = 3, 5                      # odd B: pairs of batch rows straddle the blocks of the launches
    u, k = oracle.gen_profile(B, H, L, decay=4.0, sqrt_norm=True, seed=L + 7)
    if io == "bf16":
        u, k = to_bf16(u), to_bf16(k)
    plan = sf.Plan(L, io=io, acc=acc, config=config)
    assert plan.info["blocks"] == int(config.split("x[")[0]) and plan.config == config and plan.N == 2 * L
    y, _ = run(plan, u, k, cuda_device)
    plan.close()
    err = rel_l2(y, oracle.direct_conv(u, k))
    assert err <= TOL[(io, acc)], f"{config} {io}/{acc}: {err:.3e}"


@pytest.mark.parametrize("L,io", [(32768, "fp32"), (32768, "bf16"), (65536, "fp32")])
def test_default_long_plans(oracle, cuda_device, L, io):
    B, H = 2, 3
    plan = sf.Plan(L, io=io)
    assert plan.info["blocks"] == L // 16384 and plan.config.endswith("x[32x32x32/w8]")
    u, k = oracle.gen_profile(B, H, L, decay=8.0, sqrt_norm=True, seed=3)
    if io == "bf16":
        u, k = to_bf16(u), to_bf16(k)
    y, Kf = run(plan, u, k, cuda_device)
    seqs = np.array([0, 4]) if L > 32768 else np.array([0, 3, 5])
    ref = oracle.direct_conv_seqs(u, k, seqs)
    err = rel_l2(y.reshape(B * H, L)[seqs], ref)
    assert err <= TOL[(io, "fp32")], f"L={L} {io}: {err:.3e}"
    # linearity at full length: y(2u) / 2 == y(u) (the rows' power-of-two scales absorb the factor; bound: a
    # fifth of the parity tolerance)
    dt = torch.bfloat16 if io == "bf16" else torch.float32
    y2 = plan.conv((2 * torch.from_numpy(u).to(cuda_device)).to(dt), Kf).float().cpu().numpy()
    plan.check()
    assert rel_l2(y2 / 2, y) <= TOL[(io, "fp32")] / 5
    plan.close()


def test_composite_host_pipe_and_fft(cuda_device):
    L = 512
    plan = sf.Plan(L, io="fp32", config="4x[16x16/w8]")
    rng = np.random.default_rng(5)
    B, H = 4, 6
    u = rng.standard_normal((B, H, L)).astype(np.float32)
    k = (rng.standard_normal((H, L)) * np.exp(-4 * np.arange(L) / L) / np.sqrt(L)).astype(np.float32)
    y_dev, Kf = run(plan, u, k, cuda_device)
    # the host-buffer pipeline gives the same result as the device call
    pipe = sf.HostPipe(plan, B, H, 4)
    u_h = torch.from_numpy(u).pin_memory()
    y_h = torch.empty_like(u_h).pin_memory()
    pipe.conv(u_h, Kf, y_h)
    torch.cuda.synchronize()
    pipe.close()
    plan.check()
    np.testing.assert_array_equal(y_h.numpy(), y_dev)
    # the standalone FFT of the composite length
    x = rng.standard_normal((2, 2 * L)).astype(np.float32)
    X = plan.rfft(torch.from_numpy(x).to(cuda_device))
    assert rel_l2(X.cpu().numpy(), np.fft.rfft(x.astype(np.float64), axis=-1)) <= 3e-6
    plan.close()


def test_composite_rejects_other_filter_layouts(cuda_device):
    plan = sf.Plan(256, config="2x[16x16/w4]")
    with pytest.raises(sf.SffftError):
        plan.filter_spectrum(torch.zeros((2, 511), device=cuda_device), layout="two_sided")
    with pytest.raises(sf.SffftError):
        sf.Plan(512, config="2x[16x16/w4]")          # 2 blocks of 128 make 256, not 512
    with pytest.raises(sf.SffftError):
        sf.Plan(384, config="3x[16x16/w4]")          # block counts are powers of two
    plan.close()


def test_composite_workspace_contract(cuda_device):
    L, B, H = 256, 3, 4
    plan = sf.Plan(L, config="2x[16x16/w4]")
    need = plan.workspace_bytes(B, H)
    # pair spectra of every input block (ceil(B/2) * H * L complex fp32 pairs) and the row energies
    assert need == 2 * H * L * 2 * 8 + 256
    assert sf.Plan(1024).workspace_bytes(B, H) == 0
    rng = np.random.default_rng(9)
    u = torch.from_numpy(rng.standard_normal((B, H, L)).astype(np.float32)).to(cuda_device)
    k = torch.from_numpy((rng.standard_normal((H, L)) / np.sqrt(L)).astype(np.float32)).to(cuda_device)
    Kf = plan.filter_spectrum(k)
    y_ref = plan.conv(u, Kf)
    lib = sf.lib()
    y = torch.empty_like(u)
    args = (plan._h, u.data_ptr(), Kf.data_ptr(), y.data_ptr(), B, H)
    assert lib.sffft_conv(*args, None) == sf.ERR_WORKSPACE            # nothing attached
    work = torch.empty(need, dtype=torch.uint8, device=cuda_device)
    assert lib.sffft_conv_ws(*args, work.data_ptr(), need - 1, None) == sf.ERR_WORKSPACE
    assert lib.sffft_conv_ws(*args, work.data_ptr() + 16, need, None) == sf.ERR_INVALID_ARGUMENT   # alignment
    assert lib.sffft_plan_set_workspace(plan._h, work.data_ptr() + 16, need) == sf.ERR_INVALID_ARGUMENT
    assert lib.sffft_plan_set_workspace(plan._h, work.data_ptr(), need) == sf.OK
    assert lib.sffft_conv(*args, None) == sf.OK
    plan.check()
    assert torch.equal(y, y_ref)
    y.zero_()
    assert lib.sffft_conv_ws(*args, work.data_ptr(), need, None) == sf.OK
    plan.check()
    assert torch.equal(y, y_ref)
    assert lib.sffft_plan_set_workspace(plan._h, None, 0) == sf.OK
    assert lib.sffft_conv(*args, None) == sf.ERR_WORKSPACE
    plan.close()


def test_composite_pairs_of_very_different_scale(oracle, cuda_device):
    # every row keeps its own relative accuracy next to a partner 1e3-1e5 times larger, or all zero: its scale
    # comes from its energy over the whole row and is shared by its blocks
    L, config = 512, "4x[16x16/w8]"
    plan = sf.Plan(L, config=config)
    u, k = scaled_pair_inputs(oracle, 2, L, "fp32", seed=4)
    y, _ = run(plan, u, k, cuda_device)
    plan.close()
    errs = per_row_rel_l2(y, oracle.direct_conv(u, k))
    assert np.all(errs <= TOL[("fp32", "fp32")]), errs
