"""Channel-sharded convolution over several devices through the C ABI (sffft_conv_multi for device-resident
shards, sffft_multi_pipe_create / sffft_conv_host_multi for one batch in host memory).  Shard g owns the
channels sffft_shard_range(H, G, g); results must equal the single-plan path and the fp64 oracle.  Runs on
every visible GPU, and with several shards on one GPU where only one is visible (shards are independent of
the device they run on)."""
import ctypes

import numpy as np
import pytest
import torch

import sffft_b200 as sf
from tests.conftest import rel_l2

pytestmark = pytest.mark.gpu


def devices(G):
    n = torch.cuda.device_count()
    return [g % n for g in range(G)]


@pytest.mark.parametrize("G,H", [(2, 37), (3, 8), (8, 96)])
def test_device_resident_shards(oracle, cuda_device, G, H):
    L, B = 1024, 6
    u, k = oracle.gen_profile(B, H, L, seed=3)
    plans = [sf.Plan(L, device=d) for d in devices(G)]
    us, Kfs, ys = [], [], []
    for g, p in enumerate(plans):
        h0, h1 = sf.shard_range(H, G, g)
        dev = torch.device("cuda", p.device)
        us.append(torch.from_numpy(np.ascontiguousarray(u[:, h0:h1])).to(dev))
        Kfs.append(p.filter_spectrum(torch.from_numpy(np.ascontiguousarray(k[h0:h1])).to(dev)))
        ys.append(torch.empty_like(us[-1]))
    sf.conv_multi(plans, us, Kfs, ys, B, H)
    for p in plans:
        p.check()
    y = np.concatenate([t.cpu().numpy() for t in ys], axis=1)
    assert y.shape == u.shape
    assert rel_l2(y, oracle.direct_conv(u, k)) <= 5e-4
    # bit-identical to one plan over the whole batch (the same kernel on the same pairs)
    whole = sf.Plan(L)
    ref = whole.conv(torch.from_numpy(u).to(cuda_device), whole.filter_spectrum(torch.from_numpy(k).to(cuda_device)))
    whole.check()
    assert np.array_equal(y, ref.cpu().numpy())


@pytest.mark.parametrize("io", ["fp32", "bf16"])
@pytest.mark.parametrize("G", [2, 4])
def test_host_batch_over_devices(oracle, cuda_device, G, io):
    L, B, H = 2048, 8, 50
    u, k = oracle.gen_profile(B, H, L, seed=4)
    dt = torch.bfloat16 if io == "bf16" else torch.float32
    u_h = torch.from_numpy(u).to(dt).pin_memory()
    y_h = torch.zeros_like(u_h).pin_memory()
    plans = [sf.Plan(L, io=io, device=d) for d in devices(G)]
    kt = torch.from_numpy(k).to(dt)
    Kfs = []
    for g, p in enumerate(plans):
        h0, h1 = sf.shard_range(H, G, g)
        Kfs.append(p.filter_spectrum(kt[h0:h1].contiguous().to(torch.device("cuda", p.device))))
    mp = sf.HostPipeMulti(plans, B, H, chunks=2)
    for _ in range(2):   # twice: the pipes' staging slots are reused across calls
        y_h.zero_()
        mp.conv(u_h, Kfs, y_h)
    mp.close()
    uo = u_h.float().numpy()
    ko = kt.float().numpy()
    tol = 3e-3 if io == "bf16" else 5e-4
    assert rel_l2(y_h.float().numpy(), oracle.direct_conv(uo, ko)) <= tol


def test_invalid_multi_calls(cuda_device):
    plans = [sf.Plan(1024), sf.Plan(1024)]
    other = sf.Plan(2048)
    lib = sf.lib()
    hs = (ctypes.c_void_p * 2)(plans[0]._h.value, other._h.value)
    h = ctypes.c_void_p()
    assert lib.sffft_multi_pipe_create(ctypes.byref(h), hs, 2, 8, 16, 0) == sf.ERR_INVALID_ARGUMENT   # lengths differ
    hs = (ctypes.c_void_p * 2)(plans[0]._h.value, plans[1]._h.value)
    assert lib.sffft_multi_pipe_create(ctypes.byref(h), hs, 2, 8, 1, 0) == sf.ERR_INVALID_ARGUMENT    # H < G
    with pytest.raises(sf.SffftError):
        sf.conv_multi(plans, [None, None], [None, None], [None, None], 8, 16)


def test_composite_plans_over_devices(oracle, cuda_device):
    # composite plans take their workspace from the caller: attached to each plan for sffft_conv_multi, allocated by
    # each device's pipe for sffft_conv_host_multi; both equal one composite plan over the whole batch
    L, B, H, G, config = 512, 4, 10, 2, "4x[16x16/w8]"
    u, k = oracle.gen_profile(B, H, L, seed=6)
    plans = [sf.Plan(L, config=config, device=d) for d in devices(G)]
    us, Kfs, ys, works = [], [], [], []
    for g, p in enumerate(plans):
        h0, h1 = sf.shard_range(H, G, g)
        dev = torch.device("cuda", p.device)
        us.append(torch.from_numpy(np.ascontiguousarray(u[:, h0:h1])).to(dev))
        Kfs.append(p.filter_spectrum(torch.from_numpy(np.ascontiguousarray(k[h0:h1])).to(dev)))
        ys.append(torch.empty_like(us[-1]))
        works.append(torch.empty(p.workspace_bytes(B, h1 - h0), dtype=torch.uint8, device=dev))
        assert sf.lib().sffft_plan_set_workspace(p._h, works[-1].data_ptr(), works[-1].numel()) == sf.OK
    sf.conv_multi(plans, us, Kfs, ys, B, H)
    for p in plans:
        p.check()
    y = np.concatenate([t.cpu().numpy() for t in ys], axis=1)
    whole = sf.Plan(L, config=config)
    ref = whole.conv(torch.from_numpy(u).to(cuda_device), whole.filter_spectrum(torch.from_numpy(k).to(cuda_device)))
    whole.check()
    assert np.array_equal(y, ref.cpu().numpy())
    assert rel_l2(y, oracle.direct_conv(u, k)) <= 5e-4
    u_h = torch.from_numpy(u).pin_memory()
    y_h = torch.zeros_like(u_h).pin_memory()
    mp = sf.HostPipeMulti(plans, B, H)
    mp.conv(u_h, Kfs, y_h)
    mp.close()
    assert np.array_equal(y_h.numpy(), y)
