"""Channel sharding across ranks (the multi-GPU path) with world-size-2 gloo ranks on CPU: each rank takes
its channel slice from sffft_shard_range, convolves it (CPU emulation of the fused kernel), and the gathered
slices must equal the unsharded result; a rank that fails is reported to the others through the process
group instead of hanging them."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

import sffft_b200 as sf
from tests.oracle_py import spectrum_digit_order


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def inputs(B, H, L, seed=3):
    rng = np.random.default_rng(seed)
    u = rng.standard_normal((B, H, L)).astype(np.float32)
    k = (rng.standard_normal((H, L)) * np.exp(-4 * np.arange(L) / L) / np.sqrt(L)).astype(np.float32)
    return u, k


def conv_slice(u, k, name):
    R = [int(x) for x in name.split("/")[0].split("x")]
    Kc = spectrum_digit_order(k, R)
    Kf = np.stack([Kc.real, Kc.imag], -1).astype(np.float32)
    return sf.emu_conv(name, np.ascontiguousarray(u), Kf)


def worker(rank, world, port, B, H, L, name, fail_rank, out_q):
    import datetime

    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    try:
        u, k = inputs(B, H, L)
        h0, h1 = sf.shard_range(H, world, rank)
        ok = torch.tensor([1], dtype=torch.int32)
        y = None
        try:
            if rank == fail_rank:
                raise RuntimeError("injected failure on this rank")
            y = conv_slice(u[:, h0:h1], k[h0:h1], name)
        except Exception:
            ok[0] = 0
        # every rank learns whether all ranks succeeded before any data collective
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        if ok.item() == 0:
            out_q.put((rank, "aborted", None))
            return
        parts = [None] * world
        dist.all_gather_object(parts, (h0, h1, y))
        if rank == 0:
            full = np.zeros((B, H, L), np.float32)
            for a, b, yy in parts:
                full[:, a:b] = yy
            out_q.put((rank, "ok", full))
        else:
            out_q.put((rank, "ok", None))
    finally:
        dist.destroy_process_group()


def run_world(world, B, H, L, name, fail_rank=-1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=worker, args=(r, world, port, B, H, L, name, fail_rank, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return res


@pytest.mark.parametrize("H", [4, 5])
def test_two_rank_channel_shards_equal_unsharded(H):
    B, L, name = 3, 128, "16x16/w4"
    res = run_world(2, B, H, L, name)
    full = [r[2] for r in res if r[0] == 0][0]
    u, k = inputs(B, H, L)
    ref = conv_slice(u, k, name)
    # per-channel results do not depend on how channels are grouped into CTAs beyond fp16 rounding order
    assert np.linalg.norm(full - ref) / np.linalg.norm(ref) < 1e-6


def test_failed_rank_is_reported_not_hung():
    res = run_world(2, 2, 4, 128, "16x16/w4", fail_rank=1)
    assert sorted(r[1] for r in res) == ["aborted", "aborted"]
