"""Benchmark of the fused causal long convolution (headline metric: ms per B=8 x H=768 batch and fraction of
the HBM / tensor roofline).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--L 1024] [--io fp32] ...
    torchrun --nproc-per-node N bench.py --gpus N ...      (one rank per GPU)

Workload (default): configuration configs[1] -- one batch of B=8 x H=768 channels, L=1024, fp32 I/O, fp32
accumulation, u ~ N(0,1), k = N(0,1) exp(-4n/L)/sqrt(L).  A step is one sffft_conv launch per GPU.  With N GPUs
the batch is sharded by channel (rank r owns sffft_shard_range(768, N, r), its u/y slices and spectrum rows;
no collective on the data path) and `value` is the fixed batch's ms = max-over-ranks step time (strong
scaling).  `weak_scaling` adds the per-GPU-fixed variant: every rank convolves a whole 8 x 768 batch of its own
and the line reports max step time / N per batch.  Inputs rotate over independent sets (u, y, Kf) whose total
exceeds the 126 MB L2, so every step reads from HBM.

At N = 1 the line also carries `sweep`: the metric's L = 128..8192 x {fp32, bf16} points (B=8, H=768, default
plan, fp32 accumulation) and configurations 2-4, each with ms per batch, roofline fraction and the cuFFT
pad/R2C/multiply/C2R/slice pipeline on the same GPU timed the same way.  `parity` compares sampled sequences of
every rank's output with the fp64 oracle (outside the timed region).

--impl reference times the reference's CPU path for the same metric -- the fp64 direct causal convolution
(sfFFT src/sffft.cu:376-378, restated in oracle/oracle.c) on all host cores -- on a bounded sample of sequences
per step, scaled to a full batch; under torchrun only rank 0 runs it.
"""
import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "ms/batch and % of roofline, B=8×H=768, L=128–8192, fp32/bf16 I/O"
UNIT = "ms/batch"
GB10_PUBLISHED_MS = {(1024, "fp32"): 0.459, (1024, "bf16"): 0.440, (128, "fp32"): 0.033, (4096, "bf16"): 1.342,
                     (8192, "bf16"): 3.434, (8192, "fp32"): 4.184}
L2_BYTES = 126e6
# The benchmark's named configurations by (B, H, L, I/O, accumulation); other shapes are "custom".
NAMED_CONFIGS = {(1, 1, 128, "fp32", "fp32"): "configs[0]", (8, 768, 1024, "fp32", "fp32"): "configs[1]",
                 (8, 768, 4096, "bf16", "fp32"): "configs[2]", (8, 768, 8192, "bf16", "fp16"): "configs[3]",
                 (16, 1024, 16384, "fp32", "fp32"): "configs[4]"}
SWEEP_EXTRA = [(8, 768, 4096, "bf16", "fp32"), (8, 768, 8192, "bf16", "fp16"), (16, 1024, 16384, "fp32", "fp32"),
               (8, 768, 65536, "fp32", "fp32")]   # the last: a composite plan (partitioned convolution, 4 blocks)


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        p = json.load(open(path))
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def flops_per_seq(radices):
    N = 1
    for r in radices:
        N *= r
    return 4 * radices[0] * N + 16 * N * sum(radices[1:])


def roofline(B, H, L, io, radices, ms):
    """(bound, achieved, peak, unit, frac, alg_bytes, alg_flops, t_roof_ms) of one batch in `ms`."""
    s_io = 4 if io == "fp32" else 2
    alg_bytes = 2 * B * H * L * s_io + H * 2 * L * 8
    alg_flops = B * H * flops_per_seq(radices)
    hbm, tc, _ = peaks()
    t_hbm, t_tc = alg_bytes / (hbm * 1e9), alg_flops / (tc * 1e12)
    if t_hbm >= t_tc:
        bound, achieved, peak, unit = "hbm", alg_bytes / (ms * 1e-3) / 1e9, hbm, "GB/s"
    else:
        bound, achieved, peak, unit = "tensor", alg_flops / (ms * 1e-3) / 1e12, tc, "TFLOP/s"
    return bound, achieved, peak, unit, achieved / peak, alg_bytes, alg_flops, max(t_hbm, t_tc) * 1e3


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--L", type=int, default=1024)
    ap.add_argument("--B", type=int, default=8)
    ap.add_argument("--H", type=int, default=768, help="channels of the whole batch (sharded over the GPUs)")
    ap.add_argument("--io", default="fp32", choices=["fp32", "bf16"])
    ap.add_argument("--acc", default="fp32", choices=["fp32", "fp16"])
    ap.add_argument("--config", default=None)
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--chunks", type=int, default=0, help="chunks of the host-buffer pipeline (0 = 4)")
    ap.add_argument("--sweep", default="auto", choices=["auto", "on", "off"],
                    help="metric sweep and configurations 2-4 (auto: at N = 1 only)")
    ap.add_argument("--weak", default="auto", choices=["auto", "on", "off"],
                    help="per-GPU-fixed batch beside the sharded one (auto: at N > 1 only)")
    return ap.parse_args()


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        time.sleep(0.3)

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.2)
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        loaded = [s for s in sm if smax and s > 0.5 * smax] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


def make_inputs(torch, dev, B, H, L, io, seed, decay=4.0, sqrt_norm=True):
    """Seeded u [B][H][L] ~ N(0,1) and k [H][L] = N(0,1) exp(-decay n / L) [/ sqrt(L)], both rounded to bf16
    for bf16 I/O."""
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    u = torch.randn((B, H, L), device=dev, generator=g)
    n = torch.arange(L, device=dev, dtype=torch.float32)
    k = torch.randn((H, L), device=dev, generator=g) * torch.exp(-decay * n / L)
    if sqrt_norm:
        k = k / L ** 0.5
    if io == "bf16":
        u, k = u.to(torch.bfloat16), k.to(torch.bfloat16)
    return u, k


def n_sets(B, H, L, io):
    """Rotating input/output/spectrum sets: enough for their total to exceed L2 about twice."""
    s_io = 4 if io == "fp32" else 2
    per = 2 * B * H * L * s_io + H * 2 * L * 8
    return int(min(64, max(2, math.ceil(2.2 * L2_BYTES / per))))


def event_time(torch, stream, fn, steps):
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(steps):
        fn(i)
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def cpu_baseline_run(args, budget_s=15.0):
    """fp64 direct convolution of a bounded sample on all host cores; returns (ms per full batch, info)."""
    import numpy as np

    from tests.oracle_py import Oracle
    oracle = Oracle()
    B, H, L = args.B, args.H, args.L
    rng = np.random.default_rng(0)
    u = rng.standard_normal((B, H, L)).astype(np.float32)
    k = (rng.standard_normal((H, L)) * np.exp(-4.0 * np.arange(L) / L) / np.sqrt(L)).astype(np.float32)
    total = B * H
    # size the sample to roughly budget_s of work from a short calibration
    t0 = time.perf_counter()
    # every host core this process may use (launchers such as torchrun set OMP_NUM_THREADS=1 per rank)
    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    oracle.direct_conv_seqs(u, k, np.arange(min(64, total)), threads=cores)
    per_seq = (time.perf_counter() - t0) / min(64, total)
    n = int(max(64, min(total, budget_s / max(per_seq, 1e-9))))
    seqs = np.linspace(0, total - 1, n).astype(np.int64)
    # a batch that takes less than the budget is repeated, so the sample is always ~budget_s of work
    reps = 0
    t0 = time.perf_counter()
    while True:
        oracle.direct_conv_seqs(u, k, seqs, threads=cores)
        reps += 1
        dt = time.perf_counter() - t0
        if n < total or dt >= budget_s or reps >= 10000:
            break
    ms_batch = dt * 1e3 * total / (n * reps)
    what = f"{n} of {total} sequences" if n < total else f"the full batch of {total} sequences x {reps}"
    return ms_batch, {"cores": cores, "sample": f"{what} (B={B} H={H} L={L}), fp64 direct causal "
                      f"convolution, {dt:.1f} s, scaled to ms per batch", "seconds": round(dt, 2)}


def run_reference(args, world, rank):
    if rank != 0:
        return
    ms_steps = []
    for _ in range(max(1, args.warmup // 3)):
        cpu_baseline_run(args, budget_s=2.0)
    for _ in range(args.steps if args.steps <= 5 else 5):
        ms, info = cpu_baseline_run(args, budget_s=10.0)
        ms_steps.append(ms)
    value = statistics.median(ms_steps)
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": args.gpus,
            "steps": len(ms_steps), "warmup": max(1, args.warmup // 3), "ms_per_step": round(value, 4),
            "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "f64",
            "data": "synthetic", "config": {"workload": f"causal long conv B={args.B} H={args.H} L={args.L}",
                                            "B": args.B, "H": args.H, "L": args.L, "io": args.io},
            "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": info["cores"], "kind": "port",
                             "sample": info["sample"]},
            "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


class Workload:
    """A plan and rotating device sets for B x H channels [h0, h0 + H) of a batch."""

    def __init__(self, torch, sf, dev, local, B, H, L, io, acc, config, seed, decay=4.0, sqrt_norm=True,
                 sets=None):
        self.torch, self.B, self.H, self.L, self.io = torch, B, H, L, io
        self.plan = sf.Plan(L, io=io, acc=acc, config=config, device=local)
        self.stream = torch.cuda.current_stream(dev)
        self.sets = []
        for s in range(sets or n_sets(B, H, L, io)):
            u, k = make_inputs(torch, dev, B, H, L, io, seed + s, decay=decay, sqrt_norm=sqrt_norm)
            Kf = self.plan.filter_spectrum(k, stream=self.stream)
            self.sets.append((u, Kf, torch.empty_like(u), k))
        torch.cuda.synchronize(dev)

    def step(self, i):
        u, Kf, y, _ = self.sets[i % len(self.sets)]
        st = self.plan.conv_ptr(u.data_ptr(), Kf.data_ptr(), y.data_ptr(), self.B, self.H, self.stream)
        if st:
            import sffft_b200 as sf
            raise sf.SffftError(st, "conv")

    def time(self, steps, warmup):
        for i in range(warmup):
            self.step(i)
        self.plan.check()
        ms = event_time(self.torch, self.stream, self.step, steps)
        self.plan.check()
        return ms

    def parity(self, oracle, nseq=6):
        """Max relative L2 of sampled sequences of set 0 against the fp64 oracle (run once more first)."""
        import numpy as np
        self.step(0)
        self.plan.check()
        u, _, y, k = self.sets[0]
        un, kn, yn = u.float().cpu().numpy(), k.float().cpu().numpy(), y.float().cpu().numpy()
        total = self.B * self.H
        seqs = np.unique(np.linspace(0, total - 1, min(nseq, total)).astype(np.int64))
        ref = oracle.direct_conv_seqs(un, kn, seqs)
        got = yn.reshape(total, self.L)[seqs].astype(np.float64)
        errs = np.sqrt(np.sum((got - ref) ** 2, axis=1) / np.maximum(np.sum(ref ** 2, axis=1), 1e-300))
        return float(errs.max()), len(seqs)

    def close(self):
        self.plan.close()
        self.sets = []


def cufft_ms(torch, sf, dev, wl, steps, warmup):
    """The cuFFT pipeline (sffft_baseline_run, full = pad -> R2C -> x spectrum -> C2R -> slice) on the same
    rotating sets (fp32: the pipeline's own type), timed like the fused kernel."""
    fsets = [(u.float(), torch.empty(u.shape, dtype=torch.float32, device=dev)) for u, _, _, _ in wl.sets]
    k = wl.sets[0][3].float().contiguous()
    bl = sf.Baseline(wl.L, wl.B, wl.H, k, device=dev.index)
    stream = torch.cuda.current_stream(dev)

    def step(i):
        u, y = fsets[i % len(fsets)]
        bl.run(u, y, full=True, stream=stream)

    for i in range(warmup):
        step(i)
    torch.cuda.synchronize(dev)
    ms = event_time(torch, stream, step, steps)
    bl.close()
    del fsets
    return ms


def run_sweep(torch, sf, dev, local, steps, warmup):
    points = [(8, 768, L, io, "fp32") for io in ("fp32", "bf16") for L in (128, 256, 512, 1024, 2048, 4096, 8192)]
    points += [c for c in SWEEP_EXTRA if c not in points]
    out = []
    for B, H, L, io, acc in points:
        decay, sqrt_norm = (8.0, True) if L == 16384 else (4.0, True)
        wl = Workload(torch, sf, dev, local, B, H, L, io, acc, None, seed=500 + L, decay=decay, sqrt_norm=sqrt_norm)
        ms = wl.time(steps, warmup)
        bound, achieved, peak, unit, frac, _, _, _ = roofline(B, H, L, io, wl.plan.radices, ms)
        try:
            cms = cufft_ms(torch, sf, dev, wl, steps, warmup)
        except Exception as exc:   # reported, not fatal: the sweep's fused numbers stand on their own
            cms = None
            print(f"cuFFT pipeline failed at L={L}: {exc}", file=sys.stderr)
        label = NAMED_CONFIGS.get((B, H, L, io, acc), "composite" if wl.plan.blocks > 1 else "sweep")
        out.append({"config": label, "B": B, "H": H, "L": L, "io": io,
                    "acc": acc, "plan": wl.plan.config, "ms": round(ms, 5), "bound": bound,
                    "achieved": round(achieved, 2), "unit": unit, "frac": round(frac, 4),
                    "cufft_ms": round(cms, 5) if cms else None,
                    "vs_cufft": round(cms / ms, 3) if cms else None, "sets": len(wl.sets)})
        wl.close()
        torch.cuda.empty_cache()
    return out


def main():
    args = parse()
    world, rank, local = dist_setup(args)
    if args.impl == "reference":
        run_reference(args, world, rank)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return

    import torch

    import sffft_b200 as sf
    from tests.oracle_py import Oracle

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    B, H, L = args.B, args.H, args.L
    h0, h1 = sf.shard_range(H, world, rank)
    Hg = h1 - h0
    # this rank's channel shard of the batch (its own seeded data of the batch's distribution)
    wl = Workload(torch, sf, dev, local, B, Hg, L, args.io, args.acc, args.config, seed=1000 + h0)
    plan = wl.plan

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier(device_ids=[local])

    def allmax(x):
        if world == 1:
            return x
        import torch.distributed as dist
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for i in range(args.warmup):
        wl.step(i)
    plan.check()
    clocks = ClockSampler(local)
    clocks.start()
    barrier()
    torch.cuda.synchronize(dev)
    ms_step = event_time(torch, wl.stream, wl.step, args.steps)
    barrier()
    clk = clocks.stop()
    plan.check()
    ms_step = allmax(ms_step)

    # parity of this rank's shard against the fp64 oracle (outside the timed region), max over ranks
    oracle = Oracle()
    perr, nchk = wl.parity(oracle)
    perr = allmax(perr)

    # end to end through the public host-buffer call (sffft_conv_host): every step uploads the shard of u from
    # pinned host memory, runs the fused convolution and downloads y, in chunks whose copies and kernels overlap
    u_h = wl.sets[0][0].cpu().pin_memory()
    y_h = torch.zeros_like(u_h).pin_memory()
    Kf_d = wl.sets[0][1]
    pipe = sf.HostPipe(plan, B, Hg, args.chunks)
    pipe_chunks = args.chunks if args.chunks > 0 else 4
    for _ in range(max(args.warmup, 30)):
        pipe.conv(u_h, Kf_d, y_h, stream=wl.stream)
    torch.cuda.synchronize(dev)
    barrier()
    e2e_step = event_time(torch, wl.stream, lambda i: pipe.conv(u_h, Kf_d, y_h, stream=wl.stream), args.e2e_steps)
    plan.check()
    pipe.close()
    e2e_step = allmax(e2e_step)
    # this rank's plain copy rates over PCIe (each direction alone, pinned buffers)
    u_d = torch.empty_like(wl.sets[0][0])
    h2d_ms = event_time(torch, wl.stream, lambda i: u_d.copy_(u_h, non_blocking=True), 5)
    d2h_ms = event_time(torch, wl.stream, lambda i: y_h.copy_(u_d, non_blocking=True), 5)
    nbytes = u_h.numel() * u_h.element_size()

    # per-GPU-fixed batch (weak scaling): every rank convolves a whole B x H batch of its own
    weak = None
    if args.weak == "on" or (args.weak == "auto" and world > 1):
        wk = Workload(torch, sf, dev, local, B, H, L, args.io, args.acc, args.config, seed=2000 + rank)
        wms = allmax(wk.time(args.steps, args.warmup))
        wk.close()
        weak = {"ms_per_step": round(wms, 5), "value": round(wms / world, 5), "unit": UNIT, "H_per_gpu": H,
                "H_total": H * world, "what": f"each of the {world} GPUs convolves its own B={B} x H={H} batch; "
                                              "value = max step time / N per batch"}

    sweep = None
    if rank == 0 and (args.sweep == "on" or (args.sweep == "auto" and world == 1)):
        sweep = run_sweep(torch, sf, dev, local, max(10, min(args.steps, 30)), max(3, args.warmup))

    if rank == 0:
        bound, achieved, peak, unit, frac, alg_bytes, alg_flops, t_roof = roofline(B, H, L, args.io, plan.radices,
                                                                                   ms_step)
        _, _, src = peaks()
        traffic = None
        tp = os.path.join(ROOT, "profiles", "traffic.json")
        if os.path.exists(tp):
            traffic = json.load(open(tp)).get(f"{plan.config}|{args.io}|{L}|{B}x{H}") if world == 1 else None
        cpu_ms, cpu_info = (None, None)
        if world == 1:
            cpu_ms, cpu_info = cpu_baseline_run(args)
        pub = GB10_PUBLISHED_MS.get((L, args.io)) if (B, H, args.acc) == (8, 768, "fp32") else None
        name = NAMED_CONFIGS.get((B, H, L, args.io, args.acc), "custom")
        line = {
            "metric": METRIC, "value": round(ms_step, 5), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 5), "higher_is_better": False, "scaling": "strong",
            "vs_baseline": round(ms_step / pub, 4) if pub else None, "dtype": "f16",
            "data": "synthetic (seeded torch.randn u; k = N(0,1) exp(-4n/L)/sqrt(L))",
            "config": {"workload": f"{name}: causal long conv B={B} H={H} L={L}, {args.io} I/O, {args.acc} "
                                   f"accumulation, channel-sharded over {world} GPU(s)",
                       "plan": plan.config, "B": B, "H_total": H, "H_per_gpu": Hg, "L": L, "io": args.io,
                       "acc": args.acc, "smem_bytes": plan.info["smem_bytes"],
                       "parallelism": f"channel-sharded x{world} (fixed batch), no collective on the data path",
                       "l2": f"{len(wl.sets)} rotating input/output/spectrum sets per GPU "
                             f"(> 126 MB L2 in aggregate at N = 1)",
                       "vs_baseline_ref": "reference GB10 published ms/batch (README.md:29-35)" if pub else None},
            "roofline": {"bound": bound, "achieved": round(achieved, 2), "peak": peak, "unit": unit,
                         "frac": round(frac, 4), "traffic": traffic,
                         "traffic_source": "ncu, one launch: dram__bytes_read.sum + lts__t_sectors_srcunit_tex_op_write.sum"
                                           " x 32 B (stores = y's write-back) (profiles/traffic.json)" if traffic else None,
                         "peak_source": f"{src} (MEASURED_PEAKS.json)" if src == "measured" else src,
                         "algorithmic_bytes": alg_bytes, "algorithmic_flops": alg_flops, "t_roof_ms": round(t_roof, 5)},
            "e2e": {"value": round(e2e_step, 5), "unit": UNIT, "h2d_bytes_per_step": nbytes,
                    "d2h_bytes_per_step": nbytes, "h2d_gbs": round(nbytes / (h2d_ms * 1e6), 2),
                    "d2h_gbs": round(nbytes / (d2h_ms * 1e6), 2),
                    "path": f"pinned host u -> sffft_conv_host (C ABI: ~{pipe_chunks} chunks, upload / fused conv / "
                            "download overlapped, one stream per stage) -> pinned host y, per step, per GPU shard "
                            "(h2d_gbs / d2h_gbs: rank 0's plain copy rate of its shard, each direction alone)"},
            "parity": {"max_rel_l2": perr, "seqs_checked": nchk, "ranks": world,
                       "what": "sampled sequences of every rank's output vs the fp64 direct convolution"},
            "gpu_launches": args.steps * world,
            "clocks": clk,
        }
        if weak:
            line["weak_scaling"] = weak
        if sweep:
            line["sweep"] = sweep
        if cpu_ms is not None:
            line["cpu_baseline"] = {"value": round(cpu_ms, 3), "unit": UNIT, "cores": cpu_info["cores"], "kind": "port",
                                    "sample": cpu_info["sample"]}
        print(json.dumps(line), flush=True)
    wl.close()
    barrier()
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
