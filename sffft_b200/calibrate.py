"""B200 calibration of every catalog plan: the measurements behind the built-in default plan per length.

    python -m sffft_b200.calibrate > sffft_b200/csrc/calibration_b200.csv
    python sffft_b200/csrc/make_calibration.py sffft_b200/csrc/calibration_b200.csv > sffft_b200/csrc/calibration.h

For L = 128 .. 16384 and every catalog plan of that length, both I/O types (fp32 accumulation, cached DFT
tables): B = 8, H = 768, seeded u ~ N(0,1) and k = N(0,1) exp(-4n/L) / sqrt(L), timed like the benchmark -- CUDA
events around `steps` launches that rotate over enough input/output/spectrum sets to exceed the 126 MB L2 about
twice, so every launch reads its operands from HBM -- and checked against an fp64 FFT convolution of one set.
Prints one row per candidate: CAL,L,plan,io,ms,rel_err.  (The `sffft` CLI's calibration instead times repeated
launches on one set of buffers, the reference's method, which keeps small problems in L2.)
"""
import math
import sys

import torch

import sffft_b200 as sf

L2_BYTES = 126 * 1024 * 1024


def fp64_conv(u, k):
    L = u.shape[-1]
    U = torch.fft.rfft(u.double(), n=2 * L)
    K = torch.fft.rfft(k.double(), n=2 * L)
    return torch.fft.irfft(U * K[None], n=2 * L)[..., :L]


def time_plan(plan, sets, B, H, steps, warmup):
    stream = torch.cuda.current_stream()
    for i in range(warmup):
        u, Kf, y = sets[i % len(sets)]
        plan.conv(u, Kf, y)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(steps):
        u, Kf, y = sets[i % len(sets)]
        st = plan.conv_ptr(u.data_ptr(), Kf.data_ptr(), y.data_ptr(), B, H, stream)
        if st:
            raise sf.SffftError(st, "conv")
    e1.record(stream)
    torch.cuda.synchronize()
    plan.check()
    return e0.elapsed_time(e1) / steps


def main(B=8, H=768, steps=20, warmup=3):
    dev = torch.device("cuda:0")
    print("# CAL,L,plan,io,ms,rel_err  (B=%d H=%d, %d timed launches over rotating sets, fp32 accumulation)" % (B, H, steps))
    by_len = {}
    for L, name in sf.catalog():
        by_len.setdefault(L, []).append(name)
    for L in sorted(by_len):
        for io in ("fp32", "bf16"):
            dt = torch.float32 if io == "fp32" else torch.bfloat16
            s_io = 4 if io == "fp32" else 2
            per = 2 * B * H * L * s_io + H * 2 * L * 8
            nsets = int(min(64, max(2, math.ceil(2.2 * L2_BYTES / per))))
            g = torch.Generator(device=dev)
            g.manual_seed(L)
            n = torch.arange(L, device=dev, dtype=torch.float32)
            raw = [(torch.randn((B, H, L), device=dev, generator=g).to(dt),
                    (torch.randn((H, L), device=dev, generator=g) * torch.exp(-4.0 * n / L) / L ** 0.5).to(dt))
                   for _ in range(nsets)]
            ref = fp64_conv(raw[0][0].float(), raw[0][1].float())
            for name in by_len[L]:
                plan = sf.Plan(L, io=io, config=name)
                sets = [(u, plan.filter_spectrum(k), torch.empty_like(u)) for u, k in raw]
                ms = time_plan(plan, sets, B, H, steps, warmup)
                y = sets[0][2].double()
                err = float(torch.linalg.vector_norm(y - ref) / torch.linalg.vector_norm(ref))
                print(f"CAL,{L},{name},{io},{ms:.5f},{err:.3e}", flush=True)
                plan.close()
                del sets
            del raw, ref
            torch.cuda.empty_cache()


if __name__ == "__main__":
    main(*[int(a) for a in sys.argv[1:]])
