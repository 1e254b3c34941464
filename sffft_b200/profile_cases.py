"""Small seeded workloads of each kernel of the library, for profiler captures of one kernel at a time.

    python -m sffft_b200.profile_cases fused <plan> <L> <fp32|bf16> <B> <H>   4 fused convolutions
    python -m sffft_b200.profile_cases spectrum <L> <H>                         3 filter spectra (digit stages)
    python -m sffft_b200.profile_cases fft <L> <rows>                           3 forward + inverse FFTs, N = 2L
    python -m sffft_b200.profile_cases composite <L> <B> <H>                    3 composite-plan convolutions
    python -m sffft_b200.profile_cases baseline <L> <B> <H>                     3 cuFFT-pipeline convolutions

Every case runs on cuda:0 with torch-generated inputs (seed 0) and prints "ok <case>" when it is done.  The
profiles of the library name the command that made them in this form.
"""
import sys

import torch

import sffft_b200 as sf


def main(argv):
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    case = argv[0]
    if case == "fused":
        name, L, io, B, H = argv[1], int(argv[2]), argv[3], int(argv[4]), int(argv[5])
        plan = sf.Plan(L, io=io, config=name)
        dt = torch.bfloat16 if io == "bf16" else torch.float32
        u = torch.randn((B, H, L), device=dev, generator=g).to(dt)
        k = (torch.randn((H, L), device=dev, generator=g) / L ** 0.5).to(dt)
        Kf = plan.filter_spectrum(k)
        for _ in range(4):
            plan.conv(u, Kf)
    elif case == "spectrum":
        L, H = int(argv[1]), int(argv[2])
        plan = sf.Plan(L)
        k = torch.randn((H, L), device=dev, generator=g)
        for _ in range(3):
            plan.filter_spectrum(k)
    elif case == "fft":
        L, rows = int(argv[1]), int(argv[2])
        plan = sf.Plan(L)
        x = torch.randn((rows, 2 * L), device=dev, generator=g)
        for _ in range(3):
            plan.irfft(plan.rfft(x))
    elif case == "composite":
        L, B, H = int(argv[1]), int(argv[2]), int(argv[3])
        plan = sf.Plan(L)
        u = torch.randn((B, H, L), device=dev, generator=g)
        k = torch.randn((H, L), device=dev, generator=g) / L ** 0.5
        Kf = plan.filter_spectrum(k)
        for _ in range(3):
            plan.conv(u, Kf)
    elif case == "baseline":
        L, B, H = int(argv[1]), int(argv[2]), int(argv[3])
        u = torch.randn((B, H, L), device=dev, generator=g)
        k = torch.randn((H, L), device=dev, generator=g) / L ** 0.5
        y = torch.empty_like(u)
        bl = sf.Baseline(L, B, H, k)
        for _ in range(3):
            bl.run(u, y, full=True)
        bl.close()
    else:
        raise SystemExit(f"unknown case {case!r}")
    torch.cuda.synchronize()
    print("ok", case)


if __name__ == "__main__":
    main(sys.argv[1:])
