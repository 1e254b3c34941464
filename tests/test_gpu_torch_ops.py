"""torch.ops.sffft.* on the device: identical results to the plan API, inside torch.compile(fullgraph=True)
too, on the current stream of a side stream, for fp32 and bf16 I/O."""
import pytest
import torch

import sffft_b200 as sf
import sffft_b200.torch_ops as ops

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("L,io,acc", [(1024, "fp32", "fp32"), (4096, "bf16", "fp32"), (128, "bf16", "fp16")])
def test_ops_equal_plan_api(L, io, acc):
    dt = torch.bfloat16 if io == "bf16" else torch.float32
    g = torch.Generator(device="cuda").manual_seed(L)
    u = torch.randn((4, 6, L), device="cuda", generator=g).to(dt)
    k = (torch.randn((6, L), device="cuda", generator=g) / L ** 0.5).to(dt)
    plan = sf.Plan(L, io=io, acc=acc)
    ref = plan.conv(u, plan.filter_spectrum(k))
    plan.check()
    y = ops.causal_conv(u, k, acc)
    torch.cuda.synchronize()
    assert torch.equal(y, ref)
    compiled = torch.compile(lambda a, b: torch.ops.sffft.conv(a, torch.ops.sffft.filter_spectrum(b), acc),
                             fullgraph=True)
    assert torch.equal(compiled(u, k), ref)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        y2 = ops.causal_conv(u, k, acc)
    s.synchronize()
    assert torch.equal(y2, ref)
    plan.close()


def test_fft_operators(cuda_device):
    x = torch.randn((2, 3, 1024), device=cuda_device)
    X = torch.ops.sffft.rfft(x)
    ref = torch.fft.rfft(x.double())
    assert (torch.linalg.norm(X.cdouble() - ref) / torch.linalg.norm(ref)).item() < 3e-6
    xr = torch.ops.sffft.irfft(X)
    assert (torch.linalg.norm(xr - x) / torch.linalg.norm(x)).item() < 3e-6
