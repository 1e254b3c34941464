"""The host-buffer pipeline (sffft_pipe_create / sffft_conv_host): channel chunks of a batch in pinned host
memory are uploaded, convolved and downloaded on three streams.  Per-pair results do not depend on how
pairs are grouped, so the output must equal sffft_conv on the whole device batch bit for bit, for chunk
counts that divide H and ones that leave a short last chunk, the default chunking, odd B, both I/O types."""
import pytest
import torch

import sffft_b200 as sf

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("L,B,H,io,chunks", [(1024, 8, 96, "fp32", 0), (512, 7, 37, "bf16", 0), (1024, 5, 37, "fp32", 4),
                                             (128, 3, 50, "bf16", 7), (4096, 2, 9, "bf16", 3),
                                             (256, 4, 3, "fp32", 8)])
def test_host_pipe_equals_device_path(L, B, H, io, chunks):
    dt = torch.bfloat16 if io == "bf16" else torch.float32
    g = torch.Generator().manual_seed(L + B + H)
    u = torch.randn((B, H, L), generator=g).to(dt)
    k = (torch.randn((H, L), generator=g) / L ** 0.5).to(dt)
    plan = sf.Plan(L, io=io)
    Kf = plan.filter_spectrum(k.cuda())
    ref = plan.conv(u.cuda(), Kf).cpu()
    u_h = u.pin_memory()
    y_h = torch.full_like(u_h, float("nan")).pin_memory()
    pipe = sf.HostPipe(plan, B, H, chunks)
    for _ in range(2):                      # the pipe is reusable; a second call overwrites y
        pipe.conv(u_h, Kf, y_h)
        torch.cuda.synchronize()
        plan.check()
        assert torch.equal(y_h, ref)
    pipe.close()
    plan.close()


def test_pipe_rejects_wrong_shapes():
    plan = sf.Plan(128)
    pipe = sf.HostPipe(plan, 2, 4)
    u = torch.zeros((2, 5, 128)).pin_memory()
    with pytest.raises(ValueError):
        pipe.conv(u, torch.zeros((4, 256, 2), device="cuda"), u)
    pipe.close()
    plan.close()
