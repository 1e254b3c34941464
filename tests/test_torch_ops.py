"""The PyTorch operators over the C ABI: registration, shape inference without a GPU (meta tensors, the path
torch.compile traces), and refusal of CPU tensors (there is no CPU path)."""
import pytest
import torch

import sffft_b200.torch_ops  # noqa: F401  (registers torch.ops.sffft.*)


def test_operators_are_registered():
    assert hasattr(torch.ops.sffft, "conv") and hasattr(torch.ops.sffft, "filter_spectrum")


def test_fake_shapes_on_meta_tensors():
    u = torch.empty((8, 768, 1024), device="meta")
    k = torch.empty((768, 1024), device="meta", dtype=torch.bfloat16)
    Kf = torch.ops.sffft.filter_spectrum(k)
    assert Kf.shape == (768, 2048, 2) and Kf.dtype == torch.float32
    y = torch.ops.sffft.conv(u.to(torch.bfloat16), Kf, "fp16")
    assert y.shape == u.shape and y.dtype == torch.bfloat16


def test_cpu_tensors_are_refused():
    with pytest.raises(ValueError):
        torch.ops.sffft.filter_spectrum(torch.zeros((2, 128)))
    with pytest.raises(ValueError):
        torch.ops.sffft.conv(torch.zeros((1, 2, 128)), torch.zeros((2, 256, 2)))


def test_fake_shapes_of_filter_layouts():
    k2 = torch.empty((6, 2 * 512 - 1), device="meta")
    assert torch.ops.sffft.filter_spectrum(k2, "", "two_sided").shape == (6, 1024, 2)
    kc = torch.empty((6, 512), device="meta")
    assert torch.ops.sffft.filter_spectrum(kc, "", "circular").shape == (6, 1024, 2)
    with pytest.raises(ValueError):
        torch.ops.sffft.filter_spectrum(torch.empty((6, 512), device="meta"), "", "two_sided")
    with pytest.raises(ValueError):
        torch.ops.sffft.filter_spectrum(kc, "", "acausal")


def test_fake_shapes_of_ffts():
    X = torch.ops.sffft.rfft(torch.empty((3, 4, 2048), device="meta"))
    assert X.shape == (3, 4, 1025) and X.dtype == torch.complex64
    x = torch.ops.sffft.irfft(X)
    assert x.shape == (3, 4, 2048) and x.dtype == torch.float32
    with pytest.raises(ValueError):
        torch.ops.sffft.rfft(torch.zeros((2, 256)))
