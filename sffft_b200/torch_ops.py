"""PyTorch operators over the C ABI (the packaging the reference names as its next step, README.md:177).

    import sffft_b200.torch_ops  # registers the operators
    Kf = torch.ops.sffft.filter_spectrum(k)            # k [H][L] fp32 or bf16 -> Kf [H][2L][2] fp32
    y = torch.ops.sffft.conv(u, Kf)                    # u [B][H][L] fp32 or bf16 -> y, same shape and type
    y = sffft_b200.torch_ops.causal_conv(u, k)         # both steps
    y = sffft_b200.torch_ops.two_sided_conv(u, k2)     # non-causal: k2 [H][2L-1], k2[:, L-1] is lag 0
    y = sffft_b200.torch_ops.circular_conv(u, kc)      # period-L circular: kc [H][L]
    X = torch.ops.sffft.rfft(x)                        # x [..., N] fp32/bf16 -> X [..., N/2+1] complex64
    x = torch.ops.sffft.irfft(X)                       # X [..., N/2+1] complex64 -> x [..., N] fp32

Both run on the current CUDA stream of the tensors' device through sffft_filter_spectrum / sffft_conv, so
they order with surrounding PyTorch work and can be captured in CUDA graphs once a first call has created
the plan (plan creation allocates).  Fake implementations give output shapes and types without running
anything, so the operators trace under torch.compile.  Forward only: the path has no backward kernel.

`acc` is "fp32" or "fp16" (accumulation mode); `config` names a catalog plan ("" = the default for L).
filter_spectrum and conv must use the same config: the spectrum is in that plan's digit order.
`layout` ("causal", "two_sided", "circular") says which convolution the spectrum makes conv compute; the
fused kernel is the same for all three.
"""
import threading

import torch
from torch import Tensor

import sffft_b200 as sf

_plans: dict = {}
_lock = threading.Lock()


def _plan(L: int, io: str, acc: str, config: str, device: int) -> "sf.Plan":
    key = (L, io, acc, config, device)
    with _lock:
        p = _plans.get(key)
        if p is None:
            p = sf.Plan(L, io=io, acc=acc, config=config or None, device=device)
            _plans[key] = p
    return p


def _check_cuda(t: Tensor, what: str):
    if t.device.type != "cuda":
        raise ValueError(f"sffft::{what} needs CUDA tensors (there is no CPU path)")


def _filter_length(k: Tensor, layout: str) -> int:
    """The sequence length L a filter row of this layout belongs to."""
    if layout not in sf.FILTER:
        raise ValueError(f"layout must be one of {sorted(sf.FILTER)}")
    if k.dim() != 2 or k.dtype not in (torch.float32, torch.bfloat16):
        raise ValueError("k must be a 2-D float32 or bfloat16 tensor")
    width = k.shape[1]
    if layout == "two_sided":
        if width % 2 == 0:
            raise ValueError("a two-sided filter has 2L-1 taps")
        return (width + 1) // 2
    return width


@torch.library.custom_op("sffft::filter_spectrum", mutates_args=())
def filter_spectrum(k: Tensor, config: str = "", layout: str = "causal") -> Tensor:
    _check_cuda(k, "filter_spectrum")
    L = _filter_length(k, layout)
    H = k.shape[0]
    dev = k.device.index if k.device.index is not None else torch.cuda.current_device()
    plan = _plan(L, "fp32", "fp32", config, dev)
    Kf = torch.empty((H, 2 * L, 2), dtype=torch.float32, device=k.device)
    return plan.filter_spectrum(k.contiguous(), Kf, stream=torch.cuda.current_stream(k.device), layout=layout)


@filter_spectrum.register_fake
def _(k: Tensor, config: str = "", layout: str = "causal") -> Tensor:
    L = _filter_length(k, layout)
    return k.new_empty((k.shape[0], 2 * L, 2), dtype=torch.float32)


@torch.library.custom_op("sffft::conv", mutates_args=())
def conv(u: Tensor, Kf: Tensor, acc: str = "fp32", config: str = "") -> Tensor:
    _check_cuda(u, "conv")
    if u.dim() != 3 or u.dtype not in (torch.float32, torch.bfloat16):
        raise ValueError("u must be [B][H][L], float32 or bfloat16")
    B, H, L = u.shape
    if tuple(Kf.shape) != (H, 2 * L, 2) or Kf.dtype != torch.float32 or Kf.device != u.device:
        raise ValueError("Kf must be the [H][2L][2] float32 spectrum on u's device")
    io = "bf16" if u.dtype == torch.bfloat16 else "fp32"
    dev = u.device.index if u.device.index is not None else torch.cuda.current_device()
    plan = _plan(L, io, acc, config, dev)
    y = torch.empty_like(u, memory_format=torch.contiguous_format)
    plan.conv(u.contiguous(), Kf.contiguous(), y, stream=torch.cuda.current_stream(u.device))
    return y


@conv.register_fake
def _(u: Tensor, Kf: Tensor, acc: str = "fp32", config: str = "") -> Tensor:
    return torch.empty_like(u, memory_format=torch.contiguous_format)


def causal_conv(u: Tensor, k: Tensor, acc: str = "fp32", config: str = "") -> Tensor:
    """y[b,h,n] = sum_{m<=n} u[b,h,m] k[h,n-m]: the spectrum of k, then the fused convolution."""
    return conv(u, filter_spectrum(k, config), acc, config)


def two_sided_conv(u: Tensor, k: Tensor, acc: str = "fp32", config: str = "") -> Tensor:
    """Non-causal: y[b,h,n] = sum_{m<L} u[b,h,m] k[h,L-1+n-m] for k [H][2L-1] (k[:, L-1] is lag 0)."""
    return conv(u, filter_spectrum(k, config, "two_sided"), acc, config)


def circular_conv(u: Tensor, k: Tensor, acc: str = "fp32", config: str = "") -> Tensor:
    """Period-L circular: y[b,h,n] = sum_{m<L} u[b,h,m] k[h,(n-m) mod L] for k [H][L]."""
    return conv(u, filter_spectrum(k, config, "circular"), acc, config)


def _fft_plan(N: int, config: str, device) -> "sf.Plan":
    if N < 256 or N & (N - 1):
        raise ValueError("the transform length must be a power of two from 256 to 32768")
    dev = device.index if device.index is not None else torch.cuda.current_device()
    return _plan(N // 2, "fp32", "fp32", config, dev)


@torch.library.custom_op("sffft::rfft", mutates_args=())
def rfft(x: Tensor, config: str = "") -> Tensor:
    """Real DFT along the last axis (numpy.fft.rfft), fp32 with exact twiddles."""
    _check_cuda(x, "rfft")
    if x.dtype not in (torch.float32, torch.bfloat16):
        raise ValueError("x must be float32 or bfloat16")
    plan = _fft_plan(x.shape[-1], config, x.device)
    return plan.rfft(x.contiguous(), stream=torch.cuda.current_stream(x.device))


@rfft.register_fake
def _(x: Tensor, config: str = "") -> Tensor:
    return x.new_empty(tuple(x.shape[:-1]) + (x.shape[-1] // 2 + 1,), dtype=torch.complex64)


@torch.library.custom_op("sffft::irfft", mutates_args=())
def irfft(X: Tensor, config: str = "") -> Tensor:
    """Inverse of rfft for an even length N = 2 (X.shape[-1] - 1) (numpy.fft.irfft)."""
    _check_cuda(X, "irfft")
    if X.dtype != torch.complex64:
        raise ValueError("X must be complex64")
    plan = _fft_plan(2 * (X.shape[-1] - 1), config, X.device)
    return plan.irfft(X.contiguous(), stream=torch.cuda.current_stream(X.device))


@irfft.register_fake
def _(X: Tensor, config: str = "") -> Tensor:
    return X.new_empty(tuple(X.shape[:-1]) + (2 * (X.shape[-1] - 1),), dtype=torch.float32)
