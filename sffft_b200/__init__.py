"""sffft_b200: B200 (sm_100a) fused causal long convolution.

    y[b, h, n] = sum_{m <= n} u[b, h, m] * k[h, n - m],   n < L

Python mirror of the C ABI in ``include/sffft.h`` (itself the drop-in for the operator surface of
sfFFT's ``src/sffft.cu`` and ``src/selection.h``).  Device buffers are torch CUDA tensors (or raw
device pointers); every native call raises :class:`SffftError` on a non-zero status.  There is no CPU
fallback: if ``lib/libsffft.so`` is missing or the device is not a B200, calls fail.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass
from typing import Optional, Sequence

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "lib", "libsffft.so")
EMU_PATH = os.path.join(_HERE, "lib", "libsffft_emu.so")
CLI_PATH = os.path.join(_HERE, "bin", "sffft")

(OK, ERR_INVALID_ARGUMENT, ERR_UNSUPPORTED, ERR_CUDA, ERR_DEVICE, ERR_TIMEOUT, ERR_NO_MATCH, ERR_ALLOC,
 ERR_SCRATCH_LIMIT, ERR_WORKSPACE) = range(10)
IO = {"fp32": 0, "bf16": 1}
ACC = {"fp32": 0, "fp16": 1}
KERNEL = {"legacy": 0, "cached": 1}
FILTER = {"causal": 0, "two_sided": 1, "circular": 2}

_lib = None
_emu = None


class SffftError(RuntimeError):
    def __init__(self, status: int, what: str):
        self.status = status
        super().__init__(f"{what}: {status_string(status) if _lib else status} (status {status})")


class PlanInfo(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in (
        "L", "N", "stages", "R0", "R1", "R2", "pairs_per_cta", "warps", "threads", "smem_bytes",
        "tmem_cols", "occupancy", "io", "acc", "kernel_mode", "device", "blocks")] + [("config", ctypes.c_char * 96)]


class _Candidate(ctypes.Structure):
    _fields_ = [("method", ctypes.c_char_p), ("io", ctypes.c_char_p), ("config", ctypes.c_char_p),
                ("ms", ctypes.c_double), ("rel_err", ctypes.c_double)]


def _declare(lib):
    P, I, V, D = ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_double
    sig = {
        "sffft_plan_create": (I, [ctypes.POINTER(P), I, I, I, ctypes.c_char_p, I, I]),
        "sffft_plan_destroy": (I, [P]),
        "sffft_plan_info": (I, [P, ctypes.POINTER(PlanInfo)]),
        "sffft_filter_spectrum": (I, [P, V, I, I, V, V]),
        "sffft_filter_spectrum_ex": (I, [P, V, I, I, I, V, V]),
        "sffft_fft_workspace_bytes": (I, [P, I, ctypes.POINTER(ctypes.c_size_t)]),
        "sffft_rfft": (I, [P, V, I, I, V, V, V]),
        "sffft_irfft": (I, [P, V, I, V, V, V]),
        "sffft_conv": (I, [P, V, V, V, I, I, V]),
        "sffft_conv_workspace_bytes": (I, [P, I, I, ctypes.POINTER(ctypes.c_size_t)]),
        "sffft_conv_ws": (I, [P, V, V, V, I, I, V, ctypes.c_size_t, V]),
        "sffft_plan_set_workspace": (I, [P, V, ctypes.c_size_t]),
        "sffft_plan_check": (I, [P]),
        "sffft_catalog_count": (I, []),
        "sffft_catalog_entry": (I, [I, ctypes.POINTER(I), ctypes.c_char_p, I]),
        "sffft_default_config": (I, [I, ctypes.c_char_p, I]),
        "sffft_select_candidate": (I, [ctypes.POINTER(_Candidate), I, D, ctypes.c_char_p]),
        "sffft_relative_l2": (D, [D, D]),
        "sffft_shard_range": (I, [I, I, I, ctypes.POINTER(I), ctypes.POINTER(I)]),
        "sffft_status_string": (ctypes.c_char_p, [I]),
        "sffft_last_cuda_error": (I, []),
        "sffft_baseline_create": (I, [ctypes.POINTER(P), I, I, I, V, I]),
        "sffft_baseline_run": (I, [P, V, V, I, V]),
        "sffft_baseline_destroy": (I, [P]),
        "sffft_debug_umma_probe": (I, [I, I, I, I, I, I, V, V, V]),
        "sffft_debug_wait_timeout": (I, [I]),
        "sffft_debug_conv_timeout": (I, [P, V, V, V, I, I, I, V]),
        "sffft_conv_noalloc": (I, [I, I, I, V, V, I, V, I, I, V, I]),
        "sffft_pipe_create": (I, [ctypes.POINTER(P), P, I, I, I]),
        "sffft_conv_host": (I, [P, V, V, V, V]),
        "sffft_pipe_destroy": (I, [P]),
        "sffft_conv_multi": (I, [ctypes.POINTER(P), I, ctypes.POINTER(V), ctypes.POINTER(V), ctypes.POINTER(V), I, I,
                                 ctypes.POINTER(V)]),
        "sffft_multi_pipe_create": (I, [ctypes.POINTER(P), ctypes.POINTER(P), I, I, I, I]),
        "sffft_conv_host_multi": (I, [P, V, ctypes.POINTER(V), V]),
        "sffft_multi_pipe_destroy": (I, [P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype, fn.argtypes = res, args
    return lib


def lib():
    """The native library (loaded once).  Raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"native library missing: {LIB_PATH} (run `make -C sffft_b200`)")
        _lib = _declare(ctypes.CDLL(LIB_PATH))
    return _lib


def _check(status: int, what: str):
    if status != OK:
        raise SffftError(status, what)


def status_string(status: int) -> str:
    return lib().sffft_status_string(status).decode()


def _ptr(x) -> Optional[int]:
    if x is None:
        return None
    if isinstance(x, int):
        return x
    return x.data_ptr()


def _stream(stream) -> Optional[int]:
    if stream is None:
        return None
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


def catalog() -> list[tuple[int, str]]:
    """(L, name) of every compiled plan."""
    L = lib()
    out = []
    buf = ctypes.create_string_buffer(96)
    for i in range(L.sffft_catalog_count()):
        n = ctypes.c_int()
        _check(L.sffft_catalog_entry(i, ctypes.byref(n), buf, 96), "catalog")
        out.append((n.value, buf.value.decode()))
    return out


def default_config(L: int) -> str:
    buf = ctypes.create_string_buffer(96)
    _check(lib().sffft_default_config(L, buf, 96), f"default config for L={L}")
    return buf.value.decode()


def relative_l2(squared_error: float, squared_reference: float) -> float:
    """relative_l2 of src/selection.h:26-29."""
    return lib().sffft_relative_l2(squared_error, squared_reference)


@dataclass
class Candidate:
    """Candidate of src/selection.h:8-11."""
    method: str
    io: str
    config: str
    ms: float
    rel_err: float


def select_candidate(candidates: Sequence[Candidate], max_error: float, io: str) -> Optional[int]:
    """Index of select_candidate's choice (src/selection.h:13-24), or None."""
    arr = (_Candidate * max(1, len(candidates)))()
    keep = []
    for i, c in enumerate(candidates):
        fields = [c.method.encode(), c.io.encode(), c.config.encode()]
        keep.append(fields)
        arr[i] = _Candidate(fields[0], fields[1], fields[2], float(c.ms), float(c.rel_err))
    idx = lib().sffft_select_candidate(arr, len(candidates), float(max_error), io.encode())
    return None if idx < 0 else idx


def shard_range(H: int, shards: int, shard: int) -> tuple[int, int]:
    """Contiguous channel range [h0, h1) owned by `shard` of `shards`."""
    h0, h1 = ctypes.c_int(), ctypes.c_int()
    _check(lib().sffft_shard_range(H, shards, shard, ctypes.byref(h0), ctypes.byref(h1)), "shard_range")
    return h0.value, h1.value


class Plan:
    """A compiled fused-convolution plan for one length, I/O type, accumulation mode and device.

    Mirrors the reference's fftconv<Plan<R0,R1,R2>,W,TIO,TAcc,CACHED> choice (src/sffft.cu:243-245)."""

    def __init__(self, L: int, io: str = "fp32", acc: str = "fp32", config: Optional[str] = None,
                 kernel: str = "cached", device: int = 0):
        self._h = ctypes.c_void_p()
        cfg = config.encode() if config else None
        _check(lib().sffft_plan_create(ctypes.byref(self._h), L, IO[io], ACC[acc], cfg, KERNEL[kernel], device),
               f"plan_create(L={L}, io={io}, acc={acc}, config={config})")
        self.L, self.io, self.acc, self.kernel, self.device = L, io, acc, kernel, device
        inf = PlanInfo()
        _check(lib().sffft_plan_info(self._h, ctypes.byref(inf)), "plan_info")
        self.info = {f: getattr(inf, f) for f, _ in PlanInfo._fields_ if f != "config"}
        self.info["config"] = inf.config.decode()
        self.config = self.info["config"]
        self.N = inf.N
        self.blocks = inf.blocks
        # digits of the length-N transform; a composite plan's last digit spans its blocks
        self.radices = [r for r in (inf.R0, inf.R1, inf.R2) if r > 1]
        self.radices[-1] *= self.blocks
        self._ws = None   # composite plans: the workspace of conv (a device byte tensor, grown on demand)

    def filter_spectrum(self, k, Kf=None, stream=None, layout="causal"):
        """Kf [H][N] complex fp32 (as float32 [H, N, 2]) in digit order from the filter k.

        layout "causal": k [H][L], conv gives y[n] = sum_{m<=n} u[m] k[n-m] (the reference's form);
        "two_sided": k [H][2L-1], y[n] = sum_{m<L} u[m] k[L-1+n-m] (k[:, L-1] is lag 0);
        "circular": k [H][L], y[n] = sum_{m<L} u[m] k[(n-m) mod L]."""
        import torch
        if layout not in FILTER:
            raise ValueError(f"layout must be one of {sorted(FILTER)}")
        width = 2 * self.L - 1 if layout == "two_sided" else self.L
        if k.dim() != 2 or k.shape[1] != width or k.dtype not in (torch.float32, torch.bfloat16) or not k.is_contiguous():
            raise ValueError(f"k must be a contiguous [H][{width}] float32 or bfloat16 tensor for layout {layout!r}")
        H = k.shape[0]
        if Kf is None:
            Kf = torch.empty((H, self.N, 2), dtype=torch.float32, device=k.device)
        kd = IO["bf16"] if k.dtype == torch.bfloat16 else IO["fp32"]
        _check(lib().sffft_filter_spectrum_ex(self._h, _ptr(k), kd, FILTER[layout], H, _ptr(Kf), _stream(stream)),
               "filter_spectrum")
        return Kf

    def _fft_work(self, rows, work, device):
        import torch
        need = ctypes.c_size_t()
        _check(lib().sffft_fft_workspace_bytes(self._h, rows, ctypes.byref(need)), "fft_workspace_bytes")
        if work is None:
            return torch.empty(need.value // 4, dtype=torch.float32, device=device)
        if work.numel() * work.element_size() < need.value:
            raise ValueError(f"workspace of {need.value} bytes needed")
        return work

    def rfft(self, x, X=None, work=None, stream=None):
        """X [..., N/2+1] complex64 = the length-N real DFT of x [..., N] (fp32 or bf16), numpy.fft.rfft's
        definition; N = 2L is the plan's transform length."""
        import torch
        if x.shape[-1] != self.N or x.dtype not in (torch.float32, torch.bfloat16) or not x.is_contiguous():
            raise ValueError(f"x must be a contiguous [..., {self.N}] float32 or bfloat16 tensor")
        rows = x.numel() // self.N
        if X is None:
            X = torch.empty(tuple(x.shape[:-1]) + (self.N // 2 + 1,), dtype=torch.complex64, device=x.device)
        work = self._fft_work(rows, work, x.device)
        kd = IO["bf16"] if x.dtype == torch.bfloat16 else IO["fp32"]
        _check(lib().sffft_rfft(self._h, _ptr(x), kd, rows, _ptr(X), _ptr(work), _stream(stream)), "rfft")
        return X

    def irfft(self, X, x=None, work=None, stream=None):
        """x [..., N] fp32 = the inverse of rfft for the half spectrum X [..., N/2+1] complex64
        (numpy.fft.irfft's definition, 1/N included)."""
        import torch
        if X.shape[-1] != self.N // 2 + 1 or X.dtype != torch.complex64 or not X.is_contiguous():
            raise ValueError(f"X must be a contiguous [..., {self.N // 2 + 1}] complex64 tensor")
        rows = X.numel() // (self.N // 2 + 1)
        if x is None:
            x = torch.empty(tuple(X.shape[:-1]) + (self.N,), dtype=torch.float32, device=X.device)
        work = self._fft_work(rows, work, X.device)
        _check(lib().sffft_irfft(self._h, _ptr(X), rows, _ptr(x), _ptr(work), _stream(stream)), "irfft")
        return x

    def workspace_bytes(self, B: int, H: int) -> int:
        """Device workspace of a B x H convolution (sffft_conv_workspace_bytes): 0 for single-pass plans."""
        need = ctypes.c_size_t()
        _check(lib().sffft_conv_workspace_bytes(self._h, B, H, ctypes.byref(need)), "conv_workspace_bytes")
        return need.value

    def _work(self, B, H, work):
        need = self.workspace_bytes(B, H)
        if need == 0:
            return None, 0
        if work is not None:
            nbytes = work.numel() * work.element_size()
            if nbytes < need:
                raise ValueError(f"workspace of {need} bytes needed, got {nbytes}")
            return work.data_ptr(), nbytes
        import torch
        if self._ws is None or self._ws.numel() < need:
            self._ws = None
            self._ws = torch.empty(need, dtype=torch.uint8, device=torch.device("cuda", self.device))
        return self._ws.data_ptr(), self._ws.numel()

    def conv(self, u, Kf, y=None, stream=None, work=None):
        """y = causal_conv(u, k) for u [B][H][L] with the spectrum Kf of k.  Composite plans use `work` (a device
        tensor of at least workspace_bytes(B, H) bytes) or a workspace the plan keeps for its calls."""
        import torch
        B, H, L = u.shape
        if L != self.L:
            raise ValueError(f"plan is for L={self.L}, got {L}")
        if y is None:
            y = torch.empty_like(u)
        wp, wn = self._work(B, H, work)
        _check(lib().sffft_conv_ws(self._h, _ptr(u), _ptr(Kf), _ptr(y), B, H, wp, wn, _stream(stream)), "conv")
        return y

    def conv_ptr(self, u_ptr: int, Kf_ptr: int, y_ptr: int, B: int, H: int, stream=None) -> int:
        """Raw-pointer form; returns the status instead of raising (for tight timing loops)."""
        wp, wn = self._work(B, H, None) if self.blocks > 1 else (None, 0)
        return lib().sffft_conv_ws(self._h, u_ptr, Kf_ptr, y_ptr, B, H, wp, wn, _stream(stream))

    def check(self):
        """Synchronise and raise if a kernel reported a device-side error."""
        _check(lib().sffft_plan_check(self._h), "device status")

    def close(self):
        if self._h:
            lib().sffft_plan_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class HostPipe:
    """Convolution of a batch held in host memory (sffft_pipe_create / sffft_conv_host): chunks of batch-row
    pairs are uploaded, convolved and downloaded on three streams so the copies and the kernels overlap."""

    def __init__(self, plan: "Plan", B: int, H: int, chunks: int = 0):
        self._h = ctypes.c_void_p()
        _check(lib().sffft_pipe_create(ctypes.byref(self._h), plan._h, B, H, chunks), "pipe_create")
        self.plan, self.B, self.H = plan, B, H

    def conv(self, u_host, Kf, y_host, stream=None):
        """y_host = causal_conv(u_host, k) for host tensors u_host, y_host [B][H][L] and the device spectrum Kf."""
        if tuple(u_host.shape) != (self.B, self.H, self.plan.L) or tuple(y_host.shape) != tuple(u_host.shape):
            raise ValueError("u_host / y_host must be [B][H][L] of the pipe's batch")
        _check(lib().sffft_conv_host(self._h, _ptr(u_host), _ptr(Kf), _ptr(y_host), _stream(stream)), "conv_host")
        return y_host

    def close(self):
        if self._h:
            lib().sffft_pipe_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _ptr_array(items):
    arr = (ctypes.c_void_p * len(items))()
    for i, x in enumerate(items):
        arr[i] = _ptr(x)
    return arr


def conv_multi(plans: Sequence["Plan"], us, Kfs, ys, B: int, H: int, streams=None):
    """Channel-sharded convolution of device-resident shards (sffft_conv_multi): shard g = channels
    shard_range(H, len(plans), g) on plans[g]'s device, u[g]/y[g] [B][h1-h0][L], Kf[g] [h1-h0][N]."""
    G = len(plans)
    hs = (ctypes.c_void_p * G)(*[p._h.value for p in plans])
    st = _ptr_array([_stream(s) for s in streams]) if streams is not None else None
    _check(lib().sffft_conv_multi(hs, G, _ptr_array(us), _ptr_array(Kfs), _ptr_array(ys), B, H, st), "conv_multi")
    return ys


class HostPipeMulti:
    """One [B][H][L] host batch convolved by several devices (sffft_multi_pipe_create / sffft_conv_host_multi):
    device g takes channels shard_range(H, len(plans), g) through a host pipe of its own; conv() returns when
    every device is done."""

    def __init__(self, plans: Sequence["Plan"], B: int, H: int, chunks: int = 0):
        self._h = ctypes.c_void_p()
        G = len(plans)
        hs = (ctypes.c_void_p * G)(*[p._h.value for p in plans])
        _check(lib().sffft_multi_pipe_create(ctypes.byref(self._h), hs, G, B, H, chunks), "multi_pipe_create")
        self.plans, self.B, self.H = list(plans), B, H

    def conv(self, u_host, Kfs, y_host):
        if tuple(u_host.shape) != (self.B, self.H, self.plans[0].L) or tuple(y_host.shape) != tuple(u_host.shape):
            raise ValueError("u_host / y_host must be [B][H][L] of the pipe's batch")
        _check(lib().sffft_conv_host_multi(self._h, _ptr(u_host), _ptr_array(Kfs), _ptr(y_host)), "conv_host_multi")
        return y_host

    def close(self):
        if self._h:
            lib().sffft_multi_pipe_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Baseline:
    """cuFFT pipeline (pad -> R2C -> x spectrum -> C2R -> slice) of src/sffft.cu:289-305,365-371."""

    def __init__(self, L: int, B: int, H: int, k, device: int = 0):
        self._h = ctypes.c_void_p()
        _check(lib().sffft_baseline_create(ctypes.byref(self._h), L, B, H, _ptr(k), device), "baseline_create")

    def run(self, u, y=None, full: bool = True, stream=None):
        _check(lib().sffft_baseline_run(self._h, _ptr(u), _ptr(y), 1 if full else 0, _stream(stream)), "baseline_run")
        return y

    def close(self):
        if self._h:
            lib().sffft_baseline_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def umma_probe(a_kind: int, a_slice: int, b_pitch: int, b_slice: int, A, Bm, acc16: bool = False):
    """One tcgen05.mma through the kernel's layout writers (debug).  A: uint16 [128,16], Bm: uint16 [n,16];
    returns uint32 [128, n] raw TMEM words."""
    import numpy as np
    A = np.ascontiguousarray(A, dtype=np.uint16)
    Bm = np.ascontiguousarray(Bm, dtype=np.uint16)
    n = Bm.shape[0]
    D = np.zeros((128, n), dtype=np.uint32)
    _check(lib().sffft_debug_umma_probe(a_kind, a_slice, b_pitch, b_slice, n, 1 if acc16 else 0,
                                        A.ctypes.data, Bm.ctypes.data, D.ctypes.data), "umma_probe")
    return D


def _emu_lib():
    global _emu
    if _emu is None:
        if not os.path.exists(EMU_PATH):
            raise RuntimeError(f"emulator library missing: {EMU_PATH}")
        _emu = ctypes.CDLL(EMU_PATH)
        _emu.sffft_emu_conv.argtypes = [ctypes.c_char_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int]
        _emu.sffft_emu_conv_composite.argtypes = [ctypes.c_char_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                  ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                                  ctypes.c_int]
    return _emu


def emu_conv_composite(config: str, P: int, u, Kf, io: str = "fp32", acc: str = "fp32"):
    """CPU emulation of the composite plan "<P>x[<config>]" (row energies, forward and inverse launches of the
    partitioned convolution); Kf: the P filter-segment spectra [P][H][N] (float32 pairs).  Test infrastructure."""
    import numpy as np
    B, H, L = u.shape
    u = np.ascontiguousarray(u)
    Kf = np.ascontiguousarray(Kf, dtype=np.float32)
    y = np.zeros_like(u)
    rc = _emu_lib().sffft_emu_conv_composite(config.encode(), P, IO[io], ACC[acc], u.ctypes.data, Kf.ctypes.data,
                                             y.ctypes.data, B, H)
    if rc == 3:
        raise RuntimeError(f"emulated kernel accessed memory out of range ({P}x[{config}])")
    if rc:
        raise ValueError(f"no partitioned-convolution kernels for {config}")
    return y


def emu_conv(config: str, u, Kf, io: str = "fp32", acc: str = "fp32"):
    """CPU emulation of the fused kernel (same stage code, emulated tcgen05); numpy in and out.
    Test infrastructure for checking layouts without a GPU."""
    import numpy as np
    B, H, L = u.shape
    u = np.ascontiguousarray(u)
    Kf = np.ascontiguousarray(Kf, dtype=np.float32)
    y = np.zeros_like(u)
    rc = _emu_lib().sffft_emu_conv(config.encode(), IO[io], ACC[acc], u.ctypes.data, Kf.ctypes.data, y.ctypes.data, B, H)
    if rc == 3:
        raise RuntimeError(f"emulated kernel accessed shared memory or TMEM out of range ({config})")
    if rc:
        raise ValueError(f"unknown config {config}")
    return y
