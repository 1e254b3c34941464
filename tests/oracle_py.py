"""ctypes access to the C oracle (oracle/liboracle.so) plus numpy restatements used by the tests.

Test infrastructure only (the product path never imports this)."""
import ctypes
import os

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "oracle", "liboracle.so")


class Oracle:
    def __init__(self):
        if not os.path.exists(LIB):
            raise RuntimeError(f"oracle library missing: {LIB} (run `make -C oracle`)")
        self.lib = ctypes.CDLL(LIB)
        V, I, D, ULL = ctypes.c_void_p, ctypes.c_int, ctypes.c_double, ctypes.c_ulonglong
        self.lib.oracle_nrand_stream.argtypes = [ULL, I, V]
        self.lib.oracle_gen_reference.argtypes = [ULL, I, I, I, D, V, V]
        self.lib.oracle_gen_profile.argtypes = [ULL, I, I, I, D, I, V, V]
        self.lib.oracle_direct_conv.argtypes = [V, V, V, I, I, I, I]
        self.lib.oracle_direct_conv_seqs.argtypes = [V, V, V, I, I, I, V, I, I]
        self.lib.oracle_direct_conv_layout_seqs.argtypes = [V, V, I, V, I, I, I, V, I, I]
        self.lib.oracle_max_threads.restype = I

    def nrand(self, seed, n):
        out = np.zeros(n, np.float64)
        self.lib.oracle_nrand_stream(seed, n, out.ctypes.data)
        return out

    def gen_reference(self, B, H, L, seed=0, input_scale=1.0):
        u = np.zeros((B, H, L), np.float32)
        k = np.zeros((H, L), np.float32)
        self.lib.oracle_gen_reference(seed, B, H, L, input_scale, u.ctypes.data, k.ctypes.data)
        return u, k

    def gen_profile(self, B, H, L, decay=4.0, sqrt_norm=True, seed=0):
        u = np.zeros((B, H, L), np.float32)
        k = np.zeros((H, L), np.float32)
        self.lib.oracle_gen_profile(seed, B, H, L, decay, 1 if sqrt_norm else 0, u.ctypes.data, k.ctypes.data)
        return u, k

    def direct_conv(self, u, k, threads=0):
        u = np.ascontiguousarray(u, np.float32)
        k = np.ascontiguousarray(k, np.float32)
        B, H, L = u.shape
        y = np.zeros((B, H, L), np.float64)
        self.lib.oracle_direct_conv(u.ctypes.data, k.ctypes.data, y.ctypes.data, B, H, L, threads)
        return y

    def direct_conv_seqs(self, u, k, seqs, threads=0):
        u = np.ascontiguousarray(u, np.float32)
        k = np.ascontiguousarray(k, np.float32)
        B, H, L = u.shape
        seqs = np.ascontiguousarray(seqs, np.int64)
        y = np.zeros((len(seqs), L), np.float64)
        self.lib.oracle_direct_conv_seqs(u.ctypes.data, k.ctypes.data, y.ctypes.data, B, H, L, seqs.ctypes.data,
                                         len(seqs), threads)
        return y

    def direct_conv_layout_seqs(self, u, k, layout, seqs, threads=0):
        """fp64 direct two-sided (k [H][2L-1]) or circular (k [H][L]) convolution of the listed sequences."""
        code = {"two_sided": 1, "circular": 2}[layout]
        u = np.ascontiguousarray(u, np.float32)
        k = np.ascontiguousarray(k, np.float32)
        B, H, L = u.shape
        assert k.shape == (H, 2 * L - 1 if code == 1 else L)
        seqs = np.ascontiguousarray(seqs, np.int64)
        y = np.zeros((len(seqs), L), np.float64)
        self.lib.oracle_direct_conv_layout_seqs(u.ctypes.data, k.ctypes.data, code, y.ctypes.data, B, H, L,
                                                seqs.ctypes.data, len(seqs), threads)
        return y

    def max_threads(self):
        return self.lib.oracle_max_threads()


def digit_order(radices):
    """Frequency held at each digit-order position (src/sffft.cu:283-288)."""
    R0, R1, R2 = (list(radices) + [1, 1])[:3]
    N = R0 * R1 * R2
    p = np.arange(N)
    if R2 > 1:
        d2 = p % R2
        d1 = (p // R2) % R1
        d0 = p // (R1 * R2)
    else:
        d2 = 0
        d1 = p % R1
        d0 = p // R1
    return d0 + R0 * (d1 + R1 * d2)


def spectrum_digit_order(k, radices):
    """Unnormalised DFT of the zero-padded filter in digit order, complex128 [H, N] (fp64 restatement of
    cufftExecC2C + permuteK, src/sffft.cu:344,365,283-288)."""
    k = np.asarray(k, np.float64)
    H, L = k.shape
    Kc = np.fft.fft(np.concatenate([k, np.zeros((H, L))], axis=1), axis=1)
    return Kc[:, digit_order(radices)]


def segment_spectra_digit_order(k, P, radices):
    """Filter-segment spectra of a composite plan of P blocks, complex128 [P, H, N] in digit order (N = 2 Lb, Lb =
    L / P): segment d is kw_d[n] = k[d Lb + n] and kw_d[Lb + m] = k[(d - 1) Lb + m] (zero for d = 0), whose
    spectrum is K_d + (-1)^f K_(d-1), the block-d term of the partitioned convolution."""
    k = np.asarray(k, np.float64)
    H, L = k.shape
    Lb = L // P
    out = []
    for d in range(P):
        kw = np.zeros((H, 2 * Lb))
        kw[:, :Lb] = k[:, d * Lb:(d + 1) * Lb]
        if d > 0:
            kw[:, Lb:] = k[:, (d - 1) * Lb:d * Lb]
        out.append(np.fft.fft(kw, axis=1)[:, digit_order(radices)])
    return np.stack(out)


def to_bf16(x):
    """Round-to-nearest-even fp32 -> bf16, returned as fp32 values."""
    x = np.ascontiguousarray(x, np.float32)
    b = x.view(np.uint32).astype(np.uint64)
    b = (b + 0x7FFF + ((b >> 16) & 1)) >> 16
    return (b.astype(np.uint32) << 16).view(np.float32).reshape(x.shape)


def bf16_bits(x):
    x = np.ascontiguousarray(x, np.float32)
    b = x.view(np.uint32).astype(np.uint64)
    return ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16).reshape(x.shape)


def bf16_from_bits(b):
    return (np.asarray(b, np.uint32) << 16).view(np.float32)


# Row scales of the pairing tests: batch rows 2j and 2j+1 share one complex transform, so each pair below
# puts rows of very different size (or an all-zero row) side by side; the last pair is all tiny.
PAIR_SCALES = [1.0, 1e-3, 1e-4, 1.0, 0.0, 1.0, 1.0, 1.0, 1e-5, 2e-5]


def scaled_pair_inputs(oracle, H, L, io, seed=0):
    """u [len(PAIR_SCALES)][H][L] with row b scaled by PAIR_SCALES[b], k of the configs' profile; both
    rounded to bf16 (and returned as fp32 values) for bf16 I/O."""
    B = len(PAIR_SCALES)
    u, k = oracle.gen_profile(B, H, L, decay=4.0, sqrt_norm=True, seed=seed)
    u = (u * np.asarray(PAIR_SCALES, np.float32)[:, None, None]).astype(np.float32)
    if io == "bf16":
        u, k = to_bf16(u), to_bf16(k)
    return u, k


def per_row_rel_l2(y, ref):
    """Relative L2 error of every (b, h) row, with relative_l2's convention for an all-zero reference row
    (0 if the row is exactly zero, else inf; sfFFT src/selection.h:26-29)."""
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    d = np.sum((y - ref) ** 2, axis=-1)
    r = np.sum(ref ** 2, axis=-1)
    out = np.where(r > 0, np.sqrt(d / np.where(r > 0, r, 1.0)), np.where(d == 0, 0.0, np.inf))
    return out
