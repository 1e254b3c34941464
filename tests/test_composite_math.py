"""The partitioned convolution behind composite plans (sffft_b200/csrc/stages.h, "Partitioned convolution"),
restated in fp64 numpy on the CPU.

A composite plan of P blocks of length Lb transforms every input block once (U_q = DFT of u_q zero-padded to
N = 2 Lb), and gets output block p as the first Lb values of the inverse DFT of W_p = sum_{q <= p} U_q K'_{p-q},
where K'_d is the spectrum of the filter segment kw_d[n] = k[d Lb + n], kw_d[Lb + m] = k[(d - 1) Lb + m]
(n, m < Lb; zero for d = 0).  These tests check that identity against the direct causal convolution (the
reference's fp64 check, src/sffft.cu:376-378) and the segment spectra against K_d + (-1)^f K_{d-1}."""
import numpy as np
import pytest


def causal(x, k):
    return np.convolve(x, k)[:len(x)]


def segment(k, d, Lb):
    kw = np.zeros(2 * Lb)
    kw[:Lb] = k[d * Lb:(d + 1) * Lb]
    if d > 0:
        kw[Lb:] = k[(d - 1) * Lb:d * Lb]
    return kw


@pytest.mark.parametrize("B,H,Lb,P", [(3, 2, 16, 2), (2, 3, 8, 4), (1, 1, 32, 8), (5, 2, 4, 16)])
def test_partitioned_convolution_equals_direct_conv(B, H, Lb, P):
    rng = np.random.default_rng(P * Lb)
    L, N = P * Lb, 2 * Lb
    u = rng.standard_normal((B, H, L))
    k = rng.standard_normal((H, L))
    ref = np.array([[causal(u[b, h], k[h]) for h in range(H)] for b in range(B)])
    # forward launch: one transform per (row, input block)
    U = np.fft.fft(np.concatenate([u.reshape(B, H, P, Lb), np.zeros((B, H, P, Lb))], axis=-1), axis=-1)
    Ks = np.stack([np.fft.fft(np.stack([segment(k[h], d, Lb) for h in range(H)]), axis=-1) for d in range(P)])
    # inverse launch: per output block, the spectrum sum and one inverse transform (first half kept)
    y = np.zeros((B, H, P, Lb))
    for p in range(P):
        W = sum(U[:, :, q] * Ks[p - q][None] for q in range(p + 1))
        y[:, :, p] = np.fft.ifft(W, axis=-1)[..., :Lb].real
    np.testing.assert_allclose(y.reshape(B, H, L), ref, rtol=0, atol=1e-9 * np.abs(ref).max())


@pytest.mark.parametrize("Lb,P", [(8, 4), (16, 2)])
def test_segment_spectrum_folds_the_previous_block(Lb, P):
    rng = np.random.default_rng(Lb)
    k = rng.standard_normal(P * Lb)
    N = 2 * Lb
    sign = (-1.0) ** np.arange(N)
    Kd = [np.fft.fft(np.concatenate([k[d * Lb:(d + 1) * Lb], np.zeros(Lb)])) for d in range(P)]
    for d in range(P):
        want = Kd[d] + (sign * Kd[d - 1] if d > 0 else 0)
        np.testing.assert_allclose(np.fft.fft(segment(k, d, Lb)), want, atol=1e-9 * np.abs(want).max())

