"""The C oracle, pinned against the reference: its generator against draws of the reference's own
nrand() (tests/golden/ref_rng.json), its fp64 direct convolution against numpy, and the digit-order
spectrum restatement against the four-step definition."""
import json
import os

import numpy as np

from tests.conftest import rel_l2
from tests.oracle_py import digit_order, spectrum_digit_order

HERE = os.path.dirname(os.path.abspath(__file__))


def test_generator_matches_reference_draws(oracle):
    gold = json.load(open(os.path.join(HERE, "golden", "ref_rng.json")))["draws"]
    for seed, draws in gold.items():
        mine = oracle.nrand(int(seed), len(draws))
        np.testing.assert_array_equal(mine, np.array(draws, np.float64))


def test_reference_recipe_uses_one_stream(oracle):
    # u = nrand()*scale over B*H*L in order, then k per channel (src/sffft.cu:339-341)
    B, H, L = 2, 3, 128
    u, k = oracle.gen_reference(B, H, L, seed=42, input_scale=2.5)
    s = oracle.nrand(42, B * H * L + H * L)
    np.testing.assert_array_equal(u.ravel(), (s[:B * H * L] * 2.5).astype(np.float32))
    a = 1.0 / (4.0 + L * np.arange(H)[:, None] / H)
    n = np.arange(L)[None, :]
    kk = (s[B * H * L:].reshape(H, L) * np.exp(-a * n) * np.sqrt(2 * a)).astype(np.float32)
    np.testing.assert_allclose(k, kk, rtol=2e-7, atol=0)


def test_profiles(oracle):
    B, H, L = 1, 2, 256
    u, k = oracle.gen_profile(B, H, L, decay=8.0, sqrt_norm=True, seed=7)
    s = oracle.nrand(7, B * H * L + H * L)
    np.testing.assert_array_equal(u.ravel(), s[:B * H * L].astype(np.float32))
    ref = s[B * H * L:].reshape(H, L) * np.exp(-8.0 * np.arange(L) / L) / np.sqrt(L)
    np.testing.assert_allclose(k, ref.astype(np.float32), rtol=2e-7)


def test_direct_conv_matches_numpy(oracle):
    rng = np.random.default_rng(0)
    u = rng.standard_normal((3, 2, 200)).astype(np.float32)
    k = rng.standard_normal((2, 200)).astype(np.float32)
    y = oracle.direct_conv(u, k)
    for b in range(3):
        for h in range(2):
            ref = np.convolve(u[b, h].astype(np.float64), k[h].astype(np.float64))[:200]
            assert rel_l2(y[b, h], ref) < 1e-14
    ys = oracle.direct_conv_seqs(u, k, [0, 3, 5])
    np.testing.assert_allclose(ys, y.reshape(6, 200)[[0, 3, 5]], rtol=0, atol=0)


def test_direct_conv_edge_cases(oracle):
    # zero filter -> zero output; unit impulse filter -> identity; single-sample input
    u = np.arange(1, 129, dtype=np.float32).reshape(1, 1, 128)
    assert not oracle.direct_conv(u, np.zeros((1, 128), np.float32)).any()
    delta = np.zeros((1, 128), np.float32)
    delta[0, 0] = 1
    np.testing.assert_array_equal(oracle.direct_conv(u, delta)[0, 0], u[0, 0])
    shift = np.zeros((1, 128), np.float32)
    shift[0, 5] = 1
    out = oracle.direct_conv(u, shift)[0, 0]
    np.testing.assert_array_equal(out[5:], u[0, 0, :123])
    assert not out[:5].any()


def _four_step(x, R):
    """fp64 four-step DFT in the reference's digit order (restating src/sffft.cu:106-113,137-241 without
    rounding): stage j is a DFT along digit j followed by the twiddle exponent of twid<P,j>."""
    R = list(R)
    N = int(np.prod(R))
    X = np.asarray(x, np.complex128).copy()
    stride = N
    pre = 1
    for j, r in enumerate(R):
        stride //= r
        pos = np.arange(N)
        out = np.zeros(N, np.complex128)
        kk = (pos // stride) % r
        base = pos - kk * stride
        for d in range(r):
            out += X[base + d * stride] * np.exp(-2j * np.pi * d * kk / r)
        if j + 1 < len(R):
            out *= np.exp(-2j * np.pi * pre * (pos % stride) * kk / N)
        X = out
        pre *= r
    return X


def test_digit_order_spectrum_is_four_step_output():
    rng = np.random.default_rng(1)
    for R in [(16, 16), (64, 32), (32, 16, 16), (16, 32, 32)]:
        N = int(np.prod(R))
        k = rng.standard_normal((1, N // 2))
        x = np.concatenate([k[0], np.zeros(N // 2)])
        np.testing.assert_allclose(_four_step(x, R), spectrum_digit_order(k, R)[0], rtol=1e-9, atol=1e-9)
        # digit order is a permutation of the frequencies
        assert sorted(digit_order(R)) == list(range(N))


def test_two_sided_and_circular_sums_match_numpy(oracle):
    # two-sided: the full linear convolution of u with the 2L-1 taps, window starting at lag 0;
    # circular: the period-L circular convolution through numpy's fp64 FFT
    rng = np.random.default_rng(3)
    B, H, L = 2, 3, 64
    u = rng.standard_normal((B, H, L)).astype(np.float32)
    k2 = rng.standard_normal((H, 2 * L - 1)).astype(np.float32)
    kc = rng.standard_normal((H, L)).astype(np.float32)
    seqs = np.arange(B * H)
    y2 = oracle.direct_conv_layout_seqs(u, k2, "two_sided", seqs)
    yc = oracle.direct_conv_layout_seqs(u, kc, "circular", seqs)
    for s in seqs:
        b, h = divmod(int(s), H)
        full = np.convolve(u[b, h].astype(np.float64), k2[h].astype(np.float64))
        assert rel_l2(y2[s], full[L - 1:2 * L - 1]) < 1e-14
        circ = np.fft.ifft(np.fft.fft(u[b, h].astype(np.float64)) * np.fft.fft(kc[h].astype(np.float64))).real
        assert rel_l2(yc[s], circ) < 1e-13


def test_two_sided_with_zero_negative_lags_is_causal(oracle):
    rng = np.random.default_rng(4)
    B, H, L = 2, 2, 128
    u = rng.standard_normal((B, H, L)).astype(np.float32)
    k = rng.standard_normal((H, L)).astype(np.float32)
    k2 = np.concatenate([np.zeros((H, L - 1), np.float32), k], axis=1)
    seqs = np.arange(B * H)
    np.testing.assert_array_equal(oracle.direct_conv_layout_seqs(u, k2, "two_sided", seqs),
                                  oracle.direct_conv_seqs(u, k, seqs))
