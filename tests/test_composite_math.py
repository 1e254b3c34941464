"""The block decomposition behind composite plans (sffft_b200/csrc/blocks.cu), checked in fp64 on the CPU.

A composite plan of P blocks of length Lb computes output block p as the causal convolution of input block p
with k[0:Lb] plus, for each lag d = 1..p, the two-sided convolution of input block p - d with the 2Lb - 1
taps k[(d-1)Lb + 1 : (d+1)Lb] (lag 0 at column Lb - 1).  The partial outputs of lag d sit at
part_offset(d) = B*H*Lb * (d*P - d*(d-1)/2) in one buffer, (P - d) blocks each.  These tests restate that
layout and compare the sum with the direct causal convolution (the reference's fp64 check,
src/sffft.cu:376-378)."""
import numpy as np
import pytest


def causal(x, k):
    return np.convolve(x, k)[:len(x)]


def two_sided(x, k2):
    Lb = len(x)
    return np.convolve(x, k2)[Lb - 1:2 * Lb - 1]


def part_offset(d, P, blk):
    return blk * (d * P - d * (d - 1) // 2)


@pytest.mark.parametrize("B,H,Lb,P", [(3, 2, 16, 2), (2, 3, 8, 4), (1, 1, 32, 8), (5, 2, 4, 16)])
def test_block_decomposition_equals_direct_conv(B, H, Lb, P):
    rng = np.random.default_rng(P * Lb)
    L = P * Lb
    u = rng.standard_normal((B, H, L))
    k = rng.standard_normal((H, L))
    ref = np.array([[causal(u[b, h], k[h]) for h in range(H)] for b in range(B)])
    blk = B * H * Lb
    ub = u.reshape(B * H, P, Lb).transpose(1, 0, 2).reshape(-1)           # block-major [P][B][H][Lb]
    parts = np.zeros(part_offset(P, P, blk))
    for d in range(P):
        src = ub[:(P - d) * blk].reshape((P - d) * B, H, Lb)
        out = np.empty_like(src)
        for h in range(H):
            taps = k[h, :Lb] if d == 0 else k[h, (d - 1) * Lb + 1:(d + 1) * Lb]
            assert len(taps) == (Lb if d == 0 else 2 * Lb - 1)
            for r in range(src.shape[0]):
                out[r, h] = causal(src[r, h], taps) if d == 0 else two_sided(src[r, h], taps)
        parts[part_offset(d, P, blk):part_offset(d, P, blk) + out.size] = out.reshape(-1)
    y = np.zeros((B * H, L))
    for row in range(B * H):
        for p in range(P):
            y[row, p * Lb:(p + 1) * Lb] = sum(
                parts[part_offset(d, P, blk) + (p - d) * blk + row * Lb:][:Lb] for d in range(p + 1))
    np.testing.assert_allclose(y.reshape(B, H, L), ref, rtol=0, atol=1e-9 * np.abs(ref).max())
