"""tcgen05 operand layouts on B200: one MMA through the fused kernel's own layout writers and
descriptors (sffft_debug_umma_probe) against a host GEMM, for every operand form the kernel uses."""
import numpy as np
import pytest

import sffft_b200 as sf

pytestmark = pytest.mark.gpu


def small_int_halves(shape, rng):
    v = rng.integers(-4, 5, size=shape).astype(np.float16)
    return v, v.view(np.uint16)


CASES = (
    [(0, s, 128, b, 128) for s in range(4) for b in range(4)] +      # MN-major SW128 A; K-major SW128 B
    [(128, s, 64, b, 64) for s in range(4) for b in range(2)] +      # K-major SW128 A; SW64 B
    [(64, s, 32, 0, 32) for s in range(2)] +                         # K-major SW64 A; SW32 B
    [(32, 0, 128, 1, 16), (0, 1, 64, 1, 32), (0, 2, 32, 0, 16)]
)


@pytest.mark.parametrize("a_kind,a_slice,b_pitch,b_slice,n", CASES)
def test_umma_layouts_fp32_accumulator(a_kind, a_slice, b_pitch, b_slice, n):
    rng = np.random.default_rng(a_kind * 100 + a_slice * 10 + b_slice + n)
    A, Ab = small_int_halves((128, 16), rng)
    Bm, Bb = small_int_halves((n, 16), rng)
    D = sf.umma_probe(a_kind, a_slice, b_pitch, b_slice, Ab, Bb)
    ref = A.astype(np.float32) @ Bm.astype(np.float32).T
    np.testing.assert_array_equal(D.view(np.float32), ref)


def test_umma_fp16_accumulator_format():
    # fp16 accumulators occupy one 32-bit TMEM column each, value in the low 16 bits
    rng = np.random.default_rng(5)
    A, Ab = small_int_halves((128, 16), rng)
    Bm, Bb = small_int_halves((32, 16), rng)
    D = sf.umma_probe(0, 0, 128, 0, Ab, Bb, acc16=True)
    ref = (A.astype(np.float32) @ Bm.astype(np.float32).T).astype(np.float16)
    np.testing.assert_array_equal((D & 0xFFFF).astype(np.uint16).view(np.float16), ref)


def test_bounded_wait_reports_timeout_and_context_survives():
    assert sf.lib().sffft_debug_wait_timeout(2000) == sf.ERR_TIMEOUT
    # the context is still usable afterwards
    rng = np.random.default_rng(0)
    A, Ab = small_int_halves((128, 16), rng)
    Bm, Bb = small_int_halves((16, 16), rng)
    D = sf.umma_probe(0, 0, 128, 0, Ab, Bb)
    np.testing.assert_array_equal(D.view(np.float32), A.astype(np.float32) @ Bm.astype(np.float32).T)
