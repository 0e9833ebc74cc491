"""Properties of the E2M1 activation split (tests/umma_split.py, the restatement
the tensor-core self-check compares against) on CPU."""

import numpy as np

from oracle import moe_oracle as mo
from tests.umma_split import e2m1_rn, e2m1_value, reconstruct, split


def bf16_values(rng, n, scale=1.0):
    x = (rng.standard_normal(n) * scale).astype(np.float32)
    return mo.bf16_bits_to_f32(mo.f32_to_bf16_bits(x))


def test_rounding_is_nearest_with_ties_to_even():
    v = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, -0.25, -5.0, 0.3, 4.9, 6.0], np.float32)
    np.testing.assert_array_equal(e2m1_value(e2m1_rn(v)), [0, 1, 1, 2, 2, 4, 4, 0, -4, 0.5, 4, 6])


def test_sixteen_terms_reconstruct_bf16_vectors_exactly():
    rng = np.random.default_rng(0)
    for scale in (1.0, 1e-3, 300.0):
        x = bf16_values(rng, 4096, scale)
        codes, scales, r = split(x, 16)
        assert np.all(r == 0)
        np.testing.assert_array_equal(reconstruct(codes, scales), x.astype(np.float64))


def test_residual_bound_and_no_saturation():
    """After t terms the block residual is at most 2^(s0 - 2(t-1)), inside the
    next term's range, so no code saturates."""
    rng = np.random.default_rng(1)
    x = bf16_values(rng, 1024)
    amax = np.abs(x).reshape(-1, 32).max(axis=1)
    codes, scales, _ = split(x, 8)
    s0 = scales[0].astype(np.int64) - 127
    assert np.all(6.0 * np.ldexp(1.0, s0) >= amax) and np.all(3.0 * np.ldexp(1.0, s0) < amax)
    for t in range(1, 8):
        _, _, r = split(x, t)
        cur = np.abs(r).reshape(-1, 32).max(axis=1)
        assert np.all(cur <= np.ldexp(1.0, s0 - 2 * (t - 1)))


def test_zero_and_tiny_blocks():
    x = np.zeros(64, np.float32)
    x[40] = 2.0 ** -120
    codes, scales, r = split(x, 4)
    assert np.all(codes == 0) and np.all(scales == 127)
    np.testing.assert_array_equal(r, x)
