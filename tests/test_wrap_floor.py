"""The angle wrap's floor (csrc/common.cuh, wrap_to_pi) without a rounding instruction.

wrap_to_pi forms floor(q), q = (x + pi) / (2 pi), as the nearest integer to q - 1/2 (adding and
subtracting 1.5 * 2^23), falling back to the division whenever the fraction q - f lies within
2e-6 of an integer or |q| > 8. These tests restate both forms in float32 numpy, one correctly
rounded operation at a time as the kernel performs them, and check that they choose the same
integer, so the wrap keeps the bits of acrobot_np.py:87-89 / pendulum_np.py:110-111.
"""

import numpy as np

PI = np.float32(3.141592653589793)
TWO_PI = np.float32(6.283185307179586)
INV_TWO_PI = np.float32(1.0) / TWO_PI
ROUND = np.float32(12582912.0)


def _fallback(x, q, f):
    y = x + PI
    r = q - f
    slow = (r < np.float32(2e-6)) | (r > np.float32(1.0) - np.float32(2e-6)) | (np.abs(q) > np.float32(8.0))
    return np.where(slow, np.floor(y / TWO_PI), f)


def floor_with_rounding(x):
    q = (x + PI) * INV_TWO_PI
    return _fallback(x, q, np.floor(q))


def floor_by_addition(x):
    q = (x + PI) * INV_TWO_PI
    f = ((q - np.float32(0.5)) + ROUND) - ROUND
    return _fallback(x, q, f)


def _near_boundaries():
    """Every float32 within 4,096 ulps of each wrap boundary (2k + 1) pi for |k| <= 12, where q
    falls within rounding of an integer."""
    out = []
    for k in range(-12, 13):
        centre = np.float32((2 * k + 1) * np.pi)
        bits = centre.view(np.int32)
        span = np.arange(-4096, 4097, dtype=np.int32)
        if centre < 0:
            out.append((bits - span).view(np.float32))
        else:
            out.append((bits + span).view(np.float32))
    return np.concatenate(out)


def test_floor_by_addition_equals_floor_near_every_boundary():
    x = _near_boundaries()
    with np.errstate(all="ignore"):
        assert np.array_equal(floor_by_addition(x), floor_with_rounding(x))


def test_floor_by_addition_equals_floor_on_random_angles():
    r = np.random.default_rng(0)
    x = np.concatenate([r.uniform(-64, 64, 2_000_000), r.uniform(-1e6, 1e6, 200_000),
                        [0.0, -0.0, 1e-30, -1e-30, 3.4e38, -3.4e38]]).astype(np.float32)
    with np.errstate(all="ignore"):
        assert np.array_equal(floor_by_addition(x), floor_with_rounding(x))
