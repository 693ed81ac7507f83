"""Constants of the kernels' sine/cosine (``sincos_fast`` and ``sincos_sfu`` in csrc/common.cuh).

Run as a script, this prints the C++ constants. tests/test_trig_coeffs.py checks that the
header holds exactly these values.

Method:
- Argument reduction by pi/2 (Cody & Waite, "Software Manual for the Elementary Functions",
  1980). Pi/2 is split into three float32 parts: each is the float32 rounding of what the
  previous parts leave of pi/2.
- The reduced argument r lies in [-pi/4, pi/4], widened by 2% because 2/pi is rounded.
- On that interval, sin r = r + r^3 P(r^2) and cos r = 1 + r^2 (-1/2 + r^2 Q(r^2)), with P and
  Q quadratics.
- P and Q are fitted for least maximum relative error by Lawson's iteratively reweighted
  least squares (C. L. Lawson, "Contributions to the theory of linear least maximum
  approximation", PhD thesis, UCLA, 1961), at float64 on 4,000 points, against mpmath
  references at 40 digits.
- The relative errors of the fits are 4.5e-9 (sine) and 1.4e-10 (cosine), well below a
  float32 ulp (6e-8 to 1.2e-7).
"""

import mpmath as mp
import numpy as np

HALF_RANGE = float(mp.pi / 4) * 1.02
POINTS = 4000
ITERATIONS = 200


def pio2_parts():
    """Pi/2 as hi + mid + lo, each a float32, hi + mid + lo equal to pi/2 to about 72 bits."""
    with mp.workdps(60):
        rest = mp.pi / 2
        parts = []
        for _ in range(3):
            p = np.float32(float(rest))
            parts.append(p)
            rest = rest - mp.mpf(float(p))
    return parts


def two_pi_parts():
    """2 pi as hi + lo, two float32s, for the reduction before the special function unit."""
    with mp.workdps(60):
        hi = np.float32(float(2 * mp.pi))
        lo = np.float32(float(2 * mp.pi - mp.mpf(float(hi))))
    return hi, lo


def _lawson(target, powers, weight, xs):
    basis = np.array([[x ** p for p in powers] for x in xs])
    y = np.array([target(x) for x in xs])
    w = np.array([weight(x) for x in xs])
    lam = np.full(len(xs), 1.0 / len(xs))
    for _ in range(ITERATIONS):
        sw = np.sqrt(lam) * w
        coef, *_ = np.linalg.lstsq(basis * sw[:, None], y * sw, rcond=None)
        err = np.abs((basis @ coef - y) * w)
        lam = lam * err
        lam /= lam.sum()
    return coef, float(err.max())


def polynomials():
    """(P, Q, sine error, cosine error): P, Q as float32 coefficients, lowest power first."""
    mp.mp.dps = 40
    xs = np.linspace(1e-4, HALF_RANGE, POINTS)
    p, es = _lawson(lambda x: float(mp.sin(x)) - x, (3, 5, 7), lambda x: 1.0 / float(mp.sin(x)), xs)
    q, ec = _lawson(lambda x: float(mp.cos(x)) - 1.0 + 0.5 * x * x, (4, 6, 8),
                    lambda x: 1.0 / float(mp.cos(x)), xs)
    return np.float32(p), np.float32(q), es, ec


def constants():
    """Name -> float32 value, as the header spells them."""
    hi, mid, lo = pio2_parts()
    p, q, _, _ = polynomials()
    out = {"kTwoOverPi": np.float32(2.0 / np.pi), "kPio2Hi": hi, "kPio2Mid": mid, "kPio2Lo": lo}
    out.update({f"kSin{i}": v for i, v in enumerate(p, 1)})
    out.update({f"kCos{i}": v for i, v in enumerate(q, 1)})
    hi2, lo2 = two_pi_parts()
    out.update({"kInvTwoPi": np.float32(1.0 / (2.0 * np.pi)), "kTwoPiHi": hi2, "kTwoPiLo": lo2})
    return out


if __name__ == "__main__":
    for name, v in constants().items():
        print(f"constexpr float {name} = {np.format_float_scientific(v, unique=True)}f;")
