"""The constants of the kernels' sine/cosine (csrc/common.cuh) are the ones trig_coeffs.py
derives, and the derivation's fits are as accurate as its docstring says."""

import re

import numpy as np

import trig_coeffs
from conftest import PKG


def test_header_constants_are_the_derived_ones():
    src = (PKG / "csrc" / "common.cuh").read_text()
    for name, value in trig_coeffs.constants().items():
        m = re.search(rf"constexpr float {name} = ([-+0-9.e]+)f;", src)
        assert m, name
        assert np.float32(m.group(1)) == value, name


def test_pio2_parts_sum_to_pi_over_2():
    import mpmath as mp

    hi, mid, lo = trig_coeffs.pio2_parts()
    with mp.workdps(50):
        rest = mp.pi / 2 - mp.mpf(float(hi)) - mp.mpf(float(mid)) - mp.mpf(float(lo))
        assert abs(rest) < mp.mpf(2) ** -70


def test_fits_are_below_a_tenth_of_an_ulp():
    _, _, sin_err, cos_err = trig_coeffs.polynomials()
    assert sin_err < 6e-9 and cos_err < 1e-9
