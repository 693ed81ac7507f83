"""The scan form of the rank-one articulated body (csrc/pendulum_aba_coop.cu), restated in
float64 numpy and checked against the oracle's articulated body (oracle/pendulum.py aba_accel,
itself pinned to the reference's pendulum_aba_np.py). The one-warp kernel evaluates exactly these
recurrences, each as a scan over the warp's lanes:
- link velocities: the exclusive prefix sum of om_j (-sin th_j, cos th_j), rotated into link i's
  frame;
- articulated masses: m_i = (1 + m_{i+1}) / (1 + s_{i+1}^2 m_{i+1}), m = 1 at the last link, a
  linear fractional map (a suffix product of 2 x 2 matrices);
- bias forces: pa1_i = alpha_i + beta_i pa1_{i+1} (a suffix affine scan);
- accelerations: (ax, z = ay + aw) -> (c ax + s z + c1, g - U1 (c ax + s z + c1)) (a prefix
  affine scan), each link's angular acceleration z - ay.
In exact arithmetic they equal the sequential articulated-body algorithm; in float64 the two
agree to rounding.
"""

import numpy as np
import pytest

from oracle import pendulum


def aba_scan_form(th, om, torque, k):
    """Absolute angular accelerations (k, n) by the scan form's recurrences."""
    n = th.shape[1]
    acc = np.zeros((k, n))
    phi = np.concatenate([th[:1], np.diff(th, axis=0)])  # joint angles
    s, c = np.sin(phi), np.cos(phi)
    qd = np.concatenate([om[:1], np.diff(om, axis=0)])
    # velocities: exclusive prefix sum in the world frame, rotated into each link's frame
    u = np.stack([-om * np.sin(th), om * np.cos(th)])
    S = np.cumsum(u, axis=1) - u
    x = np.cos(th) * S[0] + np.sin(th) * S[1]
    y = -np.sin(th) * S[0] + np.cos(th) * S[1]
    w = om
    # the next link's joint trig (zero past the chain: no child)
    s1 = np.concatenate([s[1:], np.zeros((1, n))])
    c1n = np.concatenate([c[1:], np.zeros((1, n))])
    # articulated masses, as the suffix product of [[1, 1], [s^2, 1]] applied to (1, 1)
    m = np.zeros((k + 1, n))
    P = np.broadcast_to(np.eye(2)[:, :, None], (2, 2, n)).copy()
    for i in range(k - 1, -1, -1):
        m[i] = (P[0, 0] + P[0, 1]) / (P[1, 0] + P[1, 1])
        if i >= 1:
            Mi = np.stack([np.stack([np.ones(n), np.ones(n)]), np.stack([s[i] ** 2, np.ones(n)])])
            P = np.einsum("abn,bcn->acn", Mi, P)
            P /= P.sum(axis=(0, 1))
    m_next = np.concatenate([m[1:k], np.zeros((1, n))])
    a00 = 1 + m_next * s1 ** 2
    a01 = m_next * s1 * c1n
    r = 1 / a00
    u1 = a01 * r
    c1 = qd * y
    c2 = -qd * x
    alpha = -w * (w + y) + m[:k] * c1 - u1 * x * w
    beta = c1n * r
    pa1 = np.zeros((k + 1, n))
    for i in range(k - 1, 0, -1):
        pa1[i] = alpha[i] + beta[i] * pa1[i + 1]
    g = -(x * w + s1 * pa1[1:]) * r
    # the root, the base accelerating at -g
    ax = np.cos(th[0]) * -pendulum.PD_GRAVITY
    ay = -np.sin(th[0]) * -pendulum.PD_GRAVITY
    qdd0 = (torque - s1[0] * pa1[1] - (a01[0] * ax + a00[0] * ay)) / a00[0]
    acc[0] = qdd0
    z = ay + qdd0
    for i in range(1, k):
        ap1 = c[i] * ax + s[i] * z + c1[i]
        ap2 = -s[i] * ax + c[i] * z + c2[i]
        z = g[i] - u1[i] * ap1
        ax = ap1
        acc[i] = z - ap2
    return acc


@pytest.mark.parametrize("k", [1, 2, 3, 4, 7, 16, 33, 64, 100])
def test_scan_form_equals_the_articulated_body(k):
    rng = np.random.default_rng(k)
    n = 40
    th = rng.uniform(-np.pi, np.pi, (k, n))
    om = rng.uniform(-3, 3, (k, n))
    tq = rng.uniform(-1, 1, n)
    want = np.asarray(pendulum.aba_accel(th, om, tq, k))
    got = aba_scan_form(th, om, tq, k)
    np.testing.assert_allclose(got, want, rtol=0, atol=1e-11 * max(1.0, float(np.abs(want).max())))
