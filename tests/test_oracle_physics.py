"""Known-answer and invariant checks of the oracle, written independently of it: the checks the
reference's own test files make (scalar Gym transcriptions, closed forms, energy, contact
laws), restated here so the oracle is pinned by physics and not only by the golden vectors."""

import math

import numpy as np
import pytest

from oracle import classic, legged, pendulum, rng


# ---- CartPole: Gym CartPole-v1's Euler step, scalar (test_cartpole.py:13-44) ---------------

def _cartpole_scalar(x, xd, th, thd, a):
    f = 10.0 if a == 1 else -10.0
    c, s = math.cos(th), math.sin(th)
    tmp = (f + 0.05 * thd * thd * s) / 1.1
    alpha = (9.8 * s - c * tmp) / (0.5 * (4.0 / 3.0 - 0.1 * c * c / 1.1))
    acc = tmp - 0.05 * alpha * c / 1.1
    return x + 0.02 * xd, xd + 0.02 * acc, th + 0.02 * thd, thd + 0.02 * alpha


def test_cartpole_matches_scalar_gym():
    r = np.random.default_rng(10)
    st = r.uniform(-1, 1, (4, 100)).astype(np.float32)
    act = r.integers(0, 2, 100)
    want = np.array([_cartpole_scalar(*col, a) for col, a in zip(st.T.tolist(), act)]).T
    np.testing.assert_allclose(classic.cartpole_physics(st, act), want, atol=1e-5)


def test_cartpole_terminal_columns():
    st = np.zeros((4, 3), dtype=np.float32)
    st[0, 0], st[2, 1] = 2.5, 0.3
    assert classic.cartpole_terminated(classic.cartpole_physics(st, np.ones(3))).tolist() == [True, True, False]


# ---- Acrobot: Gym's rk4 on the torque-augmented state and its while-loop wrap -------------

def _acrobot_scalar(t1, t2, w1, w2, a):
    g, dt = 9.8, 0.2
    tau = [-1.0, 0.0, 1.0][a]

    def f(y):
        th1, th2, d1_, d2_ = y
        d1 = 0.25 + (1.0 + 0.25 + 2 * 0.5 * math.cos(th2)) + 2.0
        d2 = (0.25 + 0.5 * math.cos(th2)) + 1.0
        phi2 = 0.5 * g * math.cos(th1 + th2 - math.pi / 2)
        phi1 = -0.5 * d2_ ** 2 * math.sin(th2) - d2_ * d1_ * math.sin(th2) + 1.5 * g * math.cos(th1 - math.pi / 2) + phi2
        dd2 = (tau + d2 / d1 * phi1 - 0.5 * d1_ ** 2 * math.sin(th2) - phi2) / (1.25 - d2 * d2 / d1)
        return [d1_, d2_, -(d2 * dd2 + phi1) / d1, dd2]

    y = [t1, t2, w1, w2]
    k1 = f(y)
    k2 = f([a_ + dt / 2 * b for a_, b in zip(y, k1)])
    k3 = f([a_ + dt / 2 * b for a_, b in zip(y, k2)])
    k4 = f([a_ + dt * b for a_, b in zip(y, k3)])
    ns = [a_ + dt / 6 * (p + 2 * q + 2 * r_ + s) for a_, p, q, r_, s in zip(y, k1, k2, k3, k4)]

    def wrap(x):
        while x > math.pi:
            x -= 2 * math.pi
        while x < -math.pi:
            x += 2 * math.pi
        return x

    return wrap(ns[0]), wrap(ns[1]), min(max(ns[2], -4 * math.pi), 4 * math.pi), min(max(ns[3], -9 * math.pi), 9 * math.pi)


def test_acrobot_matches_scalar_gym():
    r = np.random.default_rng(11)
    st = np.stack([r.uniform(-np.pi, np.pi, 200), r.uniform(-np.pi, np.pi, 200),
                   r.uniform(-2, 2, 200), r.uniform(-2, 2, 200)]).astype(np.float32)
    act = r.integers(0, 3, 200)
    want = np.array([_acrobot_scalar(*col, a) for col, a in zip(st.T.tolist(), act)]).T
    got = classic.acrobot_physics(st, act)
    diff = np.abs(got - want)
    diff[:2] = np.minimum(diff[:2], 2 * np.pi - diff[:2])  # the two wraps may disagree exactly at +-pi
    assert diff.max() < 1e-3


def test_acrobot_stays_in_bounds_under_random_actions():
    r = np.random.default_rng(0)
    st = r.uniform(-0.1, 0.1, (4, 512)).astype(np.float32)
    for _ in range(300):
        st = classic.acrobot_physics(st, r.integers(0, 3, 512))
    assert np.isfinite(st).all() and np.all(np.abs(st[:2]) <= np.pi)
    assert np.all(np.abs(st[2]) <= classic.AC_MAX_VEL_1 + 1e-5) and np.all(np.abs(st[3]) <= classic.AC_MAX_VEL_2 + 1e-5)


# ---- K-link pendulum ---------------------------------------------------------------------

def _double_pendulum(t1, t2, w1, w2, tau):
    """Unit masses and rods, absolute angles, Cramer's rule (test_pendulum.py:14-23)."""
    g = 9.8
    m12 = math.cos(t1 - t2)
    b1 = tau - math.sin(t1 - t2) * w2 * w2 - 2 * g * math.sin(t1)
    b2 = math.sin(t1 - t2) * w1 * w1 - g * math.sin(t2)
    det = 2.0 - m12 * m12
    return (b1 - m12 * b2) / det, (2.0 * b2 - m12 * b1) / det


def _state(k, n, seed):
    r = np.random.default_rng(seed)
    return (np.concatenate([r.uniform(-np.pi, np.pi, (k, n)), r.uniform(-1, 1, (k, n))]).astype(np.float32),
            r.integers(0, 3, n))


def test_two_links_match_double_pendulum():
    st, act = _state(2, 100, 0)
    tau = ((act - 1) * 1.0).astype(np.float32)
    want = np.array([_double_pendulum(*col, t) for col, t in zip(st.T.tolist(), tau)]).T
    np.testing.assert_allclose(pendulum.mm_accel(st[:2], st[2:], tau, 2), want, rtol=1e-3, atol=1e-3)
    np.testing.assert_allclose(pendulum.aba_accel(st[:2], st[2:], tau, 2), want, rtol=1e-3, atol=1e-3)


def test_aba_single_link_closed_form():
    r = np.random.default_rng(0)
    st = r.uniform(-3, 3, (2, 50)).astype(np.float32)
    tau = r.uniform(-1, 1, 50).astype(np.float32)
    np.testing.assert_allclose(pendulum.aba_accel(st[:1], st[1:], tau, 1)[0], tau - 9.8 * np.sin(st[0]), atol=1e-5)


@pytest.mark.parametrize("k", [2, 3, 4, 8, 16])
def test_aba_equals_mass_matrix(k):
    st, act = _state(k, 300, k)
    tau = ((act - 1) * 1.0).astype(np.float32)
    np.testing.assert_allclose(pendulum.aba_accel(st[:k], st[k:], tau, k), pendulum.mm_accel(st[:k], st[k:], tau, k),
                               atol=1e-3)


@pytest.mark.parametrize("k,tol,form", [(2, 0.01, "mm"), (4, 0.01, "mm"), (8, 0.01, "mm"), (16, 0.01, "mm"),
                                        (16, 0.01, "aba"), (32, 0.03, "aba"), (64, 0.1, "aba")])
def test_energy_drift_without_torque(k, tol, form):
    r = np.random.default_rng(k)
    n = 32
    st = np.concatenate([r.uniform(-0.5, 0.5, (k, n)), r.uniform(-0.3, 0.3, (k, n))]).astype(np.float32)
    e0 = pendulum.energy(st, k)
    phys = pendulum.mm_physics if form == "mm" else pendulum.aba_physics
    for _ in range(200):
        st = phys(st, np.ones(n, dtype=np.int64), k)
    drift = np.abs(pendulum.energy(st, k) - e0) / (np.abs(e0) + 1e-6)
    assert drift.max() < tol, (k, form, drift.max())


# ---- Hopper and legged bodies -----------------------------------------------------------

def _run(q, v, tau, n, mu=legged.LG_MU):
    for _ in range(n):
        q, v = legged.substep(q, v, [tau], 1, iters=1, mu=mu)
    return q, v


def _col(*vals):
    return np.asarray(vals, np.float32).reshape(-1, 1)


def test_airborne_body_follows_a_ballistic_arc():
    q, v = _run(_col(0.0, 10.0, 0.0, 0.0), _col(0.3, 0.0, 0.0, 0.0), np.zeros(1, np.float32), 100)
    assert abs(q[1, 0] - (10.0 - 0.5 * 9.8 * 1.0)) < 0.06 and abs(q[0, 0] - 0.3) < 1e-4


def test_standing_hopper_does_not_drift():
    q, v = _run(_col(0.0, 1.0, 0.0, 0.0), _col(0.0, 0.0, 0.0, 0.0), np.zeros(1, np.float32), 400)
    assert np.abs(q[:, 0] - [0.0, 1.0, 0.0, 0.0]).max() < 1e-3 and np.abs(v[:, 0]).max() < 1e-3


def test_inelastic_drop_lands_without_bounce():
    q, v = _col(0.0, 1.5, 0.0, 0.0), _col(0.0, 0.0, 0.0, 0.0)
    low = 0.0
    for _ in range(300):
        q, v = _run(q, v, np.zeros(1, np.float32), 1)
        low = min(low, float(q[1, 0] - np.cos(q[2, 0] + q[3, 0])))
    assert low > -0.02 and abs(q[1, 0] - 1.0) < 0.01 and abs(v[1, 0]) < 1e-2


def test_friction_slows_a_sliding_foot():
    q0, v0 = _col(0.0, 1.0, 0.0, 0.0), _col(1.0, 0.0, 0.0, 0.0)

    def foot_speed(q, v):
        return float(v[0, 0] + np.cos(q[2, 0] + q[3, 0]) * (v[2, 0] + v[3, 0]))

    assert 0.0 <= foot_speed(*_run(q0, v0, np.zeros(1, np.float32), 5)) < 1.0
    assert abs(foot_speed(*_run(q0, v0, np.zeros(1, np.float32), 5, mu=0.0)) - 1.0) < 0.05


def test_contact_impulse_complementarity():
    r = np.random.default_rng(0)
    n = 2000
    b = r.uniform(-1, 1, (n, 2, 2))
    A = np.einsum("nij,nkj->nik", b, b) + 0.05 * np.eye(2)
    att, atn, ann = (A[:, i, j].astype(np.float32) for i, j in ((0, 0), (0, 1), (1, 1)))
    wt, wn = r.uniform(-2, 2, n).astype(np.float32), r.uniform(-2, 2, n).astype(np.float32)
    depth = r.uniform(-0.1, 0.1, n).astype(np.float32)
    lt, ln = legged.contact_impulse(att, atn, ann, wt, wn, depth)
    target = 20.0 * np.maximum(depth, 0.0)
    wt2, wn2 = wt + att * lt + atn * ln, wn + atn * lt + ann * ln
    assert ln.min() >= 0 and not ln[depth < 0].any()
    ok = ann > legged.LG_MU * np.abs(atn)
    push_ = ok & (ln > 0)
    np.testing.assert_allclose(wn2[push_], target[push_], atol=1e-3)
    assert (np.abs(lt[ok]) <= legged.LG_MU * ln[ok] + 1e-5).all()
    inside = push_ & (np.abs(lt) < legged.LG_MU * ln - 1e-4)
    np.testing.assert_allclose(wt2[inside], 0.0, atol=1e-3)


def test_one_leg_one_sweep_is_the_hopper():
    from conftest import golden

    g = golden("hopper")
    np.testing.assert_allclose(legged.physics(g["state"], g["action"], 1, iters=1), g["stepped"], rtol=1e-5, atol=1e-5)


def _standing_drift(c, iters, substeps=400):
    pose = legged.static_pose(c)
    d = 3 + c
    q, v = pose[:d].astype(np.float32)[:, None], np.zeros((d, 1), np.float32)
    for _ in range(substeps):
        q, v = legged.substep(q, v, [np.zeros(1, np.float32)] * c, c, iters=iters)
    return float(np.max(np.abs(q[:, 0] - pose[:d])))


def test_two_leg_stand_converges_with_sweeps():
    drifts = [_standing_drift(2, k) for k in (1, 4, 8, 32, 256)]
    assert np.all(np.diff(drifts) < 0), drifts  # more sweeps, less drift
    assert drifts[2] < 1e-2 and drifts[4] < 1e-6, drifts


@pytest.mark.parametrize("c", [1, 2, 4])
def test_step_impulses_carry_the_weight_of_a_standing_body(c):
    """At rest on every foot, the normal impulses of one step (four substeps of 0.01) add up
    to the body's weight times 0.04 (plus the Baumgarte correction of a resting contact), and
    the step with impulses is the same step."""
    pose = legged.static_pose(c)[:, None]
    hold = np.full(1, (3**c - 1) // 2)  # zero torque on every leg
    imp = legged.step_impulses(pose, hold, c)
    weight = (legged.LG_M_T + c * legged.LG_M_F) * legged.LG_GRAVITY * legged.LG_H * legged.LG_SUBSTEPS
    assert imp.shape == (2 * c, 1) and imp.dtype == np.float32
    assert abs(float(imp[1::2].sum()) / weight - 1.0) < 0.06
    # symmetric stance: the tangential impulses nearly cancel (the sweep order is not symmetric)
    assert abs(float(imp[0::2].sum())) < 0.01 * weight


def test_step_impulses_cone_and_flight():
    r = np.random.default_rng(5)
    for c in (2, 4):
        st = legged.stand_pose(c)[:, None] + r.uniform(-0.05, 0.05, (2 * (3 + c), 512)).astype(np.float32)
        act = r.integers(0, 3**c, 512)
        imp = legged.step_impulses(st, act, c)
        lt, ln = imp[0::2], imp[1::2]
        assert (ln >= 0).all() and (ln > 0).any()
        # each substep's impulse is inside the cone, so the sum is too
        assert (np.abs(lt) <= legged.LG_MU * ln + 1e-5).all()
    high = legged.stand_pose(2)[:, None].copy()
    high[1] += 1.0  # every foot a metre above the floor
    assert (legged.step_impulses(high, np.zeros(1, np.int64), 2) == 0).all()


def test_random_policy_keeps_legged_bodies_above_the_floor():
    r = np.random.default_rng(0)
    for c in (2, 4):
        st = legged.stand_pose(c)[:, None] + r.uniform(-0.05, 0.05, (2 * (3 + c), 256)).astype(np.float32)
        worst = 0.0
        for _ in range(60):
            st = legged.physics(st, r.integers(0, 3**c, 256), c)
            worst = min(worst, float(legged.foot_heights(st, c).min()))
        assert np.isfinite(st).all() and worst > -0.08


# ---- random streams ------------------------------------------------------------------------

def _pcg_int(v):
    s = (v * 747796405 + 2891336453) & 0xFFFFFFFF
    w = (((s >> ((s >> 28) + 4)) ^ s) * 277803737) & 0xFFFFFFFF
    return ((w >> 22) ^ w) & 0xFFFFFFFF


def test_pcg_hash_matches_python_integers():
    vals = np.array([0, 1, 2, 12345, 0x9E3779B9, 0xFFFFFFFF, 0x85EBCA6B], dtype=np.uint64)
    assert rng.pcg_hash(vals).tolist() == [_pcg_int(int(v)) for v in vals]


def test_reset_stream_statistics():
    out = rng.reset_rows(7, 16384, 4, 0.05, offsets=rng.CLASSIC_ROW_OFFSETS)
    assert np.all(np.abs(out) <= 0.05)
    assert len(np.unique(out[0])) > 0.99 * 16384
    assert abs(out.mean()) < 0.002 and abs(out.std() - 0.05 / np.sqrt(3)) < 0.002
    assert not np.allclose(out, rng.reset_rows(8, 16384, 4, 0.05, offsets=rng.CLASSIC_ROW_OFFSETS))


def test_philox_known_answers():
    """The Random123 known-answer vectors for Philox-4x32-10."""
    cases = [((0, 0, 0, 0), (0, 0), (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
             ((0xFFFFFFFF,) * 4, (0xFFFFFFFF,) * 2, (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
             ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
              (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1))]
    for ctr, key, want in cases:
        got = rng.philox4x32_10(*(np.array([c], np.uint64) for c in ctr), *(np.array([k], np.uint64) for k in key))
        assert tuple(int(g[0]) for g in got) == want


def test_noise_is_standard_normal_and_keyed():
    z = rng.noise(3, 1, np.arange(512), 64)
    assert abs(z.mean()) < 0.02 and abs(z.std() - 1.0) < 0.02
    np.testing.assert_array_equal(z[100:110], rng.noise(3, 1, np.arange(100, 110), 64))
    assert not np.allclose(z, rng.noise(3, 2, np.arange(512), 64))
