"""K-link pendulum dynamics in float32 numpy: mass-matrix and articulated-body forms.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

State (2K, N): K absolute angles from the downward vertical, then K angular
velocities. Unit point masses on unit massless rods, gravity 9.8, root torque
(action - 1) * 1.0, RK4 with dt 0.02, angles wrapped to [-pi, pi), velocities
clipped to +-10 pi (pendulum_np.py:27-66).
"""

import numpy as np

from oracle.classic import wrap_angle

PD_GRAVITY = 9.8
PD_DT = 0.02
PD_TORQUE = 1.0
PD_MAX_VEL = 10 * np.pi
PD_RESET_BOUND = 0.1


def hanging_mass(k):
    """mu_ij = K - max(i, j): the unit masses beyond the outer of joints i and j (pendulum_np.py:37-39)."""
    idx = np.arange(k)
    return (k - np.maximum(idx[:, None], idx[None, :])).astype(np.float32)


def chol_solve(M, b, k):
    """Solve M x = b for symmetric positive definite M (k, k, N), b (k, N), batched over N:
    Cholesky row by row, then forward and back substitution, each a scalar loop over
    vector operations (pendulum_np.py:83-107)."""
    L = {}
    for i in range(k):
        for j in range(i + 1):
            acc = M[i, j]
            for p in range(j):
                acc = acc - L[i, p] * L[j, p]
            L[i, j] = np.sqrt(acc) if i == j else acc / L[j, j]
    y = []
    for i in range(k):
        acc = b[i]
        for p in range(i):
            acc = acc - L[i, p] * y[p]
        y.append(acc / L[i, i])
    x = [None] * k
    for i in range(k - 1, -1, -1):
        acc = y[i]
        for p in range(i + 1, k):
            acc = acc - L[p, i] * x[p]
        x[i] = acc / L[i, i]
    return np.stack(x)


def mm_accel(th, om, torque, k):
    """Angular accelerations (k, N) from M(t) a = tau - c(t, w) - g(t) (pendulum_np.py:68-78)."""
    mu = hanging_mass(k)
    c, s = np.cos(th), np.sin(th)
    cos_d = c[:, None, :] * c[None, :, :] + s[:, None, :] * s[None, :, :]
    sin_d = s[:, None, :] * c[None, :, :] - c[:, None, :] * s[None, :, :]
    M = mu[:, :, None] * cos_d
    coriolis = (mu[:, :, None] * sin_d * (om**2)[None, :, :]).sum(axis=1)
    rhs = -coriolis - PD_GRAVITY * np.diag(mu)[:, None] * s
    rhs[0] = rhs[0] + torque
    return chol_solve(M, rhs, k)


def aba_accel(th, om, torque, k):
    """Absolute angular accelerations by Featherstone's articulated-body algorithm
    (pendulum_aba_np.py:30-99): outward link velocities and velocity-product biases,
    inward articulated inertias and bias forces, outward accelerations with the base
    accelerating at -g, then a prefix sum from joint to absolute accelerations.
    Planar motion vectors (w, vx, vy); inertias as (00, 01, 02, 11, 12, 22)."""
    z = np.zeros_like(th[0])
    q = [th[0], *np.diff(th[:k], axis=0)]  # joint angle: each link relative to its parent
    qd = [om[0], *np.diff(om[:k], axis=0)]
    cs = [np.cos(qi) for qi in q]
    sn = [np.sin(qi) for qi in q]
    vel, bias_c, p, inertia = [], [], [], []
    prev = (z, z, z)
    for i in range(k):
        r = 0.0 if i == 0 else 1.0
        w, x, y = prev
        xy = y + w * r
        v = (w + qd[i], cs[i] * x + sn[i] * xy, -sn[i] * x + cs[i] * xy)
        vel.append(v)
        bias_c.append((z, qd[i] * v[2], -qd[i] * v[1]))
        fx, fy = v[1], v[0] + v[2]
        p.append([v[1] * fy - v[2] * fx, -v[0] * fy, v[0] * fx])
        inertia.append([z + 1.0, z, z + 1.0, z + 1.0, z, z + 1.0])
        prev = v
    U, D, u = {}, {}, {}
    for i in range(k - 1, -1, -1):
        a00, a01, a02, a11, a12, a22 = inertia[i]
        U[i] = (a00, a01, a02)
        D[i] = a00
        u[i] = (torque if i == 0 else z) - p[i][0]
        if i == 0:
            break
        u0, u1, u2 = U[i]
        d = D[i]
        ia = (a00 - u0 * u0 / d, a01 - u0 * u1 / d, a02 - u0 * u2 / d,
              a11 - u1 * u1 / d, a12 - u1 * u2 / d, a22 - u2 * u2 / d)
        cc = bias_c[i]
        iac = (ia[0] * cc[0] + ia[1] * cc[1] + ia[2] * cc[2],
               ia[1] * cc[0] + ia[3] * cc[1] + ia[4] * cc[2],
               ia[2] * cc[0] + ia[4] * cc[1] + ia[5] * cc[2])
        g = u[i] / d
        pa = [p[i][j] + iac[j] + U[i][j] * g for j in range(3)]
        c_, s_ = cs[i], sn[i]
        x1, x2 = s_ * 1.0, c_ * 1.0
        rows = ((ia[0], ia[1], ia[2]), (ia[1], ia[3], ia[4]), (ia[2], ia[4], ia[5]))
        B = [(m0 + m1 * x1 + m2 * x2, m1 * c_ - m2 * s_, m1 * s_ + m2 * c_) for m0, m1, m2 in rows]
        cols = ((1.0, x1, x2), (0.0, c_, -s_), (0.0, s_, c_))

        def xtb(a, b):
            return cols[a][0] * B[0][b] + cols[a][1] * B[1][b] + cols[a][2] * B[2][b]

        par = inertia[i - 1]
        inertia[i - 1] = [par[0] + xtb(0, 0), par[1] + xtb(0, 1), par[2] + xtb(0, 2),
                          par[3] + xtb(1, 1), par[4] + xtb(1, 2), par[5] + xtb(2, 2)]
        pp = p[i - 1]
        p[i - 1] = [pp[0] + pa[0] + x1 * pa[1] + x2 * pa[2], pp[1] + c_ * pa[1] - s_ * pa[2],
                    pp[2] + s_ * pa[1] + c_ * pa[2]]
    acc_prev = (z, z - PD_GRAVITY, z)
    run, out = z, []
    for i in range(k):
        r = 0.0 if i == 0 else 1.0
        w, x, y = acc_prev
        xy = y + w * r
        ap = (w + bias_c[i][0], cs[i] * x + sn[i] * xy + bias_c[i][1], -sn[i] * x + cs[i] * xy + bias_c[i][2])
        qdd = (u[i] - (U[i][0] * ap[0] + U[i][1] * ap[1] + U[i][2] * ap[2])) / D[i]
        acc_prev = (ap[0] + qdd, ap[1], ap[2])
        run = run + qdd
        out.append(run)
    return np.stack(out)


def rk4(state, action, k, accel):
    """RK4 of dt 0.02 on (t, w) with root torque (action - 1) (pendulum_np.py:60-66)."""
    s = np.asarray(state, dtype=np.float32)
    tq = ((np.asarray(action) - 1) * PD_TORQUE).astype(np.float32)

    def deriv(x):
        return np.concatenate([x[k:], accel(x[:k], x[k:], tq, k)])

    k1 = deriv(s)
    k2 = deriv(s + PD_DT / 2 * k1)
    k3 = deriv(s + PD_DT / 2 * k2)
    k4 = deriv(s + PD_DT * k3)
    nxt = s + PD_DT / 6 * (k1 + 2 * k2 + 2 * k3 + k4)
    return np.concatenate([wrap_angle(nxt[:k]), np.clip(nxt[k:], -PD_MAX_VEL, PD_MAX_VEL)]).astype(np.float32)


def mm_physics(state, action, k):
    return rk4(state, action, k, mm_accel)


def aba_physics(state, action, k):
    return rk4(state, action, k, aba_accel)


def terminated(state, k):
    """The tip above half the chain's length: -sum cos t > K / 2 (pendulum_np.py:79-80)."""
    return -np.cos(state[:k]).sum(axis=0) > k / 2


def reward(done):
    return np.where(done, np.float32(0.0), np.float32(-1.0)).astype(np.float32)


def energy(state, k):
    """Kinetic plus potential energy per env, unit masses and rods (pendulum_np.py:114-120)."""
    th, om = state[:k], state[k:2 * k]
    joint_vel = np.cumsum(np.stack([om * np.cos(th), om * np.sin(th)]), axis=1)  # (2, K, N)
    kinetic = 0.5 * np.square(joint_vel).sum(axis=0).sum(axis=0)
    return kinetic + PD_GRAVITY * np.cumsum(-np.cos(th), axis=0).sum(axis=0)
