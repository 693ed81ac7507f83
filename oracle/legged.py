"""Hopper and legged-body contact dynamics in float32 numpy.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

A torso disk (mass 1, inertia 0.1) at the hip (x, y, phi) and C massless legs
of length 1 at relative angles psi_k, each with a 0.2 point mass at its foot.
q = (x, y, phi, psi_1..psi_C), state (2(3+C), N) = q then q_dot. Each foot is a
hard inelastic contact with Coulomb friction 0.7 and Baumgarte 0.2; four
semi-implicit Euler substeps of 0.01 per step; multiple contacts are combined
by block projected Gauss-Seidel (hopper_np.py:24-35, legged_np.py:24-97).
C = 1 with one sweep is the hopper.
"""

import numpy as np

from oracle.pendulum import chol_solve

LG_M_T, LG_I_T, LG_M_F, LG_L = 1.0, 0.1, 0.2, 1.0
LG_GRAVITY = 9.8
LG_TORQUE = 2.0
LG_MU = 0.7
LG_H, LG_SUBSTEPS = 0.01, 4
LG_BAUMGARTE = 0.2
LG_FALL_HEIGHT, LG_FALL_ANGLE = 0.6, 1.0
LG_RESET_BOUND = 0.05
LG_ITERS = 8
HOPPER_STAND = np.array([0.0, LG_L, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0], dtype=np.float32)


def leg_angles(c):
    """Resting leg angles, spread symmetrically 0.5 rad apart (legged_np.py:28-30)."""
    return 0.5 * (np.arange(c) - 0.5 * (c - 1))


def _pose(angles):
    """Zero-velocity state with the hip at the height where the innermost foot touches."""
    c = len(angles)
    s = np.zeros(2 * (3 + c), dtype=np.float32)
    s[1] = LG_L * np.cos(np.abs(angles).min())
    s[3:3 + c] = angles
    return s


def stand_pose(c):
    """Reset pose: hip at the height where the innermost feet touch the floor (legged_np.py:43-46)."""
    return _pose(leg_angles(c))


def static_pose(c):
    """Every foot on the floor with legs at +-0.25 rad: a true equilibrium (legged_np.py:33-40)."""
    return _pose(np.repeat([-0.25, 0.25], c // 2) if c > 1 else np.zeros(1))


def torques(action, c):
    """Action index in [0, 3^C) to per-leg torques ((a // 3^k) % 3 - 1) * 2 (legged_np.py:49-54)."""
    a = np.asarray(action)
    return [((a // 3**k) % 3 - 1).astype(np.float32) * LG_TORQUE for k in range(c)]


def contact_impulse(att, atn, ann, wt, wn, depth, mu=LG_MU, f32=False):
    """Exact single-contact impulse (lt, ln), branch-free (hopper_np.py:80-109): stick when
    the sticking impulse lies in the friction cone, else slide on the cone's edge in the
    direction that opposes the residual slip; nothing above the floor, when pulling, or when
    the free motion already separates. A sliding direction with a non-positive denominator
    (the Painleve regime) contributes nothing. As in the reference, the sliding sign is a
    float64 array, so lt (and every state it touches afterwards) is float64. With f32 the sign
    is float32 and every value stays float32, as in the reference's Metal kernels and its MLX
    step loop (legged_metal.py:53-71), which its rollout test compares (test_es.py:46-68)."""
    touching = depth >= 0.0
    target = LG_BAUMGARTE / LG_H * np.maximum(depth, 0.0)
    det = att * ann - atn * atn
    ln_st = (att * (target - wn) + atn * wt) / det
    lt_st = (-ann * wt - atn * (target - wn)) / det
    stick = np.abs(lt_st) <= mu * ln_st
    dp, dm = ann + mu * atn, ann - mu * atn
    ln_p = np.where(dp > 0.0, np.maximum((target - wn) / np.where(dp > 0.0, dp, 1.0), 0.0), 0.0)
    ln_m = np.where(dm > 0.0, np.maximum((target - wn) / np.where(dm > 0.0, dm, 1.0), 0.0), 0.0)
    slip = wt + (att * mu + atn) * ln_p
    one = np.float32(1.0) if f32 else 1.0
    direction = np.where(slip <= 0.0, one, -one)
    ln_sl = np.where(slip <= 0.0, ln_p, ln_m)
    lt_sl = mu * direction * ln_sl
    ln = np.where(stick, ln_st, ln_sl)
    lt = np.where(stick, lt_st, lt_sl)
    on = touching & (ln > 0.0) & (wn < target)
    return np.where(on, lt, 0.0), np.where(on, ln, 0.0)


def substep(q, v, tq, c, iters=LG_ITERS, mu=LG_MU, assist=0.0, return_impulses=False, f32=False):
    """One substep of 0.01 for C legs (legged_np.py:57-97). q, v: (3+C, N); tq: C arrays.
    f32 keeps every value float32 (see contact_impulse)."""
    n = 3 + c
    z = np.zeros_like(q[0])
    one = z + 1.0

    def foot(k):
        # Rows of the foot's tangential and normal Jacobians, the velocity-product term of its
        # acceleration, and its penetration below the floor.
        ang = q[2] + q[3 + k]
        ca, sa = np.cos(ang), np.sin(ang)
        rate = v[2] + v[3 + k]
        leg_t = [LG_L * ca if j == k else z for j in range(c)]
        leg_n = [LG_L * sa if j == k else z for j in range(c)]
        return ([one, z, LG_L * ca, *leg_t], [z, one, LG_L * sa, *leg_n],
                (-LG_L * sa * rate * rate, LG_L * ca * rate * rate), -(q[1] - LG_L * ca))

    Jt, Jn, drift, depth = (list(col) for col in zip(*(foot(k) for k in range(c))))
    base = [[0.0] * n for _ in range(n)]  # Python floats: weak scalars in float32 expressions
    base[0][0] = base[1][1] = LG_M_T
    base[2][2] = LG_I_T
    M = np.stack([np.stack([base[i][j] + LG_M_F * sum(Jt[k][i] * Jt[k][j] + Jn[k][i] * Jn[k][j] for k in range(c))
                            for j in range(n)]) for i in range(n)])
    f = [-LG_M_F * sum(Jt[k][i] * drift[k][0] + Jn[k][i] * drift[k][1] for k in range(c))
         - LG_GRAVITY * (LG_M_F * sum(Jn[k][i] for k in range(c)) + (LG_M_T if i == 1 else 0.0)) for i in range(n)]
    for k in range(c):
        f[3 + k] = f[3 + k] + tq[k]
    f[2] = f[2] - assist * q[2] - 0.1 * assist * v[2]
    vfree = [v[i] + LG_H * a for i, a in enumerate(chol_solve(M, np.stack(f), n))]
    MiJt = [chol_solve(M, np.stack(Jt[k]), n) for k in range(c)]
    MiJn = [chol_solve(M, np.stack(Jn[k]), n) for k in range(c)]

    def dot(a, b):
        return sum(a[i] * b[i] for i in range(n))

    A = [[(dot(Jt[k], MiJt[l]), dot(Jt[k], MiJn[l]), dot(Jn[k], MiJt[l]), dot(Jn[k], MiJn[l])) for l in range(c)]
         for k in range(c)]
    w0 = [(dot(Jt[k], vfree), dot(Jn[k], vfree)) for k in range(c)]
    lt, ln = [z] * c, [z] * c

    def coupled(k, row):
        # Velocity that the other contacts' current impulses add along row 0 (tangent) or 1 (normal).
        return sum(A[k][l][2 * row] * lt[l] + A[k][l][2 * row + 1] * ln[l] for l in range(c) if l != k)

    for _ in range(iters):
        for k in range(c):
            rel_t, rel_n = w0[k][0] + coupled(k, 0), w0[k][1] + coupled(k, 1)
            lt[k], ln[k] = contact_impulse(A[k][k][0], A[k][k][1], A[k][k][3], rel_t, rel_n, depth[k], mu, f32)
    vnew = np.stack([vfree[i] + sum(MiJt[k][i] * lt[k] + MiJn[k][i] * ln[k] for k in range(c)) for i in range(n)])
    out = q + LG_H * vnew, vnew
    return out + (np.stack(lt), np.stack(ln)) if return_impulses else out


def physics(state, action, c, iters=LG_ITERS, assist=0.0, f32=False):
    """Four substeps from state (2(3+C), N) under the decoded per-leg torques (legged_np.py:121-128).
    f32 keeps every value float32 (see contact_impulse)."""
    s = np.asarray(state)
    d = 3 + c
    q, v = s[:d], s[d:]
    tq = torques(action, c)
    for _ in range(LG_SUBSTEPS):
        q, v = substep(q, v, tq, c, iters, assist=assist, f32=f32)
    return np.r_[q, v]


def step_impulses(state, action, c, iters=LG_ITERS, assist=0.0):
    """The contact impulses of one step, (2C, N): row 2k the tangential and row 2k + 1 the
    normal impulse of foot k, each the final (lt, ln) of a substep's Gauss-Seidel solve
    (legged_np.py:89-96) summed over the four substeps. The reference's step computes them
    and drops them; this is the checker for the step's optional impulse output."""
    s = np.asarray(state)
    d = 3 + c
    q, v = s[:d], s[d:]
    tq = torques(action, c)
    total = np.zeros((2 * c, s.shape[1]), dtype=np.float64)
    for _ in range(LG_SUBSTEPS):
        q, v, lt, ln = substep(q, v, tq, c, iters, assist=assist, return_impulses=True)
        total[0::2] += lt
        total[1::2] += ln
    return total.astype(np.float32)


def terminated(state):
    """Torso below 0.6 or tilted past 1 rad (legged_np.py:130-132)."""
    return (state[1] < LG_FALL_HEIGHT) | (np.abs(state[2]) > LG_FALL_ANGLE)


def reward(stepped, done, c):
    """Forward velocity plus one, zero on the terminating step (legged_np.py:115-119)."""
    return np.where(done, np.float32(0.0), stepped[3 + c] + np.float32(1.0)).astype(np.float32)


def foot_heights(state, c):
    """Height of every foot above the floor (C, N)."""
    return state[1] - LG_L * np.cos(state[2] + state[3:3 + c])
