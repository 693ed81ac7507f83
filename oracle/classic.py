"""CartPole and Acrobot dynamics in float32 numpy, restated from the reference.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Arrays are structure-of-arrays (4, N) float32. Python-float constants enter
float32 expressions the way numpy >= 2 treats weak scalars: cast to float32,
so the arithmetic below is float32 throughout, as in the reference.
"""

import numpy as np

# ---- CartPole (cartpole_np.py:20-31) ----------------------------------------
CP_GRAVITY = 9.8
CP_CART_MASS = 1.0
CP_POLE_MASS = 0.1
CP_TOTAL_MASS = CP_CART_MASS + CP_POLE_MASS
CP_HALF_POLE = 0.5
CP_POLE_MASS_LENGTH = CP_POLE_MASS * CP_HALF_POLE
CP_FORCE = 10.0
CP_TAU = 0.02
CP_X_LIMIT = 2.4
CP_THETA_LIMIT = 12 * 2 * np.pi / 360
CP_RESET_BOUND = 0.05


def cartpole_physics(state, action):
    """One explicit-Euler step of Gym CartPole-v1 (cartpole_np.py:58-77). action == 1 pushes right."""
    x, x_dot, th, th_dot = (np.asarray(r, dtype=np.float32) for r in state)
    push = np.float32(CP_FORCE) * np.where(np.asarray(action) == 1, np.float32(1), np.float32(-1))
    cth, sth = np.cos(th), np.sin(th)
    temp = (push + CP_POLE_MASS_LENGTH * th_dot**2 * sth) / CP_TOTAL_MASS
    alpha = (CP_GRAVITY * sth - cth * temp) / (CP_HALF_POLE * (4.0 / 3.0 - CP_POLE_MASS * cth**2 / CP_TOTAL_MASS))
    acc = temp - CP_POLE_MASS_LENGTH * alpha * cth / CP_TOTAL_MASS
    rows = (x + CP_TAU * x_dot, x_dot + CP_TAU * acc, th + CP_TAU * th_dot, th_dot + CP_TAU * alpha)
    return np.stack(rows).astype(np.float32)


def cartpole_terminated(state):
    """|x| beyond 2.4 or |theta| beyond 12 degrees (cartpole_np.py:80-83)."""
    return (np.abs(state[0]) > CP_X_LIMIT) | (np.abs(state[2]) > CP_THETA_LIMIT)


def cartpole_reward(done):
    return np.ones(np.shape(done), dtype=np.float32)


# ---- Acrobot (acrobot_np.py:19-30) --------------------------------------------
AC_L1 = 1.0
AC_M1 = 1.0
AC_M2 = 1.0
AC_LC1 = 0.5
AC_LC2 = 0.5
AC_MOI = 1.0
AC_GRAVITY = 9.8
AC_DT = 0.2
AC_MAX_VEL_1 = 4 * np.pi
AC_MAX_VEL_2 = 9 * np.pi
AC_RESET_BOUND = 0.1


def _acrobot_derivative(th1, th2, w1, w2, torque):
    """Gym AcrobotEnv._dsdt, book dynamics, torque alongside the state (acrobot_np.py:64-86)."""
    m1, m2, l1, lc1, lc2 = AC_M1, AC_M2, AC_L1, AC_LC1, AC_LC2
    i1 = i2 = AC_MOI
    g = AC_GRAVITY
    c2, s2 = np.cos(th2), np.sin(th2)
    d1 = m1 * lc1**2 + m2 * (l1**2 + lc2**2 + 2 * l1 * lc2 * c2) + i1 + i2
    d2 = m2 * (lc2**2 + l1 * lc2 * c2) + i2
    phi2 = m2 * lc2 * g * np.cos(th1 + th2 - np.pi / 2)
    phi1 = (-m2 * l1 * lc2 * w2**2 * s2 - 2 * m2 * l1 * lc2 * w2 * w1 * s2
            + (m1 * lc1 + m2 * l1) * g * np.cos(th1 - np.pi / 2) + phi2)
    alpha2 = (torque + d2 / d1 * phi1 - m2 * l1 * lc2 * w1**2 * s2 - phi2) / (m2 * lc2**2 + i2 - d2**2 / d1)
    alpha1 = -(d2 * alpha2 + phi1) / d1
    return np.stack([w1, w2, alpha1, alpha2])


def wrap_angle(x):
    """To [-pi, pi) without branches (acrobot_np.py:87-89)."""
    period = 2 * np.pi
    return x - period * np.floor((x + np.pi) / period)


def acrobot_physics(state, action):
    """One RK4 step of dt 0.2, then wrap and clip (acrobot_np.py:47-61); action in {0,1,2} is torque a - 1."""
    s = np.asarray(state, dtype=np.float32)
    tq = (np.asarray(action) - 1).astype(np.float32)
    k1 = _acrobot_derivative(*s, tq)
    k2 = _acrobot_derivative(*(s + AC_DT / 2 * k1), tq)
    k3 = _acrobot_derivative(*(s + AC_DT / 2 * k2), tq)
    k4 = _acrobot_derivative(*(s + AC_DT * k3), tq)
    nxt = s + AC_DT / 6 * (k1 + 2 * k2 + 2 * k3 + k4)
    return np.stack([wrap_angle(nxt[0]), wrap_angle(nxt[1]),
                     np.clip(nxt[2], -AC_MAX_VEL_1, AC_MAX_VEL_1),
                     np.clip(nxt[3], -AC_MAX_VEL_2, AC_MAX_VEL_2)]).astype(np.float32)


def acrobot_terminated(state):
    """Tip above height 1: -cos t1 - cos(t1 + t2) > 1 (acrobot_np.py:92-93)."""
    return np.cos(state[0]) + np.cos(state[0] + state[1]) < -1.0


def acrobot_reward(done):
    return np.where(done, np.float32(0.0), np.float32(-1.0)).astype(np.float32)
