"""Semantics of the fused ES rollout kernels, vectorised over the population in numpy.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Member i runs the MLP policy in row i of theta_pop (es.unflatten's layout)
against its own environment from column i of the initial state until its first
termination or `horizon` steps:

- cartpole, acrobot: fitness = steps before the first termination
  (cartpole_rollout_metal.py:53-76, acrobot_rollout_metal.py:31-57);
- legged: fitness = sum over non-falling steps of (y >= gate ? x_dot : 0) + alive,
  minus `fall` once at the fall; steps = steps taken including the falling one
  (legged_rollout_metal.py:36-58).

The policy is greedy with the first index winning ties, as numpy's argmax.
A terminated member's state is frozen; it no longer affects anything.
"""

import numpy as np

from oracle import classic, legged


def policy_logits(obs, theta_pop, hidden, obs_dim, n_out):
    """(P, n_out) logits of an obs-H-out tanh MLP per member (es.py:156-171)."""
    P, H = theta_pop.shape[0], hidden
    i = 0
    w1 = theta_pop[:, i:i + obs_dim * H].reshape(P, obs_dim, H); i += obs_dim * H
    b1 = theta_pop[:, i:i + H]; i += H
    w2 = theta_pop[:, i:i + H * n_out].reshape(P, H, n_out); i += H * n_out
    b2 = theta_pop[:, i:i + n_out]
    h = np.tanh(np.einsum("pi,pih->ph", obs, w1) + b1)
    return np.einsum("ph,pho->po", h, w2) + b2


def _theta_rows(theta, p):
    theta = np.asarray(theta, dtype=np.float32)
    return np.broadcast_to(theta.reshape(1, -1), (p, theta.size)) if theta.ndim == 1 or theta.shape[0] == 1 else theta


def cartpole(state, theta, hidden, horizon):
    s = np.array(state, dtype=np.float32)
    P = s.shape[1]
    theta = _theta_rows(theta, P)
    alive = np.ones(P, dtype=bool)
    survived = np.zeros(P, dtype=np.float32)
    for _ in range(horizon):
        if not alive.any():
            break
        act = np.argmax(policy_logits(s.T, theta, hidden, 4, 2), axis=-1)
        nxt = classic.cartpole_physics(s, act)
        term = classic.cartpole_terminated(nxt)
        survived += (alive & ~term).astype(np.float32)
        s = np.where(alive[None, :], nxt, s)
        alive &= ~term
    return survived


def acrobot_obs(s):
    return np.stack([np.cos(s[0]), np.sin(s[0]), np.cos(s[1]), np.sin(s[1]), s[2], s[3]], axis=1)


def acrobot(state, theta, hidden, horizon):
    s = np.array(state, dtype=np.float32)
    P = s.shape[1]
    theta = _theta_rows(theta, P)
    alive = np.ones(P, dtype=bool)
    survived = np.zeros(P, dtype=np.float32)
    for _ in range(horizon):
        if not alive.any():
            break
        act = np.argmax(policy_logits(acrobot_obs(s), theta, hidden, 6, 3), axis=-1)
        nxt = classic.acrobot_physics(s, act)
        term = classic.acrobot_terminated(nxt)
        survived += (alive & ~term).astype(np.float32)
        s = np.where(alive[None, :], nxt, s)
        alive &= ~term
    return survived


def legged_action(logits, c):
    """Per-leg three-way heads to one action index: sum_k argmax(head k) * 3^k (es.py:86-93)."""
    out = np.zeros(logits.shape[0], dtype=np.int64)
    for k in range(c):
        out += np.argmax(logits[:, 3 * k:3 * k + 3], axis=-1) * 3**k
    return out


def legged_rollout(state, theta, hidden, horizon, c, alive_bonus=1.0, fall_penalty=0.0, height_gate=0.0,
                   assist=0.0, iters=legged.LG_ITERS, f32=False):
    """f32 runs the physics in float32 throughout (legged.contact_impulse); by default it
    follows the reference numpy's float64 promotion."""
    s = np.array(state)
    P = s.shape[1]
    theta = _theta_rows(theta, P)
    alive = np.ones(P, dtype=bool)
    fit = np.zeros(P)
    steps = np.zeros(P)
    for _ in range(horizon):
        if not alive.any():
            break
        act = legged_action(policy_logits(s[1:].T, theta, hidden, 5 + 2 * c, 3 * c), c)
        nxt = legged.physics(s, act, c, iters, assist, f32=f32)
        fell = legged.terminated(nxt)
        steps += alive
        forward = np.where(nxt[1] >= height_gate, nxt[3 + c], 0.0)
        fit += np.where(alive & ~fell, forward + alive_bonus, 0.0) - np.where(alive & fell, fall_penalty, 0.0)
        s = np.where(alive[None, :], nxt, s)
        alive &= ~fell
    return fit.astype(np.float32), steps.astype(np.float32)
