"""A whole ES rollout on a legged body as one sm_100a kernel launch.

Drop-in for the reference module of the same name (legged_rollout_metal.py:1-83):
`rollout(state, theta_pop, hidden, horizon, c, alive_bonus=1.0, fall_penalty=0.0,
height_gate=0.0, assist=0.0) -> (fitness (P,), steps (P,))`. Member i runs its
(5+2C)-H-3C tanh MLP (one three-way head per leg, greedy, first index on ties)
on the state without x, then four contact substeps with 8 Gauss-Seidel sweeps,
until it falls or `horizon` steps pass. Fitness sums (y >= height_gate ? x_dot : 0)
+ alive_bonus over the steps before the fall and subtracts fall_penalty once at
the fall; steps counts the steps taken including the falling one.

The reference passes the bonus, gate and penalty to Metal as integer template
constants (hundredths for the bonus and gate, whole units for the penalty); the
same quantisation is applied here, so the kernel sees the reference's values.
hidden in {1, 2, 4, 8, 16, 32}, c in 1..4.
"""

import numpy as np
import torch

import rlenv_lib as _rl

ITERS = 8


def _centi(x):
    return float(np.float32(int(round(100 * x))) / np.float32(100.0))


def rollout(state, theta_pop, hidden, horizon, c, alive_bonus=1.0, fall_penalty=0.0, height_gate=0.0, assist=0.0):
    state = _rl.as_state(state, 2 * (3 + c))
    p = state.shape[1]
    obs, out = 5 + 2 * c, 3 * c
    theta, stride = _rl.as_theta(theta_pop, p, obs * hidden + hidden + hidden * out + out, state.device)
    fit = torch.empty(p, dtype=torch.float32, device=state.device)
    steps = torch.empty(p, dtype=torch.float32, device=state.device)
    _rl.check(_rl.lib().legged_rollout(c, hidden, int(horizon), ITERS, _centi(alive_bonus),
                                       float(int(round(fall_penalty))), _centi(height_gate),
                                       _rl.float_scalar(assist), state.data_ptr(), theta.data_ptr(), stride, p,
                                       fit.data_ptr(), steps.data_ptr(), _rl.stream_ptr(state.device)))
    return fit, steps
