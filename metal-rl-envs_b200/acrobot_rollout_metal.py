"""A whole ES rollout on Acrobot as one sm_100a kernel launch.

Drop-in for the reference module of the same name (acrobot_rollout_metal.py:1-81):
`rollout_steps(state, theta_pop, hidden, horizon) -> steps (P,)` before each
member's tip first clears height 1 (the horizon if never), each running its own
6-H-3 tanh MLP on Gym's observation (cos, sin of both angles, both velocities).
Rows of theta_pop (P, 10H + 3): w1 (6, H), b1 (H), w2 (H, 3), b2 (3).
hidden in {1, 2, 4, 8, 16, 32, 64}.
"""

import torch

import rlenv_lib as _rl


def rollout_steps(state, theta_pop, hidden, horizon):
    state = _rl.as_state(state, 4)
    p = state.shape[1]
    theta, stride = _rl.as_theta(theta_pop, p, 10 * hidden + 3, state.device)
    fit = torch.empty(p, dtype=torch.float32, device=state.device)
    _rl.check(_rl.lib().acrobot_rollout(state.data_ptr(), theta.data_ptr(), stride, p, hidden, int(horizon),
                                        fit.data_ptr(), _rl.stream_ptr(state.device)))
    return fit
