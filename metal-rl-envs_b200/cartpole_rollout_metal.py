"""A whole ES rollout on CartPole as one sm_100a kernel launch.

Drop-in for the reference module of the same name (cartpole_rollout_metal.py:1-100):
`rollout_steps(state, theta_pop, hidden, horizon) -> fitness (P,)`, the steps each
member survived (its terminating step excluded) running its own 4-H-2 tanh MLP,
greedy with the first index winning ties, from column i of `state` (4, P). Rows
of theta_pop (P, 7H + 2) follow es.unflatten: w1 (4, H), b1 (H), w2 (H, 2), b2 (2).
A single row (7H + 2,) is shared by every member. A group of min(H, 32) warp
lanes runs each member, one hidden unit (or two at H = 64) per lane, with its
weights in registers for the whole horizon. hidden in {1, 2, 4, 8, 16, 32, 64}.
"""

import torch

import rlenv_lib as _rl


def rollout_steps(state, theta_pop, hidden, horizon):
    state = _rl.as_state(state, 4)
    p = state.shape[1]
    theta, stride = _rl.as_theta(theta_pop, p, 7 * hidden + 2, state.device)
    fit = torch.empty(p, dtype=torch.float32, device=state.device)
    _rl.check(_rl.lib().cartpole_rollout(state.data_ptr(), theta.data_ptr(), stride, p, hidden, int(horizon),
                                         fit.data_ptr(), _rl.stream_ptr(state.device)))
    return fit
