"""Batched Acrobot stepped by a hand-written sm_100a CUDA kernel.

Drop-in for the reference module of the same name (acrobot_metal.py:1-111):
`step(state, action)`, `reseed(seed=0)`, `reset(n)`. State (4, N) float32,
rows theta1, theta2, dtheta1, dtheta2; action in {0, 1, 2} is torque -1, 0, +1.
One launch per call runs RK4 with dt 0.2 (four derivative evaluations of Gym's
book dynamics), wrap and clip, the termination test (tip above height 1), the
hash-stream reset of terminated columns and the reward (-1, 0 on termination).

`step_many(state, actions)` runs T steps per launch with the state in registers.
"""

import rlenv_lib as _rl

DT = 0.2
MAX_VEL_1 = 4 * 3.141592653589793
MAX_VEL_2 = 9 * 3.141592653589793
RESET_BOUND = 0.1
ROWS = 4

_counter = _rl.StepCounter()


def reseed(seed=0):
    _counter.calls = seed


def reset(n):
    """Fresh initial states for n environments: every variable uniform in +-RESET_BOUND."""
    return _rl.reset_uniform(ROWS, n, RESET_BOUND)


def step(state, action):
    state = _rl.as_state(state, ROWS)
    n = state.shape[1]
    if isinstance(action, _rl.PackedActions):  # rlenv_lib.pack_actions of one step
        if action.steps != 1:
            raise ValueError(f"step takes the packed actions of one step; got {action.steps}")
        action, dt = action.checked(n, state.device), _rl.U2
    else:
        action, dt = _rl.as_actions(action, n, state.device)
    nxt, reward, done = _rl.step_outputs(ROWS, n, state.device)
    _rl.check(_rl.lib().acrobot_step(state.data_ptr(), action.data_ptr(), dt, _counter.next(), n, 0,
                                     nxt.data_ptr(), reward.data_ptr(), done.data_ptr(),
                                     _rl.stream_ptr(state.device)))
    return nxt, reward, done


def step_many(state, actions, rewards=True, dones=True, sums=False, out=None):
    """T steps in one launch for actions (T, N). Returns (final_state, rewards (T, N) or None,
    dones (T, N) or None[, reward_sum (N,), done_count (N,)] if sums). `out` may give the
    final-state tensor (it may be `state` itself). actions may also be rlenv_lib.pack_actions'
    PackedActions, four steps to a byte: the same results from a quarter of the uint8 bytes (for a
    caller that streams actions from host memory)."""
    return _rl.run_step_many(_rl.lib().acrobot_step_many, ROWS, _counter, state, actions, rewards, dones, sums, out)
