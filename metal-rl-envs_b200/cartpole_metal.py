"""Batched CartPole stepped by a hand-written sm_100a CUDA kernel.

Drop-in for the reference module of the same name (cartpole_metal.py:1-125):
`step(state, action) -> (next_state, reward, done)`, `reseed(seed=0)` and
`reset(n)`, with torch CUDA tensors where the reference used MLX arrays.

State is (4, N) float32, rows x, x_dot, theta, theta_dot, one column per
environment. One kernel launch per call does the physics (Gym CartPole-v1,
explicit Euler with tau 0.02), the termination test, the in-place reset of
terminated columns from the in-kernel hash stream, the reward (always 1) and
the done flag. The per-call seed is a counter incremented before each call,
as in the reference; reseed sets it.

`step_many(state, actions)` is an addition: T steps in one launch with the
state held in registers, equal to T calls of `step` with the same actions.
"""

import rlenv_lib as _rl

GRAVITY = 9.8
CART_MASS = 1.0
POLE_MASS = 0.1
TOTAL_MASS = CART_MASS + POLE_MASS
HALF_POLE_LENGTH = 0.5
POLE_MASS_LENGTH = POLE_MASS * HALF_POLE_LENGTH
FORCE_MAG = 10.0
TAU = 0.02
X_LIMIT = 2.4
THETA_LIMIT = 12 * 2 * 3.141592653589793 / 360
RESET_BOUND = 0.05
ROWS = 4

_counter = _rl.StepCounter()


def reseed(seed=0):
    _counter.calls = seed


def reset(n):
    """Fresh initial states for n environments: every variable uniform in +-RESET_BOUND."""
    return _rl.reset_uniform(ROWS, n, RESET_BOUND)


def step(state, action):
    """Advance all N environments by one step in one kernel launch."""
    state = _rl.as_state(state, ROWS)
    n = state.shape[1]
    if isinstance(action, _rl.PackedActions):  # rlenv_lib.pack_actions of one step
        if action.steps != 1:
            raise ValueError(f"step takes the packed actions of one step; got {action.steps}")
        action, dt = action.checked(n, state.device), _rl.U2
    else:
        action, dt = _rl.as_actions(action, n, state.device)
    nxt, reward, done = _rl.step_outputs(ROWS, n, state.device)
    _rl.check(_rl.lib().cartpole_step(state.data_ptr(), action.data_ptr(), dt, _counter.next(), n, 0,
                                      nxt.data_ptr(), reward.data_ptr(), done.data_ptr(),
                                      _rl.stream_ptr(state.device)))
    return nxt, reward, done


def step_many(state, actions, rewards=True, dones=True, sums=False, out=None):
    """T steps in one launch for actions (T, N). Returns (final_state, rewards (T, N) or None,
    dones (T, N) or None[, reward_sum (N,), done_count (N,)] if sums). `out` may give the
    final-state tensor (it may be `state` itself). actions may also be rlenv_lib.pack_actions'
    PackedActions, four steps to a byte: the same results from a quarter of the uint8 bytes (for a
    caller that streams actions from host memory)."""
    return _rl.run_step_many(_rl.lib().cartpole_step_many, ROWS, _counter, state, actions, rewards, dones, sums, out)
