"""The K-link pendulum by Featherstone's articulated-body algorithm, one thread per environment.

Drop-in for the reference module of the same name (pendulum_aba_metal.py:1-144):
`Pendulum(k)` with `.step(state, action)`, `.reseed(seed)`, `.reset(n)`. Same
state, action, reward and reset conventions as pendulum_metal; the
accelerations come from three O(K) passes over the links (outward velocities,
inward articulated inertias and bias forces, outward accelerations) instead of
a K x K solve. Built for any K from 1 to 192 (K > 16 with its per-link arrays in
shared memory).
"""

import rlenv_lib as _rl
from pendulum_metal import RESET_BOUND


class Pendulum(_rl.StepBody):
    def __init__(self, k):
        super().__init__()
        self.k = k
        self.rows = 2 * k

    def reset(self, n):
        return _rl.reset_uniform(self.rows, n, RESET_BOUND)

    def step(self, state, action):
        return self._launch(_rl.lib().pendulum_aba_step, (self.k,), state, action)

    def step_many(self, state, actions, rewards=True, dones=True):
        """T steps in one launch for actions (T, N): equal bit for bit to T `step` calls (the same
        seeds are drawn). Returns (final_state, rewards (T, N) or None, dones (T, N) or None)."""
        return self._launch_many(_rl.lib().pendulum_aba_step_many, (self.k,), state, actions, rewards=rewards,
                                 dones=dones)
