"""The K-link pendulum by Featherstone's articulated-body algorithm, one thread per environment.

Drop-in for the reference module of the same name (pendulum_aba_metal.py:1-144):
`Pendulum(k)` with `.step(state, action)`, `.reseed(seed)`, `.reset(n)`. Same
state, action, reward and reset conventions as pendulum_metal; the
accelerations come from three O(K) passes over the links (outward velocities,
inward articulated inertias and bias forces, outward accelerations) instead of
a K x K solve. Built for any K from 1 to 192 (K > 16 with its per-link arrays in
shared memory; K > 64, or any K with cooperative=True, one warp per environment).
"""

import rlenv_lib as _rl
from pendulum_metal import RESET_BOUND


class Pendulum(_rl.StepBody):
    """cooperative=True runs one warp per environment (rlenv_pendulum_aba_coop_step_many: the
    recurrences along the chain as scans over the lanes), the faster form for batches that do not
    fill the GPU with one thread per environment (K = 64: 6x at N = 256, 2.2x at N = 4,096);
    above 64 links the library runs it for every batch."""

    def __init__(self, k, cooperative=False):
        super().__init__()
        self.k = k
        self.rows = 2 * k
        self.cooperative = bool(cooperative)

    def reset(self, n):
        return _rl.reset_uniform(self.rows, n, RESET_BOUND)

    def step(self, state, action):
        if self.cooperative:  # one step is the T-step launch with T = 1
            state = _rl.as_state(state, self.rows)
            action, _ = _rl.as_actions(action, state.shape[1], state.device)
            nxt, rew, done = self._launch_many(_rl.lib().pendulum_aba_coop_step_many, (self.k,), state,
                                               action.reshape(1, -1))
            return nxt, rew[0], done[0]
        return self._launch(_rl.lib().pendulum_aba_step, (self.k,), state, action)

    def step_many(self, state, actions, rewards=True, dones=True):
        """T steps in one launch for actions (T, N): equal bit for bit to T `step` calls (the same
        seeds are drawn). Returns (final_state, rewards (T, N) or None, dones (T, N) or None)."""
        fn = _rl.lib().pendulum_aba_coop_step_many if self.cooperative else _rl.lib().pendulum_aba_step_many
        return self._launch_many(fn, (self.k,), state, actions, rewards=rewards, dones=dones)
