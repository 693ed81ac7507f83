"""The K-link pendulum step with K warp lanes cooperating on each environment.

Drop-in for the reference module of the same name (pendulum_metal_coop.py:1-149):
`Pendulum(k)` with `.step(state, action)`, `.reseed(seed)`, `.reset(n)`. Lane j
of an environment's K-lane segment owns row j of the mass matrix and of its
Cholesky factor; the factorisation, the two substitutions and the termination
height are formed with warp shuffles. K must be a power of two no larger than
32, so segments tile a 32-lane warp.
"""

import rlenv_lib as _rl
from pendulum_metal import RESET_BOUND


class Pendulum(_rl.StepBody):
    def __init__(self, k):
        if k not in (2, 4, 8, 16, 32):
            raise ValueError("K lanes must tile a 32-lane warp: k in {2, 4, 8, 16, 32}")
        super().__init__()
        self.k = k
        self.rows = 2 * k

    def reset(self, n):
        return _rl.reset_uniform(self.rows, n, RESET_BOUND)

    def step(self, state, action):
        return self._launch(_rl.lib().pendulum_coop_step, (self.k,), state, action)

    def step_many(self, state, actions, rewards=True, dones=True):
        """T steps in one launch for actions (T, N): equal bit for bit to T `step` calls (the same
        seeds are drawn). Returns (final_state, rewards (T, N) or None, dones (T, N) or None)."""
        return self._launch_many(_rl.lib().pendulum_coop_step_many, (self.k,), state, actions, rewards=rewards,
                                 dones=dones)
