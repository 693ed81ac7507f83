"""Batched K-link pendulum, mass-matrix form, one thread per environment on sm_100a.

Drop-in for the reference module of the same name (pendulum_metal.py:1-131):
`Pendulum(k, pairwise_trig=False)` with `.step(state, action)`, `.reseed(seed)`
and `.reset(n)`. State (2K, N) float32: K absolute angles, then K angular
velocities. One launch per call builds each environment's K x K mass matrix,
solves it by Cholesky at each of the four RK4 stages, wraps and clips, tests
termination (tip above K/2), resets terminated columns from the hash stream
and writes the reward (-1, 0 on termination). `pairwise_trig` evaluates every
angle-difference cosine and sine directly (the reference's v9 variant).
Built for K = 1..16; other K raise ValueError.
"""

import rlenv_lib as _rl

GRAVITY = 9.8
DT = 0.02
TORQUE = 1.0
MAX_VEL = 10 * 3.141592653589793
RESET_BOUND = 0.1


class Pendulum(_rl.StepBody):
    def __init__(self, k, pairwise_trig=False):
        super().__init__()
        self.k = k
        self.rows = 2 * k
        self.pairwise_trig = bool(pairwise_trig)

    def reset(self, n):
        """Angles and velocities uniform in +-RESET_BOUND."""
        return _rl.reset_uniform(self.rows, n, RESET_BOUND)

    def step(self, state, action):
        return self._launch(_rl.lib().pendulum_mm_step, (self.k, int(self.pairwise_trig)), state, action)

    def step_many(self, state, actions, rewards=True, dones=True):
        """T steps in one launch for actions (T, N): equal bit for bit to T `step` calls (the same
        seeds are drawn). Returns (final_state, rewards (T, N) or None, dones (T, N) or None)."""
        return self._launch_many(_rl.lib().pendulum_mm_step_many, (self.k, int(self.pairwise_trig)), state, actions,
                                 rewards=rewards, dones=dones)
