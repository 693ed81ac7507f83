"""The planar hopper with one hard contact, stepped by an sm_100a CUDA kernel.

Drop-in for the reference module of the same name (hopper_metal.py:1-138):
`Hopper(branchy=False)` with `.step(state, action)`, `.reseed(seed)`,
`.reset(n)`. State (8, N): q = (x, y, phi, psi) then q_dot; action in {0, 1, 2}
is a hip torque of (a - 1) * 2. Four substeps of 0.01 with the exact
single-contact impulse (stick, slide or separate). The hopper is the legged
body with one leg and one contact sweep. `branchy` skips the contact solve of
airborne environments with a branch instead of computing it and selecting zero.
"""

import numpy as np

import rlenv_lib as _rl
from legged_metal import FALL_ANGLE, FALL_HEIGHT, L, RESET_BOUND, _OnDevice  # noqa: F401

STAND = np.zeros(8, dtype=np.float32)
STAND[1] = L  # upright at rest, the hip one leg length above the floor


class Hopper(_rl.StepBody):
    rows = 8

    def __init__(self, branchy=False):
        super().__init__()
        self.branchy = bool(branchy)
        self._stand = _OnDevice(STAND)

    def reset(self, n):
        return _rl.reset_uniform(self.rows, n, RESET_BOUND, center=STAND)

    def step(self, state, action):
        state = _rl.as_state(state, self.rows)
        stand = self._stand.on(state.device)
        return self._launch(_rl.lib().hopper_step, (int(self.branchy),), state, action, tail=(stand.data_ptr(),))

    def step_many(self, state, actions, rewards=True, dones=True):
        """T steps in one launch for actions (T, N): equal bit for bit to T `step` calls (the same
        seeds are drawn). Returns (final_state, rewards (T, N) or None, dones (T, N) or None)."""
        state = _rl.as_state(state, self.rows)
        stand = self._stand.on(state.device)
        return self._launch_many(_rl.lib().hopper_step_many, (int(self.branchy),), state, actions,
                                 tail=(stand.data_ptr(),), rewards=rewards, dones=dones)
