"""Planar legged bodies with C hard ground contacts, stepped by an sm_100a CUDA kernel.

Drop-in for the reference module of the same name (legged_metal.py:1-185):
`Legged(c, iters=8)` with `.step(state, action, assist=None)`, `.reseed(seed)`,
`.reset(n)`, `.stand`, `.n_actions`. State (2(3+C), N) float32: q = (x, y, phi,
psi_1..psi_C) then q_dot. The action is an index in [0, 3^C): leg k's torque is
((a // 3^k) % 3 - 1) * 2. One thread per environment runs four substeps of 0.01:
the (3+C) x (3+C) mass matrix and its Cholesky factor, 2C + 1 solves, the
Delassus blocks, and `iters` sweeps of block projected Gauss-Seidel over the
feet, each foot's exact stick/slide/separate impulse given the others. Then the
fall test (torso below 0.6 or tilted past 1 rad), the reset to the standing
pose plus uniform +-0.05 on every row, and the reward x_dot + 1.
`assist` (a float or a one-element CUDA tensor) is the stiffness of the
curriculum's torso-upright spring-damper. Built for C = 1..4.
"""

import numpy as np
import torch

import rlenv_lib as _rl

M_T, I_T, M_F, L = 1.0, 0.1, 0.2, 1.0
GRAVITY = 9.8
TORQUE = 2.0
MU = 0.7
H, SUBSTEPS = 0.01, 4
BAUMGARTE = 0.2
FALL_HEIGHT, FALL_ANGLE = 0.6, 1.0
RESET_BOUND = 0.05
ITERS = 8


def leg_angles(c):
    """Resting leg angles, 0.5 rad apart and symmetric about the vertical."""
    return (2.0 * np.arange(c) - (c - 1)) * 0.25


def _at_rest(angles):
    """State (2(3+C),) at rest with the given leg angles, the hip as high as the innermost leg."""
    angles = np.asarray(angles, dtype=np.float64)
    q = np.zeros(3 + angles.size)
    q[1] = L * np.cos(np.min(np.abs(angles)))
    q[3:] = angles
    return np.pad(q, (0, q.size)).astype(np.float32)


def stand_pose(c):
    """The reset pose (2(3+C),): hip at the height of the innermost feet, at rest."""
    return _at_rest(leg_angles(c))


def static_pose(c):
    """A true equilibrium with every foot on the floor, legs at +-0.25 rad (C even)."""
    return _at_rest(np.where(np.arange(c) < c // 2, -0.25, 0.25) if c > 1 else [0.0])


class _OnDevice:
    """A small constant array uploaded once per device."""

    def __init__(self, host):
        self.host = np.ascontiguousarray(host, dtype=np.float32)
        self._dev = {}

    def on(self, dev):
        t = self._dev.get(dev)
        if t is None:
            t = self._dev[dev] = torch.from_numpy(self.host).to(dev)
        return t


class Legged(_rl.StepBody):
    def __init__(self, c, iters=ITERS):
        if c not in (1, 2, 3, 4):
            raise ValueError("legged bodies are built for c in 1..4")
        super().__init__()
        self.c, self.iters = c, int(iters)
        self.rows = 2 * (3 + c)
        self.n_actions = 3**c
        self._stand = _OnDevice(stand_pose(c))

    @property
    def stand(self):
        return self._stand.on(_rl.device())

    def reset(self, n):
        return _rl.reset_uniform(self.rows, n, RESET_BOUND, center=self._stand.host)

    @staticmethod
    def _assist(assist):
        """(value, device tensor or None) of the torso-assist stiffness argument."""
        if isinstance(assist, torch.Tensor) and assist.device.type == "cuda":
            return 0.0, assist.reshape(-1)[:1].float().contiguous()
        return (0.0 if assist is None else _rl.float_scalar(assist)), None

    def step(self, state, action, assist=None, impulses=False):
        """(next_state, reward, done), and with impulses=True a fourth output: the (2c, n)
        contact impulses of the step, row 2k the tangential and row 2k + 1 the normal impulse
        of foot k, each summed over the four substeps (the lt, ln of legged_np.py:89-96)."""
        state = _rl.as_state(state, self.rows)
        stand = self._stand.on(state.device)
        a_val, a_ptr = self._assist(assist)
        imp = torch.empty((2 * self.c, state.shape[1]), dtype=torch.float32, device=state.device) if impulses else None
        out = self._launch(_rl.lib().legged_step, (self.c, self.iters), state, action,
                           tail=(stand.data_ptr(), a_val, _rl.ptr(a_ptr)), outs=(_rl.ptr(imp),))
        return out + (imp,) if impulses else out

    def step_many(self, state, actions, assist=None, impulses=False, rewards=True, dones=True):
        """T steps in one launch for actions (T, N): equal bit for bit to T `step` calls (the same
        seeds are drawn). Returns (final_state, rewards (T, N) or None, dones (T, N) or None), and
        with impulses=True a fourth output (T, 2c, N): each step's impulses as `step` returns them."""
        state = _rl.as_state(state, self.rows)
        stand = self._stand.on(state.device)
        a_val, a_ptr = self._assist(assist)
        steps = len(actions)
        imp = (torch.empty((steps, 2 * self.c, state.shape[1]), dtype=torch.float32, device=state.device),) \
            if impulses else ()
        out = self._launch_many(_rl.lib().legged_step_many, (self.c, self.iters), state, actions,
                                tail=(stand.data_ptr(), a_val, _rl.ptr(a_ptr)), rewards=rewards, dones=dones,
                                extra=imp or (None,))
        return out if impulses else out[:3]
