"""Step semantics of the reference's Metal kernels, in numpy.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

A reference step kernel computes the numpy physics, tests termination on the
stepped state, and replaces a terminated column with a reset drawn from its
in-kernel hash stream, not from a numpy Generator (cartpole_metal.py:84-96,
pendulum_metal.py:84-92, hopper_metal.py:100-107, legged_metal.py:145-155).
These functions return exactly that: (next_state, reward, done, stepped) with
`stepped` the post-physics state before any reset, so a test can compare live
columns to tolerance and reset columns bit for bit.
"""

import numpy as np

from oracle import classic, legged, pendulum, rng


def _select(done, fresh, stepped):
    return np.where(done[None, :], fresh, np.asarray(stepped, dtype=np.float32)).astype(np.float32)


def cartpole_step(state, action, seed, index_offset=0):
    stepped = classic.cartpole_physics(state, action)
    done = classic.cartpole_terminated(stepped)
    fresh = rng.reset_rows(seed, stepped.shape[1], 4, classic.CP_RESET_BOUND, index_offset,
                           offsets=rng.CLASSIC_ROW_OFFSETS)
    return _select(done, fresh, stepped), classic.cartpole_reward(done), done, stepped


def acrobot_step(state, action, seed, index_offset=0):
    stepped = classic.acrobot_physics(state, action)
    done = classic.acrobot_terminated(stepped)
    fresh = rng.reset_rows(seed, stepped.shape[1], 4, classic.AC_RESET_BOUND, index_offset,
                           offsets=rng.CLASSIC_ROW_OFFSETS)
    return _select(done, fresh, stepped), classic.acrobot_reward(done), done, stepped


def pendulum_step(state, action, seed, k, form="mass_matrix", index_offset=0):
    """form: "mass_matrix" (pendulum_metal, pendulum_metal_coop) or "aba" (pendulum_aba_metal)."""
    stepped = pendulum.aba_physics(state, action, k) if form == "aba" else pendulum.mm_physics(state, action, k)
    done = pendulum.terminated(stepped, k)
    fresh = rng.reset_rows(seed, stepped.shape[1], 2 * k, pendulum.PD_RESET_BOUND, index_offset)
    return _select(done, fresh, stepped), pendulum.reward(done), done, stepped


def legged_step(state, action, seed, c, iters=legged.LG_ITERS, assist=0.0, index_offset=0, stand=None):
    """The legged kernel; with c = 1 and iters = 1 it is the hopper kernel."""
    stand = legged.stand_pose(c) if stand is None else np.asarray(stand, dtype=np.float32)
    stepped = legged.physics(state, action, c, iters, assist)
    done = legged.terminated(stepped)
    fresh = rng.reset_rows(seed, stepped.shape[1], 2 * (3 + c), legged.LG_RESET_BOUND, index_offset, center=stand)
    return _select(done, fresh, stepped), legged.reward(stepped, done, c), done, stepped


def hopper_step(state, action, seed, index_offset=0):
    return legged_step(state, action, seed, 1, 1, 0.0, index_offset, stand=legged.HOPPER_STAND)
