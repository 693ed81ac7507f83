"""Helpers for the GPU parity tests: compare one step kernel's outputs with the reference's
golden physics and the oracle's kernel semantics, and record the measured error."""

import json
import os

import numpy as np


def to_np(t):
    return t.detach().cpu().numpy()


def record(name, **fields):
    """Append measured parity figures to $RLENV_PARITY_LOG (one JSON line per check)."""
    path = os.environ.get("RLENV_PARITY_LOG")
    if path:
        with open(path, "a") as f:
            f.write(json.dumps({"check": name, **{k: (float(v) if isinstance(v, (np.floating, float)) else v)
                                                  for k, v in fields.items()}}) + "\n")


def max_rel(a, b, atol):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float((np.abs(a - b) / (np.abs(b) + atol)).max()) if a.size else 0.0


def check_step(name, out, ref_stepped, ref_done, oracle_next, rtol, atol, ref_reward=None):
    """out = (next_state, reward, done) from the GPU. Live columns (ref_done False) must match
    ref_stepped within rtol/atol; done must equal ref_done exactly; reset columns must equal the
    oracle's hash-stream resets bit for bit."""
    nxt, reward, done = (to_np(t) for t in out)
    assert nxt.dtype == np.float32 and reward.dtype == np.float32 and done.dtype == np.bool_
    flips = int((done != ref_done).sum())
    live = ~ref_done
    err = np.abs(nxt[:, live].astype(np.float64) - np.asarray(ref_stepped, np.float64)[:, live])
    record(name, n=int(done.size), done_flips=flips, live=int(live.sum()),
           max_abs=float(err.max()) if err.size else 0.0,
           max_rel=max_rel(nxt[:, live], np.asarray(ref_stepped)[:, live], atol))
    assert flips == 0, f"{name}: {flips} done flags differ"
    np.testing.assert_allclose(nxt[:, live], np.asarray(ref_stepped)[:, live], rtol=rtol, atol=atol, err_msg=name)
    np.testing.assert_array_equal(nxt[:, ~live], oracle_next[:, ~live], err_msg=f"{name}: reset columns")
    if ref_reward is not None:
        np.testing.assert_allclose(reward, ref_reward, rtol=rtol, atol=atol, err_msg=f"{name}: reward")


# The legged rollout cases pinned at the reference's horizon (test_es.py:46-104): (legs, alive
# bonus, fall penalty, height gate, assist). Plain reward for both bodies; the shaped and
# assisted variants of the reference's legged2 tasks.
LEGGED_ROLLOUT_CASES = [(2, 1.0, 0.0, 0.0, 0.0), (2, 0.1, 20.0, 0.0, 0.0), (2, 0.0, 0.0, 0.85, 0.0),
                        (2, 0.0, 0.0, 0.0, 20.0), (4, 1.0, 0.0, 0.0, 0.0), (4, 0.1, 20.0, 0.0, 0.0)]
LEGGED_ROLLOUT_P, LEGGED_ROLLOUT_HORIZON, LEGGED_ROLLOUT_HIDDEN = 1024, 200, 16


def legged_rollout_inputs(index):
    """(initial states (2(3+C), P), parameter rows (P, D)) of case `index`: the reset pose plus
    uniform +-0.05 on every row, and normal parameters scaled by 0.3 (the reference test's
    scale), from numpy's default generator seeded with 100 + index."""
    from oracle import legged

    c = LEGGED_ROLLOUT_CASES[index][0]
    h, p = LEGGED_ROLLOUT_HIDDEN, LEGGED_ROLLOUT_P
    rng = np.random.default_rng(100 + index)
    state = (legged.stand_pose(c)[:, None] + rng.uniform(-0.05, 0.05, (2 * (3 + c), p))).astype(np.float32)
    d = (5 + 2 * c) * h + h + h * 3 * c + 3 * c
    theta = (rng.normal(size=(p, d)) * 0.3).astype(np.float32)
    return state, theta
