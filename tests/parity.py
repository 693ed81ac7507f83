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
