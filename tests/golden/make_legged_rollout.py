"""Oracle outputs of the legged ES rollout at the reference's horizon, for
tests/test_gpu_rollouts.py.

For every case of parity.LEGGED_ROLLOUT_CASES (1,024 members, horizon 200, inputs from
parity.legged_rollout_inputs) the script runs oracle.rollout.legged_rollout twice: in float32
throughout (the arithmetic of the reference's Metal kernel and its MLX step loop) and with the
reference numpy's float64 promotion. It stores both (fitness, steps) and writes
legged_rollout.npz next to this file. Run from the repository root:
python tests/golden/make_legged_rollout.py
"""

import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))

import parity  # noqa: E402
from oracle import rollout  # noqa: E402


def run(index, f32, p=None):
    c, alive, fall, gate, assist = parity.LEGGED_ROLLOUT_CASES[index]
    state, theta = parity.legged_rollout_inputs(index)
    if p is not None:
        state, theta = state[:, :p], theta[:p]
    return rollout.legged_rollout(state, theta, parity.LEGGED_ROLLOUT_HIDDEN, parity.LEGGED_ROLLOUT_HORIZON, c,
                                  alive, fall, gate, assist, f32=f32)


def main():
    out = {}
    for i in range(len(parity.LEGGED_ROLLOUT_CASES)):
        t0 = time.time()
        for f32 in (True, False):
            fit, steps = run(i, f32)
            tag = "f32" if f32 else "f64"
            out[f"case{i}_{tag}_fitness"] = fit
            out[f"case{i}_{tag}_steps"] = steps
        print(f"case {i} {parity.LEGGED_ROLLOUT_CASES[i]}: {time.time() - t0:.0f} s", flush=True)
    np.savez_compressed(Path(__file__).resolve().parent / "legged_rollout.npz", **out)


if __name__ == "__main__":
    main()
