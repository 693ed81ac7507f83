"""Generations-to-solve of the ES reference over 10 seeds, for the distribution check in
tests/test_gpu_es_seeds.py.

The reference's es.train evaluates the mean policy through MLX even with its numpy backend
(es.py:308-322), so it cannot run here. This script runs the oracle's train loop
(oracle/es.py). Its generation reproduces the reference's numpy generation exactly; that is
pinned by tests/test_oracle_golden.py against es.npz. Its evaluation restates es.py:308-322 in
numpy. For seeds 0..9 and two tasks the script records whether the task was solved, the number
of generations, the env steps taken and the final score, and writes es_solve.npz next to this
file. Run from the repository root: python tests/golden/make_es_solve.py
"""

import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle import es as oes  # noqa: E402

# task -> (population, max generations); sigma 0.1, lr 0.1, horizon 500 as es.py's Config
RUNS = {"cartpole": (256, 100), "acrobot": (1024, 40)}
SEEDS = range(10)


def main():
    out = {}
    for task, (pop, max_gen) in RUNS.items():
        rows = []
        for seed in SEEDS:
            t0 = time.time()
            cfg = oes.Config(task=task, pop=pop, max_generations=max_gen, time_budget=1e9)
            r = oes.train(cfg, seed)
            rows.append((r.solved, r.generations, r.env_steps, r.score))
            print(f"{task} P={pop} seed={seed}: solved={r.solved} generations={r.generations} "
                  f"score={r.score:.1f} ({time.time() - t0:.0f} s)", flush=True)
        arr = np.array(rows, dtype=np.float64)
        out[f"{task}_solved"] = arr[:, 0].astype(bool)
        out[f"{task}_generations"] = arr[:, 1].astype(np.int64)
        out[f"{task}_env_steps"] = arr[:, 2].astype(np.int64)
        out[f"{task}_score"] = arr[:, 3]
        out[f"{task}_config"] = np.array([pop, max_gen], dtype=np.int64)
    np.savez_compressed(Path(__file__).resolve().parent / "es_solve.npz", **out)


if __name__ == "__main__":
    main()
