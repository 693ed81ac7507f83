"""Generations-to-solve of the ES reference over 10 seeds, for the distribution check in
tests/test_gpu_es_seeds.py.

The reference's es.train evaluates the mean policy through MLX even with its numpy backend
(es.py:308-322), so it cannot run here. This script runs the oracle's train loop
(oracle/es.py). Its generation reproduces the reference's numpy generation exactly; that is
pinned by tests/test_oracle_golden.py against es.npz. Its evaluation restates es.py:308-322 in
numpy. For seeds 0..9 the script records whether the task was solved, the number of
generations, the env steps taken and the final score, for CartPole and Acrobot at es.py's
defaults (lr 0.1, small populations) and at BASELINE's settings (P = 4,096, lr 0.03).

legged4 cannot be trained to its threshold here: one numpy evaluation alone steps 2,048
bodies for 500 steps. For it the script records the learning curve instead: the population's
mean training fitness in each of 30 generations at P = 256, horizon 100, sigma 0.1, lr 0.03,
for seeds 0..9. Everything goes to es_solve.npz next to this file. Run from the repository
root: python tests/golden/make_es_solve.py
"""

import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle import es as oes  # noqa: E402

# key -> (task, population, max generations, lr); sigma 0.1 and horizon 500 as es.py's Config
RUNS = {"cartpole": ("cartpole", 256, 100, 0.1), "acrobot": ("acrobot", 1024, 40, 0.1),
        "cartpole_p4096": ("cartpole", 4096, 120, 0.03), "acrobot_p4096": ("acrobot", 4096, 60, 0.03)}
SEEDS = range(10)
# legged4 learning curves: population, horizon, generations, lr
LEGGED = ("legged4", 256, 100, 30, 0.03)


def legged_curves():
    task_name, pop, horizon, gens, lr = LEGGED
    task = oes.TASKS[task_name]
    cfg = oes.Config(task=task_name, pop=pop, horizon=horizon, sigma=0.1, lr=lr)
    curves = []
    for seed in SEEDS:
        t0 = time.time()
        rng = np.random.default_rng(seed)
        theta = rng.normal(size=(oes.n_params(task.hidden, task),)).astype(np.float32) * 0.1
        curve = []
        for gen in range(1, gens + 1):
            theta, fit, _ = oes.generation(task, theta, cfg, task.hidden, rng, gen)
            curve.append(float(np.mean(fit)))
        curves.append(curve)
        print(f"{task_name} P={pop} seed={seed}: fitness {curve[0]:.1f} -> {curve[-1]:.1f} ({time.time() - t0:.0f} s)",
              flush=True)
    return np.array(curves, dtype=np.float64)


def main():
    out = {}
    for key, (task, pop, max_gen, lr) in RUNS.items():
        rows = []
        for seed in SEEDS:
            t0 = time.time()
            cfg = oes.Config(task=task, pop=pop, lr=lr, max_generations=max_gen, time_budget=1e9)
            r = oes.train(cfg, seed)
            rows.append((r.solved, r.generations, r.env_steps, r.score))
            print(f"{key} P={pop} lr={lr} seed={seed}: solved={r.solved} generations={r.generations} "
                  f"score={r.score:.1f} ({time.time() - t0:.0f} s)", flush=True)
        arr = np.array(rows, dtype=np.float64)
        out[f"{key}_solved"] = arr[:, 0].astype(bool)
        out[f"{key}_generations"] = arr[:, 1].astype(np.int64)
        out[f"{key}_env_steps"] = arr[:, 2].astype(np.int64)
        out[f"{key}_score"] = arr[:, 3]
        out[f"{key}_config"] = np.array([pop, max_gen], dtype=np.int64)
        out[f"{key}_lr"] = np.float64(lr)
    out["legged4_curves"] = legged_curves()
    out["legged4_config"] = np.array(LEGGED[1:4], dtype=np.int64)
    out["legged4_lr"] = np.float64(LEGGED[4])
    np.savez_compressed(Path(__file__).resolve().parent / "es_solve.npz", **out)


if __name__ == "__main__":
    main()
