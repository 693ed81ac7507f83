"""ES over 10 seeds against the reference's distribution (the north star's "ES
generations-to-solve distributions consistent over 10 seeds").

The reference side is tests/golden/es_solve.npz: the oracle's train loop for seeds 0..9, whose
generation reproduces the reference's numpy generation exactly (made by
tests/golden/make_es_solve.py). The GPU run draws its noise from a counter-based stream, so
individual seeds differ; the distributions must agree.
- CartPole and Acrobot at es.py's defaults (lr 0.1) and at BASELINE's settings (P = 4,096,
  lr 0.03): generations to solve.
- legged4 (P = 256, horizon 100, lr 0.03): the population's mean training fitness over the last
  five of 30 generations, since the oracle cannot train it to its threshold in reasonable time."""

import numpy as np
import pytest

from conftest import golden
from parity import record

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("key", ["cartpole", "acrobot", "cartpole_p4096", "acrobot_p4096"])
def test_generations_to_solve_match_the_reference_distribution(cuda, key):
    import es
    from scipy.stats import mannwhitneyu

    g = golden("es_solve")
    task = key.split("_")[0]
    pop, max_gen = (int(x) for x in g[f"{key}_config"])
    lr = float(g[f"{key}_lr"]) if f"{key}_lr" in g else 0.1
    ref_solved, ref_gens = g[f"{key}_solved"], g[f"{key}_generations"]
    results = [es.train(es.Config(task=task, pop=pop, lr=lr, max_generations=max_gen, time_budget=1e9), "metal", seed)
               for seed in range(10)]
    gens = np.array([r.generations for r in results])
    solved = np.array([r.solved for r in results])
    p = float(mannwhitneyu(gens, ref_gens).pvalue)
    record(f"es_{key}_10_seeds", population=pop, lr=lr, gpu_generations=gens.tolist(),
           reference_generations=ref_gens.tolist(), gpu_solved=int(solved.sum()),
           reference_solved=int(ref_solved.sum()), mann_whitney_p=p)
    assert solved.sum() >= ref_solved.sum() - 1, (solved, ref_solved)
    # a two-sided rank-sum test at the 1% level, and medians within a factor of two
    assert p > 0.01, (gens, ref_gens, p)
    assert 0.5 <= np.median(gens) / np.median(ref_gens) <= 2.0, (gens, ref_gens)


def test_legged4_learning_curves_match_the_reference_distribution(cuda):
    import es
    from scipy.stats import mannwhitneyu

    g = golden("es_solve")
    pop, horizon, gens = (int(x) for x in g["legged4_config"])
    lr = float(g["legged4_lr"])
    ref = g["legged4_curves"]
    task = es.TASKS["legged4"]
    cfg = es.Config(task="legged4", pop=pop, horizon=horizon, sigma=0.1, lr=lr)
    curves = []
    for seed in range(10):
        backend = es.MetalBackend(task, seed)
        theta = backend.normal((es.n_params(task.hidden, task),)) * 0.1
        curve = []
        for gen in range(1, gens + 1):
            theta, fit, _ = es.generation(backend, theta, cfg, task.hidden, gen)
            curve.append(float(fit.mean().item()))
        curves.append(curve)
    curves = np.array(curves)
    late, ref_late = curves[:, -5:].mean(axis=1), ref[:, -5:].mean(axis=1)
    p = float(mannwhitneyu(late, ref_late).pvalue)
    record("es_legged4_curves_10_seeds", population=pop, horizon=horizon, generations=gens, lr=lr,
           gpu_first=curves[:, 0].round(2).tolist(), reference_first=ref[:, 0].round(2).tolist(),
           gpu_last5=late.round(2).tolist(), reference_last5=ref_late.round(2).tolist(), mann_whitney_p=p)
    # both sides learn: the last generations beat the first on most seeds
    assert (late > curves[:, :3].mean(axis=1)).sum() >= 7 and (ref_late > ref[:, :3].mean(axis=1)).sum() >= 7
    assert p > 0.01, (late, ref_late, p)
    assert 0.75 <= np.median(late) / np.median(ref_late) <= 1.33, (late, ref_late)
