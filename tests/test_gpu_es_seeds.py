"""ES over 10 seeds against the reference's distribution (the north star's "ES
generations-to-solve distributions consistent over 10 seeds").

The reference side is tests/golden/es_solve.npz: the oracle's train loop for seeds 0..9, whose
generation reproduces the reference's numpy generation exactly (made by
tests/golden/make_es_solve.py). The GPU run draws its noise from a counter-based stream, so
individual seeds differ; the distributions must agree.
- CartPole and Acrobot at es.py's defaults (lr 0.1) and at BASELINE's settings (P = 4,096,
  lr 0.03): generations to solve.
- legged4 (P = 256, horizon 100, lr 0.03): the learning curve of the population's mean training
  fitness over 30 generations (its mean, and the generations it takes to reach 60), since the
  oracle cannot train legged4 to its threshold in reasonable time."""

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

    def to_60(c):
        return np.array([int(np.argmax(r >= 60)) + 1 if (r >= 60).any() else gens + 1 for r in c])

    # the area under the learning curve (the late generations sit near the horizon's cap of about
    # 100 on both sides, so they would not tell distributions apart) and generations to reach 60
    area, ref_area = curves.mean(axis=1), ref.mean(axis=1)
    p = float(mannwhitneyu(area, ref_area).pvalue)
    p60 = float(mannwhitneyu(to_60(curves), to_60(ref)).pvalue)
    record("es_legged4_curves_10_seeds", population=pop, horizon=horizon, generations=gens, lr=lr,
           gpu_area=area.round(2).tolist(), reference_area=ref_area.round(2).tolist(),
           gpu_generations_to_60=to_60(curves).tolist(), reference_generations_to_60=to_60(ref).tolist(),
           mann_whitney_p_area=p, mann_whitney_p_to_60=p60)
    assert (to_60(curves) <= gens).sum() >= 9 and (to_60(ref) <= gens).sum() >= 9, "both sides learn"
    assert p > 0.01 and p60 > 0.01, (area, ref_area, p, p60)
    assert 0.8 <= np.median(area) / np.median(ref_area) <= 1.25, (area, ref_area)
