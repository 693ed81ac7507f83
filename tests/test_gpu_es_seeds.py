"""ES generations-to-solve over 10 seeds against the reference's distribution (the north star's
"ES generations-to-solve distributions consistent over 10 seeds").

The reference side is tests/golden/es_solve.npz: the oracle's train loop for seeds 0..9, whose
generation reproduces the reference's numpy generation exactly (made by
tests/golden/make_es_solve.py). The GPU run draws its noise from a counter-based stream, so
individual seeds differ; the distributions must agree."""

import numpy as np
import pytest

from conftest import golden
from parity import record

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("task", ["cartpole", "acrobot"])
def test_generations_to_solve_match_the_reference_distribution(cuda, task):
    import es
    from scipy.stats import mannwhitneyu

    g = golden("es_solve")
    pop, max_gen = (int(x) for x in g[f"{task}_config"])
    ref_solved, ref_gens = g[f"{task}_solved"], g[f"{task}_generations"]
    results = [es.train(es.Config(task=task, pop=pop, max_generations=max_gen, time_budget=1e9), "metal", seed)
               for seed in range(10)]
    gens = np.array([r.generations for r in results])
    solved = np.array([r.solved for r in results])
    p = float(mannwhitneyu(gens, ref_gens).pvalue)
    record(f"es_{task}_10_seeds", gpu_generations=gens.tolist(), reference_generations=ref_gens.tolist(),
           gpu_solved=int(solved.sum()), reference_solved=int(ref_solved.sum()), mann_whitney_p=p)
    assert solved.sum() >= ref_solved.sum() - 1, (solved, ref_solved)
    # a two-sided rank-sum test at the 1% level, and medians within a factor of two
    assert p > 0.01, (gens, ref_gens, p)
    assert 0.5 <= np.median(gens) / np.median(ref_gens) <= 2.0, (gens, ref_gens)
