"""ES generation kernels and the GPU es.py on a B200 (mirrors test_es.py of the reference)."""

import numpy as np
import pytest
import torch

from oracle import es as oes
from oracle import rng
from parity import record, to_np

pytestmark = pytest.mark.gpu


def test_noise_matches_oracle(cuda):
    import rlenv_lib as rl

    rows, d = 300, 226
    out = torch.empty((rows, d), device=cuda)
    rl.check(rl.lib().es_noise(out.data_ptr(), rows, d, 12345, 7, 100, rl.stream_ptr()))
    want = rng.noise(12345, 7, np.arange(100, 100 + rows), d)
    got = to_np(out)
    record("es_noise", max_abs=float(np.abs(got - want).max()))
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=2e-6)
    assert abs(got.mean()) < 0.02 and abs(got.std() - 1) < 0.02


def test_perturb_is_antithetic_and_matches_noise(cuda):
    import rlenv_lib as rl

    pairs, d, sigma = 64, 50, 0.1
    theta = torch.from_numpy(np.random.default_rng(0).normal(size=d).astype(np.float32)).to(cuda)
    pop = torch.empty((2 * pairs, d), device=cuda)
    rl.check(rl.lib().es_perturb(theta.data_ptr(), d, sigma, 9, 3, pairs, 0, 2 * pairs, pop.data_ptr(), rl.stream_ptr()))
    half = torch.empty((pairs, d), device=cuda)
    rl.check(rl.lib().es_noise(half.data_ptr(), pairs, d, 9, 3, 0, rl.stream_ptr()))
    th, p, h = to_np(theta), to_np(pop), to_np(half)
    np.testing.assert_array_equal(p[:pairs], (th + (np.float32(sigma) * h)).astype(np.float32))
    np.testing.assert_array_equal(p[pairs:], (th + (np.float32(sigma) * -h)).astype(np.float32))
    shard = torch.empty((40, d), device=cuda)
    rl.check(rl.lib().es_perturb(theta.data_ptr(), d, sigma, 9, 3, pairs, 50, 40, shard.data_ptr(), rl.stream_ptr()))
    np.testing.assert_array_equal(to_np(shard), p[50:90])


@pytest.mark.parametrize("p", [2, 3, 1000, 4096, 16384])
def test_centered_ranks_stable(cuda, p):
    import es

    r = np.random.default_rng(p)
    vals = r.integers(0, max(2, p // 8), p).astype(np.float32)  # many ties
    got = to_np(es.centered_ranks(torch, torch.from_numpy(vals).to(cuda)))
    np.testing.assert_allclose(got, oes.centered_ranks(vals, stable=True), atol=1e-7)
    known = to_np(es.centered_ranks(torch, torch.tensor([3.0, 1.0, 2.0, 10.0], device=cuda)))
    np.testing.assert_allclose(known, [1 / 6, -0.5, -1 / 6, 0.5], atol=1e-6)


def _ranks_both(cuda, vals):
    """The counting kernel's and the sort kernel's ranks of the same fitness."""
    import es

    t = torch.from_numpy(vals).to(cuda)
    return (to_np(es.centered_ranks(torch, t, sorted_kernel=False)),
            to_np(es.centered_ranks(torch, t, sorted_kernel=True)))


@pytest.mark.parametrize("p", [2, 3, 1000, 4095, 4096, 4097, 8192, 10000, 65536, 100003])
def test_sorted_ranks_equal_counting_and_oracle(cuda, p):
    """One tile, one tile plus one, whole and ragged merge passes: the same bits everywhere."""
    vals = np.random.default_rng(p).integers(0, max(2, p // 8), p).astype(np.float32)  # many ties
    count, srt = _ranks_both(cuda, vals)
    np.testing.assert_array_equal(srt, count)
    np.testing.assert_array_equal(srt, oes.centered_ranks(vals, stable=True))


def test_ranks_order_special_values_as_numpy(cuda):
    """NaN after every number (NaNs tied), -0 equal to +0, infinities at the ends; across tiles."""
    base = [np.nan, 1.0, -0.0, 0.0, np.inf, -np.inf, np.nan, 0.0, -1.0, 1.0, -0.0, 3.0e38, -3.0e38, 1e-45]
    vals = np.array(base * 700, dtype=np.float32)
    count, srt = _ranks_both(cuda, vals)
    np.testing.assert_array_equal(srt, count)
    np.testing.assert_array_equal(srt, oes.centered_ranks(vals, stable=True))


def test_sorted_ranks_at_the_references_largest_population(cuda):
    """P = 262,144 (the reference's own largest ES runs): a permutation, equal to the counting
    kernel and to numpy's stable double argsort."""
    p = 262_144
    vals = np.random.default_rng(7).normal(size=p).astype(np.float32)
    vals[::97] = np.round(vals[::97])  # some ties among many distinct values
    count, srt = _ranks_both(cuda, vals)
    np.testing.assert_array_equal(srt, count)
    np.testing.assert_array_equal(srt, oes.centered_ranks(vals, stable=True))
    pos = np.rint((srt.astype(np.float64) + 0.5) * (p - 1)).astype(np.int64)
    assert np.array_equal(np.sort(pos), np.arange(p))


def test_update_matches_float64(cuda):
    import rlenv_lib as rl

    pairs, d, lr, sigma = 2048, 428, 0.03, 0.1
    theta = torch.from_numpy(np.random.default_rng(1).normal(size=d).astype(np.float32) * 0.1).to(cuda)
    ranks = torch.from_numpy(oes.centered_ranks(np.random.default_rng(2).normal(size=2 * pairs).astype(np.float32))).to(cuda)
    out = torch.empty_like(theta)
    rl.check(rl.lib().es_update(theta.data_ptr(), ranks.data_ptr(), d, pairs, lr, sigma, 5, 11, out.data_ptr(), rl.stream_ptr()))
    half = torch.empty((pairs, d), device=cuda)
    rl.check(rl.lib().es_noise(half.data_ptr(), pairs, d, 5, 11, 0, rl.stream_ptr()))
    h = to_np(half).astype(np.float64)
    rk = to_np(ranks).astype(np.float64)
    eps = np.concatenate([h, -h])
    want = to_np(theta) + lr * (rk[:, None] * eps).sum(0) / (2 * pairs * sigma)
    got = to_np(out)
    record("es_update", max_abs=float(np.abs(got - want).max()))
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-6)
    # fixed summation order: the same bits every call
    out2 = torch.empty_like(theta)
    rl.check(rl.lib().es_update(theta.data_ptr(), ranks.data_ptr(), d, pairs, lr, sigma, 5, 11, out2.data_ptr(), rl.stream_ptr()))
    assert torch.equal(out, out2)


def test_generation_uses_antithetic_pairs_and_moves_theta(cuda):
    import es

    pop, horizon, width = 8, 5, 4
    backend = es.MetalBackend(es.TASKS["cartpole"], 0)
    theta = torch.zeros(es.n_params(width, es.TASKS["cartpole"]), device=cuda)
    new, fit, steps = es.generation(backend, theta, es.Config(pop=pop, horizon=horizon), width)
    assert tuple(fit.shape) == (pop,) and steps.max().item() <= horizon
    assert not torch.allclose(new, torch.zeros_like(new))


def test_generation_is_deterministic(cuda):
    import es

    task = es.TASKS["legged2"]
    cfg = es.Config(task="legged2", pop=256, horizon=50)
    outs = []
    for _ in range(2):
        backend = es.MetalBackend(task, 3)
        theta = backend.normal((es.n_params(task.hidden, task),)) * 0.1
        for gen in range(1, 4):
            theta, fit, steps = es.generation(backend, theta, cfg, task.hidden, gen)
        outs.append(theta)
    assert torch.equal(outs[0], outs[1])


@pytest.mark.parametrize("name,scale", [("cartpole", 0.5), ("acrobot", 0.5), ("legged2", 0.3), ("legged2_alive10_fall", 0.3)])
def test_fused_kernel_matches_step_loop(cuda, name, scale):
    """Same population, same initial states: the fused rollout and the step-by-step loop (torch
    policy + CUDA step kernel) agree on reward sum and step count for almost every member."""
    import es

    task = es.TASKS[name]
    pop, horizon = 1024, 200
    theta = torch.from_numpy((np.random.default_rng(0).normal(size=(pop, es.n_params(task.hidden, task))) * scale)
                             .astype(np.float32)).to(cuda)
    backend = es.MLXBackend(task, 0)
    state = backend.reset(pop, gen=5)
    fk, sk = task.rollout(state, theta, task.hidden, horizon)
    fl, sl = es.loop_fitness(backend, es.unflatten(theta, task.hidden, task), horizon, state=state)
    fk, fl, sk, sl = to_np(fk), to_np(fl), to_np(sk), to_np(sl)
    # the reference's criterion (test_es.py): fitness within 1e-3 relative (floor 1) plus 1e-2,
    # and equal step counts, for more than 95% of the members
    fitness_agree = float(np.mean(np.isclose(fk, fl, rtol=0.0, atol=1e-2 + 1e-3 * np.maximum(np.abs(fl), 1.0))))
    steps_agree = float(np.mean(sk == sl))
    record(f"es_kernel_vs_loop_{name}", fitness_agree=fitness_agree, steps_agree=steps_agree)
    assert min(fitness_agree, steps_agree) > 0.95, (fitness_agree, steps_agree)
    if name.startswith("legged"):
        assert 5 < sl.mean() < 200


def test_evaluate_theta_equals_actor_loop(cuda):
    import es

    for name in ("cartpole", "acrobot", "legged2"):
        task = es.TASKS[name]
        theta = torch.from_numpy((np.random.default_rng(4).normal(size=es.n_params(task.hidden, task)) * 0.3)
                                 .astype(np.float32)).to(cuda)
        state = es.MetalBackend(task, 0).reset(512, gen=9)
        fused = es.evaluate_theta(task, theta, task.hidden, n=512, steps=200, state=state)
        actor = es.mean_policy(theta, task.hidden, task)
        # the loop from the same states: reuse evaluate's arithmetic with a fixed initial state
        alive = torch.ones(512, dtype=torch.bool, device=cuda)
        fit = torch.zeros(512, device=cuda)
        s = state
        for _ in range(200):
            s, r, d = task.metal.step(s, task.action(torch, actor(task.obs(torch, s))))
            alive = alive & ~d
            fit = fit + (r - 1.0 + task.eval_bonus) * alive.float()
        assert abs(fused - fit.mean().item()) <= 0.05 * max(1.0, abs(fused)), (name, fused, fit.mean().item())


def test_es_learns_cartpole(cuda):
    import es

    r = es.train(es.Config(pop=256, time_budget=60.0, solved_at=150.0), "metal", seed=0)
    record("es_cartpole_p256", solved=r.solved, generations=r.generations, score=r.score, seconds=r.train_seconds)
    assert r.score >= 150.0, r


def test_es_learns_acrobot(cuda):
    import es

    goal = -250.0  # the reference's learning check for Acrobot at P = 4,096
    result = es.train(es.Config(task="acrobot", pop=4096, time_budget=60.0, solved_at=goal), "metal", seed=0)
    record("es_acrobot_p4096", solved=result.solved, generations=result.generations, score=result.score,
           seconds=result.train_seconds)
    assert result.score >= goal, result


def test_es_biped_learns_to_stay_up(cuda):
    import es

    fitness_by_generation = []

    def keep(*entry):  # (gen, env_steps, seconds, mean training fitness, score)
        fitness_by_generation.append(entry[3])

    es.train(es.Config(task="legged2", pop=1024, time_budget=30.0, max_generations=60), "metal", seed=0, log=keep)
    final = fitness_by_generation[-1]
    record("es_legged2_p1024_60gens", final_fitness=final, generations=len(fitness_by_generation))
    assert final >= 300.0, final  # the biped stands for most of its 500-step episodes


def test_generation_runs_a_backend_written_against_the_reference_interface(cuda):
    """es.generation with a backend that has only the reference's interface (xp, normal,
    rollout, sync; es.py:218-227) follows the reference's generation: eps = [half; -half],
    g = sum_i rank_i eps_i / (P sigma), theta + lr g."""
    import es

    task = es.TASKS["cartpole"]
    p, hidden = 64, 8
    state = task.mlx.reset(p)
    drawn = []

    class Outside:
        xp = torch

        def __init__(self):
            self.g = torch.Generator(device=cuda).manual_seed(5)

        def normal(self, shape):
            drawn.append(torch.randn(shape, device=cuda, generator=self.g))
            return drawn[-1]

        def rollout(self, theta_pop, hidden, horizon, assist=0.0, start_velocity=0.0):
            return task.rollout(state, theta_pop, hidden, horizon)

        def sync(self, *arrays):
            torch.cuda.synchronize()

    cfg = es.Config(pop=p, horizon=50, sigma=0.1, lr=0.1)
    theta = torch.zeros(es.n_params(hidden, task), device=cuda)
    new, fit, steps = es.generation(Outside(), theta, cfg, hidden)
    eps = torch.cat([drawn[0], -drawn[0]])
    ranks = torch.argsort(torch.argsort(fit, stable=True), stable=True).float() / (p - 1) - 0.5
    expect = theta + cfg.lr * (ranks[:, None] * eps).sum(0) / (p * cfg.sigma)
    assert fit.shape == (p,) and steps.shape == (p,)
    torch.testing.assert_close(new, expect, rtol=1e-5, atol=1e-6)


def test_generation_runs_a_subclass_with_the_reference_reset(cuda):
    """A backend subclass that overrides reset(self, n), as the reference's tests do
    (test_es.py:53-56), runs inside es.generation and gets its fixed states."""
    import es

    task = es.TASKS["legged2"]
    p = 128
    fixed = task.mlx.reset(p)

    class Fixed(es.MetalBackend):
        def reset(self, n):
            return fixed

    class FixedLoop(es.MLXBackend):
        def reset(self, n):
            return fixed

    cfg = es.Config(task="legged2", pop=p, horizon=30)
    theta = torch.from_numpy((np.random.default_rng(1).normal(size=es.n_params(task.hidden, task)) * 0.1)
                             .astype(np.float32)).to(cuda)
    outs = [es.generation(b(task, 0), theta, cfg, task.hidden, 1) for b in (Fixed, FixedLoop)]
    for new, fit, steps in outs:
        assert fit.shape == (p,) and steps.max().item() <= 30 and not torch.equal(new, theta)
    # same initial states, same perturbations: the fused rollout and the loop take the same steps
    # for almost every member (their policies round the MLP differently)
    assert (outs[0][2] == outs[1][2]).float().mean().item() > 0.95


def test_train_resumes_from_a_checkpoint_exactly(cuda, tmp_path):
    """A run stopped after 3 generations and resumed from its checkpoint ends with the same theta,
    the same per-generation fitness and scores, and the same Result counts as the run that was
    never stopped (noise and initial states are functions of (seed, generation, member), and the
    checkpoint carries every seed counter)."""
    import es
    import rlenv_lib

    def run(max_gen, path, logs):
        cfg = es.Config(task="cartpole", pop=256, max_generations=max_gen, time_budget=1e9, solved_at=1e9)
        return es.train(cfg, "metal", 3, log=lambda *e: logs.append((e[0], e[1], e[3], e[4])),
                        checkpoint=str(path), checkpoint_every=2)

    rlenv_lib._reset_calls = 0
    whole_log = []
    whole = run(6, tmp_path / "whole.pt", whole_log)
    rlenv_lib._reset_calls = 0
    part_log = []
    run(3, tmp_path / "part.pt", part_log)
    rlenv_lib._reset_calls = 12345  # whatever the process did meanwhile: the checkpoint restores it
    resumed = run(6, tmp_path / "part.pt", part_log)
    assert (resumed.generations, resumed.env_steps, resumed.solved) == (whole.generations, whole.env_steps, whole.solved)
    assert part_log == whole_log
    a = torch.load(tmp_path / "whole.pt", weights_only=False)
    b = torch.load(tmp_path / "part.pt", weights_only=False)
    assert a["gen"] == b["gen"] == 6 and torch.equal(a["theta"], b["theta"])
    with pytest.raises(ValueError):  # another run's checkpoint is refused
        es.train(es.Config(task="acrobot", pop=256, max_generations=1), "metal", 3, checkpoint=str(tmp_path / "part.pt"))
