"""The oracle reproduces the reference's own numpy outputs (tests/golden, made by running the
reference's *_np.py and es.py). These pins are what lets every GPU test trust the oracle."""

import sys

import numpy as np
import pytest

from conftest import GOLDEN, golden
from oracle import classic, es, legged, pendulum

TIGHT = dict(rtol=1e-6, atol=1e-6)


def test_cartpole_matches_reference():
    g = golden("cartpole")
    out = classic.cartpole_physics(g["state"], g["action"])
    np.testing.assert_allclose(out, g["stepped"], **TIGHT)
    assert (classic.cartpole_terminated(g["stepped"]) == g["done"]).all()
    s = g["traj_state"]
    ck = 0
    for t, a in enumerate(g["traj_actions"], 1):
        s = classic.cartpole_physics(s, a)
        if t in (1, 10, 25, 50, 100):
            np.testing.assert_allclose(s, g["traj"][ck], rtol=1e-5, atol=1e-5, err_msg=f"step {t}")
            ck += 1


def test_acrobot_matches_reference():
    g = golden("acrobot")
    out = classic.acrobot_physics(g["state"], g["action"])
    np.testing.assert_allclose(out, g["stepped"], **TIGHT)
    assert (classic.acrobot_terminated(g["stepped"]) == g["done"]).all()
    s = g["traj_state"]
    ck = 0
    for t, a in enumerate(g["traj_actions"], 1):
        s = classic.acrobot_physics(s, a)
        if t in (1, 10, 25, 50, 100):
            np.testing.assert_allclose(s, g["traj"][ck], rtol=1e-5, atol=1e-5, err_msg=f"step {t}")
            ck += 1


@pytest.mark.parametrize("k", [2, 3, 4, 8, 16, 32, 64])
def test_pendulum_matches_reference(k):
    g = golden("pendulum")
    st, ac = g[f"state_k{k}"], g[f"action_k{k}"]
    tq = ((ac - 1) * 1.0).astype(np.float32)
    np.testing.assert_allclose(pendulum.aba_accel(st[:k], st[k:], tq, k), g[f"aba_acc_k{k}"], **TIGHT)
    np.testing.assert_allclose(pendulum.aba_physics(st, ac, k), g[f"aba_stepped_k{k}"], **TIGHT)
    assert (pendulum.terminated(g[f"aba_stepped_k{k}"], k) == g[f"aba_done_k{k}"]).all()
    if k <= 16:
        np.testing.assert_allclose(pendulum.mm_accel(st[:k], st[k:], tq, k), g[f"mm_acc_k{k}"], **TIGHT)
        np.testing.assert_allclose(pendulum.mm_physics(st, ac, k), g[f"mm_stepped_k{k}"], **TIGHT)
        assert (pendulum.terminated(g[f"mm_stepped_k{k}"], k) == g[f"mm_done_k{k}"]).all()


@pytest.mark.parametrize("k", [4, 16])
def test_pendulum_trajectories_match_reference(k):
    g = golden("pendulum")
    for form, phys in (("mm", pendulum.mm_physics), ("aba", pendulum.aba_physics)):
        s, ck = g[f"traj_state_k{k}"], 0
        for t, a in enumerate(g[f"traj_actions_k{k}"], 1):
            s = phys(s, a, k)
            if t in (1, 10, 25, 50):
                np.testing.assert_allclose(s, g[f"{form}_traj_k{k}"][ck], rtol=1e-5, atol=1e-5, err_msg=f"{form} step {t}")
                ck += 1


def test_hopper_matches_reference():
    g = golden("hopper")
    out = legged.physics(g["state"], g["action"], 1, iters=1)
    np.testing.assert_allclose(out, g["stepped"], **TIGHT)
    assert (legged.terminated(g["stepped"]) == g["done"]).all()
    lt, ln = legged.contact_impulse(g["att"], g["atn"], g["ann"], g["wt"], g["wn"], g["depth"])
    np.testing.assert_allclose(lt, g["lt"], **TIGHT)
    np.testing.assert_allclose(ln, g["ln"], **TIGHT)


@pytest.mark.parametrize("c", [1, 2, 4])
def test_legged_matches_reference(c):
    g = golden("legged")
    st, ac = g[f"state_c{c}"], g[f"action_c{c}"]
    for iters in (1, 4, 8, 16):
        out = legged.physics(st, ac, c, iters)
        np.testing.assert_allclose(out, g[f"stepped_c{c}_i{iters}"], **TIGHT, err_msg=f"iters={iters}")
        assert (legged.terminated(out) == g[f"done_c{c}_i{iters}"]).all()
    np.testing.assert_allclose(legged.physics(st, ac, c, 8, assist=20.0), g[f"assist_stepped_c{c}"], **TIGHT)
    np.testing.assert_array_equal(legged.stand_pose(c), g[f"stand_c{c}"])
    np.testing.assert_array_equal(legged.static_pose(c), g[f"static_c{c}"])


def test_es_pieces_match_reference():
    g = golden("es")
    np.testing.assert_allclose(es.centered_ranks(g["ranks_in"], stable=False), g["ranks_out"], atol=1e-7)
    np.testing.assert_allclose(es.centered_ranks(g["ranks_in"]), g["ranks_out"], atol=1e-7)  # no ties: same
    np.testing.assert_allclose(es.centered_ranks(g["ranks_known_in"]), g["ranks_known_out"], atol=1e-7)
    from oracle.rollout import legged_action
    np.testing.assert_array_equal(legged_action(g["leg_logits"], 2), g["leg_action"])


@pytest.mark.parametrize("name,pop,horizon", [("cartpole", 64, 60), ("acrobot", 64, 40), ("legged2", 32, 25)])
def test_es_generation_matches_reference(name, pop, horizon):
    """The numpy ES generation draws from one Generator in the reference's order, so the oracle
    reproduces the reference's fitness, steps and updated parameters from the same seed."""
    g = golden("es")
    task = es.TASKS[name]
    rng = np.random.default_rng(3)
    theta = rng.normal(size=(es.n_params(task.hidden, task),)).astype(np.float32) * 0.1
    np.testing.assert_array_equal(theta, g[f"{name}_theta0"])
    cfg = es.Config(task=name, pop=pop, horizon=horizon, sigma=0.1, lr=0.1)
    new, fit, steps = es.generation(task, theta, cfg, task.hidden, rng, 1, stable_ranks=False)
    np.testing.assert_allclose(fit, g[f"{name}_fit"], rtol=1e-5, atol=1e-5)
    np.testing.assert_array_equal(steps, g[f"{name}_steps"])
    np.testing.assert_allclose(new, g[f"{name}_theta1"], rtol=1e-5, atol=1e-6)


def test_es_solve_fixture_reproduces():
    """tests/golden/es_solve.npz (10-seed generations-to-solve of the oracle's train loop) is
    what the committed script computes: seed 3 of each task rerun here."""
    from oracle import es as oes

    g = golden("es_solve")
    for task in ("cartpole", "acrobot"):
        pop, max_gen = (int(x) for x in g[f"{task}_config"])
        r = oes.train(oes.Config(task=task, pop=pop, max_generations=max_gen, time_budget=1e9), 3)
        assert (r.solved, r.generations, r.env_steps) == (bool(g[f"{task}_solved"][3]), int(g[f"{task}_generations"][3]),
                                                          int(g[f"{task}_env_steps"][3]))


def test_legged_rollout_fixture_is_the_oracles():
    """tests/golden/legged_rollout.npz (the GPU rollout test's reference side) is what the oracle
    computes from parity.legged_rollout_inputs: recomputed here on the first 48 members."""
    sys.path.insert(0, str(GOLDEN))
    import make_legged_rollout

    g = golden("legged_rollout")
    for index, f32 in ((0, True), (0, False), (4, True)):
        fit, steps = make_legged_rollout.run(index, f32, p=48)
        tag = "f32" if f32 else "f64"
        np.testing.assert_array_equal(fit, g[f"case{index}_{tag}_fitness"][:48])
        np.testing.assert_array_equal(steps, g[f"case{index}_{tag}_steps"][:48])
