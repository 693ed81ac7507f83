"""Evolution Strategies with es.py's numpy backend, restated.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Everything runs on the CPU with one numpy Generator per run, as es.py's
NumpyBackend does (es.py:270-296): antithetic noise, the population stepped
together through the numpy environment with auto-reset (loop_fitness,
es.py:174-193), centred ranks, the rank-weighted update (es.py:214-227), and a
numpy restatement of the greedy evaluation (es.py:302-322).
"""

import time
from dataclasses import dataclass

import numpy as np

from oracle import classic, legged
from oracle.rollout import acrobot_obs, legged_action

# ---- tasks (es.py:47-132) ------------------------------------------------------


@dataclass(frozen=True)
class TaskSpec:
    name: str
    obs_dim: int
    n_out: int
    hidden: int
    solved_at: float
    legs: int = 0                # 0 for CartPole / Acrobot
    alive_bonus: float = 1.0
    fall_penalty: float = 0.0
    eval_bonus: float = 1.0
    height_gate: float = 0.0
    xdot_row: int | None = None
    assistable: bool = False


def _legged(c, suffix, alive=1.0, fall=0.0, gate=0.0):
    return TaskSpec(f"legged{c}{suffix}", 5 + 2 * c, 3 * c, 16, 100.0, c, alive, fall, 0.0, gate, 3 + c, True)


TASKS = {
    "cartpole": TaskSpec("cartpole", 4, 2, 32, 475.0),
    "acrobot": TaskSpec("acrobot", 6, 3, 32, -100.0),
    "legged2": _legged(2, ""),
    "legged4": _legged(4, ""),
    "legged2_distance": _legged(2, "_distance", alive=0.0),
    "legged4_distance": _legged(4, "_distance", alive=0.0),
    "legged2_alive10": _legged(2, "_alive10", alive=0.1),
    "legged2_fall": _legged(2, "_fall", alive=0.0, fall=20.0),
    "legged2_alive10_fall": _legged(2, "_alive10_fall", alive=0.1, fall=20.0),
    "legged4_alive10": _legged(4, "_alive10", alive=0.1),
    "legged2_gated": _legged(2, "_gated", alive=0.0, gate=0.85),
}


def n_params(hidden, task):
    """Weights and biases of both layers of the obs-H-out MLP (es.py:152-153)."""
    return (task.obs_dim + 1 + task.n_out) * hidden + task.n_out


def unflatten(theta_pop, hidden, task):
    """(P, D) rows to w1 (P, obs, H), b1 (P, H), w2 (P, H, out), b2 (P, out) (es.py:156-164)."""
    rows, n_in, n_out = theta_pop.shape[0], task.obs_dim, task.n_out
    w1, b1, w2, b2 = np.split(theta_pop, np.cumsum([n_in * hidden, hidden, hidden * n_out]), axis=1)
    return w1.reshape(rows, n_in, hidden), b1, w2.reshape(rows, hidden, n_out), b2


def population_logits(obs, params):
    w1, b1, w2, b2 = params
    h = np.tanh(np.einsum("pi,pih->ph", obs, w1) + b1)
    return np.einsum("ph,pho->po", h, w2) + b2


def centered_ranks(values, stable=True):
    """argsort(argsort(v)) / (P - 1) - 0.5 (es.py:214-215). stable=True breaks ties by index,
    as the GPU kernel does; stable=False uses numpy's default sort like the reference."""
    kind = "stable" if stable else None
    r = np.argsort(np.argsort(values, kind=kind), kind=kind).astype(values.dtype)
    return r / (values.shape[0] - 1) - 0.5


# ---- environment hooks ---------------------------------------------------------


def observe(task, state):
    if task.legs:
        return state[1:].T
    return acrobot_obs(state) if task.name == "acrobot" else state.T


def act(task, logits):
    return legged_action(logits, task.legs) if task.legs else np.argmax(logits, axis=-1)


def reset(task, n, rng):
    if task.legs:
        c = task.legs
        return legged.stand_pose(c)[:, None] + rng.uniform(-legged.LG_RESET_BOUND, legged.LG_RESET_BOUND,
                                                           size=(2 * (3 + c), n)).astype(np.float32)
    bound = classic.AC_RESET_BOUND if task.name == "acrobot" else classic.CP_RESET_BOUND
    return rng.uniform(-bound, bound, size=(4, n)).astype(np.float32)


def env_step(task, state, action, rng, assist=0.0):
    """The numpy environment's step with auto-reset from `rng` (cartpole_np.py:39-55 and siblings)."""
    if task.legs:
        stepped = legged.physics(state, action, task.legs, legged.LG_ITERS, assist)
        done = legged.terminated(stepped)
        reward = legged.reward(stepped, done, task.legs)
    elif task.name == "acrobot":
        stepped = classic.acrobot_physics(state, action)
        done = classic.acrobot_terminated(stepped)
        reward = classic.acrobot_reward(done)
    else:
        stepped = classic.cartpole_physics(state, action)
        done = classic.cartpole_terminated(stepped)
        reward = classic.cartpole_reward(done)
    fresh = reset(task, stepped.shape[1], rng)
    return np.where(done[None, :], fresh, stepped), reward, done


def push(task, state, start_velocity):
    """Initial states with start_velocity added to the forward velocity row (es.py:196-203)."""
    if start_velocity and task.xdot_row is not None:
        state = state.copy()
        state[task.xdot_row] += start_velocity
    return state


# ---- learner -------------------------------------------------------------------


@dataclass
class Config:
    task: str = "cartpole"
    pop: int = 1024
    hidden: int | None = None
    sigma: float = 0.1
    lr: float = 0.1
    horizon: int = 500
    solved_at: float | None = None
    max_generations: int = 500
    time_budget: float = 120.0
    assist_k0: float = 0.0
    start_velocity: float = 0.0
    anneal_gens: int = 300


def curriculum(cfg, gen):
    """(assist, push) at generation gen: linear from the configured values at generation 1 to
    zero at generation anneal_gens + 1; zero when anneal_gens is not positive (es.py:206-211)."""
    weight = 1.0 - min(1.0, (gen - 1) / cfg.anneal_gens) if cfg.anneal_gens > 0 else 0.0
    return cfg.assist_k0 * weight, cfg.start_velocity * weight


def loop_fitness(task, params, horizon, rng, state=None, assist=0.0, start_velocity=0.0):
    """(reward sum to the first termination, steps taken) per member, the whole population
    stepped together with auto-reset (es.py:174-193)."""
    P = params[0].shape[0]
    s = push(task, reset(task, P, rng) if state is None else np.array(state), start_velocity)
    alive = np.ones(P, dtype=bool)
    fit = np.zeros(P, dtype=np.float32)
    steps = np.zeros(P, dtype=np.float32)
    for _ in range(horizon):
        a = act(task, population_logits(observe(task, s), params))
        s, r, done = env_step(task, s, a, rng, assist)
        steps += alive
        fell = alive & done
        alive = alive & ~done
        fwd = (r - 1.0) * (s[1] >= task.height_gate).astype(fit.dtype) if task.height_gate else r - 1.0
        fit = fit + (fwd + task.alive_bonus) * alive.astype(fit.dtype) - task.fall_penalty * fell.astype(fit.dtype)
    return fit, steps


def generation(task, theta, cfg, hidden, rng, gen=1, stable_ranks=True):
    """One generation of es.py:218-227. stable_ranks=False ranks ties with numpy's default sort,
    exactly as the reference; True breaks them by index, as the GPU kernel does."""
    half = rng.normal(size=(cfg.pop // 2, theta.shape[0])).astype(np.float32)
    eps = np.concatenate([half, -half], axis=0)
    assist, sv = curriculum(cfg, gen)
    fit, steps = loop_fitness(task, unflatten(theta[None, :] + cfg.sigma * eps, hidden, task), cfg.horizon,
                              rng, assist=assist, start_velocity=sv)
    grad = (centered_ranks(fit, stable_ranks)[:, None] * eps).sum(axis=0) / (cfg.pop * cfg.sigma)
    return theta + cfg.lr * grad, fit, steps


def evaluate(task, theta, hidden, rng, n=2048, steps=500):
    """Greedy mean policy over n fresh episodes: sum of (reward - 1 + eval_bonus) to the first
    termination, averaged (es.py:308-322)."""
    params = tuple(np.broadcast_to(p, (n,) + p.shape[1:]) for p in unflatten(theta[None, :], hidden, task))
    s = reset(task, n, rng)
    alive = np.ones(n, dtype=bool)
    fit = np.zeros(n, dtype=np.float32)
    for _ in range(steps):
        a = act(task, population_logits(observe(task, s), params))
        s, r, done = env_step(task, s, a, rng)
        alive = alive & ~done
        fit = fit + (r - 1.0 + task.eval_bonus) * alive.astype(np.float32)
    return float(fit.mean())


@dataclass
class Result:
    solved: bool
    generations: int
    env_steps: int
    train_seconds: float
    score: float


def train(cfg, seed, log=lambda *_: None):
    """es.py:334-354 with the numpy backend and the numpy evaluation above: generations until
    the mean policy's score reaches the threshold, the generation cap or the time budget. One
    numpy Generator seeded with `seed` draws theta, then each generation's noise and initial
    states, then each evaluation's episodes, in that order."""
    if cfg.pop % 2:
        raise ValueError("the population must be even")
    task = TASKS[cfg.task]
    width = cfg.hidden if cfg.hidden is not None else task.hidden
    target = cfg.solved_at if cfg.solved_at is not None else task.solved_at
    rng = np.random.default_rng(seed)
    theta = rng.normal(size=(n_params(width, task),)).astype(np.float32) * 0.1
    clock, taken, score, gen = 0.0, 0, 0.0, 0
    while gen < cfg.max_generations:
        gen += 1
        start = time.perf_counter()
        theta, fit, steps = generation(task, theta, cfg, width, rng, gen)
        clock += time.perf_counter() - start
        taken += int(steps.sum())
        score = evaluate(task, theta, width, rng)
        log(gen, taken, clock, float(fit.mean()), score)
        if score >= target:
            return Result(True, gen, taken, clock, score)
        if clock >= cfg.time_budget:
            break
    return Result(False, gen, taken, clock, score)
