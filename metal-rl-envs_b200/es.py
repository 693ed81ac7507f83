"""Evolution Strategies on the batched environments, every generation on the GPU.

Drop-in for the reference's es.py (es.py:1-383): the same Task table, Config,
`n_params`, `unflatten`, `population_logits`, `loop_fitness`, `push`,
`curriculum`, `centered_ranks`, `generation`, `evaluate`, `mean_policy`,
`train` and command line, on torch CUDA tensors.

Backends:
- "metal" (alias "cuda"): the B200 path. Per generation: one kernel writes the
  perturbed population theta +- sigma * eps with eps regenerated from
  (seed, generation, pair) (Philox-4x32-10 + Box-Muller, no noise matrix is
  stored); one fused rollout kernel runs every member's policy and physics for
  the whole horizon; one kernel forms stable centred ranks; one kernel applies
  the rank-weighted antithetic update, regenerating the noise with a fixed
  summation order.
- "mlx" (alias "loop"): the reference's step-by-step loop (es.py:174-193): the
  population's MLP in torch, the environment through the CUDA step kernel. It
  is the kernel-versus-loop cross-check.
There is no numpy backend here: the CPU implementation is the test oracle.

Multi-GPU: when torch.distributed is initialised with world size G, rank r
rolls out members [r P/G, (r+1) P/G) (P divisible by G), then one
all_gather_into_tensor of (fitness, steps) over NCCL gives every rank the full
vectors, and every rank computes the same ranks and the same update bits, so
theta never needs to be broadcast.

Deviation from the reference, stated: eps comes from a counter-based generator
keyed by (seed, gen, pair) rather than MLX's global normal stream, and ties in
centred_ranks are broken by member index (a stable sort) where numpy's default
sort leaves their order unspecified. Generations therefore do not match the
reference bit for bit; parity is the distribution of generations to solve.
"""

import argparse
import inspect
import os
import time
from dataclasses import dataclass
from typing import Any, Callable

import torch
import torch.distributed as dist

import acrobot_metal
import acrobot_rollout_metal
import cartpole_metal
import cartpole_rollout_metal
import legged_metal
import legged_rollout_metal
import rlenv_lib as _rl


# ---- tasks -------------------------------------------------------------------------------------

@dataclass(frozen=True)
class Task:
    """A learning problem: its bodies, the policy's shape, how states become observations and
    logits become actions, the fused rollout, and the shaping of the fitness. The field names
    are es.py's (es.py:48-70), so code written against the reference reads them unchanged;
    `np` is always None here (the numpy bodies are the tests' oracle)."""
    name: str
    obs_dim: int
    n_out: int
    hidden: int
    solved_at: float
    np: Any
    mlx: Any
    metal: Any
    obs: Callable
    action: Callable
    rollout: Callable
    alive_bonus: float = 1.0
    fall_penalty: float = 0.0
    eval_bonus: float = 1.0
    height_gate: float = 0.0
    xdot_row: int | None = None
    assistable: bool = False


def _greedy(xp, logits):
    """The index of the largest logit (the first one on ties)."""
    return logits.argmax(dim=-1)


def _state_as_obs(xp, state):
    """CartPole observes its state as it is: (N, 4)."""
    return state.t()


def _acrobot_features(xp, state):
    """cos t1, sin t1, cos t2, sin t2, then both angular velocities: (N, 6)."""
    c, s = torch.cos(state[:2]), torch.sin(state[:2])
    return torch.stack((c[0], s[0], c[1], s[1], state[2], state[3]), dim=1)


def _obs_without_x(xp, state):
    """A legged body observes every state row except its horizontal position, so the policy
    cannot depend on where the body is."""
    return state[1:].t()


def _per_leg_action(c):
    """Three logits per leg, one argmax per leg, combined as the base-3 digits of one action."""
    place = 3 ** torch.arange(c, dtype=torch.int32)

    def action(xp, logits):
        digits = logits.reshape(logits.shape[0], c, 3).argmax(dim=-1).to(torch.int32)
        return (digits * place.to(digits.device)).sum(dim=1, dtype=torch.int32)
    return action


def _survival(rollout_steps, sign):
    """Adapt a rollout that counts the steps an episode survived (its terminating step not
    counted) to the (fitness, steps taken) pair: fitness is the count with the task's sign,
    steps taken include the terminating step and stop at the horizon (es.py:96-103)."""
    def rollout(state, theta_pop, hidden, horizon):
        survived = rollout_steps(state, theta_pop, hidden, horizon)
        return sign * survived, torch.clamp(survived + 1, max=horizon)
    return rollout


class _LeggedEnv:
    """The legged body with C legs as es.py's `mlx` and `metal` slots use it: reset around the
    standing pose, step with the torso assist."""

    RESET_BOUND = legged_metal.RESET_BOUND

    def __init__(self, c):
        self.body = legged_metal.Legged(c)
        self.ROWS = self.body.rows
        self.CENTER = legged_metal.stand_pose(c)

    def reset(self, n):
        return self.body.reset(n)

    def step(self, state, action, assist=None):
        return self.body.step(state, action, assist)

    def reseed(self, seed=0):
        self.body.reseed(seed)


def _classic_task(name, module, rollout_module, obs_dim, n_out, solved_at, observe, sign):
    return Task(name, obs_dim, n_out, 32, solved_at, None, module, module, observe, _greedy,
                _survival(rollout_module.rollout_steps, sign))


def _legged_variant(name, c, alive, fall, gate):
    """A legged task: training fitness is forward velocity (counted only while the torso is at
    least `gate` high) plus `alive` per step, minus `fall` on the step that falls; the score
    that decides "solved" is the distance walked before the first fall, 100 for every variant."""
    env = _LeggedEnv(c)

    def rollout(state, theta, hidden, horizon, assist=0.0):
        return legged_rollout_metal.rollout(state, theta, hidden, horizon, c, alive, fall, gate, assist)

    return Task(name, 5 + 2 * c, 3 * c, 16, 100.0, None, env, env, _obs_without_x, _per_leg_action(c), rollout,
                alive_bonus=alive, fall_penalty=fall, eval_bonus=0.0, height_gate=gate, xdot_row=3 + c,
                assistable=True)


# name -> (legs, alive bonus, fall penalty, height gate): es.py's table of legged tasks
_LEGGED_TASKS = {
    "legged2": (2, 1.0, 0.0, 0.0),
    "legged4": (4, 1.0, 0.0, 0.0),
    "legged2_distance": (2, 0.0, 0.0, 0.0),
    "legged4_distance": (4, 0.0, 0.0, 0.0),
    "legged2_alive10": (2, 0.1, 0.0, 0.0),
    "legged2_fall": (2, 0.0, 20.0, 0.0),
    "legged2_alive10_fall": (2, 0.1, 20.0, 0.0),
    "legged4_alive10": (4, 0.1, 0.0, 0.0),
    "legged2_gated": (2, 0.0, 0.0, 0.85),
}

TASKS = {
    "cartpole": _classic_task("cartpole", cartpole_metal, cartpole_rollout_metal, 4, 2, 475.0, _state_as_obs, 1.0),
    "acrobot": _classic_task("acrobot", acrobot_metal, acrobot_rollout_metal, 6, 3, -100.0, _acrobot_features, -1.0),
    **{name: _legged_variant(name, *spec) for name, spec in _LEGGED_TASKS.items()},
}


@dataclass
class Config:
    """Hyper-parameters of a run, with es.py's names and defaults. hidden and solved_at of None
    take the task's; assist_k0 and start_velocity are the curricula's starting values, both
    annealed to zero over anneal_gens generations."""
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


# ---- the policy --------------------------------------------------------------------------------

def n_params(hidden, task):
    """Parameters of an obs-H-out MLP with biases on both layers."""
    return (task.obs_dim + 1 + task.n_out) * hidden + task.n_out


def unflatten(theta_pop, hidden, task):
    """Views of the (P, D) parameter rows as the MLP's weights: w1 (P, obs, H), b1 (P, H),
    w2 (P, H, out), b2 (P, out), stored in that order (es.py:156-164)."""
    p, i, o = theta_pop.shape[0], task.obs_dim, task.n_out
    w1, b1, w2, b2 = torch.split(theta_pop, (i * hidden, hidden, hidden * o, o), dim=1)
    return w1.reshape(p, i, hidden), b1, w2.reshape(p, hidden, o), b2


def population_logits(xp, obs, params):
    """Each environment evaluated by its own member's MLP: two batched matrix products."""
    w1, b1, w2, b2 = params
    hidden = torch.tanh(torch.bmm(obs.unsqueeze(1), w1).squeeze(1) + b1)
    return torch.bmm(hidden.unsqueeze(1), w2).squeeze(1) + b2


# ---- curricula ---------------------------------------------------------------------------------

def push(xp, task, state, start_velocity):
    """Start every episode with start_velocity added to the forward velocity (es.py:196-203);
    the state is returned unchanged when there is no push or the task has no forward row."""
    if start_velocity and task.xdot_row is not None:
        state = state.clone()
        state[task.xdot_row] += start_velocity
    return state


def curriculum(cfg, gen):
    """(assist stiffness, start push) of generation gen: the configured values at generation 1,
    falling linearly to zero by generation anneal_gens + 1, zero throughout when anneal_gens is
    not positive (es.py:206-211)."""
    if cfg.anneal_gens <= 0:
        return 0.0, 0.0
    weight = 1.0 - min(1.0, (gen - 1) / cfg.anneal_gens)
    return cfg.assist_k0 * weight, cfg.start_velocity * weight


# Populations from this size up are ranked by the O(P log P) sort kernel, smaller ones by the
# one-launch O(P^2) counting kernel; both give the same bits. Measured per call on a B200: the
# counting kernel is faster up to P = 8,192 (34 us against 44), the sort from P = 16,384 (50 us
# against 101; 90 us against 19 ms at P = 262,144).
SORTED_RANKS_FROM = 16384
_rank_scratch = {}


def _scratch(dev, nbytes):
    buf = _rank_scratch.get(dev)
    if buf is None or buf.numel() < nbytes:
        buf = _rank_scratch[dev] = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    return buf


def centered_ranks(xp, values, sorted_kernel=None):
    """rank / (P - 1) - 0.5 with ranks from a stable ascending sort (NaN last), on the device.
    sorted_kernel forces the sort (True) or the counting kernel (False); None picks by size."""
    values = values.contiguous().float()
    out = torch.empty_like(values)
    p, sp = values.shape[0], _rl.stream_ptr(values.device)
    if sorted_kernel if sorted_kernel is not None else p >= SORTED_RANKS_FROM:
        need = _rl.lib().es_ranks_scratch_bytes(p)
        scratch = _scratch(values.device, need) if need > 0 else None
        _rl.check(_rl.lib().es_centered_ranks_sorted(values.data_ptr(), p, out.data_ptr(), _rl.ptr(scratch),
                                                     need, sp))
    else:
        _rl.check(_rl.lib().es_centered_ranks(values.data_ptr(), p, out.data_ptr(), sp))
    return out


def loop_fitness(backend, params, horizon, assist=0.0, start_velocity=0.0, state=None):
    """(fitness, steps taken) per member by the step-at-a-time loop of es.py:174-193: the
    population's MLPs in torch, the bodies through the CUDA step kernel, every member stepped
    each iteration and credited only until its first termination."""
    task = backend.task
    n = params[0].shape[0]
    if state is None:
        state = backend.reset(n)
    state = push(torch, task, state, start_velocity)
    dev = state.device
    running = torch.ones(n, dtype=torch.bool, device=dev)
    fitness = torch.zeros(n, device=dev)
    taken = torch.zeros(n, device=dev)
    for _ in range(horizon):
        action = task.action(torch, population_logits(torch, task.obs(torch, state), params))
        if task.assistable:
            state, reward, done = backend.step(state, action, assist)
        else:
            state, reward, done = backend.step(state, action)
        taken += running.float()
        fell = running & done
        running = running & ~done
        progress = reward - 1.0
        if task.height_gate:
            progress = progress * (state[1] >= task.height_gate).float()
        fitness += (progress + task.alive_bonus) * running.float() - task.fall_penalty * fell.float()
    return fitness, taken


def _reset(backend, n, gen, member_offset):
    """backend.reset for n members of generation gen from global member member_offset; a subclass
    that overrides reset with the reference's signature reset(self, n) (as test_es.py:53-56 does)
    gets just n."""
    try:
        params = inspect.signature(backend.reset).parameters.values()
    except (TypeError, ValueError):
        params = ()
    takes = sum(p.kind in (p.POSITIONAL_ONLY, p.POSITIONAL_OR_KEYWORD) for p in params)
    if takes >= 3 or any(p.kind == p.VAR_POSITIONAL for p in params):
        return backend.reset(n, gen, member_offset)
    return backend.reset(n)


def _world():
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(), dist.get_world_size()
    return 0, 1


class MetalBackend:
    """The fused B200 path: perturbation, rollout, ranks and update are device kernels."""

    xp = torch

    def __init__(self, task, seed):
        self.task = task
        self.seed = int(seed) & 0xFFFFFFFFFFFFFFFF
        self.rank, self.world = _world()
        self._normal_calls = 0
        task.metal.reseed(seed)

    # -- the reference backend interface ------------------------------------------------
    def normal(self, shape):
        """Standard normals (rows, d) from the counter-based generator (a fresh stream per call)."""
        rows, d = shape if len(shape) == 2 else (1, shape[0])
        self._normal_calls += 1
        out = torch.empty((rows, d), dtype=torch.float32, device=_rl.device())
        _rl.check(_rl.lib().es_noise(out.data_ptr(), rows, d, self.seed ^ 0xC0FFEE, self._normal_calls, 0,
                                     _rl.stream_ptr()))
        return out if len(shape) == 2 else out[0]

    def reset(self, n, gen=0, index_offset=0):
        """Fresh states for n members, a function of (seed, gen, global member index) only."""
        env = self.task.mlx
        return _rl.reset_uniform(env.ROWS, n, env.RESET_BOUND, center=getattr(env, "CENTER", None),
                                 seed=self._reset_seed(gen), index_offset=index_offset)

    def step(self, state, action, assist=None):
        return self.task.metal.step(state, action) if assist is None else self.task.metal.step(state, action, assist)

    def obs(self, state):
        return self.task.obs(torch, state)

    def sync(self, *arrays):
        torch.cuda.synchronize()

    def to_mx(self, theta):
        return theta

    # -- the fused generation -------------------------------------------------------------
    def _reset_seed(self, gen):
        x = (self.seed * 0x9E3779B97F4A7C15 + (gen + 1) * 0xBF58476D1CE4E5B9) & 0xFFFFFFFFFFFFFFFF
        return ((x >> 29) ^ x) & 0xFFFFFFFF

    def shard(self, pop):
        if pop % self.world:
            raise ValueError(f"population {pop} is not divisible by the world size {self.world}")
        per = pop // self.world
        return self.rank * per, per

    def perturb(self, theta, sigma, gen, pairs, member_offset, rows):
        theta = theta.contiguous()
        out = torch.empty((rows, theta.shape[0]), dtype=torch.float32, device=theta.device)
        _rl.check(_rl.lib().es_perturb(theta.data_ptr(), theta.shape[0], sigma, self.seed, gen, pairs, member_offset,
                                       rows, out.data_ptr(), _rl.stream_ptr(theta.device)))
        return out

    def centered_ranks(self, fit):
        return centered_ranks(torch, fit)

    def update(self, theta, ranks, lr, sigma, gen, pairs):
        out = torch.empty_like(theta)
        _rl.check(_rl.lib().es_update(theta.data_ptr(), ranks.data_ptr(), theta.shape[0], pairs, lr, sigma, self.seed,
                                      gen, out.data_ptr(), _rl.stream_ptr(theta.device)))
        return out

    def rollout(self, theta_pop, hidden, horizon, assist=0.0, start_velocity=0.0, gen=0, member_offset=0):
        state = push(torch, self.task, _reset(self, theta_pop.shape[0], gen, member_offset), start_velocity)
        extra = (assist,) if self.task.assistable else ()
        return self.task.rollout(state, theta_pop, hidden, horizon, *extra)

    def gather(self, local):
        """All ranks' shards concatenated in rank order (one collective per tensor stack)."""
        if self.world == 1:
            return local
        local = local.contiguous()
        if dist.get_backend() == "nccl":
            full = torch.empty((self.world,) + tuple(local.shape), dtype=local.dtype, device=local.device)
            dist.all_gather_into_tensor(full, local)
        else:  # gloo (CPU tests of this orchestration)
            parts = [torch.empty_like(local) for _ in range(self.world)]
            dist.all_gather(parts, local)
            full = torch.stack(parts)
        return full.reshape((-1,) + tuple(local.shape[1:]))


class MLXBackend(MetalBackend):
    """The step-by-step loop (es.py:230-257): torch policy, CUDA step kernel, per-step launches."""

    def rollout(self, theta_pop, hidden, horizon, assist=0.0, start_velocity=0.0, gen=0, member_offset=0):
        state = _reset(self, theta_pop.shape[0], gen, member_offset)
        return loop_fitness(self, unflatten(theta_pop, hidden, self.task), horizon, assist, start_velocity, state)


BACKENDS = {"metal": MetalBackend, "cuda": MetalBackend, "mlx": MLXBackend, "loop": MLXBackend}


_FUSED = ("shard", "perturb", "update", "centered_ranks")


def reference_generation(backend, theta, cfg, hidden, gen=1):
    """es.py:218-227 as the reference writes it, for a backend that offers only the reference's
    interface (xp, normal, rollout, sync): half = normal((P/2, D)), eps = [half; -half], fitness
    of theta + sigma eps, g = sum_i rank_i eps_i / (P sigma), theta + lr g. The ranks come from
    this module's centred-rank kernel when the arrays are CUDA tensors."""
    xp = getattr(backend, "xp", torch)
    half = backend.normal((cfg.pop // 2, theta.shape[0]))
    eps = xp.concatenate([half, -half], axis=0) if xp is not torch else torch.cat([half, -half], dim=0)
    assist, start_velocity = curriculum(cfg, gen)
    fit, steps = backend.rollout(theta[None, :] + cfg.sigma * eps, hidden, cfg.horizon, assist, start_velocity)
    if isinstance(fit, torch.Tensor) and fit.is_cuda:
        ranks = centered_ranks(xp, fit)
    else:  # es.py:214-215 as written, for host arrays
        ranks = xp.argsort(xp.argsort(fit)).astype(fit.dtype) / (fit.shape[0] - 1) - 0.5
    grad = (ranks[:, None] * eps).sum(axis=0) / (cfg.pop * cfg.sigma)
    theta = theta + cfg.lr * grad
    backend.sync(theta)
    return theta, fit, steps


def generation(backend, theta, cfg, hidden, gen=1):
    """One generation of es.py:218-227 on this rank's shard of the population: perturb, roll
    out, gather every shard's (fitness, steps), rank, update. Returns (theta, fitness, steps)
    with fitness and steps of the whole population. A backend without the fused pieces (shard,
    perturb, update, centered_ranks), one written against the reference's interface, runs
    reference_generation instead."""
    if not all(callable(getattr(backend, m, None)) for m in _FUSED):
        return reference_generation(backend, theta, cfg, hidden, gen)
    pairs = cfg.pop // 2
    first, count = backend.shard(cfg.pop)
    members = backend.perturb(theta, cfg.sigma, gen, pairs, first, count)
    stiffness, velocity = curriculum(cfg, gen)
    fit, steps = backend.rollout(members, hidden, cfg.horizon, stiffness, velocity, gen, first)
    if backend.world > 1:
        gathered = backend.gather(torch.stack([fit.float(), steps.float()], dim=1))
        fit, steps = gathered[:, 0].contiguous(), gathered[:, 1].contiguous()
    theta = backend.update(theta, backend.centered_ranks(fit), cfg.lr, cfg.sigma, gen, pairs)
    backend.sync(theta)
    return theta, fit, steps


CHECK_EVERY = 10  # generations between cross-rank checks of theta in train()


def theta_checksum(theta):
    """An order-dependent checksum of theta's bits (an int64 tensor of one element)."""
    bits = theta.detach().contiguous().view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    weight = torch.arange(bits.numel(), device=bits.device, dtype=torch.int64) % 1021 + 1
    return (bits * weight).sum().reshape(1)


def assert_ranks_agree(theta):
    """Every rank must hold the same theta bits (each computes the update itself). One MIN and one
    MAX all-reduce of a checksum; a mismatch raises on every rank."""
    rank, world = _world()
    if world == 1:
        return
    lo = theta_checksum(theta)
    hi = lo.clone()
    dist.all_reduce(lo, op=dist.ReduceOp.MIN)
    dist.all_reduce(hi, op=dist.ReduceOp.MAX)
    if int(lo.item()) != int(hi.item()):
        raise RuntimeError(f"rank {rank}: theta diverged across ranks (checksums {int(lo.item())} .. {int(hi.item())})")


def mean_policy(theta, hidden, task):
    """theta (D,) as a function from (n, obs_dim) observations to (n, out) logits."""
    w1, b1, w2, b2 = (part[0] for part in unflatten(theta.reshape(1, -1), hidden, task))

    def actor(obs):
        return torch.tanh(obs @ w1 + b1) @ w2 + b2
    return actor


def evaluate(task, actor, n=2048, steps=500):
    """The score that decides "solved" (es.py:308-322): n fresh episodes of the greedy actor,
    each crediting reward - 1 + task.eval_bonus per step until its first termination (the
    environment's own reward for CartPole and Acrobot, forward distance for legged bodies);
    the mean over episodes. The actor and the bodies run on the GPU."""
    state = task.mlx.reset(n)
    running = torch.ones(n, dtype=torch.bool, device=state.device)
    total = torch.zeros(n, device=state.device)
    for _ in range(steps):
        state, reward, done = task.metal.step(state, task.action(torch, actor(task.obs(torch, state))))
        running &= ~done
        total += (reward - 1.0 + task.eval_bonus) * running.float()
    return total.mean().item()


def evaluate_theta(task, theta, hidden, n=2048, steps=500, state=None):
    """The same score for the mean policy theta as one fused rollout launch: every one of the n
    members shares theta's row (stride 0). Equal to evaluate(task, mean_policy(theta, ...)) from
    the same initial states."""
    state = task.mlx.reset(n) if state is None else state
    if isinstance(task.mlx, _LeggedEnv):
        fit, _ = legged_rollout_metal.rollout(state, theta, hidden, steps, task.mlx.body.c, task.eval_bonus, 0.0, 0.0)
    else:
        fit, _ = task.rollout(state, theta, hidden, steps)
    return fit.mean().item()


@dataclass
class Result:
    """Outcome of `train`, with es.py's fields: env_steps counts the steps members actually
    took (each episode ends at its first termination); train_seconds covers the generations
    only, not the evaluations of the mean policy."""
    solved: bool
    generations: int
    env_steps: int
    train_seconds: float
    score: float


def _seed_counters(task):
    """Every counter that seeds a later draw of a training run: the library's reset counter (the
    evaluation's fresh states) and the task's step-kernel call counter (the step loop's resets)."""
    m = task.metal
    holder = getattr(m, "body", None) or getattr(m, "_counter", None) or m
    return {"reset_calls": _rl._reset_calls, "step_calls": getattr(holder, "calls", None)}


def _restore_seed_counters(task, counters):
    _rl._reset_calls = int(counters["reset_calls"])
    m = task.metal
    holder = getattr(m, "body", None) or getattr(m, "_counter", None) or m
    if counters.get("step_calls") is not None and hasattr(holder, "calls"):
        holder.calls = int(counters["step_calls"])


def train(cfg, backend_name, seed, log=lambda *_: None, *, checkpoint=None, checkpoint_every=10):
    """Run generations until the mean policy's score reaches the threshold, the generation cap
    or the time budget (es.py:334-354). log(gen, env_steps, train_seconds, mean fitness,
    score) is called after every generation.

    checkpoint: a file path. Every checkpoint_every generations, and when training ends, theta,
    the generation, the bookkeeping and every seed counter are saved there (written to a
    temporary file, then renamed over it; rank 0 writes). If the file exists when train starts,
    the run resumes from it. The noise and the initial states of a generation are functions of
    (seed, generation, member), so a resumed run continues exactly as the uninterrupted run
    would have. The reference keeps theta only in memory (es.py:325-354)."""
    if cfg.pop % 2:
        raise ValueError(f"the population must be even (antithetic pairs); got {cfg.pop}")
    if backend_name not in BACKENDS:
        raise ValueError(f"backend {backend_name!r}: this build runs on the GPU only ({sorted(BACKENDS)}); "
                         "the numpy reference is the test oracle")
    task = TASKS[cfg.task]
    width = task.hidden if cfg.hidden is None else cfg.hidden
    target = task.solved_at if cfg.solved_at is None else cfg.solved_at
    make_backend = BACKENDS[backend_name]
    backend = make_backend(task, seed)
    theta = backend.normal((n_params(width, task),)) * 0.1
    backend.sync(theta)
    clock, taken, score, gen = 0.0, 0, 0.0, 0
    run = {"task": cfg.task, "pop": cfg.pop, "width": width, "seed": int(seed), "backend": backend_name}
    if checkpoint is not None and os.path.exists(checkpoint):
        saved = torch.load(checkpoint, map_location="cpu", weights_only=False)
        if saved["run"] != run:
            raise ValueError(f"checkpoint {checkpoint} belongs to another run: {saved['run']} != {run}")
        theta = saved["theta"].to(theta.device)
        gen, taken, clock, score = saved["gen"], saved["taken"], saved["clock"], saved["score"]
        backend._normal_calls = saved["normal_calls"]
        _restore_seed_counters(task, saved["counters"])

    def save():
        if checkpoint is None or backend.rank != 0:
            return
        tmp = f"{checkpoint}.tmp"
        torch.save({"run": run, "theta": theta.detach().cpu(), "gen": gen, "taken": taken, "clock": clock,
                    "score": score, "normal_calls": backend._normal_calls, "counters": _seed_counters(task)}, tmp)
        os.replace(tmp, checkpoint)

    while gen < cfg.max_generations:
        gen += 1
        t0 = time.perf_counter()
        theta, fit, steps = generation(backend, theta, cfg, width, gen)
        clock += time.perf_counter() - t0
        taken += int(steps.sum().item())
        if backend.world > 1 and gen % CHECK_EVERY == 0:
            assert_ranks_agree(theta)
        score = evaluate_theta(task, theta, width)
        log(gen, taken, clock, float(fit.mean().item()), score)
        if score >= target:
            save()
            return Result(True, gen, taken, clock, score)
        if checkpoint_every > 0 and gen % checkpoint_every == 0:
            save()
        if clock >= cfg.time_budget:
            break
    save()
    return Result(False, gen, taken, clock, score)


# es.py's command line: flag -> (type, default, help)
_FLAGS = {
    "--task": (str, "cartpole", "the task to learn"),
    "--pop": (int, 1024, "population size (even: antithetic pairs)"),
    "--backend": (str, "metal", "metal (alias cuda): the fused kernels; mlx (alias loop): the step loop"),
    "--seed": (int, 0, "seed of parameters, noise and initial states"),
    "--lr": (float, 0.1, "learning rate"),
    "--sigma": (float, 0.1, "perturbation scale"),
    "--time-budget": (float, 120.0, "seconds of training after which the run stops"),
    "--max-generations": (int, 500, "generation cap"),
    "--assist": (float, 0.0, "curriculum: torso-assist stiffness at generation 1, annealed to zero"),
    "--start-velocity": (float, 0.0, "curriculum: forward push at the start of every episode, annealed to zero"),
    "--anneal": (int, 300, "generation by which both curricula have reached zero"),
    # this build's own: checkpoint and resume (train's checkpoint arguments)
    "--checkpoint": (str, None, "file to save the run to every --checkpoint-every generations, and to resume from"),
    "--checkpoint-every": (int, 10, "generations between checkpoints"),
}


def main(argv=None):
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    for flag, (kind, default, text) in _FLAGS.items():
        choices = {"--task": TASKS, "--backend": BACKENDS}.get(flag)
        parser.add_argument(flag, type=kind, default=default, help=text, choices=choices)
    args = parser.parse_args(argv)
    renamed = {"assist": "assist_k0", "anneal": "anneal_gens"}  # flags whose Config field is named otherwise
    own = ("backend", "seed", "checkpoint", "checkpoint_every")
    cfg = Config(**{renamed.get(k, k): v for k, v in vars(args).items() if k not in own})

    def report(gen, env_steps, seconds, fitness, score):
        print(f"generation {gen:4d} | {env_steps:>14,} env steps | {seconds:8.2f} s | population fitness "
              f"{fitness:8.1f} | score {score:8.1f}", flush=True)

    print(train(cfg, args.backend, args.seed, log=report, checkpoint=args.checkpoint,
                checkpoint_every=args.checkpoint_every))
    return 0


if __name__ == "__main__":
    main()
