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


@dataclass(frozen=True)
class Task:
    name: str
    obs_dim: int
    n_out: int               # policy outputs
    hidden: int
    solved_at: float         # threshold on the greedy mean policy's mean fitness
    np: Any                  # the numpy environment: not part of this build (see oracle/ in the tests)
    mlx: Any                 # environment with reset(n) on the device
    metal: Any               # the CUDA step kernel: step(state, action), reseed(seed)
    obs: Callable            # (xp, state) -> (P, obs_dim)
    action: Callable         # (xp, logits (P, n_out)) -> action index (P,)
    rollout: Callable        # (state, theta_pop, hidden, horizon[, assist]) -> (fitness, steps)
    alive_bonus: float = 1.0
    fall_penalty: float = 0.0
    eval_bonus: float = 1.0
    height_gate: float = 0.0
    xdot_row: int | None = None
    assistable: bool = False


def _argmax(xp, logits):
    return torch.argmax(logits, dim=-1)


def _cartpole_obs(xp, state):
    return state.T


def _acrobot_obs(xp, state):
    th1, th2, dth1, dth2 = state
    return torch.stack([torch.cos(th1), torch.sin(th1), torch.cos(th2), torch.sin(th2), dth1, dth2], dim=1)


def _legged_obs(xp, state):
    """Everything but x, so the policy is translation-invariant."""
    return state[1:].T


def _legged_action(c):
    def action(xp, logits):
        out = None
        for k in range(c):
            a_k = torch.argmax(logits[:, 3 * k:3 * k + 3], dim=-1).to(torch.int32) * 3**k
            out = a_k if out is None else out + a_k
        return out
    return action


def _steps_fitness(kernel, sign):
    """Steps survived (the terminating step excluded) to (fitness, steps taken): fitness has the
    task's sign; steps taken counts the terminating step, capped at the horizon (es.py:96-103)."""
    def rollout(state, theta_pop, hidden, horizon):
        steps = kernel(state, theta_pop, hidden, horizon)
        return sign * steps, torch.clamp(steps + 1, max=horizon)
    return rollout


class _LeggedEnv:
    """Legged step kernel plus a device reset around the standing pose, shared per C."""

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


def _legged_task(c, name, alive=1.0, fall=0.0, gate=0.0):
    env = _LeggedEnv(c)
    return Task(f"legged{c}{name}", 5 + 2 * c, 3 * c, 16, 100.0, None, env, env,
                _legged_obs, _legged_action(c),
                lambda state, theta, hidden, horizon, assist=0.0: legged_rollout_metal.rollout(
                    state, theta, hidden, horizon, c, alive, fall, gate, assist),
                alive, fall, 0.0, gate, 3 + c, True)


TASKS = {
    "cartpole": Task("cartpole", 4, 2, 32, 475.0, None, cartpole_metal, cartpole_metal,
                     _cartpole_obs, _argmax, _steps_fitness(cartpole_rollout_metal.rollout_steps, 1.0)),
    "acrobot": Task("acrobot", 6, 3, 32, -100.0, None, acrobot_metal, acrobot_metal,
                    _acrobot_obs, _argmax, _steps_fitness(acrobot_rollout_metal.rollout_steps, -1.0)),
    "legged2": _legged_task(2, ""),
    "legged4": _legged_task(4, ""),
    "legged2_distance": _legged_task(2, "_distance", alive=0.0),
    "legged4_distance": _legged_task(4, "_distance", alive=0.0),
    "legged2_alive10": _legged_task(2, "_alive10", alive=0.1),
    "legged2_fall": _legged_task(2, "_fall", alive=0.0, fall=20.0),
    "legged2_alive10_fall": _legged_task(2, "_alive10_fall", alive=0.1, fall=20.0),
    "legged4_alive10": _legged_task(4, "_alive10", alive=0.1),
    "legged2_gated": _legged_task(2, "_gated", alive=0.0, gate=0.85),
}


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


def n_params(hidden, task):
    return task.obs_dim * hidden + hidden + hidden * task.n_out + task.n_out


def unflatten(theta_pop, hidden, task):
    """(P, D) parameter rows to the four batched weight arrays of an obs-H-out MLP."""
    P, H, I, O = theta_pop.shape[0], hidden, task.obs_dim, task.n_out
    i = 0
    w1 = theta_pop[:, i:i + I * H].reshape(P, I, H); i += I * H
    b1 = theta_pop[:, i:i + H]; i += H
    w2 = theta_pop[:, i:i + H * O].reshape(P, H, O); i += H * O
    b2 = theta_pop[:, i:i + O]
    return w1, b1, w2, b2


def population_logits(xp, obs, params):
    """Every environment runs its own policy: one batched contraction per layer."""
    w1, b1, w2, b2 = params
    h = torch.tanh(torch.einsum("pi,pih->ph", obs, w1) + b1)
    return torch.einsum("ph,pho->po", h, w2) + b2


def push(xp, task, state, start_velocity):
    """The starting-push curriculum: add a forward velocity to every episode's initial state."""
    if not start_velocity or task.xdot_row is None:
        return state
    state = state.clone()
    state[task.xdot_row] += start_velocity
    return state


def curriculum(cfg, gen):
    """Assistance stiffness and starting push at generation `gen`, annealed linearly to zero by anneal_gens."""
    ramp = max(0.0, 1.0 - (gen - 1) / cfg.anneal_gens) if cfg.anneal_gens > 0 else 0.0
    return cfg.assist_k0 * ramp, cfg.start_velocity * ramp


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
    """(reward sum until first termination, steps taken) for each member, stepping the whole
    population once per iteration through the CUDA step kernel (es.py:174-193)."""
    task = backend.task
    P = params[0].shape[0]
    state = push(torch, task, backend.reset(P) if state is None else state, start_velocity)
    alive = torch.ones(P, dtype=torch.bool, device=state.device)
    fit = torch.zeros(P, device=state.device)
    steps = torch.zeros(P, device=state.device)
    for _ in range(horizon):
        action = task.action(torch, population_logits(torch, task.obs(torch, state), params))
        state, reward, done = backend.step(state, action, assist) if task.assistable else backend.step(state, action)
        steps = steps + alive.float()
        fell = alive & done
        alive = alive & ~done
        forward = (reward - 1.0) * (state[1] >= task.height_gate).float() if task.height_gate else reward - 1.0
        fit = fit + (forward + task.alive_bonus) * alive.float() - task.fall_penalty * fell.float()
    return fit, steps


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
        state = push(torch, self.task, self.reset(theta_pop.shape[0], gen, member_offset), start_velocity)
        if self.task.assistable:
            return self.task.rollout(state, theta_pop, hidden, horizon, assist)
        return self.task.rollout(state, theta_pop, hidden, horizon)

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
        state = self.reset(theta_pop.shape[0], gen, member_offset)
        return loop_fitness(self, unflatten(theta_pop, hidden, self.task), horizon, assist, start_velocity, state)


BACKENDS = {"metal": MetalBackend, "cuda": MetalBackend, "mlx": MLXBackend, "loop": MLXBackend}


def generation(backend, theta, cfg, hidden, gen=1):
    """One ES generation: perturb, roll out, rank, update (es.py:218-227)."""
    pairs = cfg.pop // 2
    offset, rows = backend.shard(cfg.pop)
    theta_pop = backend.perturb(theta, cfg.sigma, gen, pairs, offset, rows)
    assist, start_velocity = curriculum(cfg, gen)
    fit, steps = backend.rollout(theta_pop, hidden, cfg.horizon, assist, start_velocity, gen, offset)
    if backend.world > 1:
        both = backend.gather(torch.stack([fit.float(), steps.float()], dim=1))
        fit, steps = both[:, 0].contiguous(), both[:, 1].contiguous()
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
    """The unperturbed policy as an actor on (n, obs_dim) observations, on the GPU."""
    w1, b1, w2, b2 = (p[0] for p in unflatten(theta[None, :], hidden, task))
    return lambda obs: torch.tanh(obs @ w1 + b1) @ w2 + b2


def evaluate(task, actor, n=2048, steps=500):
    """Canonical score of a greedy actor over n fresh episodes (es.py:308-322): the environment's
    reward minus one plus task.eval_bonus, summed to the first termination, on the GPU."""
    state = task.mlx.reset(n)
    alive = torch.ones(n, dtype=torch.bool, device=state.device)
    fit = torch.zeros(n, device=state.device)
    for _ in range(steps):
        action = task.action(torch, actor(task.obs(torch, state)))
        state, reward, done = task.metal.step(state, action)
        alive = alive & ~done
        fit = fit + (reward - 1.0 + task.eval_bonus) * alive.float()
    return fit.mean().item()


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
    solved: bool
    generations: int
    env_steps: int        # steps actually taken: a member's episode ends at its first termination
    train_seconds: float  # training only; evaluation of the mean policy is outside the clock
    score: float


def train(cfg, backend_name, seed, log=lambda *_: None):
    assert cfg.pop % 2 == 0
    if backend_name not in BACKENDS:
        raise ValueError(f"backend {backend_name!r}: this build runs on the GPU only ({sorted(BACKENDS)}); "
                         "the numpy reference is the test oracle")
    task = TASKS[cfg.task]
    hidden = task.hidden if cfg.hidden is None else cfg.hidden
    solved_at = task.solved_at if cfg.solved_at is None else cfg.solved_at
    backend = BACKENDS[backend_name](task, seed)
    theta = backend.normal((n_params(hidden, task),)) * 0.1
    backend.sync(theta)
    train_seconds, env_steps, score, gen = 0.0, 0, 0.0, 0
    for gen in range(1, cfg.max_generations + 1):
        start = time.perf_counter()
        theta, fit, steps = generation(backend, theta, cfg, hidden, gen)
        train_seconds += time.perf_counter() - start
        env_steps += int(steps.sum().item())
        if backend.world > 1 and gen % CHECK_EVERY == 0:
            assert_ranks_agree(theta)
        score = evaluate_theta(task, theta, hidden)
        log(gen, env_steps, train_seconds, float(fit.mean().item()), score)
        if score >= solved_at:
            return Result(True, gen, env_steps, train_seconds, score)
        if train_seconds >= cfg.time_budget:
            break
    return Result(False, gen, env_steps, train_seconds, score)


def main():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--task", choices=TASKS, default="cartpole")
    p.add_argument("--pop", type=int, default=1024)
    p.add_argument("--backend", choices=BACKENDS, default="metal")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--lr", type=float, default=0.1)
    p.add_argument("--sigma", type=float, default=0.1)
    p.add_argument("--time-budget", type=float, default=120.0)
    p.add_argument("--max-generations", type=int, default=500)
    p.add_argument("--assist", type=float, default=0.0, help="torso-assist spring stiffness at generation 1, annealed to zero")
    p.add_argument("--start-velocity", type=float, default=0.0, help="forward push at episode start, annealed to zero")
    p.add_argument("--anneal", type=int, default=300, help="generation by which both curricula reach zero")
    args = p.parse_args()
    cfg = Config(task=args.task, pop=args.pop, lr=args.lr, sigma=args.sigma, time_budget=args.time_budget,
                 max_generations=args.max_generations, assist_k0=args.assist,
                 start_velocity=args.start_velocity, anneal_gens=args.anneal)
    result = train(
        cfg, args.backend, args.seed,
        log=lambda gen, es_, secs, fit, score: print(
            f"gen {gen:4d}  env_steps {es_:>13,}  train {secs:7.2f}s  pop fitness {fit:8.1f}  score {score:8.1f}", flush=True),
    )
    print(result)


if __name__ == "__main__":
    main()
