"""Steps/s sweeps over N and ES population sweeps, written in the reference's results/*.csv format.

The reference's bench scripts each sweep a batch size and write one CSV under results/
(bench.py:85-101, bench_acrobot.py:32-33, bench_hopper.py:73-74, bench_kernel.py:29-30,
bench_pendulum.py:121-133, bench_aba.py:117-123, bench_legged.py:74-82, bench_es.py:19-33 with
bench_ppo.write_csv :37-41). This module runs the same sweeps through this build's CUDA kernels
and writes files with the same names and columns, so B200 rows can sit beside the reference's:

    python metal-rl-envs_b200/bench_sweep.py steps --body cartpole     # results/steps_per_sec.csv
    python metal-rl-envs_b200/bench_sweep.py steps --body legged --cs 1 2 4
    python metal-rl-envs_b200/bench_sweep.py es --task acrobot --ns 1024 16384 --seeds 0 1

Timing follows the reference's rule (bench.py:3-12): steps/s = N x iterations / wall-clock
seconds of the timed loop, warm-up untimed, random actions drawn inside the timed loop on the
same device, the device drained before the clock stops, the median of the repeats. The
configurations are this build's: the step kernel synchronised every step (the reference's
"eval every step"), every `eval_every` steps (its lazy window), and for CartPole and Acrobot
the T-step kernel that runs the whole loop in one launch. Kernel-only device timings with the
roofline live in bench.py at the repository root; these are the reference-comparable ones.
"""

import argparse
import csv
import statistics
import sys
import time
from pathlib import Path

import torch

_HERE = Path(__file__).resolve().parent
if str(_HERE) not in sys.path:
    sys.path.insert(0, str(_HERE))

import rlenv_lib as _rl  # noqa: E402

RESULTS = Path("results")

# Column orders of the reference's files.
STEPS_COLUMNS = ["config", "n", "steps_per_sec", "iters", "warmup", "repeats"]            # bench.py:98
K_COLUMNS = ["k", "config", "n", "steps_per_sec", "iters", "warmup", "repeats"]           # bench_pendulum.py:131
LEGGED_COLUMNS = ["c", "config", "n", "steps_per_sec", "sweeps", "iters", "warmup", "repeats"]  # bench_legged.py:80
ES_COLUMNS = ["backend", "lr", "series", "n", "seed", "solved", "generations", "env_steps", "train_seconds",
              "score", "steps_per_sec"]                                                   # bench_es.py:27-28

# body -> (results file, extra key column or None)
STEP_FILES = {
    "cartpole": ("steps_per_sec.csv", None),
    "kernel": ("kernel.csv", None),
    "acrobot": ("acrobot.csv", None),
    "hopper": ("hopper.csv", None),
    "pendulum": ("pendulum.csv", "k"),
    "aba": ("aba.csv", "k"),
    "legged": ("legged.csv", "c"),
}


def _sync():
    torch.cuda.synchronize()


def kernel_rollout(body, n_actions, every):
    """The reference's rollout loop (bench.py:47-60) on this build's step: `iters` steps of N
    environments from a fresh reset, actions drawn on the device each step, the device drained
    every `every` steps and at the end."""
    dev = _rl.device()

    def run(n, iters):
        state = body.reset(n)
        for done_steps in range(iters):
            state, _, _ = body.step(state, torch.randint(0, n_actions, (n,), device=dev, dtype=torch.int32))
            if (done_steps + 1) % every == 0:
                _sync()
        _sync()
        return state

    return run


def chain_rollout(module, n_actions):
    """The same loop as one launch of the T-step kernel (`step_many`): all T x N actions drawn on
    the device, then every step, reward and done flag of the chain written by one kernel."""
    dev = _rl.device()

    def run(n, iters):
        state = module.reset(n)
        actions = torch.randint(0, n_actions, (iters, n), device=dev, dtype=torch.uint8)
        state = module.step_many(state, actions)[0]
        _sync()
        return state

    return run


def configs(body, eval_every, k=None, c=None, sweeps=None):
    """Config name -> rollout(n, iters) for one body, in the reference's naming style."""
    import acrobot_metal
    import cartpole_metal

    if body in ("cartpole", "kernel", "acrobot"):
        mod, n_act = (acrobot_metal, 3) if body == "acrobot" else (cartpole_metal, 2)
        return {
            "cuda kernel, sync every step": kernel_rollout(mod, n_act, 1),
            f"cuda kernel, sync every {eval_every}": kernel_rollout(mod, n_act, eval_every),
            "cuda T-step kernel, one launch": chain_rollout(mod, n_act),
        }
    if body == "hopper":
        import hopper_metal

        sel, br = hopper_metal.Hopper(), hopper_metal.Hopper(branchy=True)
        return {
            "cuda kernel, sync every step": kernel_rollout(sel, 3, 1),
            f"cuda kernel, sync every {eval_every}": kernel_rollout(sel, 3, eval_every),
            f"cuda branchy kernel, sync every {eval_every}": kernel_rollout(br, 3, eval_every),
            "cuda T-step kernel, one launch": chain_rollout(sel, 3),
        }
    if body == "pendulum":
        import pendulum_metal
        import pendulum_metal_coop

        mm, v9, co = pendulum_metal.Pendulum(k), pendulum_metal.Pendulum(k, pairwise_trig=True), pendulum_metal_coop.Pendulum(k)
        return {
            "cuda kernel, sync every step": kernel_rollout(mm, 3, 1),
            f"cuda kernel, sync every {eval_every}": kernel_rollout(mm, 3, eval_every),
            f"cuda cooperative kernel, sync every {eval_every}": kernel_rollout(co, 3, eval_every),
            f"cuda kernel (pairwise trig), sync every {eval_every}": kernel_rollout(v9, 3, eval_every),
            "cuda T-step kernel, one launch": chain_rollout(mm, 3),
            "cuda cooperative T-step kernel, one launch": chain_rollout(co, 3),
        }
    if body == "aba":
        import pendulum_aba_metal
        import pendulum_metal

        ab = pendulum_aba_metal.Pendulum(k)
        cfg = {
            "cuda articulated-body kernel, sync every step": kernel_rollout(ab, 3, 1),
            f"cuda articulated-body kernel, sync every {eval_every}": kernel_rollout(ab, 3, eval_every),
            "cuda articulated-body T-step kernel, one launch": chain_rollout(ab, 3),
        }
        if k <= 16:
            cfg[f"cuda mass-matrix kernel, sync every {eval_every}"] = kernel_rollout(pendulum_metal.Pendulum(k), 3, eval_every)
        return cfg
    if body == "legged":
        import legged_metal

        lg = legged_metal.Legged(c, sweeps)
        return {
            "cuda kernel, sync every step": kernel_rollout(lg, 3**c, 1),
            f"cuda kernel, sync every {eval_every}": kernel_rollout(lg, 3**c, eval_every),
            "cuda T-step kernel, one launch": chain_rollout(lg, 3**c),
        }
    raise ValueError(f"unknown body {body!r}; choose from {sorted(STEP_FILES)}")


def steps_per_sec(rollout, n, iters, warmup, repeats):
    """The reference's timing rule (bench.py:74-82): an untimed warm-up run, then the median
    wall-clock time of `repeats` runs of `iters` steps over N environments."""
    rollout(n, warmup)

    def timed_run():
        _sync()
        t0 = time.perf_counter()
        rollout(n, iters)
        return time.perf_counter() - t0

    return n * iters / statistics.median(timed_run() for _ in range(repeats))


def sweep(cfg, max_exp, iters, warmup, repeats, key=None, log=print):
    """Every config at N = 2^0 .. 2^max_exp (bench.py:85-93). `key` is an extra leading column
    such as {"k": 8} or {"c": 4}."""
    rows = []
    for name, rollout in cfg.items():
        for exp in range(max_exp + 1):
            n = 2**exp
            sps = steps_per_sec(rollout, n, iters, warmup, repeats)
            rows.append({**(key or {}), "config": name, "n": n, "steps_per_sec": round(sps)})
            log(f"{name:48s} N={n:>9d}  {sps:>16,.0f} steps/s")
    return rows


def write_steps_csv(rows, path, iters, warmup, repeats, sweeps=None):
    """The reference's writers: bench.py:96-101 (no key), bench_pendulum.py:129-133 and
    bench_aba.py:121-125 (k), bench_legged.py:78-82 (c, with the Gauss-Seidel sweeps)."""
    if rows and "c" in rows[0]:
        cols = LEGGED_COLUMNS
    elif rows and "k" in rows[0]:
        cols = K_COLUMNS
    else:
        cols = STEPS_COLUMNS
    fixed = {"iters": iters, "warmup": warmup, "repeats": repeats, "sweeps": sweeps}
    with open(path, "w", newline="") as out:
        table = csv.writer(out)
        table.writerow(cols)
        table.writerows([r.get(c, fixed.get(c)) for c in cols] for r in rows)


def write_dict_csv(rows, path):
    """The reference's ES writer (bench_ppo.py:37-41): a header of the first row's keys in
    their order, then one line per row."""
    columns = list(rows[0].keys())
    Path(path).parent.mkdir(parents=True, exist_ok=True)
    with open(path, "w", newline="") as out:
        writer = csv.writer(out)
        writer.writerow(columns)
        writer.writerows([row[c] for c in columns] for row in rows)


def es_sweep(task, ns, seeds, lrs, sigma, time_budget, assist=0.0, start_velocity=0.0, anneal=300,
             series="backend", backend="cuda", max_generations=None, log=print):
    """bench_es.py:19-33 through this build's ES loop: one row per (lr, population, seed)."""
    import es

    rows = []
    for lr in lrs:
        for pop in ns:
            for seed in seeds:
                extra = {} if max_generations is None else {"max_generations": max_generations}
                cfg = es.Config(task=task, pop=pop, lr=lr, sigma=sigma, time_budget=time_budget, assist_k0=assist,
                                start_velocity=start_velocity, anneal_gens=anneal, **extra)
                result = es.train(cfg, backend, seed)
                rate = result.env_steps / result.train_seconds
                rows.append({"backend": backend, "lr": lr, "series": backend if series == "backend" else f"lr {lr}",
                             "n": pop, "seed": seed, **vars(result), "steps_per_sec": rate})
                outcome = "solved" if result.solved else "not solved"
                log(f"{backend} lr={lr:g} P={pop} seed={seed}: {outcome} after {result.generations} generations, "
                    f"{result.train_seconds:.1f} s, {result.env_steps:,} env steps ({rate / 1e6:.1f} M/s), "
                    f"score {result.score:.1f}")
    return rows


def _parse(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--results", default=str(RESULTS), help="output folder (the reference writes results/)")
    sub = p.add_subparsers(dest="cmd", required=True)
    s = sub.add_parser("steps", help="steps/s over N = 2^0 .. 2^max_exp for one body")
    s.add_argument("--body", choices=sorted(STEP_FILES), default="cartpole")
    s.add_argument("--max-exp", type=int, default=None, help="default 20 (classic bodies) or 16 (the others)")
    s.add_argument("--iters", type=int, default=None, help="timed steps per run; default 256 or 64")
    s.add_argument("--warmup", type=int, default=None, help="untimed steps first; default 16 or 8")
    s.add_argument("--repeats", type=int, default=3)
    s.add_argument("--eval-every", type=int, default=32)
    s.add_argument("--ks", type=int, nargs="+", default=None, help="pendulum links; default 2 4 8 16 (aba: up to 64)")
    s.add_argument("--cs", type=int, nargs="+", default=[1, 2, 4], help="legs of the legged body")
    s.add_argument("--sweeps", type=int, default=8, help="Gauss-Seidel sweeps of the legged body")
    e = sub.add_parser("es", help="ES training runs over population sizes, seeds and learning rates")
    e.add_argument("--task", default="cartpole")
    e.add_argument("--ns", type=int, nargs="+", default=[64, 256, 1024, 4096, 16384, 65536])
    e.add_argument("--seeds", type=int, nargs="+", default=[0, 1, 2, 3, 4])
    e.add_argument("--lrs", type=float, nargs="+", default=[0.1])
    e.add_argument("--sigma", type=float, default=0.1)
    e.add_argument("--assist", type=float, default=0.0)
    e.add_argument("--start-velocity", type=float, default=0.0)
    e.add_argument("--anneal", type=int, default=300)
    e.add_argument("--series", choices=["backend", "lr"], default="backend")
    e.add_argument("--time-budget", type=float, default=300.0)
    e.add_argument("--max-generations", type=int, default=None)
    e.add_argument("--out", default=None, help="results file stem; default es or es_<task>")
    return p.parse_args(argv)


def main(argv=None):
    args = _parse(argv)
    out_dir = Path(args.results)
    out_dir.mkdir(parents=True, exist_ok=True)
    log = lambda s: print(s, flush=True)  # noqa: E731
    if args.cmd == "es":
        rows = es_sweep(args.task, args.ns, args.seeds, args.lrs, args.sigma, args.time_budget, args.assist,
                        args.start_velocity, args.anneal, args.series, max_generations=args.max_generations, log=log)
        stem = args.out or ("es" if args.task == "cartpole" else f"es_{args.task}")
        path = out_dir / f"{stem}.csv"
        write_dict_csv(rows, path)
        log(f"wrote {path}")
        return path
    classic = args.body in ("cartpole", "kernel", "acrobot", "hopper")
    max_exp = args.max_exp if args.max_exp is not None else (20 if classic else 16)
    iters = args.iters if args.iters is not None else (256 if classic else 64)
    warmup = args.warmup if args.warmup is not None else (16 if classic else 8)
    fname, key = STEP_FILES[args.body]
    rows = []
    if key is None:
        rows = sweep(configs(args.body, args.eval_every), max_exp, iters, warmup, args.repeats, log=log)
    elif key == "k":
        ks = args.ks or ([2, 4, 8, 16] if args.body == "pendulum" else [2, 4, 8, 16, 32, 64])
        for k in ks:
            log(f"--- K = {k}")
            rows += sweep(configs(args.body, args.eval_every, k=k), max_exp, iters, warmup, args.repeats, {"k": k}, log)
    else:
        for c in args.cs:
            log(f"--- C = {c}")
            rows += sweep(configs(args.body, args.eval_every, c=c, sweeps=args.sweeps), max_exp, iters, warmup,
                          args.repeats, {"c": c}, log)
    path = out_dir / fname
    write_steps_csv(rows, path, iters, warmup, args.repeats, args.sweeps)
    log(f"wrote {path}")
    return path


if __name__ == "__main__":
    main()
