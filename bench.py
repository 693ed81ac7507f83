"""Benchmark of the batched environment step on B200, one JSON line per run.

Workload: Acrobot batched step, N = 262,144 environments per
GPU, 1,000 environment steps per bench step, actions uniform over {0, 1, 2} drawn once
from a seeded generator and resident in HBM, initial state uniform in +-0.1.

One bench step is one launch of the T-step Acrobot kernel over the whole batch: the state
stays in registers for the 1,000 steps; every step reads one action byte per environment
and writes the reward (float32) and done flag (byte) of every environment to (T, N)
buffers, with the terminated environments reset from the in-kernel hash stream. Inputs
and outputs (262 MB of actions, 1.3 GB of rewards and flags per step) are larger than
the 126 MB L2, so nothing is served from L2 across steps.

  value  env steps/s of the whole job: N x 1000 x K x world / max-over-ranks device time
  e2e    the same metric through the public API (acrobot_metal.step_many) with host
         buffers: each step copies the state and the actions from pinned host memory and
         reads back the final state and the per-environment reward sum and done count
  roofline  the step kernel against the FP32 issue roofline (algorithmic flops from
         rlenv_flops.py over CUDA-event time; peak = cuBLAS SGEMM measured in this run,
         TF32 off) with the HBM view beside it
  cpu_baseline  the numpy oracle port of the reference's acrobot_np.step loop on the
         host cores (rank 0, N = 1 only), a bounded sample

`--impl reference` times the reference's CPU implementation of the path (the oracle
port of acrobot_np.step, the reference's own numpy code restated) on all host cores
and prints the same line with "impl": "reference".

Multi-GPU (torchrun): every rank steps its own 262,144 environments (global indices
offset by rank, so each rank draws its own resets); there is no collective on the data
path, only barriers and one max-reduction of the elapsed time. Weak scaling.
"""

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
PKG = ROOT / "metal-rl-envs_b200"
sys.path.insert(0, str(PKG))

N_ENVS = 262_144
T_STEPS = 1000
METRIC = "env steps/s"
WORKLOAD = "acrobot_batched_step"
# workload -> (config it measures, default N, default T)
NOMINAL_FP32_TFLOPS = 148 * 128 * 2 * 1.965e9 / 1e12  # 74.4: FMA lanes x 2 flops x max SM clock

WORKLOADS = {
    "acrobot_step": ("BASELINE configs[1]: Acrobot batched step", N_ENVS, T_STEPS),
    "cartpole_step": ("BASELINE configs[0]: CartPole batched step, T-step kernel", 131_072, T_STEPS),
    "cartpole_single": ("BASELINE configs[0]: CartPole single-step kernel, one launch per step, N past L2", 1 << 24, 20),
    "acrobot_single": ("BASELINE configs[1]: Acrobot single-step kernel, one launch per step, N past L2", 1 << 24, 20),
    "pendulum_aba": ("BASELINE configs[2]: K-link pendulum, articulated body", 65_536, 100),
    "pendulum_mm": ("BASELINE configs[2]: K-link pendulum, mass matrix", 65_536, 100),
    "pendulum_coop": ("BASELINE configs[2]: K-link pendulum, K lanes per env", 65_536, 100),
    "pendulum_aba_coop": ("BASELINE configs[2]: K-link pendulum, articulated body, one warp per env", 65_536, 100),
    "legged_step": ("BASELINE configs[3]: legged body with C contacts", N_ENVS, 50),
    "es_cartpole": ("BASELINE configs[4]: ES generation, CartPole P=4096 H=32 horizon 500", 4096, 500),
    "es_acrobot": ("BASELINE configs[4]: ES generation, Acrobot P=4096 H=32 horizon 500", 4096, 500),
    "es_legged4": ("BASELINE configs[4]: ES generation, legged4 P=16384 H=16 horizon 1000", 16_384, 1000),
    "es_ranks": ("es.py:214-215 centred ranks of P fitness values: sort kernel and counting kernel", 262_144, 1),
}


# The reference's own published numbers (Apple M3 Pro through Metal/MLX, listed in the build's
# baseline notes with their README.md / results/*.csv sources), keyed by the exact configuration
# they were measured on: vs_baseline is reported only for a line whose configuration matches.
PUBLISHED = {
    ("acrobot_step", 262_144): (1.123e9, "Acrobot step kernel, N = 262,144, M3 Pro (README.md:403)"),
    ("cartpole_step", 131_072): (1.133e9, "CartPole step kernel, N = 131,072, M3 Pro (README.md:307)"),
    ("cartpole_step", 1_048_576): (1.249e9, "CartPole step kernel, N = 1,048,576, M3 Pro (README.md:310)"),
    ("pendulum_mm", 256, 4): (4.44e6, "pendulum mass matrix K = 4, N = 256, M3 Pro (results/pendulum.csv)"),
    ("pendulum_mm", 65_536, 4): (298e6, "pendulum mass matrix K = 4, N = 65,536, M3 Pro (README.md:1127)"),
    ("pendulum_mm", 256, 16): (495e3, "pendulum mass matrix K = 16, N = 256, M3 Pro (results/pendulum.csv)"),
    ("pendulum_mm", 65_536, 16): (12.1e6, "pendulum mass matrix K = 16, N = 65,536, M3 Pro (README.md:1129)"),
    ("pendulum_coop", 256, 16): (643e3, "pendulum cooperative K = 16, N = 256, M3 Pro (README.md:1215)"),
    ("pendulum_coop", 65_536, 16): (4.33e6, "pendulum cooperative K = 16, N = 65,536, M3 Pro (README.md:1223)"),
    ("pendulum_aba", 256, 4): (3.48e6, "articulated body K = 4, N = 256, M3 Pro (results/aba.csv)"),
    ("pendulum_aba", 65_536, 4): (450e6, "articulated body K = 4, N = 65,536, M3 Pro (README.md:1295)"),
    ("pendulum_aba", 256, 16): (2.40e6, "articulated body K = 16, N = 256, M3 Pro (results/aba.csv)"),
    ("pendulum_aba", 65_536, 16): (68.2e6, "articulated body K = 16, N = 65,536, M3 Pro (README.md:1297)"),
    ("pendulum_aba", 256, 64): (713e3, "articulated body K = 64, N = 256, M3 Pro (results/aba.csv)"),
    ("pendulum_aba", 65_536, 64): (3.96e6, "articulated body K = 64, N = 65,536, M3 Pro (README.md:1301)"),
    ("legged_step", 65_536, 2, 8): (94.6e6, "legged C = 2, 8 sweeps, N = 65,536, M3 Pro (README.md:1685)"),
    ("legged_step", 65_536, 4, 4): (26.2e6, "legged C = 4, 4 sweeps, N = 65,536, M3 Pro (README.md:1609)"),
    ("legged_step", 65_536, 4, 8): (24.3e6, "legged C = 4, 8 sweeps, N = 65,536, M3 Pro (README.md:1610)"),
    ("legged_step", 65_536, 4, 16): (21.2e6, "legged C = 4, 16 sweeps, N = 65,536, M3 Pro (README.md:1611)"),
    ("legged_step", 262_144, 1, 1): (617e6, "hopper (C = 1, one sweep), N = 262,144, M3 Pro (README.md:1552)"),
}


def published(*key):
    """(value, source) of the reference's number for this exact configuration, or (None, None)."""
    return PUBLISHED.get(tuple(key), (None, None))


def parse():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--n", type=int, default=N_ENVS, help="environments per GPU")
    p.add_argument("--t", type=int, default=T_STEPS, help="environment steps per bench step")
    p.add_argument("--cpu-seconds", type=float, default=12.0, help="budget of the CPU baseline sample")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--workload", default="acrobot_step", choices=sorted(WORKLOADS),
                   help="acrobot_step is the default line (BASELINE.json configs[1]); the others measure "
                        "the remaining configs for the design record")
    p.add_argument("--k", type=int, default=16, help="pendulum links (pendulum workloads)")
    p.add_argument("--c", type=int, default=4, help="legs (legged workload)")
    p.add_argument("--iters", type=int, default=8, help="Gauss-Seidel sweeps (legged workload)")
    p.add_argument("--no-impulses", action="store_true", help="legged workload without the contact-impulse output")
    p.add_argument("--pop", type=int, default=None, help="ES population (es_* workloads)")
    p.add_argument("--horizon", type=int, default=None, help="ES horizon (es_* workloads)")
    return p.parse_args()


# ---- the CPU arm: the oracle port of the reference's numpy step loop ------------------------------

def _cpu_worker(args):
    """Step n environments of the numpy Acrobot (physics, termination, numpy-RNG reset: the shape of
    acrobot_np.step) for `steps` steps; returns the elapsed seconds."""
    n, steps, seed = args
    import os as _os

    _os.environ.setdefault("OMP_NUM_THREADS", "1")
    sys.path.insert(0, str(ROOT))
    from oracle import classic

    rng = np.random.default_rng(seed)
    state = rng.uniform(-0.1, 0.1, size=(4, n)).astype(np.float32)
    acts = rng.integers(0, 3, size=(steps, n))
    t0 = time.perf_counter()
    for t in range(steps):
        stepped = classic.acrobot_physics(state, acts[t])
        done = classic.acrobot_terminated(stepped)
        fresh = rng.uniform(-0.1, 0.1, size=(4, n)).astype(np.float32)
        state = np.where(done[None, :], fresh, stepped)
        classic.acrobot_reward(done)
    return time.perf_counter() - t0


def cpu_throughput(n, budget_s, processes):
    """(steps/s, sample description, cores) of the numpy step loop on `processes` host processes,
    the batch sharded across them, sized to about budget_s seconds of wall time."""
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    per = max(1, n // processes)
    # calibrate on one process with a short run
    probe = _cpu_worker((per, 3, 0))
    steps = max(3, min(T_STEPS, int(budget_s / max(probe / 3, 1e-6))))
    with ctx.Pool(processes) as pool:
        secs = pool.map(_cpu_worker, [(per, steps, r) for r in range(processes)])
    total = per * processes * steps
    sample = f"N={per * processes} environments ({processes} shards of {per}), {steps} steps, numpy {np.__version__}"
    return total / max(secs), sample, processes


def _steps_baseline(step, make, n, budget_s, label):
    """Single-thread env steps/s of an oracle step loop: one untimed warm-up step, then at least
    5 timed steps (more while the budget lasts) over n environments."""
    state, acts = make(n)
    state = step(state, acts(0), 0)
    t0, steps = time.perf_counter(), 0
    while steps < 5 or (time.perf_counter() - t0 < budget_s and steps < 1000):
        state = step(state, acts(steps + 1), steps + 1)
        steps += 1
    secs = time.perf_counter() - t0
    sample = f"{label}: N={n} environments, {steps} timed steps after 1 warm-up, numpy {np.__version__}, 1 thread"
    return {"value": n * steps / secs, "unit": "env steps/s", "cores": 1, "kind": "port", "sample": sample}


def cpu_workload_baseline(workload, args, n, budget_s=10.0):
    """The reference's numpy path for a bench workload, restated in oracle/ and timed on one host
    core over a bounded sample of the workload (the reference reports numpy single-threaded)."""
    sys.path.insert(0, str(ROOT))
    from oracle import es as oes
    from oracle import kernels, legged

    rng = np.random.default_rng(0)
    if workload in ("cartpole_step", "cartpole_single", "acrobot_single"):
        cp = workload.startswith("cartpole")
        fn, n_act, bound = (kernels.cartpole_step, 2, 0.05) if cp else (kernels.acrobot_step, 3, 0.1)
        make = lambda m: (rng.uniform(-bound, bound, (4, m)).astype(np.float32), lambda t: rng.integers(0, n_act, m))
        return _steps_baseline(lambda s, a, t: fn(s, a, 1 + t)[0], make, min(n, 131_072), budget_s,
                               "cartpole_np.step" if cp else "acrobot_np.step")
    if workload in ("pendulum_aba", "pendulum_aba_coop", "pendulum_mm", "pendulum_coop"):
        k, form = args.k, ("aba" if workload.startswith("pendulum_aba") else "mass_matrix")
        make = lambda m: (np.concatenate([rng.uniform(-0.1, 0.1, (k, m)), np.zeros((k, m))]).astype(np.float32),
                          lambda t: rng.integers(0, 3, m))
        return _steps_baseline(lambda s, a, t: kernels.pendulum_step(s, a, 1 + t, k, form=form)[0], make,
                               min(n, 4096), budget_s,
                               f"pendulum_{'aba_' if form == 'aba' else ''}np.Pendulum({k}).step")
    if workload == "legged_step":
        c, iters = args.c, args.iters
        stand = legged.stand_pose(c)[:, None]
        make = lambda m: ((stand + rng.uniform(-0.05, 0.05, (2 * (3 + c), m))).astype(np.float32),
                          lambda t: rng.integers(0, 3 ** c, m))
        return _steps_baseline(lambda s, a, t: kernels.legged_step(s, a, 1 + t, c, iters)[0], make,
                               min(n, 4096), budget_s, f"legged_np.Legged({c}, {iters}).step")
    # es_*: one generation of es.py's numpy backend at a bounded population and horizon
    task = {"es_cartpole": "cartpole", "es_acrobot": "acrobot", "es_legged4": "legged4"}[workload]
    spec = oes.TASKS[task]
    pop = min(args.pop or WORKLOADS[workload][1], 1024 if task != "legged4" else 256)
    horizon = min(args.horizon or WORKLOADS[workload][2], 500 if task != "legged4" else 100)
    cfg = oes.Config(task=task, pop=pop, horizon=horizon, sigma=0.1, lr=0.03)
    theta = rng.normal(size=(oes.n_params(spec.hidden, spec),)).astype(np.float32) * 0.1
    oes.generation(spec, theta, cfg, spec.hidden, rng, 1)  # warm-up
    t0, gens, taken = time.perf_counter(), 0, 0.0
    while gens < 1 or (time.perf_counter() - t0 < budget_s and gens < 20):
        theta, _, steps = oes.generation(spec, theta, cfg, spec.hidden, rng, gens + 2)
        taken += float(steps.sum())
        gens += 1
    secs = time.perf_counter() - t0
    return {"value": taken / secs, "unit": "env steps/s (steps taken)", "cores": 1, "kind": "port",
            "ms_per_generation_of_sample": 1e3 * secs / gens,
            "sample": f"es.generation, numpy backend: P={pop}, horizon {horizon}, {gens} timed generations "
                      f"after 1 warm-up, numpy {np.__version__}, 1 thread"}


def default_config(n, T, world):
    """The default line's workload, printed identically by both arms."""
    return {"workload": WORKLOAD, "n_envs_per_gpu": n, "env_steps_per_step": T,
            "actions": "uniform over {0, 1, 2}, seeded", "state0": "uniform in +-0.1, seeded",
            "parallelism": f"env-sharded x{world}, no data-path collective"}


def _ref_step_fn():
    """(step(state, action, rng) -> (next, reward, done), kind): the reference's own
    acrobot_np.step where an install of the reference is importable (baseline/_ref), else the
    oracle's restatement of it."""
    ref = ROOT / "baseline" / "_ref"
    if (ref / "acrobot_np.py").exists():
        sys.path.insert(0, str(ref))
        try:
            import acrobot_np

            return acrobot_np.step, "reference"
        except Exception:
            pass
    sys.path.insert(0, str(ROOT))
    from oracle import classic

    def step(state, action, rng):
        stepped = classic.acrobot_physics(state, action)
        done = classic.acrobot_terminated(stepped)
        fresh = rng.uniform(-0.1, 0.1, size=state.shape).astype(np.float32)
        return np.where(done[None, :], fresh, stepped), classic.acrobot_reward(done), done
    return step, "port"


def _ref_worker(args):
    """Step a shard of n environments of the numpy Acrobot `steps` times (the shape of the
    reference's bench loop: actions drawn inside the loop); returns the elapsed seconds."""
    n, steps, seed = args
    os.environ.setdefault("OMP_NUM_THREADS", "1")
    step, _ = _ref_step_fn()
    rng = np.random.default_rng(seed)
    state = rng.uniform(-0.1, 0.1, size=(4, n)).astype(np.float32)
    t0 = time.perf_counter()
    for _ in range(steps):
        state, _, _ = step(state, rng.integers(0, 3, size=n), rng)
    return time.perf_counter() - t0


def run_reference(args):
    """The reference's CPU implementation of the path on every host core: the batch sharded over
    one process per core, each bench step a bounded sample of the workload (the same N, fewer
    environment steps), K timed steps after W warm-up steps, sized to finish in about
    --cpu-seconds."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import multiprocessing as mp

    cores = len(os.sched_getaffinity(0))
    n = args.n
    per = max(1, n // cores)
    _, kind = _ref_step_fn()
    probe = _ref_worker((per, 2, 0)) / 2  # seconds per step of one shard
    budget = max(args.cpu_seconds, 5.0) / max(1, args.steps + args.warmup)
    sample_steps = int(max(1, min(args.t, budget / max(probe, 1e-6))))
    secs = []
    with mp.get_context("spawn").Pool(cores) as pool:
        for k in range(args.warmup + args.steps):
            t0 = time.perf_counter()
            pool.map(_ref_worker, [(per, sample_steps, 1000 * k + r) for r in range(cores)])
            if k >= args.warmup:
                secs.append(time.perf_counter() - t0)
    total = per * cores * sample_steps
    value = total * len(secs) / sum(secs)
    sample = (f"{'acrobot_np.step (the reference, baseline/_ref)' if kind == 'reference' else 'acrobot_np.step restated in oracle/'}: "
              f"N={per * cores} environments in {cores} shards, {sample_steps} environment steps per bench step, "
              f"numpy {np.__version__}, one process per core")
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "env steps/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * n * args.t / value,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded uniform states and actions)",
            "config": default_config(n, args.t, args.gpus),
            "cpu_baseline": {"value": value, "unit": "env steps/s", "cores": cores, "kind": kind, "sample": sample},
            "e2e": {"value": value, "unit": "env steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "timing": "wall clock over the K timed bench steps; ms_per_step is the time of a full step "
                      "(N x env_steps_per_step) at the measured rate"}
    print(json.dumps(line), flush=True)


# ---- GPU helpers ---------------------------------------------------------------------------------

class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons while the timed region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.rows = []
        self._stop = threading.Event()
        self._thread = None

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                                      "--format=csv,noheader,nounits"], capture_output=True, text=True, timeout=5)
                for line in out.stdout.strip().splitlines():
                    self.rows.append([x.strip() for x in line.split(",")])
            except Exception:
                return
            self._stop.wait(0.2)

    def __enter__(self):
        self._thread = threading.Thread(target=self._run, daemon=True)
        self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        self._thread.join(timeout=10)

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if len(r) > 5 + i and "Active" in r[5 + i]
                          and "Not" not in r[5 + i]})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(self.rows[0][2]) if self.rows[0][2].replace(".", "").isdigit() else None,
                "reasons": reasons, "samples": len(self.rows)}


def measured_sgemm_tflops(torch):
    """cuBLAS fp32 GEMM throughput with TF32 off: the measured FP32 FMA ceiling used for the roofline."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        n = 8192
        a = torch.randn(n, n, device="cuda")
        b = torch.randn(n, n, device="cuda")
        a @ b
        torch.cuda.synchronize()
        best = float("inf")
        for _ in range(3):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            a @ b
            e.record()
            e.synchronize()
            best = min(best, s.elapsed_time(e) / 1e3)
        return 2 * n ** 3 / best / 1e12
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def hbm_peak_gbs():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        return float(json.loads(path.read_text())["hbm_gbs"]), "measured (MEASURED_PEAKS.json)"
    return 6650.0, "fallback"


def north_star_records(torch, dist, world, rank, local, dev, sgemm):
    """Sub-records of the default run: the north star's other figures, each timed here with CUDA
    events over its own region (warm-up untimed, max over ranks). Every rank runs every record in
    the same order (the ES record's all-gather and the barriers are collectives).
    - cartpole_fused_n1m: CartPole, N = 1,048,576 per GPU, 1,000 steps per launch (T-step kernel,
      per-step rewards and done flags to HBM); target 1e9 env-steps/s per GPU.
    - cartpole_single_n16m: the drop-in single step at N = 2^24 per GPU, 20 launches per CUDA graph,
      41 B per env-step streamed (int32 actions): against measured HBM bandwidth.
    - acrobot_single_like_reference: the reference's published configuration (README.md:403):
      N = 262,144, one step kernel launch per step, actions drawn on the device every step, 32
      steps per CUDA graph (the reference evaluates every 32); vs_baseline against its 1.123e9.
    - legged4_step: C = 4, 8 sweeps, N = 262,144 per GPU, 50 steps per launch, states, rewards,
      fall flags and contact impulses out: against the FP32 rate.
    - es_legged4: one ES generation (perturb, rollout, ranks, update), P = 16,384 split over the
      ranks (strong scaling), horizon 1,000, H = 16, sigma 0.1, lr 0.03; with more than one rank
      also es_legged4_weak, P = 16,384 per rank."""
    import es
    import legged_metal
    import rlenv_flops
    import rlenv_lib as rl

    lib = rl.load()
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream
    g = torch.Generator(device=dev).manual_seed(777 + rank)
    hbm, hbm_kind = hbm_peak_gbs()
    out = {}

    def timed(fn, steps, warmup):
        return _timed(torch, dist, world, stream, fn, steps, warmup, local)

    def fp32(flops_per_s):
        return {"achieved_tflops": flops_per_s / 1e12, "peak_tflops": sgemm,
                "frac": flops_per_s / 1e12 / sgemm if sgemm else None, "peak_kind": "cuBLAS SGEMM, TF32 off, this run"}

    # CartPole fused
    n, T = 1 << 20, 1000
    acts = torch.randint(0, 2, (T, n), device=dev, generator=g).to(torch.uint8)
    s0 = rl.reset_uniform(4, n, 0.05, seed=7, index_offset=rank * n, dev=dev)
    s1 = torch.empty_like(s0)
    rew, dn = torch.empty((T, n), device=dev), torch.empty((T, n), device=dev, dtype=torch.bool)
    secs, clk = timed(lambda: rl.check(lib.cartpole_step_many(s0.data_ptr(), acts.data_ptr(), rl.U8, 1, T, n, rank * n,
                                                              s1.data_ptr(), rew.data_ptr(), dn.data_ptr(), 0, 0, sp)), 5, 3)
    v = n * T * 5 / secs
    out["cartpole_fused_n1m"] = {"value": v * world, "unit": "env steps/s", "per_gpu": v, "target_per_gpu": 1e9,
                                 "n_envs_per_gpu": n, "env_steps_per_launch": T, "launches": 5, "ms_per_launch": 1e3 * secs / 5,
                                 "fp32": fp32(v * rlenv_flops.CARTPOLE["flops"]), "sm_mhz": clk["sm_mhz"]}
    del acts, s0, s1, rew, dn

    # CartPole and Acrobot single steps
    def singles(env, n, T, dtype, sample_on_device):
        n_act = 2 if env == "cartpole" else 3
        abi = getattr(lib, f"{env}_step")
        acts = (torch.empty((T, n), device=dev, dtype=torch.int32) if sample_on_device else
                torch.randint(0, n_act, (T, n), device=dev, generator=g, dtype=torch.int32))
        sa = rl.reset_uniform(4, n, 0.05 if env == "cartpole" else 0.1, seed=7, index_offset=rank * n, dev=dev)
        sb = torch.empty_like(sa)
        rew, dn = torch.empty((T, n), device=dev), torch.empty((T, n), device=dev, dtype=torch.bool)

        def one(t):
            if sample_on_device:
                acts[t].random_(0, n_act)
            src, dst = (sa, sb) if t % 2 == 0 else (sb, sa)
            rl.check(abi(src.data_ptr(), acts[t].data_ptr(), rl.I32, 1 + t, n, rank * n, dst.data_ptr(),
                         rew[t].data_ptr(), dn[t].data_ptr(), torch.cuda.current_stream().cuda_stream))
        graph = _graph_steps(torch, one, T)
        secs, clk = timed(graph.replay, 3, 3)
        del graph
        return n * T * 3 / secs, secs / 3, clk

    v, per, clk = singles("cartpole", 1 << 24, 20, torch.int32, False)
    gbs = v * rlenv_flops.step_bytes(4, 4) / 1e9
    out["cartpole_single_n16m"] = {"value": v * world, "unit": "env steps/s", "per_gpu": v, "n_envs_per_gpu": 1 << 24,
                                   "launches_per_graph": 20, "bytes_per_env_step": rlenv_flops.step_bytes(4, 4),
                                   "hbm": {"achieved_gbs": gbs, "peak_gbs": hbm, "frac": gbs / hbm, "peak_kind": hbm_kind},
                                   "sm_mhz": clk["sm_mhz"]}
    v, per, clk = singles("acrobot", 262_144, 32, torch.int32, True)
    pub, src = published("acrobot_step", 262_144)
    out["acrobot_single_like_reference"] = {
        "value": v * world, "unit": "env steps/s", "per_gpu": v, "n_envs_per_gpu": 262_144, "launches_per_graph": 32,
        "actions": "drawn on the device every step (torch random_, inside the graph), as the reference's bench does",
        "vs_baseline": v / pub, "vs_baseline_source": src, "sm_mhz": clk["sm_mhz"],
        "gpu_launches_per_step": 1}

    # legged4 step with contact impulses
    c, iters, n, T = 4, 8, 262_144, 50
    stand = torch.from_numpy(legged_metal.stand_pose(c)).to(dev)
    la = rl.reset_uniform(2 * (3 + c), n, 0.05, center=stand, seed=3, index_offset=rank * n, dev=dev)
    lb = torch.empty_like(la)
    acts = torch.randint(0, 3 ** c, (T, n), device=dev, generator=g).to(torch.uint8)
    rew, dn = torch.empty((T, n), device=dev), torch.empty((T, n), device=dev, dtype=torch.bool)
    imp = torch.empty((T, 2 * c, n), device=dev)
    secs, clk = timed(lambda: rl.check(lib.legged_step_many(c, iters, la.data_ptr(), acts.data_ptr(), rl.U8, 1,
                                                            stand.data_ptr(), 0.0, None, T, n, rank * n, lb.data_ptr(),
                                                            rew.data_ptr(), dn.data_ptr(), imp.data_ptr(), sp)), 5, 3)
    v = n * T * 5 / secs
    fl = rlenv_flops.legged_flops(c, iters)["flops"]
    out["legged4_step"] = {"value": v * world, "unit": "env steps/s", "per_gpu": v, "legs": c, "sweeps": iters,
                           "n_envs_per_gpu": n, "env_steps_per_launch": T, "impulses": True,
                           "flops_per_env_step": fl, "fp32": fp32(v * fl),
                           "flops_per_env_step_reference_algorithm": rlenv_flops.legged_reference_flops(c, iters)["flops"],
                           "sm_mhz": clk["sm_mhz"]}
    del la, lb, acts, rew, dn, imp

    # legged4 ES generation
    def es_record(pop):
        task = es.TASKS["legged4"]
        cfg = es.Config(task="legged4", pop=pop, horizon=1000, sigma=0.1, lr=0.03)
        backend = es.MetalBackend(task, 0)
        st = {"theta": backend.normal((es.n_params(task.hidden, task),)) * 0.1, "gen": 0, "taken": 0.0}

        def gen():
            st["gen"] += 1
            st["theta"], _, steps = es.generation(backend, st["theta"], cfg, task.hidden, st["gen"])
            st["taken"] += float(steps.sum().item())
        for _ in range(3):
            gen()
        st["taken"] = 0.0
        secs, clk = timed(gen, 5, 0)
        taken = st["taken"] / 5 * world  # every rank's shard takes about as many steps as rank 0's
        fl = rlenv_flops.es_member_step_flops("legged4")["flops"]
        return {"value": 1e3 * secs / 5, "unit": "ms per generation", "higher_is_better": False, "population": pop,
                "horizon": 1000, "hidden": task.hidden, "generations": 5, "after_generations": 3,
                "member_steps_taken_per_generation": taken, "member_steps_nominal": pop * 1000,
                "env_steps_per_s": taken / (secs / 5), "fp32_steps_taken": fp32(taken / (secs / 5) * fl),
                "sm_mhz": clk["sm_mhz"]}
    out["es_legged4"] = {**es_record(16_384), "scaling": "strong (P split over the ranks, one all-gather per generation)"}
    if world > 1:
        out["es_legged4_weak"] = {**es_record(16_384 * world), "scaling": "weak (P = 16,384 per rank)"}
    return out


def _cpulist(text):
    cpus = set()
    for part in text.strip().split(","):
        if "-" in part:
            a, b = part.split("-")
            cpus.update(range(int(a), int(b) + 1))
        elif part:
            cpus.add(int(part))
    return cpus


def pin_to_gpu_numa(torch, dev):
    """Run this process on the CPUs next to the GPU (its PCI device's local_cpulist), so that the
    pinned host buffers of the e2e run are allocated on the GPU's NUMA node: host-to-device copies
    from a remote node ran at half the bandwidth. Returns what was done, for the JSON line."""
    try:
        p = torch.cuda.get_device_properties(dev)
        path = Path(f"/sys/bus/pci/devices/{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0/local_cpulist")
        cpus = _cpulist(path.read_text()) & set(os.sched_getaffinity(0))
        if not cpus:
            return "no local CPUs found; affinity unchanged"
        os.sched_setaffinity(0, cpus)
        return f"pinned to the {len(cpus)} CPUs local to the GPU before allocating pinned buffers"
    except Exception as e:  # no sysfs entry, or affinity not settable
        return f"affinity unchanged ({type(e).__name__})"


def run_ours(args):
    import torch
    import torch.distributed as dist

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    import acrobot_metal
    import rlenv_flops
    import rlenv_lib as rl

    lib = rl.load()
    n, T = args.n, args.t
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    actions = torch.randint(0, 3, (T, n), device=dev, generator=g, dtype=torch.int64).to(torch.uint8)
    state0 = rl.reset_uniform(4, n, 0.1, seed=99, index_offset=rank * n, dev=dev)
    state = torch.empty_like(state0)
    rew = torch.empty((T, n), device=dev)
    dn = torch.empty((T, n), device=dev, dtype=torch.bool)
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream
    off = rank * n

    def launch(seed0):
        rl.check(lib.acrobot_step_many(state0.data_ptr(), actions.data_ptr(), rl.U8, seed0, T, n, off, state.data_ptr(),
                                       rew.data_ptr(), dn.data_ptr(), 0, 0, sp))

    def barrier():
        if world > 1:
            dist.barrier()

    for w in range(args.warmup):
        launch(1 + w * T)
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        start.record(stream)
        for k in range(args.steps):
            launch(1 + (args.warmup + k) * T)
        end.record(stream)
        torch.cuda.synchronize()
    barrier()
    secs = start.elapsed_time(end) / 1e3
    t = torch.tensor([secs], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    secs_max = float(t.item())
    per_launch = secs / args.steps
    value = world * n * T * args.steps / secs_max

    # ---- e2e through the public API with host buffers ---------------------------------------------
    # Each step's state and actions come from pinned host memory and its final state, reward sum
    # and done count go back to pinned host memory. Two steps are in flight: the copy stream moves
    # step k+1's inputs while the compute stream runs step k (two device input buffers), which is
    # how a caller streaming batches from the host would drive acrobot_metal.step_many.
    # The actions stream packed along time (rlenv_lib.pack_actions: four steps to a byte, two bits
    # each), which step_many takes as PackedActions: 65.5 MB per step instead of 262 MB of uint8.
    # The uint8 stream is timed the same way beside it and reported in the e2e record.
    numa = pin_to_gpu_numa(torch, dev)
    pin_state = state0.cpu().pin_memory()
    packed_bits = rl.pack_actions(actions).bits
    outs = [(torch.empty((4, n), pin_memory=True), torch.empty(n, pin_memory=True), torch.empty(n, pin_memory=True))
            for _ in range(2)]
    copy_s, comp_s, back_s = torch.cuda.Stream(dev), torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    keep = [None, None]

    def e2e_time(host_actions, packed):
        pin_actions = host_actions.cpu().pin_memory()
        dev_in = [(torch.empty_like(state0), torch.empty_like(host_actions, device=dev)) for _ in range(2)]
        as_input = (lambda bits: rl.PackedActions(bits, T)) if packed else (lambda a: a)

        def e2e_run(steps):
            # three streams: inputs in (copy_s), the T steps (comp_s), results out (back_s), so that
            # neither copy waits for the other direction or delays the next launch
            h2d_done = [torch.cuda.Event() for _ in range(2)]
            comp_done = [torch.cuda.Event() for _ in range(2)]
            for k in range(steps + 1):
                b = k % 2
                if k < steps:
                    with torch.cuda.stream(copy_s):
                        if k >= 2:
                            copy_s.wait_event(comp_done[b])  # input buffer b is free once step k-2 ran
                        dev_in[b][0].copy_(pin_state, non_blocking=True)
                        dev_in[b][1].copy_(pin_actions, non_blocking=True)
                        h2d_done[b].record(copy_s)
                if k >= 1:  # launch step k-1, then queue its read-back
                    pb = (k - 1) % 2
                    with torch.cuda.stream(comp_s):
                        comp_s.wait_event(h2d_done[pb])
                        res = acrobot_metal.step_many(dev_in[pb][0], as_input(dev_in[pb][1]), rewards=False,
                                                      dones=False, sums=True)
                        comp_done[pb].record(comp_s)
                    with torch.cuda.stream(back_s):
                        back_s.wait_event(comp_done[pb])
                        for t_out, t_dev in zip(outs[pb], (res[0], res[3], res[4])):
                            t_dev.record_stream(back_s)
                            t_out.copy_(t_dev, non_blocking=True)
                        keep[pb] = res

        e2e_run(max(4, args.warmup))
        torch.cuda.synchronize()
        barrier()
        steps = max(20, args.steps // 10)
        torch.cuda.synchronize()
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s2.record(copy_s)
        e2e_run(steps)
        back_s.wait_stream(copy_s)
        back_s.wait_stream(comp_s)
        e2.record(back_s)
        torch.cuda.synchronize()
        barrier()
        t2 = torch.tensor([s2.elapsed_time(e2) / 1e3], device=dev)
        if world > 1:
            dist.all_reduce(t2, op=dist.ReduceOp.MAX)
        return world * n * T * steps / float(t2.item()), steps, pin_actions.numel() * pin_actions.element_size()

    e2e_value, e2e_steps, e2e_action_bytes = e2e_time(packed_bits, True)
    e2e_u8_value, _, e2e_u8_action_bytes = e2e_time(actions, False)

    # ---- roofline of the step kernel -----------------------------------------------------------------
    flops = rlenv_flops.ACROBOT["flops"] * n * T
    sgemm = measured_sgemm_tflops(torch) if rank == 0 else None
    bytes_per_launch = rlenv_flops.step_many_bytes(4, n, T, 1, True)
    hbm, hbm_kind = hbm_peak_gbs()
    clock_summary = clocks.summary()
    subs = north_star_records(torch, dist, world, rank, local, dev, sgemm)

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        v, sample, cores = cpu_throughput(n, args.cpu_seconds, 1)
        cpu = {"value": v, "unit": "env steps/s", "cores": cores, "kind": "port",
               "sample": sample + " (single thread, as the reference reports numpy)"}
    achieved = flops / per_launch / 1e12
    line = {
        "metric": METRIC, "value": value, "unit": "env steps/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * secs_max / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "vs_baseline_note": "the reference publishes no fused multi-step figure; its single-step kernel figure "
                            "is compared on north_star.acrobot_single_like_reference",
        "dtype": "f32", "data": "synthetic (seeded uniform states, uniform actions in {0,1,2})",
        "config": default_config(n, T, world),
        "kernel": "rlenv_acrobot_step_many: T steps per launch, state in registers, uint8 actions resident in "
                  "HBM, per-step rewards and done flags written to HBM",
        "l2": "inputs and outputs larger than L2 (actions 262 MB, rewards and done flags 1.3 GB per step)",
        "roofline": {"bound": "fp32", "achieved": achieved, "peak": sgemm, "unit": "TFLOP/s",
                     "frac": achieved / sgemm if sgemm else None,
                     "peak_kind": "cuBLAS SGEMM (TF32 off) measured in this run; nominal FP32 FMA 74.4 TFLOP/s",
                     "flops_per_env_step": rlenv_flops.ACROBOT["flops"],
                     "transcendentals_per_env_step": rlenv_flops.ACROBOT["transcendentals"],
                     "traffic": None, "algorithmic_bytes_per_launch": bytes_per_launch,
                     "traffic_note": "DRAM bytes per launch are an ncu figure, kept in profiles/ (not read here)",
                     "hbm": {"achieved": bytes_per_launch / per_launch / 1e9, "peak": hbm, "unit": "GB/s",
                             "frac": bytes_per_launch / per_launch / 1e9 / hbm, "peak_kind": hbm_kind},
                     "launch_ms": per_launch * 1e3},
        "cpu_baseline": cpu,
        "e2e": {"value": e2e_value, "unit": "env steps/s", "h2d_bytes_per_step": 4 * 4 * n + e2e_action_bytes,
                "d2h_bytes_per_step": 4 * 4 * n + 8 * n, "api": "acrobot_metal.step_many(state, PackedActions)",
                "actions": "packed along time, four steps to a byte (rlenv_lib.pack_actions), streamed from pinned "
                           "host memory",
                "steps": e2e_steps, "pipelined": "input, compute and output streams, two steps in flight", "host": numa,
                "uint8_actions": {"value": e2e_u8_value, "h2d_bytes_per_step": 4 * 4 * n + e2e_u8_action_bytes,
                                  "api": "acrobot_metal.step_many"}},
        "gpu_launches": args.steps,
        "clocks": clock_summary,
        "north_star": subs,
    }
    print(json.dumps(line), flush=True)


# ---- the other configurations --------------------------------------------------------------------

def _setup_dist(torch):
    import torch.distributed as dist

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=dev)
    return dist, rank, world, local, dev


def _timed(torch, dist, world, stream, fn, steps, warmup, local):
    """Run fn() warmup times, then time `steps` calls with CUDA events on `stream` inside
    barriers; returns (max-over-ranks seconds, clock summary)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        a.record(stream)
        for _ in range(steps):
            fn()
        b.record(stream)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t = torch.tensor([a.elapsed_time(b) / 1e3], device=stream.device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item()), clocks.summary()


def _graph_steps(torch, launch_one, T):
    """A CUDA graph of T single-step launches (launch_one(t) enqueues step t on the current
    stream): one replay runs T per-step kernel launches without host overhead."""
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for t in range(T):  # warm the launches once outside the capture
            launch_one(t)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    with torch.cuda.graph(g):
        for t in range(T):
            launch_one(t)
    torch.cuda.synchronize()
    return g


def run_workload(args):
    import torch

    import rlenv_flops
    import rlenv_lib as rl

    dist, rank, world, local, dev = _setup_dist(torch)
    lib = rl.load()
    desc, n_def, t_def = WORKLOADS[args.workload]
    n = args.n if args.n != N_ENVS else n_def
    T = args.t if args.t != T_STEPS else t_def
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream
    g = torch.Generator(device=dev).manual_seed(4321 + rank)
    extra = {}
    hbm_bound = False
    sgemm = measured_sgemm_tflops(torch) if rank == 0 else None
    if args.workload == "cartpole_step":
        actions = torch.randint(0, 2, (T, n), device=dev, generator=g).to(torch.uint8)
        s0 = rl.reset_uniform(4, n, 0.05, seed=7, index_offset=rank * n, dev=dev)
        s1 = torch.empty_like(s0)
        rew, dn = torch.empty((T, n), device=dev), torch.empty((T, n), device=dev, dtype=torch.bool)

        def fn():
            rl.check(lib.cartpole_step_many(s0.data_ptr(), actions.data_ptr(), rl.U8, 1, T, n, rank * n,
                                            s1.data_ptr(), rew.data_ptr(), dn.data_ptr(), 0, 0, sp))
        units, unit, metric, flops = n * T, "env steps/s", METRIC, rlenv_flops.CARTPOLE["flops"]
        bytes_launch = rlenv_flops.step_many_bytes(4, n, T)
    elif args.workload in ("cartpole_single", "acrobot_single"):
        # The drop-in single step (cartpole_metal.step / acrobot_metal.step): state in, next state,
        # reward and done out, int32 actions as the reference draws them; N is large enough that
        # every step streams 688 MB through HBM, far past the 126 MB L2.
        env = args.workload.split("_")[0]
        n_act = 2 if env == "cartpole" else 3
        abi = getattr(lib, f"{env}_step")
        actions = torch.randint(0, n_act, (T, n), device=dev, generator=g, dtype=torch.int32)
        state_a = rl.reset_uniform(4, n, 0.05, seed=7, index_offset=rank * n, dev=dev)
        state_b = torch.empty_like(state_a)
        rew, dn = torch.empty((T, n), device=dev), torch.empty((T, n), device=dev, dtype=torch.bool)

        def launch_one(t):
            src, dst = (state_a, state_b) if t % 2 == 0 else (state_b, state_a)
            rl.check(abi(src.data_ptr(), actions[t].data_ptr(), rl.I32, 1 + t, n, rank * n, dst.data_ptr(),
                         rew[t].data_ptr(), dn[t].data_ptr(), torch.cuda.current_stream().cuda_stream))
        graph = _graph_steps(torch, launch_one, T)

        def fn():
            graph.replay()
        units, unit, metric = n * T, "env steps/s", METRIC
        flops = (rlenv_flops.CARTPOLE if env == "cartpole" else rlenv_flops.ACROBOT)["flops"]
        bytes_launch = n * T * rlenv_flops.step_bytes(4, 4)
        extra = {"action_dtype": "int32", "bytes_per_env_step": rlenv_flops.step_bytes(4, 4),
                 "l2": "state, actions and outputs (688 MB per step at N = 2^24) exceed L2"}
        hbm_bound = True
    elif args.workload in ("pendulum_aba", "pendulum_aba_coop", "pendulum_mm", "pendulum_coop", "legged_step"):
        if args.workload == "legged_step":
            c = args.c
            rows, n_act = 2 * (3 + c), 3 ** c
            import legged_metal

            stand = torch.from_numpy(legged_metal.stand_pose(c)).to(dev)
            state_a = rl.reset_uniform(rows, n, 0.05, center=stand, seed=3, index_offset=rank * n, dev=dev)

            # BASELINE's legged outputs per step: state, contact impulses and the fall flag
            imp = torch.empty((T, 2 * c, n), device=dev) if not args.no_impulses else None

            def launch_many(src, dst, r, d):
                rl.check(lib.legged_step_many(c, args.iters, src.data_ptr(), actions.data_ptr(), rl.U8, 1,
                                              stand.data_ptr(), 0.0, None, T, n, rank * n, dst.data_ptr(),
                                              r.data_ptr(), d.data_ptr(), rl.ptr(imp), sp))
            fl = rlenv_flops.legged_flops(c, args.iters)["flops"]
            extra = {"legs": c, "sweeps": args.iters, "impulses": imp is not None,
                     "flops_per_env_step_reference_algorithm": rlenv_flops.legged_reference_flops(c, args.iters)["flops"]}
        else:
            k = args.k
            rows, n_act = 2 * k, 3
            state_a = rl.reset_uniform(rows, n, 0.1, seed=3, index_offset=rank * n, dev=dev)
            fn_name = {"pendulum_aba": "pendulum_aba_step_many", "pendulum_mm": "pendulum_mm_step_many",
                       "pendulum_coop": "pendulum_coop_step_many",
                       "pendulum_aba_coop": "pendulum_aba_coop_step_many"}[args.workload]
            head = (k, 0) if args.workload == "pendulum_mm" else (k,)
            abi = getattr(lib, fn_name)

            def launch_many(src, dst, r, d):
                rl.check(abi(*head, src.data_ptr(), actions.data_ptr(), rl.U8, 1, T, n, rank * n, dst.data_ptr(),
                             r.data_ptr(), d.data_ptr(), sp))
            aba = args.workload.startswith("pendulum_aba")
            fl = (rlenv_flops.aba_flops(k) if aba else rlenv_flops.mass_matrix_flops(k))["flops"]
            extra = {"links": k}
            if aba:
                # the roofline counts the reference's 4 x 140 K + 12 K (bench_aba.py:53-55); this
                # build's rank-one form does fewer
                extra["flops_per_env_step_this_algorithm"] = rlenv_flops.aba_rank_one_flops(k)["flops"]
        actions = torch.randint(0, n_act, (T, n), device=dev, generator=g).to(torch.uint8 if n_act < 256 else torch.int32)
        state_b = torch.empty_like(state_a)
        rew, dn = torch.empty((T, n), device=dev), torch.empty((T, n), device=dev, dtype=torch.bool)
        extra["kernel"] = "T-step kernel: T steps per launch, state on chip between steps"

        def fn():
            launch_many(state_a, state_b, rew, dn)
        units, unit, metric, flops = n * T, "env steps/s", METRIC, fl
        # the state is read and written once per launch; actions, rewards, dones (and impulses) every step
        bytes_launch = n * 2 * 4 * rows + n * T * (1 + 5 + (8 * args.c if extra.get("impulses") else 0))
    elif args.workload == "es_ranks":
        import es

        pop = args.pop or n_def
        fit = torch.randn(pop, device=dev, generator=g)
        ms = {}
        for kind in (True, False):
            secs, clocks = _timed(torch, dist, world, stream, lambda: es.centered_ranks(torch, fit, sorted_kernel=kind),
                                  args.steps, args.warmup, local)
            ms[kind] = 1e3 * secs / args.steps
        if rank == 0:
            line = {"metric": "ES centred ranks ms", "value": ms[True], "unit": "ms", "n_gpus": world,
                    "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms[True], "higher_is_better": False,
                    "scaling": "replicas", "vs_baseline": None, "dtype": "f32", "data": "synthetic (normal fitness)",
                    "config": {"workload": args.workload, "config": desc, "population": pop,
                               "kernel": "rlenv_es_centered_ranks_sorted (bitonic tiles, merge-by-rank passes)",
                               "counting_kernel_ms": ms[False], "l2": "fitness and keys (12 B per member) stay in L2"},
                    "clocks": clocks}
            print(json.dumps(line), flush=True)
        if world > 1:
            dist.destroy_process_group()
        return
    else:  # es_*
        import es

        task = {"es_cartpole": "cartpole", "es_acrobot": "acrobot", "es_legged4": "legged4"}[args.workload]
        pop = args.pop or n_def
        horizon = args.horizon or t_def
        cfg = es.Config(task=task, pop=pop, horizon=horizon, sigma=0.1, lr=0.03)
        backend = es.MetalBackend(es.TASKS[task], 0)
        hidden = es.TASKS[task].hidden
        state = {"theta": backend.normal((es.n_params(hidden, es.TASKS[task]),)) * 0.1, "gen": 0, "steps": 0.0}

        def fn():
            state["gen"] += 1
            state["theta"], fit, steps = es.generation(backend, state["theta"], cfg, hidden, state["gen"])
            state["steps"] += float(steps.sum().item())
        for _ in range(args.warmup):
            fn()
        state["steps"] = 0.0
        secs, clocks = _timed(torch, dist, world, stream, fn, args.steps, 0, local)
        value = 1e3 * secs / args.steps
        if rank == 0:
            fl = rlenv_flops.es_member_step_flops(task)
            taken_per_s = state["steps"] / secs  # rank 0's shard; every shard takes about as many
            achieved = fl["flops"] * taken_per_s * world / 1e12
            line = {"metric": "ES generation ms", "value": value, "unit": "ms", "n_gpus": world, "steps": args.steps,
                    "warmup": args.warmup, "ms_per_step": value, "higher_is_better": False, "scaling": "strong",
                    "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded parameters and initial states)",
                    "config": {"workload": args.workload, "config": desc, "population": pop, "horizon": horizon,
                               "hidden": hidden, "sigma": 0.1, "lr": 0.03,
                               "member_steps_nominal_per_generation": pop * horizon,
                               "member_steps_taken_per_generation": state["steps"] * world / args.steps,
                               "env_steps_per_s": taken_per_s * world},
                    "roofline": {"bound": "fp32", "achieved": achieved, "peak": sgemm, "unit": "TFLOP/s",
                                 "frac": achieved / sgemm if sgemm else None, "flops_per_member_step": fl["flops"],
                                 "scope": "whole generation (perturb, rollout, ranks, update) over steps taken"},
                    "clocks": clocks}
            if world == 1 and not args.no_cpu_baseline:
                line["cpu_baseline"] = cpu_workload_baseline(args.workload, args, pop)
            print(json.dumps(line), flush=True)
        if world > 1:
            dist.destroy_process_group()
        return
    secs, clocks = _timed(torch, dist, world, stream, fn, args.steps, args.warmup, local)
    per = secs / args.steps
    if rank == 0:
        achieved = flops * units / per / 1e12
        gbs, hbm_peak = bytes_launch / per / 1e9, hbm_peak_gbs()[0]
        fp32 = {"bound": "fp32", "achieved": achieved, "peak": sgemm, "unit": "TFLOP/s",
                "frac": achieved / sgemm if sgemm else None, "flops_per_env_step": flops}
        ref_flops = extra.get("flops_per_env_step_reference_algorithm")
        if ref_flops:
            # the same run in the reference algorithm's count (its dense or full 3x3 form), against the
            # measured SGEMM rate and the nominal FP32 FMA rate of 148 SMs x 128 lanes at 1,965 MHz
            ref = ref_flops * units / per / 1e12
            fp32["reference_algorithm"] = {"achieved": ref, "frac": ref / sgemm if sgemm else None,
                                           "frac_of_nominal": ref / NOMINAL_FP32_TFLOPS}
        hbm = {"bound": "hbm", "achieved": gbs, "peak": hbm_peak, "unit": "GB/s", "frac": gbs / hbm_peak,
               "bytes_per_launch": bytes_launch / T, "peak_kind": "measured (MEASURED_PEAKS.json)"}
        roof = {**hbm, "fp32": fp32} if hbm_bound else {**fp32, "hbm": hbm}
        # the one-warp articulated body computes the reference's articulated-body configuration
        key = ("pendulum_aba" if args.workload == "pendulum_aba_coop" else args.workload, n) + \
            ((args.k,) if args.workload.startswith("pendulum") else ()) + \
            ((args.c, args.iters) if args.workload == "legged_step" else ())
        pub, pub_src = published(*key)
        if extra.get("impulses"):
            # the last timed step's normal impulses: the share of feet in active contact
            extra["contact_active_fraction"] = float((imp[-1, 1::2] > 0).float().mean().item())
        line = {"metric": metric, "value": world * units * args.steps / secs, "unit": unit, "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * per, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": (world * units * args.steps / secs / pub) if pub else None,
                "vs_baseline_source": pub_src, "dtype": "f32", "data": "synthetic",
                "config": {"workload": args.workload, "config": desc, "n_envs_per_gpu": n, "env_steps_per_step": T, **extra},
                "roofline": roof, "clocks": clocks}
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_workload_baseline(args.workload, args, n)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    elif args.workload != "acrobot_step":
        run_workload(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
