"""The multi-GPU ES orchestration of es.py on gloo ranks (CPU): sharded perturbation and
rollout, the (fitness, steps) all-gather, and every rank's own update must give each rank the
same theta, equal to the single-process run; failures surface on the host as errors.

The kernels are replaced by the CPU oracle through a backend subclass, so this exercises only
the host logic that multi-GPU runs add (shard offsets, gather order, cross-rank checks)."""

import os
import socket
import sys
import traceback

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import PKG, ROOT

HIDDEN, POP, HORIZON, GENS = 8, 64, 40, 3


def _backend_cls():
    import es
    from oracle import rng, rollout
    from oracle import es as oes

    class OracleBackend(es.MetalBackend):
        """MetalBackend's orchestration with the device kernels replaced by the oracle."""

        def perturb(self, theta, sigma, gen, pairs, member_offset, rows):
            m = np.arange(member_offset, member_offset + rows)
            z = rng.noise(self.seed, gen, np.where(m < pairs, m, m - pairs), theta.numel())
            z = np.where((m >= pairs)[:, None], -z, z)
            return torch.from_numpy((theta.numpy() + np.float32(sigma) * z).astype(np.float32))

        def rollout(self, theta_pop, hidden, horizon, assist=0.0, start_velocity=0.0, gen=0, member_offset=0):
            st = rng.reset_rows(self._reset_seed(gen), theta_pop.shape[0], 4, 0.05, member_offset)
            fit = rollout.cartpole(st, theta_pop.numpy(), hidden, horizon)
            return torch.from_numpy(fit), torch.from_numpy(np.minimum(fit + 1, horizon).astype(np.float32))

        def centered_ranks(self, fit):
            return torch.from_numpy(oes.centered_ranks(fit.numpy(), stable=True).astype(np.float32))

        def update(self, theta, ranks, lr, sigma, gen, pairs):
            z = rng.noise(self.seed, gen, np.arange(pairs), theta.numel()).astype(np.float64)
            r = ranks.numpy().astype(np.float64)
            g = ((r[:pairs] - r[pairs:])[:, None] * z).sum(0)
            return torch.from_numpy((theta.numpy() + lr / (2 * pairs * sigma) * g).astype(np.float32))

        def sync(self, *arrays):
            pass

    return OracleBackend


def _run_generations(world_rank=None):
    import es

    cls = _backend_cls()
    task = es.TASKS["cartpole"]
    backend = cls(task, 17)
    theta = torch.from_numpy((np.random.default_rng(0).normal(size=es.n_params(HIDDEN, task)) * 0.1).astype(np.float32))
    cfg = es.Config(pop=POP, horizon=HORIZON, lr=0.03)
    fits = []
    for gen in range(1, GENS + 1):
        theta, fit, steps = es.generation(backend, theta, cfg, HIDDEN, gen)
        fits.append(fit.numpy())
    return theta.numpy(), np.stack(fits)


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, outdir):
    sys.path[:0] = [str(ROOT), str(PKG)]
    try:
        from datetime import timedelta

        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=timedelta(seconds=15))
        import es

        if mode == "generations":
            theta, fits = _run_generations()
            np.save(os.path.join(outdir, f"theta{rank}.npy"), theta)
            np.save(os.path.join(outdir, f"fits{rank}.npy"), fits)
            es.assert_ranks_agree(torch.from_numpy(theta))
        elif mode == "diverged":
            theta = torch.ones(10) * (1.0 + rank)
            try:
                es.assert_ranks_agree(theta)
                open(os.path.join(outdir, f"nodetect{rank}"), "w").close()
            except RuntimeError:
                open(os.path.join(outdir, f"detected{rank}"), "w").close()
        elif mode == "dead_rank":
            if rank == 1:
                raise SystemExit(3)  # leaves between steps, before the gather
            backend = es.MetalBackend.__new__(es.MetalBackend)
            backend.rank, backend.world = rank, world
            try:
                backend.gather(torch.zeros(4))
                open(os.path.join(outdir, "gathered"), "w").close()
            except Exception:
                open(os.path.join(outdir, "error0"), "w").close()
        dist.destroy_process_group()
    except SystemExit:
        raise
    except Exception:
        traceback.print_exc()
        raise


def _spawn(mode, tmp_path, world=2):
    ctx = mp.get_context("spawn")
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
            pytest.fail(f"{mode}: a rank did not finish")
    return [p.exitcode for p in procs]


def test_sharded_generations_equal_single_process(tmp_path):
    theta1, fits1 = _run_generations()
    codes = _spawn("generations", tmp_path)
    assert codes == [0, 0]
    t0, t1 = np.load(tmp_path / "theta0.npy"), np.load(tmp_path / "theta1.npy")
    np.testing.assert_array_equal(t0, t1)
    np.testing.assert_array_equal(t0, theta1)
    np.testing.assert_array_equal(np.load(tmp_path / "fits0.npy"), fits1)


def test_diverged_theta_is_detected_on_every_rank(tmp_path):
    assert _spawn("diverged", tmp_path) == [0, 0]
    assert (tmp_path / "detected0").exists() and (tmp_path / "detected1").exists()


def test_dead_rank_surfaces_as_error(tmp_path):
    codes = _spawn("dead_rank", tmp_path)
    assert codes[1] == 3
    assert (tmp_path / "error0").exists() and not (tmp_path / "gathered").exists()
