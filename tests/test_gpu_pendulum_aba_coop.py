"""The articulated-body pendulum with one warp per environment (rlenv_pendulum_aba_coop_step_many:
its recurrences along the chain as scans over the lanes) against the reference (golden) and the
oracle, on a B200: the same gates as the one-thread articulated body (tests/test_gpu_bodies.py),
at every lane width (K up to 32, 64, 128 and 192), plus chained steps against one T-step launch."""

import numpy as np
import pytest
import torch

from conftest import golden
from oracle import kernels
from parity import check_step, record, to_np

pytestmark = pytest.mark.gpu


def _tol(k):
    # the one-thread articulated body's gates: 1e-5 up to K = 4, 1e-4 up to 16, the reference's
    # own 1e-3 above
    return (1e-5, 1e-5) if k <= 4 else (1e-4, 1e-4) if k <= 16 else (1e-3, 1e-3)


def coop_steps(k, state, actions, seed0, index_offset=0):
    """T steps of the cooperative articulated body in one launch: (final state, rewards (T, N),
    dones (T, N)); actions (T, N) int64."""
    import rlenv_lib as rl

    n = state.shape[1]
    T = actions.shape[0]
    nxt = torch.empty_like(state)
    rew = torch.empty((T, n), device=state.device)
    done = torch.empty((T, n), dtype=torch.bool, device=state.device)
    rl.check(rl.lib().pendulum_aba_coop_step_many(k, state.data_ptr(), actions.data_ptr(), rl.I64, seed0, T, n,
                                                  index_offset, nxt.data_ptr(), rew.data_ptr(), done.data_ptr(),
                                                  rl.stream_ptr()))
    return nxt, rew, done


@pytest.mark.parametrize("k", [2, 3, 4, 8, 16, 32, 64])
def test_cooperative_articulated_body_matches_reference(cuda, k):
    g = golden("pendulum")
    st, ac = g[f"state_k{k}"], g[f"action_k{k}"]
    acts = torch.from_numpy(np.asarray(ac)).to(cuda, torch.int64)[None]
    nxt, rew, done = coop_steps(k, torch.from_numpy(st).to(cuda), acts, 41)
    onext, _, _, _ = kernels.pendulum_step(st, ac, 41, k, form="aba")
    rtol, atol = _tol(k)
    check_step(f"pendulum_aba_coop_k{k}", (nxt, rew[0], done[0]), g[f"aba_stepped_k{k}"], g[f"aba_done_k{k}"],
               onext, rtol, atol)


@pytest.mark.parametrize("k", [1, 17, 33, 65, 100, 129, 192])
def test_cooperative_articulated_body_matches_oracle_at_every_width(cuda, k):
    """K values with no golden vector, across the lane widths (one, two, four and six links per
    lane, the last lane part padding): the oracle on seeded states of the reference test's
    distribution."""
    r = np.random.default_rng(300 + k)
    n = 96
    st = np.concatenate([r.uniform(-np.pi, np.pi, (k, n)), r.uniform(-1, 1, (k, n))]).astype(np.float32)
    ac = r.integers(0, 3, n)
    nxt, rew, done = coop_steps(k, torch.from_numpy(st).to(cuda), torch.from_numpy(ac).to(cuda)[None], 46)
    onext, _, odone, stepped = kernels.pendulum_step(st, ac, 46, k, form="aba")
    rtol, atol = _tol(k)
    check_step(f"pendulum_aba_coop_k{k}", (nxt, rew[0], done[0]), stepped, odone, onext, rtol, atol)


@pytest.mark.parametrize("k,n", [(1, 5), (2, 17), (3, 13), (5, 11), (16, 7), (16, 1), (31, 3)])
def test_cooperative_articulated_body_ragged_batches(cuda, k, n):
    """Up to 32 links an environment takes a segment of the next power of two of lanes, so a warp
    holds several; batches that leave the last warp part empty (its spare segments mirror the
    last environment and store nothing) against the oracle, with a shard offset."""
    r = np.random.default_rng(700 + k + n)
    st = np.concatenate([r.uniform(-np.pi, np.pi, (k, n)), r.uniform(-1, 1, (k, n))]).astype(np.float32)
    ac = r.integers(0, 3, n)
    st_t = torch.from_numpy(st).to(cuda)
    nxt, rew, done = coop_steps(k, st_t, torch.from_numpy(ac).to(cuda)[None], 52, index_offset=9)
    onext, _, odone, stepped = kernels.pendulum_step(st, ac, 52, k, form="aba", index_offset=9)
    rtol, atol = _tol(k)
    check_step(f"pendulum_aba_coop_ragged_k{k}_n{n}", (nxt, rew[0], done[0]), stepped, odone, onext, rtol, atol)
    assert torch.equal(st_t, torch.from_numpy(st).to(cuda))  # the input is not written


@pytest.mark.parametrize("k", [20, 64, 150])
def test_cooperative_articulated_body_trajectory(cuda, k):
    """50 chained steps against the oracle's chain with the same resets: done flags equal and
    states within the reference's 1e-3 up to 64 links; a 150-link chain's rounding grows with its
    length (1.6e-3 after 50 steps, measured), gated at 5e-3."""
    r = np.random.default_rng(500 + k)
    n = 64
    st = np.concatenate([r.uniform(-0.1, 0.1, (k, n)), r.uniform(-0.1, 0.1, (k, n))]).astype(np.float32)
    s_gpu, s_np = torch.from_numpy(st).to(cuda), st
    worst, flips = 0.0, 0
    for t in range(50):
        ac = r.integers(0, 3, n)
        s_gpu, _, d_gpu = coop_steps(k, s_gpu, torch.from_numpy(ac).to(cuda)[None], 71 + t)
        s_np, _, d_np, _ = kernels.pendulum_step(s_np, ac, 71 + t, k, form="aba")
        flips += int((to_np(d_gpu[0]) != d_np).sum())
        worst = max(worst, float(np.abs(to_np(s_gpu) - s_np).max()))
    record(f"pendulum_aba_coop_k{k}_traj50", max_abs=worst, done_flips=flips)
    assert flips == 0 and worst < (1e-3 if k <= 64 else 5e-3), (worst, flips)


@pytest.mark.parametrize("k", [5, 40, 100])
def test_cooperative_step_many_equals_chained_steps(cuda, k):
    """One T-step launch equals T single-step launches bit for bit (the same seeds), with a shard
    offset, and the one-warp form stays within rounding of the one-thread articulated body."""
    import pendulum_aba_metal

    r = np.random.default_rng(k)
    n, T = 300, 12
    st = torch.from_numpy(np.concatenate([r.uniform(-0.1, 0.1, (k, n)), r.uniform(-0.1, 0.1, (k, n))])
                          .astype(np.float32)).to(cuda)
    acts = torch.from_numpy(r.integers(0, 3, (T, n))).to(cuda)
    fin, rew, done = coop_steps(k, st, acts, 900, index_offset=77)
    s = st
    for t in range(T):
        s, rt, dt = coop_steps(k, s, acts[t:t + 1], 900 + t, index_offset=77)
        assert torch.equal(rt[0], rew[t]) and torch.equal(dt[0], done[t])
    assert torch.equal(s, fin)
    fin0, _, done0 = coop_steps(k, st, acts, 900)
    body = pendulum_aba_metal.Pendulum(k)
    body.reseed(899)
    one, _, odone = body.step_many(st, acts)
    assert torch.equal(odone, done0)
    np.testing.assert_allclose(to_np(fin0), to_np(one), rtol=1e-3, atol=1e-3)


@pytest.mark.parametrize("k", [16, 64])
def test_cooperative_option_of_the_drop_in_module(cuda, k):
    """pendulum_aba_metal.Pendulum(k, cooperative=True) steps through the one-warp kernel with the
    reference's seed counter: its single steps equal the entry point's, and it matches the golden
    vectors as the one-thread body does."""
    import pendulum_aba_metal

    g = golden("pendulum")
    st, ac = g[f"state_k{k}"], g[f"action_k{k}"]
    p = pendulum_aba_metal.Pendulum(k, cooperative=True)
    p.reseed(40)
    out = p.step(torch.from_numpy(st).to(cuda), torch.from_numpy(np.asarray(ac)).to(cuda))
    want = coop_steps(k, torch.from_numpy(st).to(cuda), torch.from_numpy(np.asarray(ac)).to(cuda, torch.int64)[None], 41)
    assert torch.equal(out[0], want[0]) and torch.equal(out[1], want[1][0]) and torch.equal(out[2], want[2][0])
    onext, _, _, _ = kernels.pendulum_step(st, ac, 41, k, form="aba")
    rtol, atol = _tol(k)
    check_step(f"pendulum_aba_coop_module_k{k}", out, g[f"aba_stepped_k{k}"], g[f"aba_done_k{k}"], onext, rtol, atol)
    assert p.calls == 41
