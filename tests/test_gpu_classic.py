"""CartPole and Acrobot step kernels against the reference (golden) and the oracle, on a B200.

Mirrors test_cartpole.py / test_acrobot.py of the reference: parity on seeded random states
(live columns to tolerance, done exact), reset statistics, chained steps, plus the B200
additions: every action dtype, ragged and empty batches, sharded index offsets, and the T-step
kernel against the chain of single steps."""

import numpy as np
import pytest
import torch

from conftest import golden
from oracle import classic, kernels, rng
from parity import check_step, record, to_np

pytestmark = pytest.mark.gpu

# north_star: single-step states within 1e-5 relative in fp32
RTOL, ATOL = 1e-5, 1e-5

ENVS = {
    "cartpole": (lambda: __import__("cartpole_metal"), kernels.cartpole_step, classic.cartpole_terminated, 2, 0.05),
    "acrobot": (lambda: __import__("acrobot_metal"), kernels.acrobot_step, classic.acrobot_terminated, 3, 0.1),
}


@pytest.mark.parametrize("name", ["cartpole", "acrobot"])
@pytest.mark.parametrize("dtype", [torch.int64, torch.int32, torch.uint8])
def test_step_matches_reference(cuda, name, dtype):
    mod, oracle_step, _, _, _ = ENVS[name]
    m = mod()
    g = golden(name)
    m.reseed(41)
    out = m.step(torch.from_numpy(g["state"]).to(cuda), torch.from_numpy(g["action"]).to(cuda, dtype))
    onext, oreward, odone, _ = oracle_step(g["state"], g["action"], 42)
    check_step(f"{name}_step_{dtype}", out, g["stepped"], g["done"], onext, RTOL, ATOL, ref_reward=oreward)


@pytest.mark.parametrize("name", ["cartpole", "acrobot"])
@pytest.mark.parametrize("n", [1, 3, 31, 33, 257, 4096])
def test_ragged_sizes_and_offsets(cuda, name, n):
    """Scalar and vector paths, tails, and a shard at a global offset draw the same resets."""
    import rlenv_lib as rl

    _, oracle_step, _, n_act, bound = ENVS[name]
    r = np.random.default_rng(n)
    st = r.uniform(-2.5, 2.5, (4, n)).astype(np.float32)
    act = r.integers(0, n_act, n).astype(np.int32)
    fn = rl.lib().cartpole_step if name == "cartpole" else rl.lib().acrobot_step
    outs = []
    for off in (0, 1000):
        nxt = torch.empty((4, n), device=cuda)
        rew = torch.empty(n, device=cuda)
        dn = torch.empty(n, dtype=torch.bool, device=cuda)
        s_t, a_t = torch.from_numpy(st).to(cuda), torch.from_numpy(act).to(cuda)
        rl.check(fn(s_t.data_ptr(), a_t.data_ptr(), rl.I32, 7, n, off, nxt.data_ptr(), rew.data_ptr(), dn.data_ptr(),
                    rl.stream_ptr()))
        onext, _, odone, stepped = oracle_step(st, act, 7, index_offset=off)
        check_step(f"{name}_n{n}_off{off}", (nxt, rew, dn), stepped, odone, onext, RTOL, ATOL)
        outs.append(to_np(nxt))


def test_empty_batch(cuda):
    import cartpole_metal

    nxt, rew, dn = cartpole_metal.step(torch.empty((4, 0), device=cuda), torch.empty(0, dtype=torch.int64, device=cuda))
    assert nxt.shape == (4, 0) and rew.shape == (0,) and dn.shape == (0,)


@pytest.mark.parametrize("name", ["cartpole", "acrobot"])
def test_resets_are_uniform_bounded_and_vary(cuda, name):
    mod, _, _, _, bound = ENVS[name]
    m = mod()
    m.reseed(0)
    n = 16384
    terminal = np.zeros((4, n), np.float32)
    if name == "cartpole":
        terminal[:] = 3.0
    else:
        terminal[0] = np.pi
    a = torch.ones(n, dtype=torch.int32, device=cuda)
    first = to_np(m.step(torch.from_numpy(terminal).to(cuda), a)[0])
    second = to_np(m.step(torch.from_numpy(terminal).to(cuda), a)[0])
    assert np.all(np.abs(first) <= bound) and not np.allclose(first, second)
    assert len(np.unique(first[0])) > 0.99 * n
    assert abs(first.mean()) < 0.002 * bound / 0.05 and abs(first.std() - bound / np.sqrt(3)) < 0.002 * bound / 0.05
    want = rng.reset_rows(1, n, 4, bound, offsets=rng.CLASSIC_ROW_OFFSETS)
    np.testing.assert_array_equal(first, want)


@pytest.mark.parametrize("name", ["cartpole", "acrobot"])
def test_chain_of_steps_stays_valid(cuda, name):
    """100 chained steps: finite, wrapped, and never left in a terminal region."""
    mod, _, terminated, n_act, _ = ENVS[name]
    m = mod()
    n = 4096
    state = m.reset(n)
    g = torch.Generator(device=cuda).manual_seed(0)
    for _ in range(100):
        state, _, _ = m.step(state, torch.randint(0, n_act, (n,), device=cuda, generator=g))
    out = to_np(state)
    assert np.isfinite(out).all() and not terminated(out).any()
    if name == "acrobot":
        assert np.all(np.abs(out[:2]) <= np.pi)


@pytest.mark.parametrize("dtype", [torch.int32, torch.uint8, torch.int64])
def test_cartpole_four_envs_per_thread_path(cuda, dtype):
    """From about 606K environments the CartPole kernels step four environments per thread
    (16-byte accesses); that path against the oracle at N = 2^20 + 4, one step and a T-step
    chain, with a shard offset."""
    import cartpole_metal
    import rlenv_lib as rl

    n = (1 << 20) + 4
    r = np.random.default_rng(5)
    st = r.uniform(-2.5, 2.5, (4, n)).astype(np.float32)
    act = r.integers(0, 2, n)
    nxt, rew, dn = (torch.empty((4, n), device=cuda), torch.empty(n, device=cuda),
                    torch.empty(n, dtype=torch.bool, device=cuda))
    a_t = torch.from_numpy(act).to(cuda, dtype)
    rl.check(rl.lib().cartpole_step(torch.from_numpy(st).to(cuda).data_ptr(), a_t.data_ptr(), rl._DTYPES[dtype], 9, n,
                                    4096, nxt.data_ptr(), rew.data_ptr(), dn.data_ptr(), rl.stream_ptr()))
    onext, oreward, odone, stepped = kernels.cartpole_step(st, act, 9, index_offset=4096)
    check_step(f"cartpole_vec4_{dtype}", (nxt, rew, dn), stepped, odone, onext, RTOL, ATOL, ref_reward=oreward)
    # the T-step kernel on the same path equals the chain of single steps
    T = 4
    acts = torch.randint(0, 2, (T, n), device=cuda, generator=torch.Generator(device=cuda).manual_seed(2)).to(dtype)
    state0 = cartpole_metal.reset(n)
    cartpole_metal.reseed(300)
    s = state0
    for t in range(T):
        s, _, _ = cartpole_metal.step(s, acts[t])
    cartpole_metal.reseed(300)
    assert torch.equal(cartpole_metal.step_many(state0, acts)[0], s)


@pytest.mark.parametrize("name", ["cartpole", "acrobot"])
@pytest.mark.parametrize("n,T", [(1, 1), (5, 3), (1030, 17), (4096, 4), (4099, 8), ((1 << 20) + 4, 6)])
def test_packed_actions_give_the_same_bits(cuda, name, n, T):
    """Actions packed along time (RLENV_U2, rlenv_lib.pack_actions: four steps to a byte) step
    the bodies with the same bits as uint8 actions: single steps and T-step launches with every
    output, for T a multiple of four and not, at ragged sizes and on CartPole's
    four-environments-per-thread path (N = 2^20 + 4)."""
    import rlenv_lib as rl

    mod, _, _, n_act, _ = ENVS[name]
    m = mod()
    gen = torch.Generator(device=cuda).manual_seed(n + T)
    acts = torch.randint(0, n_act, (T, n), device=cuda, generator=gen).to(torch.uint8)
    packed = rl.pack_actions(acts)
    assert packed.bits.shape == ((T + 3) // 4, n) and packed.steps == T
    state0 = m.reset(n)
    m.reseed(7)
    want = m.step(state0, acts[0])
    m.reseed(7)
    got = m.step(state0, rl.pack_actions(acts[0]))
    assert all(torch.equal(a, b) for a, b in zip(got, want))
    m.reseed(70)
    want = m.step_many(state0, acts, sums=True)
    m.reseed(70)
    got = m.step_many(state0, packed, sums=True)
    assert all(torch.equal(a, b) for a, b in zip(got, want))
    m.reseed(70)
    fin, _, _ = m.step_many(state0, packed, rewards=False, dones=False)
    assert torch.equal(fin, want[0])
    if T > 1:
        with pytest.raises(ValueError):
            m.step(state0, packed)  # the packed actions of more than one step


@pytest.mark.parametrize("name", ["cartpole", "acrobot"])
@pytest.mark.parametrize("dtype", [torch.uint8, torch.int64])
def test_step_many_equals_chained_steps(cuda, name, dtype):
    """T steps in one launch are bit-identical to T single-step launches with the same seeds."""
    mod, _, _, n_act, _ = ENVS[name]
    m = mod()
    n, T = 2048, 50
    state0 = m.reset(n)
    acts = torch.randint(0, n_act, (T, n), device=cuda, generator=torch.Generator(device=cuda).manual_seed(1)).to(dtype)
    m.reseed(100)
    s = state0
    rews, dones = [], []
    for t in range(T):
        s, r, d = m.step(s, acts[t])
        rews.append(r)
        dones.append(d)
    m.reseed(100)
    fin, rseq, dseq, rsum, dcnt = m.step_many(state0, acts, sums=True)
    assert torch.equal(fin, s)
    assert torch.equal(rseq, torch.stack(rews)) and torch.equal(dseq, torch.stack(dones))
    assert torch.equal(rsum, torch.stack(rews).sum(0)) and torch.equal(dcnt, torch.stack(dones).float().sum(0))
    assert m._counter.calls == 100 + T


@pytest.mark.parametrize("name", ["cartpole", "acrobot"])
def test_trajectory_matches_oracle_kernel_semantics(cuda, name):
    """100 chained GPU steps against the oracle's chain with the same hash-stream resets: the
    done sequences agree and the states stay within a stated tolerance."""
    mod, oracle_step, _, n_act, _ = ENVS[name]
    m = mod()
    g = golden(name)
    s_np = g["traj_state"]
    acts = g["traj_actions"]
    m.reseed(500)
    s_gpu = torch.from_numpy(s_np).to(cuda)
    flips, worst = 0, 0.0
    for t in range(acts.shape[0]):
        s_gpu, _, d_gpu = m.step(s_gpu, torch.from_numpy(acts[t]).to(cuda))
        s_np, _, d_np, _ = oracle_step(s_np, acts[t], 501 + t)
        flips += int((to_np(d_gpu) != d_np).sum())
        worst = max(worst, float(np.abs(to_np(s_gpu) - s_np).max()))
    record(f"{name}_traj100", done_flips=flips, max_abs=worst, n=int(s_np.shape[1]))
    assert flips == 0
    # about ten times the measured worst (8.2e-6 CartPole, 2.3e-5 Acrobot), so a change that
    # degrades the arithmetic shows here before it shows anywhere else
    assert worst < (1e-4 if name == "cartpole" else 3e-4), worst


def test_reference_pure_physics_trajectory(cuda):
    """Against the reference's own 100-step CartPole physics chain (no resets): every column that
    the reference never terminates agrees with the chained GPU steps at each checkpoint."""
    import cartpole_metal

    g = golden("cartpole")
    s = torch.from_numpy(g["traj_state"]).to(cuda)
    alive = np.ones(s.shape[1], dtype=bool)
    ck = 0
    ref_s = g["traj_state"]
    for t, a in enumerate(g["traj_actions"], 1):
        s, _, d = cartpole_metal.step(s, torch.from_numpy(a).to(cuda))
        ref_s = classic.cartpole_physics(ref_s, a)
        alive &= ~classic.cartpole_terminated(ref_s) & ~to_np(d)
        if t in (1, 10, 25, 50, 100):
            if alive.any():
                np.testing.assert_allclose(to_np(s)[:, alive], g["traj"][ck][:, alive], rtol=1e-4, atol=1e-4)
            ck += 1
