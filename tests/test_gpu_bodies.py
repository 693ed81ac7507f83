"""K-link pendulum (mass matrix, pairwise trig, warp-cooperative, articulated body), hopper and
legged step kernels against the reference (golden) and the oracle, on a B200.

Mirrors test_pendulum.py, test_pendulum_aba.py, test_hopper.py and test_legged.py of the
reference: parity of live columns to tolerance with exact done flags on seeded random states,
resets (here bit-exact against the oracle's hash stream) and chained steps."""

import numpy as np
import pytest
import torch

from conftest import golden
from oracle import kernels, legged, pendulum
from parity import check_step, record, to_np

pytestmark = pytest.mark.gpu

# The reference's own Metal gate is rtol = atol = 1e-3 (test_pendulum.py:76, test_legged.py:107).
# These bodies are checked tighter; each test states its tolerance.


def _pend_tol(k):
    return (1e-5, 1e-5) if k <= 4 else (1e-4, 1e-4)


@pytest.mark.parametrize("k", [2, 3, 4, 8, 16])
@pytest.mark.parametrize("pairwise", [False, True])
def test_mass_matrix_matches_reference(cuda, k, pairwise):
    import pendulum_metal

    g = golden("pendulum")
    st, ac = g[f"state_k{k}"], g[f"action_k{k}"]
    p = pendulum_metal.Pendulum(k, pairwise_trig=pairwise)
    p.reseed(10)
    out = p.step(torch.from_numpy(st).to(cuda), torch.from_numpy(ac).to(cuda))
    onext, orew, _, _ = kernels.pendulum_step(st, ac, 11, k)
    rtol, atol = _pend_tol(k)
    check_step(f"pendulum_mm{'_pairwise' if pairwise else ''}_k{k}", out, g[f"mm_stepped_k{k}"], g[f"mm_done_k{k}"],
               onext, rtol, atol, ref_reward=orew)


@pytest.mark.parametrize("k", [2, 4, 8, 16])
def test_cooperative_matches_reference(cuda, k):
    import pendulum_metal_coop

    g = golden("pendulum")
    st, ac = g[f"state_k{k}"], g[f"action_k{k}"]
    p = pendulum_metal_coop.Pendulum(k)
    p.reseed(20)
    out = p.step(torch.from_numpy(st).to(cuda), torch.from_numpy(ac).to(cuda))
    onext, orew, _, _ = kernels.pendulum_step(st, ac, 21, k)
    rtol, atol = _pend_tol(k)
    check_step(f"pendulum_coop_k{k}", out, g[f"mm_stepped_k{k}"], g[f"mm_done_k{k}"], onext, rtol, atol,
               ref_reward=orew)


def test_cooperative_k32_matches_articulated_oracle(cuda):
    """K = 32 has no mass-matrix golden (the reference's own numpy stops at 16 there); the
    articulated-body reference is the same dynamics."""
    import pendulum_metal_coop

    g = golden("pendulum")
    st, ac = g["state_k32"], g["action_k32"]
    p = pendulum_metal_coop.Pendulum(32)
    p.reseed(30)
    out = p.step(torch.from_numpy(st).to(cuda), torch.from_numpy(ac).to(cuda))
    onext, _, _, _ = kernels.pendulum_step(st, ac, 31, 32)
    check_step("pendulum_coop_k32", out, g["aba_stepped_k32"], g["aba_done_k32"], onext, 1e-3, 1e-3)


@pytest.mark.parametrize("k", [2, 3, 4, 8, 16, 32, 64])
def test_articulated_body_matches_reference(cuda, k):
    import pendulum_aba_metal

    g = golden("pendulum")
    st, ac = g[f"state_k{k}"], g[f"action_k{k}"]
    p = pendulum_aba_metal.Pendulum(k)
    p.reseed(40)
    out = p.step(torch.from_numpy(st).to(cuda), torch.from_numpy(ac).to(cuda))
    onext, _, _, _ = kernels.pendulum_step(st, ac, 41, k, form="aba")
    rtol, atol = _pend_tol(k) if k <= 16 else (1e-3, 1e-3)
    check_step(f"pendulum_aba_k{k}", out, g[f"aba_stepped_k{k}"], g[f"aba_done_k{k}"], onext, rtol, atol)


@pytest.mark.parametrize("k", [17, 24, 37, 48, 100, 192])
def test_articulated_body_long_chains_match_oracle(cuda, k):
    """K values with no golden vector, any K up to 192 as the reference's template accepts any K
    (pendulum_aba_metal.py:121-144): the oracle (itself pinned to the reference's numpy at
    K = 2..64) on seeded states of the reference test's distribution."""
    import pendulum_aba_metal

    r = np.random.default_rng(k)
    st = np.concatenate([r.uniform(-np.pi, np.pi, (k, 64)), r.uniform(-1, 1, (k, 64))]).astype(np.float32)
    ac = r.integers(0, 3, 64)
    p = pendulum_aba_metal.Pendulum(k)
    p.reseed(45)
    out = p.step(torch.from_numpy(st).to(cuda), torch.from_numpy(ac).to(cuda))
    onext, _, odone, stepped = kernels.pendulum_step(st, ac, 46, k, form="aba")
    check_step(f"pendulum_aba_k{k}", out, stepped, odone, onext, 1e-3, 1e-3)


def test_unsupported_k_raises(cuda):
    import pendulum_aba_metal
    import pendulum_metal

    with pytest.raises(ValueError):
        pendulum_metal.Pendulum(17).step(torch.zeros((34, 4), device=cuda), torch.ones(4, dtype=torch.int64, device=cuda))
    with pytest.raises(ValueError):
        pendulum_aba_metal.Pendulum(193).step(torch.zeros((386, 4), device=cuda), torch.ones(4, dtype=torch.int64, device=cuda))


@pytest.mark.parametrize("k", [20, 64])
def test_articulated_body_long_chain_trajectory(cuda, k):
    """50 chained steps of a long chain against the oracle's chain with the same resets (the
    velocities walked back through the inverse joint transforms and the approximate reciprocals
    must not drift): done flags equal and states within the reference's 1e-3."""
    import pendulum_aba_metal

    r = np.random.default_rng(100 + k)
    st = np.concatenate([r.uniform(-0.1, 0.1, (k, 96)), r.uniform(-0.1, 0.1, (k, 96))]).astype(np.float32)
    p = pendulum_aba_metal.Pendulum(k)
    p.reseed(70)
    s_gpu, s_np = torch.from_numpy(st).to(cuda), st
    worst, flips = 0.0, 0
    for t in range(50):
        ac = r.integers(0, 3, 96)
        s_gpu, _, d_gpu = p.step(s_gpu, torch.from_numpy(ac).to(cuda))
        s_np, _, d_np, _ = kernels.pendulum_step(s_np, ac, 71 + t, k, form="aba")
        flips += int((to_np(d_gpu) != d_np).sum())
        worst = max(worst, float(np.abs(to_np(s_gpu) - s_np).max()))
    record(f"pendulum_aba_k{k}_traj50", max_abs=worst, done_flips=flips)
    assert flips == 0 and worst < 1e-3, (worst, flips)


@pytest.mark.parametrize("k", [32, 48, 64])
def test_articulated_body_tensor_and_shared_memory_warps_agree(cuda, k):
    """For 32 <= K <= 64 and a batch that fills the GPU, a block's first four warps keep their
    environments in tensor memory and the others in shared memory (seven warps here). The same environments rolled by 128 positions, with
    index_offset moved back by as much so that their resets draw the same numbers, change kind
    of warp: states, rewards and done flags are the same bits."""
    import rlenv_lib as rl

    lib = rl.lib()
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    n = 32 * sms * 7  # seven warps per SM: four in tensor memory, three in shared memory
    T, off, roll = 6, 1000, 128
    r = np.random.default_rng(k)
    st = r.uniform(-0.1, 0.1, (2 * k, n)).astype(np.float32)
    st[:k, ::5] = np.pi  # a fifth start upright: resets in the first step
    act = r.integers(0, 3, (T, n)).astype(np.int32)

    def run(state, actions, index_offset):
        s, a = torch.from_numpy(state).to(cuda), torch.from_numpy(actions).to(cuda)
        nxt = torch.empty_like(s)
        rew = torch.empty((T, n), device=cuda)
        done = torch.empty((T, n), dtype=torch.bool, device=cuda)
        rl.check(lib.pendulum_aba_step_many(k, s.data_ptr(), a.data_ptr(), rl.I32, 7, T, n, index_offset,
                                            nxt.data_ptr(), rew.data_ptr(), done.data_ptr(),
                                            torch.cuda.current_stream().cuda_stream))
        return to_np(nxt), to_np(rew), to_np(done)

    first = run(st, act, off)
    moved = run(np.roll(st, roll, axis=1), np.roll(act, roll, axis=1), off - roll)
    assert first[2].any(), "the window should include resets"
    for a, b in zip(first, moved):
        a = np.ascontiguousarray(a[..., : n - roll])  # the environments that moved without wrapping
        b = np.ascontiguousarray(b[..., roll:])
        np.testing.assert_array_equal(a.view(np.uint8), b.view(np.uint8))


@pytest.mark.parametrize("cls_name", ["pendulum_metal", "pendulum_metal_coop", "pendulum_aba_metal"])
def test_pendulum_resets_and_chain(cuda, cls_name):
    mod = __import__(cls_name)
    p = mod.Pendulum(4)
    n = 4096
    up = np.zeros((8, n), dtype=np.float32)
    up[:4] = np.pi
    a = torch.ones(n, dtype=torch.int32, device=cuda)
    first = to_np(p.step(torch.from_numpy(up).to(cuda), a)[0])
    second = to_np(p.step(torch.from_numpy(up).to(cuda), a)[0])
    assert np.all(np.abs(first) <= 0.1) and not np.allclose(first, second)
    assert abs(first.std() - 0.1 / np.sqrt(3)) < 0.002
    state = p.reset(n)
    gen = torch.Generator(device=cuda).manual_seed(0)
    for _ in range(100):
        state, _, _ = p.step(state, torch.randint(0, 3, (n,), device=cuda, generator=gen))
    out = to_np(state)
    assert np.all(np.isfinite(out)) and np.abs(out[:4]).max() <= np.pi


# ---- hopper and legged ----------------------------------------------------------------------

@pytest.mark.parametrize("branchy", [False, True])
def test_hopper_matches_reference(cuda, branchy):
    import hopper_metal

    g = golden("hopper")
    h = hopper_metal.Hopper(branchy=branchy)
    h.reseed(50)
    out = h.step(torch.from_numpy(g["state"]).to(cuda), torch.from_numpy(g["action"]).to(cuda))
    onext, orew, _, _ = kernels.hopper_step(g["state"], g["action"], 51)
    check_step(f"hopper{'_branchy' if branchy else ''}", out, g["stepped"], g["done"], onext, 1e-4, 1e-4,
               ref_reward=orew)
    contacts = (legged.foot_heights(g["state"], 1) <= 0).mean()
    assert 0.2 < contacts < 0.8


@pytest.mark.parametrize("c", [1, 2, 4])
@pytest.mark.parametrize("iters", [1, 4, 8, 16])
def test_legged_matches_reference(cuda, c, iters):
    import legged_metal

    g = golden("legged")
    st, ac = g[f"state_c{c}"], g[f"action_c{c}"]
    body = legged_metal.Legged(c, iters)
    body.reseed(60)
    out = body.step(torch.from_numpy(st).to(cuda), torch.from_numpy(ac).to(cuda))
    onext, orew, _, _ = kernels.legged_step(st, ac, 61, c, iters)
    check_step(f"legged_c{c}_i{iters}", out, g[f"stepped_c{c}_i{iters}"], g[f"done_c{c}_i{iters}"], onext, 1e-4, 1e-4,
               ref_reward=orew)
    touching = (legged.foot_heights(st, c) <= 0).mean()
    assert 0.2 < touching < 0.8


@pytest.mark.parametrize("as_tensor", [False, True])
def test_legged_assist(cuda, as_tensor):
    import legged_metal

    g = golden("legged")
    st, ac = g["state_c2"], g["action_c2"]
    body = legged_metal.Legged(2)
    body.reseed(70)
    assist = torch.tensor([20.0], device=cuda) if as_tensor else 20.0
    out = body.step(torch.from_numpy(st).to(cuda), torch.from_numpy(ac).to(cuda), assist)
    ref = g["assist_stepped_c2"]
    done = legged.terminated(ref)
    onext, _, _, _ = kernels.legged_step(st, ac, 71, 2, assist=20.0)
    check_step(f"legged_c2_assist_{'tensor' if as_tensor else 'float'}", out, ref, done, onext, 1e-4, 1e-4)


def test_legged_resets_and_chain(cuda):
    import legged_metal

    p = legged_metal.Legged(4)
    n = 2048
    tilted = np.tile(legged.stand_pose(4)[:, None], (1, n))
    tilted[2] = 2.0
    a = torch.zeros(n, dtype=torch.int32, device=cuda)
    first = to_np(p.step(torch.from_numpy(tilted).to(cuda), a)[0])
    second = to_np(p.step(torch.from_numpy(tilted).to(cuda), a)[0])
    assert np.all(np.abs(first - legged.stand_pose(4)[:, None]) <= 0.05 + 1e-7) and not np.allclose(first, second)
    state = p.reset(n)
    gen = torch.Generator(device=cuda).manual_seed(0)
    worst = 0.0
    for _ in range(100):
        state, _, _ = p.step(state, torch.randint(0, 81, (n,), device=cuda, generator=gen))
        worst = min(worst, float(legged.foot_heights(to_np(state), 4).min()))
    assert np.isfinite(to_np(state)).all() and worst > -0.08
    record("legged4_chain100", min_foot=worst)


@pytest.mark.parametrize("c", [2, 4])
def test_legged_trajectory_matches_oracle(cuda, c):
    """50 chained steps from the reset pose against the oracle's chain with the same resets."""
    import legged_metal

    body = legged_metal.Legged(c)
    n = 512
    r = np.random.default_rng(c)
    s_np = legged.stand_pose(c)[:, None] + r.uniform(-0.05, 0.05, (2 * (3 + c), n)).astype(np.float32)
    acts = r.integers(0, 3**c, (50, n))
    body.reseed(900)
    s_gpu = torch.from_numpy(s_np).to(cuda)
    flips, worst = 0, 0.0
    for t in range(acts.shape[0]):
        s_gpu, _, d_gpu = body.step(s_gpu, torch.from_numpy(acts[t]).to(cuda))
        s_np, _, d_np, _ = kernels.legged_step(s_np, acts[t], 901 + t, c)
        flips += int((to_np(d_gpu) != d_np).sum())
        both_live = ~to_np(d_gpu) & ~d_np
        worst = max(worst, float(np.abs(to_np(s_gpu)[:, both_live] - s_np[:, both_live]).max()))
    record(f"legged{c}_traj50", done_flips=flips, max_abs=worst, n=n)
    assert flips <= n // 100, flips


@pytest.mark.parametrize("c", [1, 2, 4])
def test_legged_impulses_match_oracle(cuda, c):
    """The optional (2c, n) contact-impulse output against the oracle's per-substep (lt, ln)
    sums on the golden states; the step itself is unchanged by asking for them."""
    import legged_metal

    g = golden("legged")
    st, ac = g[f"state_c{c}"], g[f"action_c{c}"]
    body = legged_metal.Legged(c)
    body.reseed(80)
    plain = body.step(torch.from_numpy(st).to(cuda), torch.from_numpy(ac).to(cuda))
    body.reseed(80)
    nxt, rew, done, imp = body.step(torch.from_numpy(st).to(cuda), torch.from_numpy(ac).to(cuda), impulses=True)
    np.testing.assert_allclose(to_np(nxt), to_np(plain[0]), rtol=1e-6, atol=1e-6)
    assert (to_np(done) == to_np(plain[2])).all()
    ref = legged.step_impulses(st, ac, c)
    got = to_np(imp)
    assert got.shape == (2 * c, st.shape[1])
    err = np.abs(got - ref)
    # impulses are sums of four Gauss-Seidel solves, as sensitive as the velocities they set
    tol = 1e-4 + 1e-3 * np.abs(ref)
    bad = (err > tol).mean()
    record(f"legged_c{c}_impulses", max_abs=float(err.max()), frac_out_of_tol=float(bad))
    assert bad <= 0.002, (float(err.max()), bad)
    assert (got[1::2] >= 0).all()


# ---- T steps per launch ----------------------------------------------------------------------

def _bodies():
    import hopper_metal
    import legged_metal
    import pendulum_aba_metal
    import pendulum_metal
    import pendulum_metal_coop

    return {
        "mm_k4": (pendulum_metal.Pendulum(4), 3),
        "mm_pairwise_k8": (pendulum_metal.Pendulum(8, pairwise_trig=True), 3),
        "mm_k16": (pendulum_metal.Pendulum(16), 3),
        "coop_k4": (pendulum_metal_coop.Pendulum(4), 3),
        "coop_k16": (pendulum_metal_coop.Pendulum(16), 3),
        "aba_k4": (pendulum_aba_metal.Pendulum(4), 3),
        "aba_k24": (pendulum_aba_metal.Pendulum(24), 3),
        "hopper": (hopper_metal.Hopper(), 3),
        "hopper_branchy": (hopper_metal.Hopper(branchy=True), 3),
        "legged2": (legged_metal.Legged(2), 9),
        "legged4": (legged_metal.Legged(4, 4), 81),
    }


@pytest.mark.parametrize("name", ["mm_k4", "mm_pairwise_k8", "mm_k16", "coop_k4", "coop_k16", "aba_k4", "aba_k24",
                                  "hopper", "hopper_branchy", "legged2", "legged4"])
def test_step_many_equals_chained_steps(cuda, name):
    """T steps in one launch are bit-identical to T single-step launches with the same seeds:
    states, rewards and done flags, across resets (started near the termination boundary)."""
    body, n_act = _bodies()[name]
    n, T = 1000, 30
    state0 = body.reset(n)
    # half the environments start past their termination test, so the window includes resets:
    # a chain standing upright (the pendulum's goal), a torso tilted past 1 rad
    if name.startswith(("mm", "coop", "aba")):
        state0[: state0.shape[0] // 2, : n // 2] = np.pi
    else:
        state0[2, : n // 2] = 1.5
    gen = torch.Generator(device=cuda).manual_seed(3)
    acts = torch.randint(0, n_act, (T, n), device=cuda, generator=gen).to(torch.int32)
    body.reseed(500)
    s, rews, dones = state0, [], []
    for t in range(T):
        s, r, d = body.step(s, acts[t])
        rews.append(r)
        dones.append(d)
    body.reseed(500)
    fin, rseq, dseq = body.step_many(state0, acts)[:3]
    assert torch.equal(fin, s), name
    assert torch.equal(rseq, torch.stack(rews)) and torch.equal(dseq, torch.stack(dones)), name
    assert body.calls == 500 + T
    assert int(dseq.sum()) > 0, "the window should include resets"


def test_legged_step_many_impulses_equal_single_steps(cuda):
    import legged_metal

    body = legged_metal.Legged(4)
    n, T = 512, 10
    state0 = body.reset(n)
    acts = torch.randint(0, 81, (T, n), device=cuda, generator=torch.Generator(device=cuda).manual_seed(4))
    body.reseed(7)
    s, imps = state0, []
    for t in range(T):
        s, _, _, imp = body.step(s, acts[t], impulses=True)
        imps.append(imp)
    body.reseed(7)
    fin, _, _, imp_seq = body.step_many(state0, acts, impulses=True)
    assert torch.equal(fin, s) and torch.equal(imp_seq, torch.stack(imps))


def _abi_launchers(name, stand):
    """(single-step launcher, T-step launcher, rows, n_actions) calling the C ABI with an index
    offset: launch(state, action, seed, n, off) -> (next, reward, done)."""
    import rlenv_lib as rl

    lib = rl.lib()
    sp = rl.stream_ptr()
    kind, arg = name.split("_")[0], int(name.split("_")[-1][1:]) if name[-1].isdigit() else 0

    def outs(rows, n, steps=None):
        shape = (n,) if steps is None else (steps, n)
        return (torch.empty((rows, n), device="cuda"), torch.empty(shape, device="cuda"),
                torch.empty(shape, dtype=torch.bool, device="cuda"))

    if kind in ("mm", "coop", "aba"):
        k, rows, n_act = arg, 2 * arg, 3
        one = {"mm": lambda *a: lib.pendulum_mm_step(k, 0, *a), "coop": lambda *a: lib.pendulum_coop_step(k, *a),
               "aba": lambda *a: lib.pendulum_aba_step(k, *a)}[kind]
        many = {"mm": lambda *a: lib.pendulum_mm_step_many(k, 0, *a),
                "coop": lambda *a: lib.pendulum_coop_step_many(k, *a),
                "aba": lambda *a: lib.pendulum_aba_step_many(k, *a)}[kind]
        tail = ()
    else:
        c = arg
        rows, n_act = 2 * (3 + c), 3 ** c
        one = lambda s, a, dt, seed, n, off, *o: lib.legged_step(c, 8, s, a, dt, seed, stand.data_ptr(), 0.0, None, n,  # noqa: E731
                                                                off, *o, None, sp)
        many = lambda s, a, dt, seed, T, n, off, *o: lib.legged_step_many(c, 8, s, a, dt, seed, stand.data_ptr(),  # noqa: E731
                                                                          0.0, None, T, n, off, *o, None, sp)

    def launch_one(state, action, seed, off):
        n = state.shape[1]
        nxt, r, d = outs(rows, n)
        if kind == "legged":
            rl.check(one(state.data_ptr(), action.data_ptr(), rl.I32, seed, n, off, nxt.data_ptr(), r.data_ptr(),
                         d.data_ptr()))
        else:
            rl.check(one(state.data_ptr(), action.data_ptr(), rl.I32, seed, n, off, nxt.data_ptr(), r.data_ptr(),
                         d.data_ptr(), sp))
        return nxt, r, d

    def launch_many(state, actions, seed, off):
        T, n = actions.shape
        nxt, r, d = outs(rows, n, T)
        if kind == "legged":
            rl.check(many(state.data_ptr(), actions.data_ptr(), rl.I32, seed, T, n, off, nxt.data_ptr(), r.data_ptr(),
                          d.data_ptr()))
        else:
            rl.check(many(state.data_ptr(), actions.data_ptr(), rl.I32, seed, T, n, off, nxt.data_ptr(), r.data_ptr(),
                          d.data_ptr(), sp))
        return nxt, r, d

    return launch_one, launch_many, rows, n_act


@pytest.mark.parametrize("name", ["mm_k4", "mm_k12", "coop_k8", "aba_k5", "aba_k32", "legged_c1", "legged_c3"])
def test_shards_at_index_offsets_equal_the_whole_batch(cuda, name):
    """Two shards stepped with index_offset = their first global environment (ragged sizes)
    reproduce the unsharded batch bit for bit, resets included: what bench.py --gpus N and a
    sharded caller rely on."""
    import legged_metal

    c = int(name[-1]) if name.startswith("legged") else 1
    stand = torch.from_numpy(legged_metal.stand_pose(c)).to(cuda)
    one, many, rows, n_act = _abi_launchers(name, stand)
    n, cut, T = 777, 301, 12
    r = np.random.default_rng(len(name))
    if name.startswith("legged"):
        st = (legged_metal.stand_pose(c)[:, None] + r.uniform(-0.05, 0.05, (rows, n))).astype(np.float32)
        st[2, ::3] = 1.5  # a third start past the tilt limit: resets in the first step
    else:
        st = r.uniform(-0.1, 0.1, (rows, n)).astype(np.float32)
        st[: rows // 2, ::3] = np.pi  # a third start upright: resets in the first step
    state = torch.from_numpy(st).to(cuda)
    act = torch.from_numpy(r.integers(0, n_act, (T, n)).astype(np.int32)).to(cuda)
    whole = one(state, act[0], 9, 0)
    parts = [one(state[:, :cut].contiguous(), act[0, :cut].contiguous(), 9, 0),
             one(state[:, cut:].contiguous(), act[0, cut:].contiguous(), 9, cut)]
    assert bool(whole[2].any()), "the batch should reset somewhere"
    for w, a, b in zip(whole, *parts):
        assert torch.equal(w, torch.cat([a, b], dim=-1)), name
    whole = many(state, act, 40, 0)
    parts = [many(state[:, :cut].contiguous(), act[:, :cut].contiguous(), 40, 0),
             many(state[:, cut:].contiguous(), act[:, cut:].contiguous(), 40, cut)]
    for w, a, b in zip(whole, *parts):
        assert torch.equal(w, torch.cat([a, b], dim=-1)), name
