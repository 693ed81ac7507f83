"""Generate the golden vectors that pin the oracle to the reference's own numpy code.

Run where a checkout of the reference exists, with $REF_PATH naming it:

    REF_PATH=<path of the reference checkout> python tests/golden/make_golden.py

It imports the reference's numpy modules (cartpole_np, acrobot_np, pendulum_np,
pendulum_aba_np, hopper_np, legged_np, and es.py with a stub `mlx` module so
that es.py's numpy backend imports without MLX), runs them on seeded inputs
shaped like the reference's own test generators, and writes one .npz per body
next to this file. Tests and the GPU parity checks read only the .npz files;
the reference itself is never needed at test time.
"""

import os
import sys
import types
from pathlib import Path
from unittest import mock

import numpy as np

OUT = Path(__file__).resolve().parent
REF = Path(os.environ["REF_PATH"]) if os.environ.get("REF_PATH") else None


def _import_reference():
    if REF is None or not REF.exists():
        raise SystemExit("set REF_PATH to the reference checkout (the directory holding cartpole_np.py)")
    mlx = types.ModuleType("mlx")
    mlx.core = mock.MagicMock()
    sys.modules["mlx"] = mlx
    sys.modules["mlx.core"] = mlx.core
    sys.path.insert(0, str(REF))
    import acrobot_np
    import cartpole_np
    import es
    import hopper_np
    import legged_np
    import pendulum_aba_np
    import pendulum_np
    return cartpole_np, acrobot_np, pendulum_np, pendulum_aba_np, hopper_np, legged_np, es


CHECKPOINTS = (1, 10, 25, 50, 100)


def _trajectory(physics, state, actions):
    """Chain the pure physics (no termination or reset) over the given action rows; keep the
    states after the CHECKPOINTS steps that the chain reaches."""
    out = []
    for t, a in enumerate(actions, 1):
        state = physics(state, a)
        if t in CHECKPOINTS:
            out.append(state)
    return np.stack(out)


def main():
    cartpole_np, acrobot_np, pendulum_np, pendulum_aba_np, hopper_np, legged_np, es = _import_reference()

    # CartPole: the reference test's batch shape (test_cartpole.py:33-37), a 100-step physics chain
    rng = np.random.default_rng(0)
    state = rng.uniform(-1, 1, size=(4, 256)).astype(np.float32)
    action = rng.integers(0, 2, size=256)
    stepped = cartpole_np._physics(state, action)
    s0 = rng.uniform(-0.05, 0.05, size=(4, 128)).astype(np.float32)
    acts = rng.integers(0, 2, size=(100, 128))
    np.savez_compressed(OUT / "cartpole.npz", state=state, action=action, stepped=stepped,
                        done=cartpole_np._terminated(stepped), traj_state=s0, traj_actions=acts,
                        traj=_trajectory(cartpole_np._physics, s0, acts))

    # Acrobot: angles anywhere, velocities +-2 (test_acrobot.py:52-56)
    rng = np.random.default_rng(1)
    state = np.stack([rng.uniform(-np.pi, np.pi, 256), rng.uniform(-np.pi, np.pi, 256),
                      rng.uniform(-2, 2, 256), rng.uniform(-2, 2, 256)]).astype(np.float32)
    action = rng.integers(0, 3, size=256)
    stepped = acrobot_np._physics(state, action)
    s0 = rng.uniform(-0.1, 0.1, size=(4, 128)).astype(np.float32)
    acts = rng.integers(0, 3, size=(100, 128))
    np.savez_compressed(OUT / "acrobot.npz", state=state, action=action, stepped=stepped,
                        done=acrobot_np._terminated(stepped), traj_state=s0, traj_actions=acts,
                        traj=_trajectory(acrobot_np._physics, s0, acts))

    # K-link pendulum, both forms (test_pendulum.py:26-28)
    arrays = {}
    for k in (2, 3, 4, 8, 16, 32, 64):
        n = 200 if k <= 16 else 64
        rng = np.random.default_rng(k)
        st = np.concatenate([rng.uniform(-np.pi, np.pi, (k, n)), rng.uniform(-1, 1, (k, n))]).astype(np.float32)
        ac = rng.integers(0, 3, n)
        arrays[f"state_k{k}"], arrays[f"action_k{k}"] = st, ac
        tq = ((ac - 1) * 1.0).astype(np.float32)
        aba = pendulum_aba_np.Pendulum(k)
        arrays[f"aba_stepped_k{k}"] = aba._physics(st, ac)
        arrays[f"aba_done_k{k}"] = aba._terminated(arrays[f"aba_stepped_k{k}"])
        arrays[f"aba_acc_k{k}"] = pendulum_aba_np.aba_accelerations(np, st[:k], st[k:], tq, k)
        if k <= 16:
            mm = pendulum_np.Pendulum(k)
            arrays[f"mm_stepped_k{k}"] = mm._physics(st, ac)
            arrays[f"mm_done_k{k}"] = mm._terminated(arrays[f"mm_stepped_k{k}"])
            arrays[f"mm_acc_k{k}"] = mm._dsdt(st, tq)[k:]
    rng = np.random.default_rng(99)
    for k in (4, 16):
        s0 = np.concatenate([rng.uniform(-0.1, 0.1, (k, 32)), np.zeros((k, 32))]).astype(np.float32)
        acts = rng.integers(0, 3, size=(50, 32))
        arrays[f"traj_state_k{k}"], arrays[f"traj_actions_k{k}"] = s0, acts
        arrays[f"mm_traj_k{k}"] = _trajectory(pendulum_np.Pendulum(k)._physics, s0, acts)
        arrays[f"aba_traj_k{k}"] = _trajectory(pendulum_aba_np.Pendulum(k)._physics, s0, acts)
    np.savez_compressed(OUT / "pendulum.npz", **arrays)

    # Hopper: mixed contact regimes (test_hopper.py:116-121), and the exact contact impulse on
    # random SPD Delassus blocks (test_hopper.py:268-281)
    rng = np.random.default_rng(0)
    n = 500
    ranges = ((-1.0, 1.0), (0.7, 1.3), (-0.6, 0.6), (-0.8, 0.8))  # x, y, phi, psi; drawn in this order
    q = np.stack([rng.uniform(lo, hi, n) for lo, hi in ranges])
    state = np.concatenate([q, rng.uniform(-2, 2, (4, n))]).astype(np.float32)
    action = rng.integers(0, 3, n)
    h = hopper_np.Hopper()
    stepped = h._physics(state, action)
    b = rng.uniform(-1, 1, (2000, 2, 2))
    A = np.einsum("nij,nkj->nik", b, b) + 0.05 * np.eye(2)
    att, atn, ann = (A[:, i, j].astype(np.float32) for i, j in ((0, 0), (0, 1), (1, 1)))
    wt, wn = rng.uniform(-2, 2, 2000).astype(np.float32), rng.uniform(-2, 2, 2000).astype(np.float32)
    depth = rng.uniform(-0.1, 0.1, 2000).astype(np.float32)
    lt, ln = hopper_np.contact_impulse(np, att, atn, ann, wt, wn, depth, hopper_np.MU)
    np.savez_compressed(OUT / "hopper.npz", state=state, action=action, stepped=stepped, done=h._terminated(stepped),
                        att=att, atn=atn, ann=ann, wt=wt, wn=wn, depth=depth, lt=lt, ln=ln)

    # Legged C in {1, 2, 4} (test_legged.py:12-17), several sweep counts and an assisted case
    arrays = {}
    for c in (1, 2, 4):
        rng = np.random.default_rng(c)
        d, n = 3 + c, 300
        q = np.concatenate([np.stack([rng.uniform(-1, 1, n), rng.uniform(0.7, 1.3, n), rng.uniform(-0.6, 0.6, n)]),
                            rng.uniform(-0.8, 0.8, (c, n))])
        st = np.concatenate([q, rng.uniform(-2, 2, (d, n))]).astype(np.float32)
        ac = rng.integers(0, 3**c, n)
        arrays[f"state_c{c}"], arrays[f"action_c{c}"] = st, ac
        for iters in (1, 4, 8, 16):
            body = legged_np.Legged(c, iters)
            out = body._physics(st, ac)
            arrays[f"stepped_c{c}_i{iters}"] = out
            arrays[f"done_c{c}_i{iters}"] = body._terminated(out)
        arrays[f"assist_stepped_c{c}"] = legged_np.Legged(c)._physics(st, ac, 20.0)
        arrays[f"stand_c{c}"] = legged_np.stand_pose(c)
        arrays[f"static_c{c}"] = legged_np.static_pose(c)
    np.savez_compressed(OUT / "legged.npz", **arrays)

    # ES pieces: centred ranks (default sort, as the reference), unflatten, per-leg actions, and
    # the numpy backend's loop fitness and one generation for three tasks
    arrays = {}
    rng = np.random.default_rng(7)
    distinct = rng.normal(size=64).astype(np.float32)
    arrays["ranks_in"], arrays["ranks_out"] = distinct, es.centered_ranks(np, distinct)
    arrays["ranks_known_in"] = np.array([3.0, 1.0, 2.0, 10.0], dtype=np.float32)
    arrays["ranks_known_out"] = es.centered_ranks(np, arrays["ranks_known_in"])
    logits = rng.normal(size=(32, 6)).astype(np.float32)
    arrays["leg_logits"], arrays["leg_action"] = logits, es.TASKS["legged2"].action(np, logits)
    for name, pop, horizon in (("cartpole", 64, 60), ("acrobot", 64, 40), ("legged2", 32, 25)):
        task = es.TASKS[name]
        hidden = task.hidden
        backend = es.NumpyBackend(task, 3)
        theta = backend.normal((es.n_params(hidden, task),)) * 0.1
        cfg = es.Config(task=name, pop=pop, horizon=horizon, sigma=0.1, lr=0.1)
        new_theta, fit, steps = es.generation(backend, theta, cfg, hidden, 1)
        arrays[f"{name}_theta0"], arrays[f"{name}_theta1"] = theta, new_theta
        arrays[f"{name}_fit"], arrays[f"{name}_steps"] = fit, steps
    np.savez_compressed(OUT / "es.npz", **arrays)
    for f in sorted(OUT.glob("*.npz")):
        print(f"{f.name}: {f.stat().st_size / 1024:.0f} KB")


if __name__ == "__main__":
    main()
