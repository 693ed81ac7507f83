"""CPU oracle for the batched environment steps and ES rollouts.

TEST INFRASTRUCTURE ONLY. Nothing in the product (the drop-in modules under
metal-rl-envs_b200/, the CUDA library, bench.py's timed GPU path) imports,
links or calls this package. It is the checker: `tests/`, the `smoke()` entry
point and bench.py's CPU-baseline leg use it to compute what the reference
computes on the same inputs.

Each module restates one reference file's algorithm in float32 numpy:

  classic.py   cartpole_np.py, acrobot_np.py
  pendulum.py  pendulum_np.py, pendulum_aba_np.py
  legged.py    hopper_np.py, legged_np.py
  rng.py       the reference kernels' in-kernel reset hash (cartpole_metal.py:40-51)
               and this build's counter-based ES noise
  kernels.py   the reference Metal kernels' step semantics: physics, termination,
               the hash-driven reset of terminated columns, reward
  rollout.py   the fused rollout kernels' semantics (cartpole_rollout_metal.py,
               acrobot_rollout_metal.py, legged_rollout_metal.py)
  es.py        es.py's numpy backend: loop_fitness, centered_ranks, generation, train

The restatement is pinned against golden vectors produced by running the
reference's own numpy modules (tests/golden/make_golden.py) and against the
reference tests' known-answer checks (tests/test_oracle_*.py).
"""
