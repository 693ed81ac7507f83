"""Algorithmic work per environment step, for the roofline figures.

Counting rule: a fused multiply-add is 2 flops; an add, multiply, divide, floor,
min or max is 1; square roots and transcendentals (sin, cos, tanh, log) are
counted separately, since on sm_100a the precise versions are instruction
sequences rather than single operations. Integer work (the reset hash, index
arithmetic) is not counted. The counts follow the formulas of the kernels in
csrc/*.cuh term by term; they are the denominators' numerators, not profiler
readings.
"""

# Acrobot: Gym's derivative as the reference writes it (acrobot_np.py:64-86) is 36 flops, 4
# divides included, and 4 transcendentals (sin and cos of theta2, two cosines for the potential
# terms); classic.cuh evaluates it with the unit constants folded, in 33.
# RK4: 4 derivatives (144) + three stage states (4 x 2 x 3 = 24) + the weighted sum and
# update (4 x 7 = 28) + two wraps (2 x 5) + two clips (2 x 2) + termination (3): 213 flops;
# transcendentals 4 x 4 + 2 (termination) = 18.
ACROBOT = dict(flops=213, transcendentals=18)

# CartPole as the reference writes it (cartpole_np.py:58-77): temp 5, theta_acc 9 (one divide
# each side), x_acc 5, four Euler updates as FMAs (8), termination 2 compares: 29 flops; sin and
# cos: 2. classic.cuh folds the divisions by the total mass into constants.
CARTPOLE = dict(flops=29, transcendentals=2)

# Bytes moved per environment step by the single-step kernel: state in and out
# (2 x 16), one action, a 4-byte reward and a 1-byte done. The T-step kernel
# moves the state once per launch and per step only the action, reward and done.
def step_bytes(rows=4, action_bytes=1):
    return 2 * 4 * rows + action_bytes + 4 + 1


def step_many_bytes(rows, n, T, action_bytes=1, write_seq=True):
    per_step = action_bytes + (5 if write_seq else 0)
    return n * (2 * 4 * rows + T * per_step)


def mass_matrix_flops(k):
    """Per step of the K-link mass-matrix form, 4 RK4 stages: matrix and right-hand side
    (addition formulas: 6K^2 for cos/sin differences and products, 3K^2 for the Coriolis sum,
    2K for gravity), Cholesky K^3/3 + K^2/2, two substitutions 2K^2, plus the RK4
    combination (12K). The reference's own count (bench_pendulum.py:29-33) is of the same form."""
    stage = 6 * k * k + 3 * k * k + 2 * k + k ** 3 / 3 + k * k / 2 + 2 * k * k
    return dict(flops=round(4 * stage + 12 * k), transcendentals=4 * 2 * k + k)


def aba_flops(k):
    """Per step of the articulated-body form as the reference counts it (bench_aba.py:53-55):
    about 140 flops per link and stage over the three passes of the full 3x3 spatial algebra,
    plus the RK4 combination. The roofline uses it."""
    return dict(flops=4 * 140 * k + 12 * k, transcendentals=4 * 6 * k + k)


def aba_rank_one_flops(k):
    """The same step as this build computes it (the rank-one form of csrc/pendulum.cuh,
    aba_accel_unrolled): per link and RK4 stage, the outward velocity 9, the inward step 24 (own
    bias 5, the joint's D, u / D, U1 / D and the projected inertia 8, its bias 4, the rank-one
    carry 7), the last pass's acceleration 16; plus the RK4 combination (12 per link).
    Transcendentals: one sine and cosine per link and stage, and the termination cosines. The
    long-chain kernel recomputes the link velocities and the joint trig instead of storing them;
    that recomputation is not counted."""
    return dict(flops=4 * 49 * k + 12 * k, transcendentals=4 * 2 * k + k)


def legged_flops(c, iters=8):
    """Per step of the legged body (4 substeps) as csrc/legged.cuh computes it.
    - The mass matrix is solved in closed form: an arrowhead structure, with the legs
      eliminated first and then a 2x2 Schur block.
    - The Delassus blocks come from the same closed form. Off the diagonal they are rank
      one, so a contact sees the others through one scalar coupling s.
    - Each contact's exact block solve is affine in s in each of its regimes, so its
      coefficients are formed once per substep and a Gauss-Seidel solve is the coupling, seven
      multiply-adds and three comparisons; the exact impulse is solved once at the end.
    Per substep, with n = 3 + C:
    - leg kinematics 12C; Schur block 6C + 12; generalised forces 15C + 12;
    - two mass solves 2 (14C + 7); free velocity and update 5n;
    - Delassus, the diagonal blocks in full and G below the diagonal, 1.5C^2 + 24.5C;
    - free relative velocities 10C; per-contact constants (three reciprocals, the slip
      coefficient, the Baumgarte target) 14C;
    - (C > 1) the affine coefficients 41C; per sweep and contact 2(C - 1) + 17; the final exact
      impulse 42C; (C = 1) one exact impulse, 42;
    - J^T lambda 9C.
    Every sweep is counted (the rollout's skipping of contacts no live member touches only
    removes zero terms). Transcendentals: C sines and cosines, 3C + 1 reciprocals."""
    n = 3 + c
    solve = (41 * c + iters * c * (2 * (c - 1) + 17) + 42 * c) if c > 1 else 42
    sub = (12 * c + 6 * c + 12 + 15 * c + 12 + 2 * (14 * c + 7) + 5 * n + 1.5 * c * c + 24.5 * c + 10 * c
           + 14 * c + solve + 9 * c)
    return dict(flops=round(4 * sub), transcendentals=4 * (2 * c + 3 * c + 1))


def legged_reference_flops(c, iters=8):
    """The same step as the reference computes it (legged_np.py:57-97): the dense (3+C)^2 mass
    matrix, its Cholesky factor and 2C + 1 dense solves, the Delassus blocks from the solves;
    the Gauss-Seidel sweeps over the full 2x2 blocks, 8(C - 1) + 40 per sweep and contact.
    For comparison only: the kernel does the closed form with affine sweeps."""
    n = 3 + c
    sub = (10 * c + (n * (n + 1) // 2) * 2 * c + 8 * n * c + n ** 3 / 3 + (2 * c + 1) * 2 * n * n
           + 24 * c * c + 12 * c + iters * c * (8 * (c - 1) + 40) + 4 * n * c + 4 * n)
    return dict(flops=round(4 * sub), transcendentals=4 * (2 * c + n))


def es_member_step_flops(task):
    """Per member-step of a fused ES rollout: the obs-H-out tanh MLP (FMA = 2, one tanh per hidden
    unit) plus the body's step. CartPole 4-32-2 and Acrobot 6-32-3 (obs = cos/sin of both angles
    and both velocities); legged4 13-16-12 (three logits per leg) plus 4 substeps at 8 sweeps."""
    if task == "cartpole":
        mlp = 2 * (4 * 32 + 32 * 2) + 32 + 2
        return dict(flops=mlp + CARTPOLE["flops"], transcendentals=32 + CARTPOLE["transcendentals"])
    if task == "acrobot":
        mlp = 2 * (6 * 32 + 32 * 3) + 32 + 3
        return dict(flops=mlp + ACROBOT["flops"], transcendentals=32 + ACROBOT["transcendentals"])
    if task == "legged4":
        mlp = 2 * (13 * 16 + 16 * 12) + 16 + 12
        body = legged_flops(4, 8)
        return dict(flops=mlp + body["flops"], transcendentals=16 + body["transcendentals"])
    raise ValueError(task)
