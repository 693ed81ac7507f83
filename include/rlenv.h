/*
 * rlenv.h — C ABI of librlenv.so, the sm_100a CUDA implementation of the batched
 * environment step kernels and the fused Evolution Strategies rollouts of
 * metal-rl-envs.
 *
 * Every entry point replaces one `mx.fast.metal_kernel` of the reference (its
 * file:line is given beside each declaration). The conventions are the same for all:
 *
 *  - State is structure-of-arrays, row-major (D, N) float32: row r of
 *    environment i is state[r * N + i]. Every pointer is a device pointer
 *    unless its comment says otherwise.
 *  - The caller allocates every buffer. The library never allocates or frees
 *    memory and holds no state between calls; the one exception is
 *    rlenv_es_centered_ranks_static, whose scratch is a fixed array of the
 *    library (its address cached per device and context).
 *  - Work is enqueued asynchronously on `stream` (a cudaStream_t; NULL is the
 *    legacy default stream). Calls are reentrant, except that overlapping calls of
 *    rlenv_es_centered_ranks_static on one device share its scratch.
 *  - Inputs are never written. Outputs must not alias inputs except where a
 *    comment says so.
 *  - The return value is 0 on success, a negative RLENV_E* code for an argument
 *    that the library rejects before launching anything, or a positive
 *    cudaError_t from the launch. Nothing aborts or traps.
 *  - `seed` is the per-call counter of the reference (`_calls`, incremented
 *    before every step call, cartpole_metal.py:106-125). A terminated
 *    environment i is reset from pcg_hash(seed ^ ((i + index_offset) *
 *    0x9E3779B9)) plus a per-row offset, so that a shard starting at global
 *    environment `index_offset` draws exactly the resets the unsharded batch
 *    would.
 *  - Actions are integer arrays of N elements whose element type is given by
 *    `action_dtype` (RLENV_I32, RLENV_I64 or RLENV_U8; the CartPole and Acrobot kernels
 *    also take RLENV_U2, four steps' actions packed into a byte).
 *  - `done` is one byte per environment, 0 or 1 (torch.bool layout).
 */
#ifndef RLENV_H
#define RLENV_H

#include <stdint.h>

#if defined(__GNUC__)
#define RLENV_API __attribute__((visibility("default")))
#else
#define RLENV_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes and dtypes ------------------------------------------- */
#define RLENV_OK 0
#define RLENV_EINVAL (-1)       /* a null pointer, a negative size, an unknown dtype        */
#define RLENV_EUNSUPPORTED (-2) /* a (K, C, H, ...) for which no kernel instance is built  */

#define RLENV_I32 0
#define RLENV_I64 1
#define RLENV_U8 2
/* Actions packed along time, CartPole and Acrobot step kernels only (the other kernels
 * answer RLENV_EINVAL): a (ceil(T / 4), N) byte array whose byte (r, i) holds environment i's
 * actions of steps 4r .. 4r + 3, step 4r + u in bits 2u .. 2u + 1 (a single step reads bits
 * 0-1 of N bytes). A caller that streams T steps of actions from host memory moves a quarter
 * of the uint8 bytes. No counterpart in the reference, whose kernels read int32 actions. */
#define RLENV_U2 3

/* Human-readable message for a status code; the string is static. */
RLENV_API const char* rlenv_strerror(int code);

/* Version of this ABI: bumped whenever a signature below changes. */
RLENV_API int rlenv_abi_version(void);

/* The check build (librlenv_checks.so, compiled with -DRLENV_CHECKS; no
 * counterpart in the reference, whose Metal kernels cannot report). Its kernels
 * record problems in a device word instead of trapping: bit 1 an action outside
 * its body's range, bit 2 a non-finite value written to an output. This reads
 * the OR of every kernel's word on the current device into *word and, with
 * clear, zeroes them. It synchronises the device. In the normal build it
 * returns RLENV_EUNSUPPORTED and touches no GPU. */
RLENV_API int rlenv_checks_status(unsigned int* word, int clear);

/* ---- CartPole ------------------------------------------------------------
 * Replaces `cartpole_step` (cartpole_metal.py:69-104, launched at :114-125).
 * state (4, n) rows x, x_dot, theta, theta_dot; action 1 pushes right, anything
 * else left; reward 1 for every environment; done when |x| > 2.4 or
 * |theta| > 12 degrees, after which the column is reset uniformly in +-0.05.
 */
RLENV_API int rlenv_cartpole_step(const float* state, const void* action, int action_dtype,
                        uint32_t seed, int64_t n, int64_t index_offset,
                        float* next_state, float* reward, uint8_t* done, void* stream);

/* T consecutive CartPole steps in one launch, the state held in registers.
 * No reference counterpart: it is what a chain of T `step` calls computes
 * (cartpole_metal.py:114-125 called T times), with step t using the per-call
 * seed seed0 + t. actions (T, n); reward_seq (T, n) and done_seq (T, n) may be
 * NULL; reward_sum and done_count (n) may be NULL and, when given, receive the
 * per-environment sums over the T steps. state_out may equal state_in. */
RLENV_API int rlenv_cartpole_step_many(const float* state_in, const void* actions, int action_dtype,
                             uint32_t seed0, int64_t steps, int64_t n, int64_t index_offset,
                             float* state_out, float* reward_seq, uint8_t* done_seq,
                             float* reward_sum, float* done_count, void* stream);

/* ---- Acrobot -------------------------------------------------------------
 * Replaces `acrobot_step` (acrobot_metal.py:24-111). state (4, n) rows theta1,
 * theta2, dtheta1, dtheta2; action in {0, 1, 2} is torque action - 1; RK4 with
 * dt 0.2; reward -1, or 0 on the terminating step; reset uniform in +-0.1. */
RLENV_API int rlenv_acrobot_step(const float* state, const void* action, int action_dtype,
                       uint32_t seed, int64_t n, int64_t index_offset,
                       float* next_state, float* reward, uint8_t* done, void* stream);

/* T Acrobot steps per launch; same contract as rlenv_cartpole_step_many. */
RLENV_API int rlenv_acrobot_step_many(const float* state_in, const void* actions, int action_dtype,
                            uint32_t seed0, int64_t steps, int64_t n, int64_t index_offset,
                            float* state_out, float* reward_seq, uint8_t* done_seq,
                            float* reward_sum, float* done_count, void* stream);

/* ---- K-link pendulum -----------------------------------------------------
 * state (2k, n): k absolute angles then k angular velocities; action in
 * {0, 1, 2} is a root torque of action - 1; RK4 with dt 0.02; reward -1, or 0 on
 * the terminating step; reset uniform in +-0.1 on all 2k rows.
 *
 * Mass-matrix form, one thread per environment. Replaces `pendulum{K}_step`
 * and its `_pairwise` variant (pendulum_metal.py:11-131). pairwise_trig != 0
 * evaluates cos and sin of every angle difference directly instead of by the
 * addition formulas. Built for k in 1..16. */
RLENV_API int rlenv_pendulum_mm_step(int k, int pairwise_trig, const float* state, const void* action,
                           int action_dtype, uint32_t seed, int64_t n, int64_t index_offset,
                           float* next_state, float* reward, uint8_t* done, void* stream);

/* `steps` consecutive steps of rlenv_pendulum_mm_step in one launch, the state
 * kept on chip: actions (steps, n); step t draws its resets from seed0 + t and
 * writes row t of reward_seq / done_seq (steps, n), each of which may be NULL.
 * Equal bit for bit to `steps` single-step calls with seeds seed0, seed0 + 1, ...
 * The reference has no multi-step call; it replaces a caller's loop of
 * Pendulum.step (bench_pendulum.py:36-48). The same holds for the *_step_many
 * entry points below. */
RLENV_API int rlenv_pendulum_mm_step_many(int k, int pairwise_trig, const float* state, const void* actions,
                                int action_dtype, uint32_t seed0, int64_t steps, int64_t n,
                                int64_t index_offset, float* state_out, float* reward_seq,
                                uint8_t* done_seq, void* stream);

/* Mass-matrix form with k lanes of a warp per environment, lane j owning row j
 * of the mass matrix. Replaces `pendulum{K}_coop_step`
 * (pendulum_metal_coop.py:28-149). k in {2, 4, 8, 16, 32}. */
RLENV_API int rlenv_pendulum_coop_step(int k, const float* state, const void* action, int action_dtype,
                             uint32_t seed, int64_t n, int64_t index_offset,
                             float* next_state, float* reward, uint8_t* done, void* stream);

RLENV_API int rlenv_pendulum_coop_step_many(int k, const float* state, const void* actions, int action_dtype,
                                  uint32_t seed0, int64_t steps, int64_t n, int64_t index_offset,
                                  float* state_out, float* reward_seq, uint8_t* done_seq,
                                  void* stream);

/* Articulated-body (Featherstone) form, O(k) per stage, one thread per
 * environment. Replaces `pendulum{K}_aba_step` (pendulum_aba_metal.py:14-144).
 * Any k from 1 to 192 (k > 192: RLENV_EUNSUPPORTED). For 32 <= k <= 64 and a
 * batch that fills the GPU the launch runs one block per SM that allocates all
 * 512 tensor-memory columns of its SM (tcgen05.alloc) and frees them before it
 * ends; a tensor-memory kernel of the caller's on another stream can delay its
 * blocks, never deadlock them (each allocation waits only for blocks that run to
 * completion). Results do not depend on which kernel a batch size selects. */
RLENV_API int rlenv_pendulum_aba_step(int k, const float* state, const void* action, int action_dtype,
                            uint32_t seed, int64_t n, int64_t index_offset,
                            float* next_state, float* reward, uint8_t* done, void* stream);

RLENV_API int rlenv_pendulum_aba_step_many(int k, const float* state, const void* actions, int action_dtype,
                                 uint32_t seed0, int64_t steps, int64_t n, int64_t index_offset,
                                 float* state_out, float* reward_seq, uint8_t* done_seq,
                                 void* stream);

/* The articulated body with one warp per environment (no counterpart in the reference, whose
 * only cooperative pendulum is the mass-matrix form): the recurrences along the chain (link
 * velocities, articulated masses, bias forces, accelerations) run as scans over the warp's
 * lanes, so a batch too small to fill the GPU with one thread per environment steps in a few
 * levels of shuffles instead of K dependent link steps. Same arguments and results as
 * rlenv_pendulum_aba_step_many, to float rounding (the sums are associated differently);
 * chained calls and one T-step call agree bit for bit. k in 1..192. */
RLENV_API int rlenv_pendulum_aba_coop_step_many(int k, const float* state, const void* actions, int action_dtype,
                                      uint32_t seed0, int64_t steps, int64_t n, int64_t index_offset,
                                      float* state_out, float* reward_seq, uint8_t* done_seq, void* stream);

/* ---- Hopper and legged bodies ---------------------------------------------
 * Legged body with c legs and c hard contacts (legged_metal.py:13-185):
 * state (2(3+c), n) = q then q_dot with q = (x, y, phi, psi_1..psi_c); action in
 * [0, 3^c) decoded per leg to a torque ((a / 3^leg) % 3 - 1) * 2; 4 substeps of
 * 0.01 with `iters` block projected Gauss-Seidel sweeps over the contacts;
 * reward x_dot + 1, or 0 on the terminating step; done when y < 0.6 or
 * |phi| > 1; reset to stand (2(3+c) floats, device) plus uniform +-0.05 on every
 * row. assist_ptr (device, one float) overrides `assist` when not NULL: it is
 * the stiffness of the torso-upright spring-damper of the curriculum.
 * impulses (2c, n), when not NULL, receives per foot k the tangential (row 2k)
 * and normal (row 2k + 1) contact impulse summed over the step's four
 * substeps: the (lt, ln) of legged_np.py:89-96. The reference's step does not
 * return them; BASELINE.json asks for them among the step's outputs.
 * Built for c in 1..4; iters >= 1. */
RLENV_API int rlenv_legged_step(int c, int iters, const float* state, const void* action, int action_dtype,
                      uint32_t seed, const float* stand, float assist, const float* assist_ptr,
                      int64_t n, int64_t index_offset,
                      float* next_state, float* reward, uint8_t* done, float* impulses,
                      void* stream);

/* `steps` legged steps in one launch (see rlenv_pendulum_mm_step_many);
 * impulse_seq, when not NULL, is (steps, 2c, n): step t's impulses as
 * rlenv_legged_step writes them. */
RLENV_API int rlenv_legged_step_many(int c, int iters, const float* state, const void* actions,
                           int action_dtype, uint32_t seed0, const float* stand, float assist,
                           const float* assist_ptr, int64_t steps, int64_t n, int64_t index_offset,
                           float* state_out, float* reward_seq, uint8_t* done_seq,
                           float* impulse_seq, void* stream);

/* Hopper: the one-legged body with an exact single-contact solve, equal to the
 * legged body with c = 1 and one sweep. Replaces `hopper_step` and
 * `hopper_step_branchy` (hopper_metal.py:13-138): branchy != 0 skips the
 * contact solve of airborne environments with a branch instead of a select.
 * state (8, n); stand as for rlenv_legged_step. */
RLENV_API int rlenv_hopper_step(int branchy, const float* state, const void* action, int action_dtype,
                      uint32_t seed, const float* stand, int64_t n, int64_t index_offset,
                      float* next_state, float* reward, uint8_t* done, void* stream);

RLENV_API int rlenv_hopper_step_many(int branchy, const float* state, const void* actions, int action_dtype,
                           uint32_t seed0, const float* stand, int64_t steps, int64_t n,
                           int64_t index_offset, float* state_out, float* reward_seq,
                           uint8_t* done_seq, void* stream);

/* ---- Fused ES rollouts ------------------------------------------------------
 * One launch runs a whole population: member i runs its own MLP policy from
 * parameter row theta + i * theta_stride (theta_stride 0 shares one row) against
 * its own environment from column i of state (D, p) until its first
 * termination or `horizon` steps. Rows are es.unflatten's layout: w1 (obs, h)
 * row-major, b1 (h), w2 (h, out) row-major, b2 (out). The policy acts greedily,
 * the first index winning ties.
 *
 * CartPole (cartpole_rollout_metal.py:46-100), obs 4, out 2: fitness = steps
 * survived (the terminating step excluded). hidden in {1, 2, 4, 8, 16, 32, 64}. */
RLENV_API int rlenv_cartpole_rollout(const float* state, const float* theta, int64_t theta_stride,
                           int64_t p, int hidden, int horizon, float* fitness, void* stream);

/* Acrobot (acrobot_rollout_metal.py:21-81), obs (cos t1, sin t1, cos t2,
 * sin t2, dt1, dt2), out 3: fitness = steps before the tip first clears height 1.
 * hidden as for CartPole. */
RLENV_API int rlenv_acrobot_rollout(const float* state, const float* theta, int64_t theta_stride,
                          int64_t p, int hidden, int horizon, float* fitness, void* stream);

/* Legged (legged_rollout_metal.py:19-83), obs = state without x (5 + 2c),
 * out 3c (one three-way head per leg): fitness = sum over steps before the
 * first fall of (y >= gate ? x_dot : 0) + alive, minus `fall` once at a fall;
 * steps = steps taken including the falling one. c in 1..4, hidden in
 * {1, 2, 4, 8, 16, 32}. */
RLENV_API int rlenv_legged_rollout(int c, int hidden, int horizon, int iters, float alive, float fall,
                         float gate, float assist, const float* state, const float* theta,
                         int64_t theta_stride, int64_t p, float* fitness, float* steps,
                         void* stream);

/* The same rollout with the lanes per member chosen by the caller: 1, 2 or 4,
 * dividing both c and hidden (2 and 4 need c even), or 0 for the library's
 * choice, which rlenv_legged_rollout uses. Lane l of a member's group owns its
 * contacts [l c / lanes, (l + 1) c / lanes) and hidden units
 * [l hidden / lanes, ...); every width gives the same bits, and the same bits as
 * stepping the body with rlenv_legged_step. The reference runs one thread per
 * member (legged_rollout_metal.py:19-83); this entry point is for tuning and for
 * tests of that equality. */
RLENV_API int rlenv_legged_rollout_lanes(int lanes, int c, int hidden, int horizon, int iters,
                               float alive, float fall, float gate, float assist,
                               const float* state, const float* theta, int64_t theta_stride,
                               int64_t p, float* fitness, float* steps, void* stream);

/* ---- ES generation pieces (es.py:214-227) ------------------------------------
 * Noise: half (rows, d) of standard normals for antithetic pairs
 * [row_offset, row_offset + rows), element (pair, j) a function of
 * (seed, gen, pair, j) only (Philox-4x32-10 and Box-Muller), so any shard of
 * the pairs regenerates the same values. Replaces es.py:220's
 * mx.random.normal((P/2, D)). */
RLENV_API int rlenv_es_noise(float* half, int64_t rows, int64_t d, uint64_t seed, uint64_t gen,
                   int64_t row_offset, void* stream);

/* Perturbed population rows for members [member_offset, member_offset + rows)
 * of a population of 2 * pairs: member m < pairs gets theta + sigma * half[m],
 * member m >= pairs gets theta - sigma * half[m - pairs] (es.py:221-223). The
 * noise is regenerated in the kernel from (seed, gen, pair), exactly as
 * rlenv_es_noise computes it. theta_pop (rows, d). */
RLENV_API int rlenv_es_perturb(const float* theta, int64_t d, float sigma, uint64_t seed, uint64_t gen,
                     int64_t pairs, int64_t member_offset, int64_t rows, float* theta_pop,
                     void* stream);

/* Centred ranks (es.py:214-215): ranks[i] = r_i / (p - 1) - 0.5 with r_i the
 * position of fitness[i] in ascending order, ties broken by index (a stable
 * sort), NaN after every number as in numpy's sort. p >= 2. O(p^2) work in
 * one launch: the faster choice up to a few thousand members. */
RLENV_API int rlenv_es_centered_ranks(const float* fitness, int64_t p, float* ranks, void* stream);

/* Device scratch in bytes that rlenv_es_centered_ranks_sorted needs for p
 * members: 16 p above 4,096 members, 0 up to that; -1 for p < 0. */
RLENV_API int64_t rlenv_es_ranks_scratch_bytes(int64_t p);

/* The ranks of rlenv_es_centered_ranks, bit for bit, in O(p log p) work: a
 * sort of unique (fitness order, index) keys instead of p^2 comparisons, for
 * large populations (the reference's own results run es.py at P = 262,144).
 * Both kernels order fitness as numpy's sort does: NaN after every number.
 * scratch: caller-allocated device memory, 8-byte aligned, of at least
 * rlenv_es_ranks_scratch_bytes(p) bytes (may be NULL when that is 0); nothing
 * in it needs to be initialised. 2 <= p <= 2^31. Same reference interface as
 * rlenv_es_centered_ranks (es.py:214-215). */
RLENV_API int rlenv_es_centered_ranks_sorted(const float* fitness, int64_t p, float* ranks,
                                             void* scratch, int64_t scratch_bytes, void* stream);

/* rlenv_es_centered_ranks_sorted for callers that cannot allocate device
 * memory: no counterpart in the reference, which has no such caller. Such
 * callers include code running inside a memory pool or allocator that forbids
 * further allocation, a framework that hands out only its own buffers, and
 * steps that must not add allocation latency or fragmentation. It allocates
 * nothing; its scratch is a fixed 1 MiB array inside the library (per device,
 * held until the process exits), so 2 <= p <= 65,536 and larger p is rejected
 * with RLENV_EINVAL. The first call on each device, with that device current,
 * looks up the array's device address once; make that first call before any
 * stream capture. The address is kept with the context it belongs to: after
 * the device's context is replaced (cudaDeviceReset, then new work), the next
 * call looks it up again, so again make that call outside a capture. Nothing in the array needs to start at zero. Calls on one
 * device whose executions overlap (different streams or host threads) share
 * the array and race; issue them on one stream. Same ranks, bit for bit, as
 * the other two rank entry points. */
RLENV_API int rlenv_es_centered_ranks_static(const float* fitness, int64_t p, float* ranks, void* stream);

/* Rank-weighted antithetic update (es.py:224-225):
 * theta_out = theta + lr / (2 * pairs * sigma) * sum_j (ranks[j] - ranks[j + pairs]) * half[j],
 * with half regenerated from (seed, gen) and a fixed summation order, so every
 * rank of a multi-GPU job computes the same bits. theta_out may equal theta. */
RLENV_API int rlenv_es_update(const float* theta, const float* ranks, int64_t d, int64_t pairs, float lr,
                    float sigma, uint64_t seed, uint64_t gen, float* theta_out, void* stream);

/* Fresh states for n environments: out (rows, n) = center[r] + uniform +-bound
 * (center NULL means 0), drawn from pcg_hash(seed ^ ((i + index_offset) *
 * 0x9E3779B9) + r * 0x85EBCA6B). Re-provides `reset(n)` of the MLX ports
 * (cartpole_mlx.py:30-31, legged_mlx.py:21-22) on the device. */
RLENV_API int rlenv_reset_uniform(float* out, int rows, int64_t n, const float* center, float bound,
                        uint32_t seed, int64_t index_offset, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* RLENV_H */
