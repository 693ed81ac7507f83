// Legged-body and hopper step kernels: one thread per environment runs four
// substeps of the contact dynamics in registers, then termination, the reset
// around the standing pose and the reward (legged_metal.py:137-155,
// hopper_metal.py:63-107). The hopper is the legged body with one leg and one
// Gauss-Seidel sweep, which the reference's own tests pin to float precision
// (test_legged.py:20-26).
#include "legged.cuh"

namespace rlenv {
namespace {

RLENV_D int action_at(const void* a, int dtype, int64_t i) {
  switch (dtype) {
    case RLENV_I64: return load_action(static_cast<const int64_t*>(a), i);
    case RLENV_I32: return load_action(static_cast<const int32_t*>(a), i);
    default: return load_action(static_cast<const uint8_t*>(a), i);
  }
}

template <int C>
constexpr int kActionsOf = C == 1 ? 3 : C == 2 ? 9 : C == 3 ? 27 : 81;  // 3^C

// Per-leg torques from an action index in [0, 3^C): leg k gets
// ((a / 3^k) % 3 - 1) * TORQUE (legged_np.py:51-54).
template <int C>
RLENV_D void decode_torques(int a, float (&tq)[C]) {
  unsigned u = unsigned(a);
#pragma unroll
  for (int k = 0; k < C; ++k) {
    tq[k] = float(int(u % 3u) - 1) * lg::TORQUE;
    u /= 3u;
  }
}

// T steps per launch with the state in registers; step t reads actions[t * n + e],
// draws its resets from seed0 + t, and writes reward_seq / done_seq row t (when not
// null) and, with IMPULSES, rows [t * 2C, t * 2C + 2C) of impulse_seq. One step is
// the launch with T = 1, so a chain of single steps and one T-step launch agree bit
// for bit.
template <int C, bool BRANCHY, bool IMPULSES, int kIters>
__global__ void __launch_bounds__(128)
legged_kernel(const float* __restrict__ state, const void* __restrict__ actions, int dtype,
              uint32_t seed0, const float* __restrict__ stand, float assist,
              const float* __restrict__ assist_ptr, int iters, int64_t T, int64_t n, int64_t off,
              float* __restrict__ next, float* __restrict__ reward_seq,
              uint8_t* __restrict__ done_seq, float* __restrict__ impulse_seq) {
  constexpr int nq = 3 + C;
  const int64_t e = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (e >= n) return;
  float qt[3], vt[3], ql[C], vl[C];  // torso (x, y, phi) and legs (psi_k), with their rates
#pragma unroll
  for (int i = 0; i < nq; ++i) {
    const float qi = __ldg(state + i * n + e), vi = __ldg(state + (nq + i) * n + e);
    if (i < 3) {
      qt[i] = qi;
      vt[i] = vi;
    } else {
      ql[i - 3] = qi;
      vl[i - 3] = vi;
    }
  }
  const float k_assist = assist_ptr ? __ldg(assist_ptr) : assist;
  int act = T > 0 ? action_at(actions, dtype, e) : 0;  // loaded one step ahead
  for (int64_t t = 0; t < T; ++t) {
    float tq[C];
    check_flag(act < 0 || act >= kActionsOf<C>, kCheckActionRange);
    decode_torques<C>(act, tq);
    if (t + 1 < T) act = action_at(actions, dtype, (t + 1) * n + e);
    float imp[2 * C];
#pragma unroll
    for (int k = 0; k < 2 * C; ++k) imp[k] = 0.0f;
#pragma unroll 1
    for (int ss = 0; ss < lg::SUBSTEPS; ++ss)
      legged_substep<C, 1, BRANCHY, IMPULSES, false, kIters>(qt, vt, ql, vl, tq, k_assist, iters, nullptr, 0,
                                                           true, imp);
    if constexpr (IMPULSES) {
#pragma unroll
      for (int k = 0; k < 2 * C; ++k) {
        check_flag(!isfinite(imp[k]), kCheckNonFinite);
        impulse_seq[(t * 2 * C + k) * n + e] = imp[k];
      }
    }
    const bool d = legged_terminated(qt);
    const float rw = d ? 0.0f : vt[0] + 1.0f;
    if (d) {
      const uint32_t h = env_hash(seed0 + uint32_t(t), off + e);
#pragma unroll
      for (int i = 0; i < 2 * nq; ++i) {
        const float fresh =
            __fadd_rn(__ldg(stand + i), uniform_pm(pcg_hash(h + uint32_t(i) * kRowStride), lg::RESET_BOUND));
        const int j = i < nq ? i : i - nq;
        float& slot = i < nq ? (j < 3 ? qt[j] : ql[j - 3]) : (j < 3 ? vt[j] : vl[j - 3]);
        slot = fresh;
      }
    }
    if (reward_seq) reward_seq[t * n + e] = rw;
    if (done_seq) done_seq[t * n + e] = d;
  }
#pragma unroll
  for (int i = 0; i < nq; ++i) {
    check_flag(!(isfinite(i < 3 ? qt[i] : ql[i - 3]) && isfinite(i < 3 ? vt[i] : vl[i - 3])), kCheckNonFinite);
    next[i * n + e] = i < 3 ? qt[i] : ql[i - 3];
    next[(nq + i) * n + e] = i < 3 ? vt[i] : vl[i - 3];
  }
}

using LeggedFn = void (*)(const float*, const void*, int, uint32_t, const float*, float,
                          const float*, int, int64_t, int64_t, int64_t, float*, float*, uint8_t*,
                          float*);

// kIters = 8 (the reference's ITERS, legged_np.py:27, and the legged tasks' sweeps) has its own
// instances with the sweeps unrolled; any other count runs the loop.
template <bool IMPULSES, int kIters>
LeggedFn pick_c(int c, bool branchy) {
  if (branchy) return c == 1 ? &legged_kernel<1, true, IMPULSES, kIters> : nullptr;
  switch (c) {
    case 1: return &legged_kernel<1, false, IMPULSES, kIters>;
    case 2: return &legged_kernel<2, false, IMPULSES, kIters>;
    case 3: return &legged_kernel<3, false, IMPULSES, kIters>;
    case 4: return &legged_kernel<4, false, IMPULSES, kIters>;
    default: return nullptr;
  }
}

LeggedFn pick(int c, bool branchy, bool impulses, int iters) {
  if (iters == 8) return impulses ? pick_c<true, 8>(c, branchy) : pick_c<false, 8>(c, branchy);
  return impulses ? pick_c<true, 0>(c, branchy) : pick_c<false, 0>(c, branchy);
}

int launch_legged(int c, bool branchy, int iters, const float* state, const void* actions,
                  int dtype, uint32_t seed0, const float* stand, float assist,
                  const float* assist_ptr, int64_t T, int64_t n, int64_t off, float* next,
                  float* reward_seq, uint8_t* done_seq, float* impulse_seq, void* stream) {
  if (n < 0 || T < 0 || !valid_dtype(dtype) || iters < 1) return RLENV_EINVAL;
  LeggedFn fn = pick(c, branchy, impulse_seq != nullptr, iters);
  if (!fn) return RLENV_EUNSUPPORTED;
  if (n == 0) return RLENV_OK;
  if (!state || (T > 0 && !actions) || !stand || !next) return RLENV_EINVAL;
  fn<<<grid_for(n, 128), 128, 0, as_stream(stream)>>>(state, actions, dtype, seed0, stand, assist,
                                                      assist_ptr, iters, T, n, off, next,
                                                      reward_seq, done_seq, impulse_seq);
  return launch_status();
}

}  // namespace
}  // namespace rlenv

extern "C" {

int rlenv_legged_step(int c, int iters, const float* state, const void* action, int action_dtype,
                      uint32_t seed, const float* stand, float assist, const float* assist_ptr,
                      int64_t n, int64_t index_offset, float* next_state, float* reward,
                      uint8_t* done, float* impulses, void* stream) {
  if (n > 0 && (!reward || !done)) return RLENV_EINVAL;
  return rlenv::launch_legged(c, false, iters, state, action, action_dtype, seed, stand, assist,
                              assist_ptr, 1, n, index_offset, next_state, reward, done, impulses,
                              stream);
}

int rlenv_legged_step_many(int c, int iters, const float* state, const void* actions,
                           int action_dtype, uint32_t seed0, const float* stand, float assist,
                           const float* assist_ptr, int64_t steps, int64_t n, int64_t index_offset,
                           float* state_out, float* reward_seq, uint8_t* done_seq,
                           float* impulse_seq, void* stream) {
  return rlenv::launch_legged(c, false, iters, state, actions, action_dtype, seed0, stand, assist,
                              assist_ptr, steps, n, index_offset, state_out, reward_seq, done_seq,
                              impulse_seq, stream);
}

int rlenv_hopper_step(int branchy, const float* state, const void* action, int action_dtype,
                      uint32_t seed, const float* stand, int64_t n, int64_t index_offset,
                      float* next_state, float* reward, uint8_t* done, void* stream) {
  if (n > 0 && (!reward || !done)) return RLENV_EINVAL;
  return rlenv::launch_legged(1, branchy != 0, 1, state, action, action_dtype, seed, stand, 0.0f,
                              nullptr, 1, n, index_offset, next_state, reward, done, nullptr,
                              stream);
}

int rlenv_hopper_step_many(int branchy, const float* state, const void* actions, int action_dtype,
                           uint32_t seed0, const float* stand, int64_t steps, int64_t n,
                           int64_t index_offset, float* state_out, float* reward_seq,
                           uint8_t* done_seq, void* stream) {
  return rlenv::launch_legged(1, branchy != 0, 1, state, actions, action_dtype, seed0, stand, 0.0f,
                              nullptr, steps, n, index_offset, state_out, reward_seq, done_seq,
                              nullptr, stream);
}

}  // extern "C"
