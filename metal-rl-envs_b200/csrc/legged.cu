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

template <int C, bool BRANCHY, bool IMPULSES>
__global__ void __launch_bounds__(128)
legged_kernel(const float* __restrict__ state, const void* __restrict__ action, int dtype,
              uint32_t seed, const float* __restrict__ stand, float assist,
              const float* __restrict__ assist_ptr, int iters, int64_t n, int64_t off,
              float* __restrict__ next, float* __restrict__ reward, uint8_t* __restrict__ done,
              float* __restrict__ impulses) {
  constexpr int nq = 3 + C;
  const int64_t e = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (e >= n) return;
  float q[nq], v[nq];
#pragma unroll
  for (int i = 0; i < nq; ++i) {
    q[i] = __ldg(state + i * n + e);
    v[i] = __ldg(state + (nq + i) * n + e);
  }
  float tq[C];
  decode_torques<C>(action_at(action, dtype, e), tq);
  const float k_assist = assist_ptr ? __ldg(assist_ptr) : assist;
  float imp[2 * C];
#pragma unroll
  for (int k = 0; k < 2 * C; ++k) imp[k] = 0.0f;
#pragma unroll 1
  for (int sub = 0; sub < lg::SUBSTEPS; ++sub)
    legged_substep<C, BRANCHY, IMPULSES>(q, v, tq, k_assist, iters, imp);
  if constexpr (IMPULSES) {
#pragma unroll
    for (int k = 0; k < 2 * C; ++k) impulses[k * n + e] = imp[k];
  }
  const bool d = legged_terminated<C>(q);
  const uint32_t h = env_hash(seed, off + e);
#pragma unroll
  for (int i = 0; i < 2 * nq; ++i) {
    const float fresh =
        __fadd_rn(__ldg(stand + i), uniform_pm(pcg_hash(h + uint32_t(i) * kRowStride), lg::RESET_BOUND));
    next[i * n + e] = d ? fresh : (i < nq ? q[i] : v[i - nq]);
  }
  reward[e] = d ? 0.0f : v[0] + 1.0f;
  done[e] = d;
}

using LeggedFn = void (*)(const float*, const void*, int, uint32_t, const float*, float,
                          const float*, int, int64_t, int64_t, float*, float*, uint8_t*, float*);

template <bool IMPULSES>
LeggedFn pick_c(int c, bool branchy) {
  if (branchy) return c == 1 ? &legged_kernel<1, true, IMPULSES> : nullptr;
  switch (c) {
    case 1: return &legged_kernel<1, false, IMPULSES>;
    case 2: return &legged_kernel<2, false, IMPULSES>;
    case 3: return &legged_kernel<3, false, IMPULSES>;
    case 4: return &legged_kernel<4, false, IMPULSES>;
    default: return nullptr;
  }
}

LeggedFn pick(int c, bool branchy, bool impulses) {
  return impulses ? pick_c<true>(c, branchy) : pick_c<false>(c, branchy);
}

int launch_legged(int c, bool branchy, int iters, const float* state, const void* action,
                  int dtype, uint32_t seed, const float* stand, float assist,
                  const float* assist_ptr, int64_t n, int64_t off, float* next, float* reward,
                  uint8_t* done, float* impulses, void* stream) {
  if (n < 0 || !valid_dtype(dtype) || iters < 1) return RLENV_EINVAL;
  LeggedFn fn = pick(c, branchy, impulses != nullptr);
  if (!fn) return RLENV_EUNSUPPORTED;
  if (n == 0) return RLENV_OK;
  if (!state || !action || !stand || !next || !reward || !done) return RLENV_EINVAL;
  fn<<<grid_for(n, 128), 128, 0, as_stream(stream)>>>(state, action, dtype, seed, stand, assist,
                                                      assist_ptr, iters, n, off, next, reward,
                                                      done, impulses);
  return launch_status();
}

}  // namespace
}  // namespace rlenv

extern "C" {

int rlenv_legged_step(int c, int iters, const float* state, const void* action, int action_dtype,
                      uint32_t seed, const float* stand, float assist, const float* assist_ptr,
                      int64_t n, int64_t index_offset, float* next_state, float* reward,
                      uint8_t* done, float* impulses, void* stream) {
  return rlenv::launch_legged(c, false, iters, state, action, action_dtype, seed, stand, assist,
                              assist_ptr, n, index_offset, next_state, reward, done, impulses,
                              stream);
}

int rlenv_hopper_step(int branchy, const float* state, const void* action, int action_dtype,
                      uint32_t seed, const float* stand, int64_t n, int64_t index_offset,
                      float* next_state, float* reward, uint8_t* done, void* stream) {
  return rlenv::launch_legged(1, branchy != 0, 1, state, action, action_dtype, seed, stand, 0.0f,
                              nullptr, n, index_offset, next_state, reward, done, nullptr, stream);
}

}  // extern "C"
