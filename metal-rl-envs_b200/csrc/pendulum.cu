// C ABI entry points of the K-link pendulum step kernels; the kernels
// themselves are instantiated in pendulum_mm_lo.cu, pendulum_mm_hi.cu,
// pendulum_aba.cu and pendulum_coop.cu.
#include "pendulum_kernels.cuh"

namespace rlenv {
namespace pend {
namespace {

int check_args(const float* state, const void* action, int dtype, int64_t n, float* next,
               float* reward, uint8_t* done) {
  if (n < 0 || !valid_dtype(dtype)) return RLENV_EINVAL;
  if (n > 0 && (!state || !action || !next || !reward || !done)) return RLENV_EINVAL;
  return RLENV_OK;
}

int launch(StepFn fn, int64_t threads, int block, const float* state, const void* action,
           int dtype, uint32_t seed, int64_t n, int64_t off, float* next, float* reward,
           uint8_t* done, void* stream) {
  if (n == 0) return RLENV_OK;
  fn<<<grid_for(threads, block), block, 0, as_stream(stream)>>>(state, action, dtype, seed, n, off,
                                                               next, reward, done);
  return launch_status();
}

}  // namespace
}  // namespace pend
}  // namespace rlenv

extern "C" {

int rlenv_pendulum_mm_step(int k, int pairwise_trig, const float* state, const void* action,
                           int action_dtype, uint32_t seed, int64_t n, int64_t index_offset,
                           float* next_state, float* reward, uint8_t* done, void* stream) {
  using namespace rlenv;
  using namespace rlenv::pend;
  if (int rc = check_args(state, action, action_dtype, n, next_state, reward, done)) return rc;
  StepFn fn = k <= 8 ? pick_mm_lo(k, pairwise_trig != 0) : pick_mm_hi(k, pairwise_trig != 0);
  if (!fn) return RLENV_EUNSUPPORTED;
  return launch(fn, n, 128, state, action, action_dtype, seed, n, index_offset, next_state, reward,
                done, stream);
}

int rlenv_pendulum_coop_step(int k, const float* state, const void* action, int action_dtype,
                             uint32_t seed, int64_t n, int64_t index_offset, float* next_state,
                             float* reward, uint8_t* done, void* stream) {
  using namespace rlenv;
  using namespace rlenv::pend;
  if (int rc = check_args(state, action, action_dtype, n, next_state, reward, done)) return rc;
  StepFn fn = pick_coop(k);
  if (!fn) return RLENV_EUNSUPPORTED;
  return launch(fn, n * k, 256, state, action, action_dtype, seed, n, index_offset, next_state,
                reward, done, stream);
}

int rlenv_pendulum_aba_step(int k, const float* state, const void* action, int action_dtype,
                            uint32_t seed, int64_t n, int64_t index_offset, float* next_state,
                            float* reward, uint8_t* done, void* stream) {
  using namespace rlenv;
  using namespace rlenv::pend;
  if (int rc = check_args(state, action, action_dtype, n, next_state, reward, done)) return rc;
  StepFn fn = pick_aba(k);
  if (!fn) return RLENV_EUNSUPPORTED;
  return launch(fn, n, 128, state, action, action_dtype, seed, n, index_offset, next_state, reward,
                done, stream);
}

}  // extern "C"
