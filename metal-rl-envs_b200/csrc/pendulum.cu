// C ABI entry points of the K-link pendulum step kernels; the kernels
// themselves are instantiated in pendulum_mm_lo.cu, pendulum_mm_hi.cu,
// pendulum_aba.cu, pendulum_long.cu, pendulum_aba_coop.cu and pendulum_coop.cu. Every kernel steps T times per launch;
// the single-step entry points launch it with T = 1.
#include "pendulum_kernels.cuh"

namespace rlenv {
namespace pend {
namespace {

int check_args(const float* state, const void* actions, int dtype, int64_t T, int64_t n,
               float* next) {
  if (n < 0 || T < 0 || !valid_dtype(dtype)) return RLENV_EINVAL;
  if (n > 0 && (!state || !next || (T > 0 && !actions))) return RLENV_EINVAL;
  return RLENV_OK;
}

int launch(StepFn fn, int64_t threads, int block, const float* state, const void* actions,
           int dtype, uint32_t seed0, int64_t T, int64_t n, int64_t off, float* next,
           float* reward_seq, uint8_t* done_seq, void* stream) {
  if (n == 0) return RLENV_OK;
  fn<<<grid_for(threads, block), block, 0, as_stream(stream)>>>(state, actions, dtype, seed0, T, n,
                                                               off, next, reward_seq, done_seq);
  return launch_status();
}

// Above 64 links the articulated body runs one warp per environment whatever the batch: measured on
// a B200 (T = 100), the one-warp form steps 2.6-2.7x as many environments per second as the
// one-thread long-chain kernel at N = 65,536 and 8.6-10x at N = 256 (K = 128, 192), while up to
// K = 64 the one-thread kernels win once the batch fills the GPU. The choice depends on K alone,
// so a shard of a batch runs the same kernel as the whole batch.
constexpr int kLongAbaMaxDefault = 64;

StepFn pick_mm(int k, int pairwise_trig) {
  return k <= 8 ? pick_mm_lo(k, pairwise_trig != 0) : pick_mm_hi(k, pairwise_trig != 0);
}

}  // namespace
}  // namespace pend
}  // namespace rlenv

extern "C" {

int rlenv_pendulum_mm_step(int k, int pairwise_trig, const float* state, const void* action,
                           int action_dtype, uint32_t seed, int64_t n, int64_t index_offset,
                           float* next_state, float* reward, uint8_t* done, void* stream) {
  using namespace rlenv::pend;
  if (n > 0 && (!reward || !done)) return RLENV_EINVAL;
  if (int rc = check_args(state, action, action_dtype, 1, n, next_state)) return rc;
  StepFn fn = pick_mm(k, pairwise_trig);
  if (!fn) return RLENV_EUNSUPPORTED;
  return launch(fn, n, 128, state, action, action_dtype, seed, 1, n, index_offset, next_state,
                reward, done, stream);
}

int rlenv_pendulum_mm_step_many(int k, int pairwise_trig, const float* state, const void* actions,
                                int action_dtype, uint32_t seed0, int64_t steps, int64_t n,
                                int64_t index_offset, float* state_out, float* reward_seq,
                                uint8_t* done_seq, void* stream) {
  using namespace rlenv::pend;
  if (int rc = check_args(state, actions, action_dtype, steps, n, state_out)) return rc;
  StepFn fn = pick_mm(k, pairwise_trig);
  if (!fn) return RLENV_EUNSUPPORTED;
  return launch(fn, n, 128, state, actions, action_dtype, seed0, steps, n, index_offset, state_out,
                reward_seq, done_seq, stream);
}

int rlenv_pendulum_coop_step(int k, const float* state, const void* action, int action_dtype,
                             uint32_t seed, int64_t n, int64_t index_offset, float* next_state,
                             float* reward, uint8_t* done, void* stream) {
  using namespace rlenv::pend;
  if (n > 0 && (!reward || !done)) return RLENV_EINVAL;
  if (int rc = check_args(state, action, action_dtype, 1, n, next_state)) return rc;
  StepFn fn = pick_coop(k);
  if (!fn) return RLENV_EUNSUPPORTED;
  return launch(fn, n * k, 256, state, action, action_dtype, seed, 1, n, index_offset, next_state,
                reward, done, stream);
}

int rlenv_pendulum_coop_step_many(int k, const float* state, const void* actions, int action_dtype,
                                  uint32_t seed0, int64_t steps, int64_t n, int64_t index_offset,
                                  float* state_out, float* reward_seq, uint8_t* done_seq,
                                  void* stream) {
  using namespace rlenv::pend;
  if (int rc = check_args(state, actions, action_dtype, steps, n, state_out)) return rc;
  StepFn fn = pick_coop(k);
  if (!fn) return RLENV_EUNSUPPORTED;
  return launch(fn, n * k, 256, state, actions, action_dtype, seed0, steps, n, index_offset,
                state_out, reward_seq, done_seq, stream);
}

int rlenv_pendulum_aba_step(int k, const float* state, const void* action, int action_dtype,
                            uint32_t seed, int64_t n, int64_t index_offset, float* next_state,
                            float* reward, uint8_t* done, void* stream) {
  using namespace rlenv::pend;
  if (n > 0 && (!reward || !done)) return RLENV_EINVAL;
  if (int rc = check_args(state, action, action_dtype, 1, n, next_state)) return rc;
  if (k > kLongAbaMaxDefault && k <= kCoopAbaMaxLinks) {
    if (n == 0) return RLENV_OK;
    return launch_aba_coop(k, state, action, action_dtype, seed, 1, n, index_offset, next_state, reward, done,
                           stream);
  }
  if (k > rlenv::kUnrollLinks)
    return launch_aba_long(k, state, action, action_dtype, seed, 1, n, index_offset, next_state,
                           reward, done, stream);
  StepFn fn = pick_aba(k);
  if (!fn) return RLENV_EUNSUPPORTED;
  return launch(fn, n, 128, state, action, action_dtype, seed, 1, n, index_offset, next_state,
                reward, done, stream);
}

int rlenv_pendulum_aba_step_many(int k, const float* state, const void* actions, int action_dtype,
                                 uint32_t seed0, int64_t steps, int64_t n, int64_t index_offset,
                                 float* state_out, float* reward_seq, uint8_t* done_seq,
                                 void* stream) {
  using namespace rlenv::pend;
  if (int rc = check_args(state, actions, action_dtype, steps, n, state_out)) return rc;
  if (k > kLongAbaMaxDefault && k <= kCoopAbaMaxLinks) {
    if (n == 0) return RLENV_OK;
    return launch_aba_coop(k, state, actions, action_dtype, seed0, steps, n, index_offset, state_out, reward_seq,
                           done_seq, stream);
  }
  if (k > rlenv::kUnrollLinks)
    return launch_aba_long(k, state, actions, action_dtype, seed0, steps, n, index_offset, state_out,
                           reward_seq, done_seq, stream);
  StepFn fn = pick_aba(k);
  if (!fn) return RLENV_EUNSUPPORTED;
  return launch(fn, n, 128, state, actions, action_dtype, seed0, steps, n, index_offset, state_out,
                reward_seq, done_seq, stream);
}

int rlenv_pendulum_aba_coop_step_many(int k, const float* state, const void* actions, int action_dtype,
                                      uint32_t seed0, int64_t steps, int64_t n, int64_t index_offset,
                                      float* state_out, float* reward_seq, uint8_t* done_seq, void* stream) {
  using namespace rlenv::pend;
  if (int rc = check_args(state, actions, action_dtype, steps, n, state_out)) return rc;
  if (k < 1 || k > kCoopAbaMaxLinks) return RLENV_EUNSUPPORTED;
  if (n == 0) return RLENV_OK;
  return launch_aba_coop(k, state, actions, action_dtype, seed0, steps, n, index_offset, state_out, reward_seq,
                         done_seq, stream);
}

}  // extern "C"
