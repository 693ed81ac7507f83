// Mass-matrix pendulum kernels, one thread per environment, K = 9..16.
#include "pendulum_kernels.cuh"

namespace rlenv {
namespace pend {

StepFn pick_mm_hi(int k, bool pairwise) {
  switch (k) {
#define RLENV_K(KK) \
  case KK: return pairwise ? &pendulum_kernel<KK, MASS_MATRIX_PAIRWISE> : &pendulum_kernel<KK, MASS_MATRIX>;
    RLENV_K(9) RLENV_K(10) RLENV_K(11) RLENV_K(12) RLENV_K(13) RLENV_K(14) RLENV_K(15) RLENV_K(16)
#undef RLENV_K
    default: return nullptr;
  }
}

}  // namespace pend
}  // namespace rlenv
