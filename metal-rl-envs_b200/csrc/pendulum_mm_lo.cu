// Mass-matrix pendulum kernels, one thread per environment, K = 1..8.
#include "pendulum_kernels.cuh"

namespace rlenv {
namespace pend {

StepFn pick_mm_lo(int k, bool pairwise) {
  switch (k) {
#define RLENV_K(KK) \
  case KK: return pairwise ? &pendulum_kernel<KK, MASS_MATRIX_PAIRWISE> : &pendulum_kernel<KK, MASS_MATRIX>;
    RLENV_K(1) RLENV_K(2) RLENV_K(3) RLENV_K(4) RLENV_K(5) RLENV_K(6) RLENV_K(7) RLENV_K(8)
#undef RLENV_K
    default: return nullptr;
  }
}

}  // namespace pend
}  // namespace rlenv
