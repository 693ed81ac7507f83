// Articulated-body pendulum kernels for K <= 16, one thread per environment with every
// per-link array in registers (longer chains: pendulum_long.cu).
#include "pendulum_kernels.cuh"

namespace rlenv {
namespace pend {

StepFn pick_aba(int k) {
  switch (k) {
#define RLENV_K(KK) \
  case KK: return &pendulum_kernel<KK, ARTICULATED>;
    RLENV_K(1) RLENV_K(2) RLENV_K(3) RLENV_K(4) RLENV_K(5) RLENV_K(6) RLENV_K(7) RLENV_K(8)
    RLENV_K(9) RLENV_K(10) RLENV_K(11) RLENV_K(12) RLENV_K(13) RLENV_K(14) RLENV_K(15) RLENV_K(16)
#undef RLENV_K
    default: return nullptr;
  }
}

}  // namespace pend
}  // namespace rlenv
