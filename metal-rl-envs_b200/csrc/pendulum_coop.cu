// Mass-matrix pendulum kernels with K warp lanes per environment.
#include "pendulum_kernels.cuh"

namespace rlenv {
namespace pend {

StepFn pick_coop(int k) {
  switch (k) {
    case 2: return &pendulum_coop_kernel<2>;
    case 4: return &pendulum_coop_kernel<4>;
    case 8: return &pendulum_coop_kernel<8>;
    case 16: return &pendulum_coop_kernel<16>;
    case 32: return &pendulum_coop_kernel<32>;
    default: return nullptr;
  }
}

}  // namespace pend
}  // namespace rlenv
