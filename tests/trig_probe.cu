// Test helper: evaluates the kernels' sine/cosine (sincos_fast in csrc/common.cuh)
// and CUDA's sincosf on the same inputs. Built by tests/test_gpu_trig.py.
#include "common.cuh"

namespace {
__global__ void trig_probe_kernel(const float* x, float* s, float* c, float* s_lib, float* c_lib,
                                  int64_t n) {
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  rlenv::sincos_fast(x[i], s + i, c + i);
  sincosf(x[i], s_lib + i, c_lib + i);
}
}  // namespace

extern "C" int trig_probe(const float* x, float* s, float* c, float* s_lib, float* c_lib,
                          int64_t n) {
  if (n <= 0) return 0;
  trig_probe_kernel<<<int((n + 255) / 256), 256>>>(x, s, c, s_lib, c_lib, n);
  return int(cudaDeviceSynchronize());
}
