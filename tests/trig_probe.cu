// Test helper: evaluates the kernels' sine/cosine (sincos_fast in csrc/common.cuh)
// and CUDA's sincosf on the same inputs. Built by tests/test_gpu_trig.py.
#include "common.cuh"

namespace {
// Both placements of the rare branch must give the same bits; the inline one is checked
// against the shared one here and a mismatch is written as NaN into s.
__global__ void trig_probe_kernel(const float* x, float* s, float* c, float* s_lib, float* c_lib,
                                  int64_t n) {
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float si, ci;
  rlenv::sincos_fast<rlenv::TrigFar::kShared>(x[i], s + i, c + i);
  rlenv::sincos_fast<rlenv::TrigFar::kInline>(x[i], &si, &ci);
  const bool same = __float_as_uint(si) == __float_as_uint(s[i]) && __float_as_uint(ci) == __float_as_uint(c[i]);
  if (!same) s[i] = __int_as_float(0x7fc00001);
  sincosf(x[i], s_lib + i, c_lib + i);
}
}  // namespace

__global__ void sfu_probe_kernel(const float* x, float* s, float* c, int64_t n) {
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) rlenv::sincos_sfu(x[i], s + i, c + i);
}

extern "C" int sfu_probe(const float* x, float* s, float* c, int64_t n) {
  if (n <= 0) return 0;
  sfu_probe_kernel<<<int((n + 255) / 256), 256>>>(x, s, c, n);
  return int(cudaDeviceSynchronize());
}

__global__ void near_probe_kernel(const float* x, float* s, float* c, int64_t n) {
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) rlenv::sincos_sfu_near(x[i], s + i, c + i);
}

extern "C" int near_probe(const float* x, float* s, float* c, int64_t n) {
  if (n <= 0) return 0;
  near_probe_kernel<<<int((n + 255) / 256), 256>>>(x, s, c, n);
  return int(cudaDeviceSynchronize());
}

extern "C" int trig_probe(const float* x, float* s, float* c, float* s_lib, float* c_lib,
                          int64_t n) {
  if (n <= 0) return 0;
  trig_probe_kernel<<<int((n + 255) / 256), 256>>>(x, s, c, s_lib, c_lib, n);
  return int(cudaDeviceSynchronize());
}
