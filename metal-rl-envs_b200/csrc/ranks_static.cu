// Centred ranks for callers that cannot allocate device memory: the sort of
// ranks.cu with its scratch in a fixed array of this library instead of a
// caller's buffer. The array holds the keys of up to kStaticRankMembers
// members (two arrays of 8-byte keys, 1 MiB); larger populations are rejected.
//
// Nothing in the array has to start at zero: every slot the sort reads was
// written earlier in the same call. Every call on a device uses the same
// array, so calls whose executions overlap (two streams, or two host threads
// with their own streams) race on it; calls in one stream are ordered and safe.
#include <cuda.h>

#include <mutex>

#include "common.cuh"

namespace rlenv {

int sorted_ranks_launch(const float* fitness, int64_t p, float* ranks, uint64_t* scratch,
                        cudaStream_t s);

namespace {

constexpr int64_t kStaticRankMembers = 65536;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) uint64_t g_rank_scratch[2 * kStaticRankMembers];

// The array's address is a property of the CUDA context that loaded this module. It is
// looked up once per device and kept together with that context; when the device's current
// context is another one (the old one was destroyed, for instance by cudaDeviceReset, and
// the module loaded again), the address is looked up again.
struct ScratchAddr {
  CUcontext ctx;
  uint64_t* addr;
};
std::mutex g_mu;
ScratchAddr g_addr[kMaxDevices] = {};

using CtxGetCurrent = CUresult (*)(CUcontext*);

// The driver's cuCtxGetCurrent, through the runtime (the library links only cudart).
CtxGetCurrent ctx_get_current() {
  static CtxGetCurrent fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<CtxGetCurrent>(nullptr);
    return reinterpret_cast<CtxGetCurrent>(f);
  }();
  return fn;
}

CUcontext current_ctx() {
  CUcontext c = nullptr;
  const CtxGetCurrent f = ctx_get_current();
  if (!f || f(&c) != CUDA_SUCCESS) return nullptr;
  return c;
}

// The array's address in the current device's context.
int scratch_for_current_device(uint64_t** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return int(e);
  if (dev < 0 || dev >= kMaxDevices) return RLENV_EUNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_mu);
  ScratchAddr& slot = g_addr[dev];
  const CUcontext ctx = current_ctx();
  if (!slot.addr || !ctx || ctx != slot.ctx) {
    void* a = nullptr;
    e = cudaGetSymbolAddress(&a, g_rank_scratch);  // makes the device's context current if none is
    if (e != cudaSuccess) return int(e);
    slot.addr = static_cast<uint64_t*>(a);
    slot.ctx = current_ctx();
  }
  *out = slot.addr;
  return RLENV_OK;
}

}  // namespace
}  // namespace rlenv

extern "C" {

int rlenv_es_centered_ranks_static(const float* fitness, int64_t p, float* ranks, void* stream) {
  using namespace rlenv;
  if (p < 2 || p > kStaticRankMembers || !fitness || !ranks) return RLENV_EINVAL;
  uint64_t* scratch = nullptr;
  const int rc = scratch_for_current_device(&scratch);
  if (rc != RLENV_OK) return rc;
  return sorted_ranks_launch(fitness, p, ranks, scratch, as_stream(stream));
}

}  // extern "C"
