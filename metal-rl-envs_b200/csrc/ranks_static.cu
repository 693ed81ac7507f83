// Centred ranks for callers that cannot allocate device memory: the sort of
// ranks.cu with its scratch in a fixed array of this library instead of a
// caller's buffer. The array holds the keys of up to kStaticRankMembers
// members (two arrays of 8-byte keys, 1 MiB); larger populations are rejected.
//
// Nothing in the array has to start at zero: every slot the sort reads was
// written earlier in the same call. Every call on a device uses the same
// array, so calls whose executions overlap (two streams, or two host threads
// with their own streams) race on it; calls in one stream are ordered and safe.
#include <mutex>

#include "common.cuh"

namespace rlenv {

int sorted_ranks_launch(const float* fitness, int64_t p, float* ranks, uint64_t* scratch,
                        cudaStream_t s);

namespace {

constexpr int64_t kStaticRankMembers = 65536;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) uint64_t g_rank_scratch[2 * kStaticRankMembers];

std::mutex g_mu;
uint64_t* g_addr[kMaxDevices] = {};

// The array's address in the current device's context, looked up once per device.
int scratch_for_current_device(uint64_t** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return int(e);
  if (dev < 0 || dev >= kMaxDevices) return RLENV_EUNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_addr[dev]) {
    void* a = nullptr;
    e = cudaGetSymbolAddress(&a, g_rank_scratch);
    if (e != cudaSuccess) return int(e);
    g_addr[dev] = static_cast<uint64_t*>(a);
  }
  *out = g_addr[dev];
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
