// Evolution Strategies generation pieces (es.py:214-227) and fresh-state
// resets, plus the library's status helpers.
//
// The noise of antithetic pair j at parameter i is a pure function of
// (seed, gen, j, i) (Philox-4x32-10 + Box-Muller, common.cuh), so no (P/2, D)
// noise matrix is ever stored: the perturbation kernel and the update kernel
// both regenerate it. That also makes every rank of a multi-GPU job agree on
// the noise without communicating it, and the update's fixed summation order
// makes every rank compute the same parameter bits.
#include "common.cuh"

namespace rlenv {
namespace {

__global__ void __launch_bounds__(256)
noise_kernel(float* __restrict__ half, int64_t rows, int64_t d, uint64_t seed, uint64_t gen,
             int64_t row_offset) {
  const int64_t blocks_per_row = (d + 3) / 4;
  const int64_t t = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (t >= rows * blocks_per_row) return;
  const int64_t r = t / blocks_per_row, b = t % blocks_per_row;
  float v[4];
  normal4(seed, gen, row_offset + r, b, v);
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int64_t j = 4 * b + u;
    if (j < d) half[r * d + j] = v[u];
  }
}

// theta_pop[r] = theta + sigma * (+-noise of its pair); the sum is two
// correctly rounded operations (no fused multiply-add), as numpy computes it.
__global__ void __launch_bounds__(256)
perturb_kernel(const float* __restrict__ theta, int64_t d, float sigma, uint64_t seed,
               uint64_t gen, int64_t pairs, int64_t member_offset, int64_t rows,
               float* __restrict__ out) {
  const int64_t blocks_per_row = (d + 3) / 4;
  const int64_t t = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (t >= rows * blocks_per_row) return;
  const int64_t r = t / blocks_per_row, b = t % blocks_per_row;
  const int64_t m = member_offset + r;
  const bool neg = m >= pairs;
  const int64_t pair = neg ? m - pairs : m;
  float v[4];
  normal4(seed, gen, pair, b, v);
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int64_t j = 4 * b + u;
    if (j < d) out[r * d + j] = __fadd_rn(__ldg(theta + j), __fmul_rn(sigma, neg ? -v[u] : v[u]));
  }
}

// Stable ranks by counting: rank_i = #{j : f_j < f_i} + #{j < i : f_j == f_i},
// in numpy's sort order: NaN after every number, NaNs equal among themselves
// (ties by index), -0 equal to +0; each fitness is compared as its order key
// (rank_order_key, common.cuh). A warp owns kRankMembersPerWarp members and its
// lanes stride over tiles of keys staged in shared memory, comparing each key
// with all of the warp's members; the per-lane counts are summed by shuffles.
// Integer counts, so the result does not depend on the split.
constexpr int kRankTile = 4096;
constexpr int kRankMembersPerWarp = 4;
constexpr int kRankThreads = 256;
constexpr int kRankMembersPerBlock = kRankThreads / 32 * kRankMembersPerWarp;

__global__ void __launch_bounds__(kRankThreads)
ranks_kernel(const float* __restrict__ f, int64_t p, float* __restrict__ ranks) {
  __shared__ uint32_t tile[kRankTile];
  const int lane = threadIdx.x & 31;
  const int64_t first = int64_t(blockIdx.x) * kRankMembersPerBlock +
                        int64_t(threadIdx.x >> 5) * kRankMembersPerWarp;
  uint32_t key[kRankMembersPerWarp];
  int cnt[kRankMembersPerWarp];
#pragma unroll
  for (int m = 0; m < kRankMembersPerWarp; ++m) {
    key[m] = first + m < p ? rank_order_key(__ldg(f + first + m)) : 0u;
    cnt[m] = 0;
  }
  for (int64_t base = 0; base < p; base += kRankTile) {
    const int len = int((p - base) < kRankTile ? (p - base) : kRankTile);
    __syncthreads();
    for (int k = threadIdx.x; k < len; k += kRankThreads) tile[k] = rank_order_key(__ldg(f + base + k));
    __syncthreads();
    for (int k = lane; k < len; k += 32) {
      const uint32_t kj = tile[k];
      const int64_t j = base + k;
#pragma unroll
      for (int m = 0; m < kRankMembersPerWarp; ++m)
        cnt[m] += (kj < key[m]) || (kj == key[m] && j < first + m);
    }
  }
#pragma unroll
  for (int m = 0; m < kRankMembersPerWarp; ++m) {
    int c = cnt[m];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
    if (lane == m && first + m < p) ranks[first + m] = centered_rank(c, p);
  }
}

// theta_out = theta + lr / (2 pairs sigma) * sum_j (ranks[j] - ranks[j + pairs]) noise_j.
// Block b owns parameters 4b .. 4b+3; its 256 threads split the pairs
// round-robin and their partial sums are combined by a fixed tree, so the
// result does not depend on the device or on the launch.
constexpr int kUpdThreads = 256;
__global__ void __launch_bounds__(kUpdThreads)
update_kernel(const float* __restrict__ theta, const float* __restrict__ ranks, int64_t d,
              int64_t pairs, float scale, uint64_t seed, uint64_t gen, float* __restrict__ out) {
  __shared__ float part[4][kUpdThreads];
  const int64_t b = blockIdx.x;
  float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  for (int64_t j = threadIdx.x; j < pairs; j += kUpdThreads) {
    const float w = __ldg(ranks + j) - __ldg(ranks + j + pairs);
    float v[4];
    normal4(seed, gen, j, b, v);
#pragma unroll
    for (int u = 0; u < 4; ++u) acc[u] += w * v[u];
  }
#pragma unroll
  for (int u = 0; u < 4; ++u) part[u][threadIdx.x] = acc[u];
  __syncthreads();
  for (int s = kUpdThreads / 2; s > 0; s >>= 1) {
    if (threadIdx.x < s) {
#pragma unroll
      for (int u = 0; u < 4; ++u) part[u][threadIdx.x] += part[u][threadIdx.x + s];
    }
    __syncthreads();
  }
  if (threadIdx.x < 4) {
    const int64_t j = 4 * b + threadIdx.x;
    if (j < d) out[j] = __fadd_rn(__ldg(theta + j), __fmul_rn(scale, part[threadIdx.x][0]));
  }
}

__global__ void __launch_bounds__(256)
reset_kernel(float* __restrict__ out, int rows, int64_t n, const float* __restrict__ center,
             float bound, uint32_t seed, int64_t off) {
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint32_t h = env_hash(seed, off + i);
  for (int r = 0; r < rows; ++r) {
    const float u = uniform_pm(pcg_hash(h + uint32_t(r) * kRowStride), bound);
    out[int64_t(r) * n + i] = center ? __fadd_rn(__ldg(center + r), u) : u;
  }
}

}  // namespace
}  // namespace rlenv

extern "C" {

const char* rlenv_strerror(int code) {
  if (code == RLENV_OK) return "ok";
  if (code == RLENV_EINVAL) return "invalid argument (null pointer, negative size or unknown dtype)";
  if (code == RLENV_EUNSUPPORTED) return "no kernel instance is built for these template parameters";
  if (code > 0) return cudaGetErrorString(static_cast<cudaError_t>(code));
  return "unknown rlenv status";
}

int rlenv_abi_version(void) { return 2; }

int rlenv_es_noise(float* half, int64_t rows, int64_t d, uint64_t seed, uint64_t gen,
                   int64_t row_offset, void* stream) {
  using namespace rlenv;
  if (rows < 0 || d < 0 || row_offset < 0) return RLENV_EINVAL;
  if (rows == 0 || d == 0) return RLENV_OK;
  if (!half) return RLENV_EINVAL;
  noise_kernel<<<grid_for(rows * ((d + 3) / 4)), 256, 0, as_stream(stream)>>>(half, rows, d, seed,
                                                                             gen, row_offset);
  return launch_status();
}

int rlenv_es_perturb(const float* theta, int64_t d, float sigma, uint64_t seed, uint64_t gen,
                     int64_t pairs, int64_t member_offset, int64_t rows, float* theta_pop,
                     void* stream) {
  using namespace rlenv;
  if (d < 0 || pairs < 0 || member_offset < 0 || rows < 0 || member_offset + rows > 2 * pairs)
    return RLENV_EINVAL;
  if (rows == 0 || d == 0) return RLENV_OK;
  if (!theta || !theta_pop) return RLENV_EINVAL;
  perturb_kernel<<<grid_for(rows * ((d + 3) / 4)), 256, 0, as_stream(stream)>>>(
      theta, d, sigma, seed, gen, pairs, member_offset, rows, theta_pop);
  return launch_status();
}

int rlenv_es_centered_ranks(const float* fitness, int64_t p, float* ranks, void* stream) {
  using namespace rlenv;
  if (p < 2 || !fitness || !ranks) return RLENV_EINVAL;
  ranks_kernel<<<grid_for(p, kRankMembersPerBlock), kRankThreads, 0, as_stream(stream)>>>(fitness, p,
                                                                                          ranks);
  return launch_status();
}

int rlenv_es_update(const float* theta, const float* ranks, int64_t d, int64_t pairs, float lr,
                    float sigma, uint64_t seed, uint64_t gen, float* theta_out, void* stream) {
  using namespace rlenv;
  if (d < 0 || pairs < 1 || !(sigma != 0.0f)) return RLENV_EINVAL;
  if (d == 0) return RLENV_OK;
  if (!theta || !ranks || !theta_out) return RLENV_EINVAL;
  const float scale = lr / (float(2 * pairs) * sigma);
  update_kernel<<<int((d + 3) / 4), kUpdThreads, 0, as_stream(stream)>>>(theta, ranks, d, pairs,
                                                                         scale, seed, gen,
                                                                         theta_out);
  return launch_status();
}

int rlenv_reset_uniform(float* out, int rows, int64_t n, const float* center, float bound,
                        uint32_t seed, int64_t index_offset, void* stream) {
  using namespace rlenv;
  if (rows < 0 || n < 0) return RLENV_EINVAL;
  if (rows == 0 || n == 0) return RLENV_OK;
  if (!out) return RLENV_EINVAL;
  reset_kernel<<<grid_for(n), 256, 0, as_stream(stream)>>>(out, rows, n, center, bound, seed,
                                                           index_offset);
  return launch_status();
}

}  // extern "C"
