// Centred ranks of a large ES population in O(P log P) work (es.py:214-215).
//
// Every member becomes one unique 64-bit key: its fitness's order key
// (rank_order_key, common.cuh) in the high half and its index in the low half.
// Ascending order of these keys is the stable ascending order of the fitness,
// so sorting them gives every member's rank with ties broken by index, exactly
// the ranks of the counting kernel in es.cu, bit for bit.
//
//  1. tile_sort_kernel: each block sorts a tile of kTile keys in shared memory
//     with a bitonic network and writes it as a sorted run.
//  2. merge_kernel: runs of width w are merged pairwise into runs of 2w. Keys
//     are unique, so an element's position in the merged run is its position
//     in its own run plus the number of keys of the sibling run below it (one
//     binary search); no merge-path partitioning is needed.
//  3. The last pass (or the tile sort, when one tile holds the whole
//     population) writes ranks[index] = position / (P - 1) - 0.5 instead of
//     the key.
//
// Scratch: two arrays of P keys (16 P bytes), ping-ponged between passes.
#include "common.cuh"

namespace rlenv {
namespace {

constexpr int kTile = 4096;         // keys per tile: 32 KB of shared memory
constexpr int kTileThreads = 1024;
constexpr int kMergeThreads = 256;

RLENV_D uint64_t member_key(const float* __restrict__ f, int64_t i) {
  return (uint64_t(rank_order_key(__ldg(f + i))) << 32) | uint64_t(uint32_t(i));
}

// Sort tile b of the population (keys past p are padding that sorts last).
// With `ranks` set, the tile is the whole population and its ranks are written
// directly; otherwise the sorted run goes to `out`.
__global__ void __launch_bounds__(kTileThreads)
tile_sort_kernel(const float* __restrict__ f, int64_t p, uint64_t* __restrict__ out,
                 float* __restrict__ ranks) {
  __shared__ uint64_t s[kTile];
  const int64_t base = int64_t(blockIdx.x) * kTile;
  for (int k = threadIdx.x; k < kTile; k += kTileThreads)
    s[k] = base + k < p ? member_key(f, base + k) : ~uint64_t(0);
  __syncthreads();
  for (int size = 2; size <= kTile; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int t = threadIdx.x; t < kTile / 2; t += kTileThreads) {
        const int lo = 2 * t - (t & (stride - 1));  // bit `stride` of lo is clear
        const int hi = lo + stride;
        const bool ascending = (lo & size) == 0;
        const uint64_t a = s[lo], b = s[hi];
        if ((a > b) == ascending) {
          s[lo] = b;
          s[hi] = a;
        }
      }
      __syncthreads();
    }
  }
  for (int k = threadIdx.x; k < kTile; k += kTileThreads) {
    if (base + k >= p) break;
    if (ranks)
      ranks[uint32_t(s[k])] = centered_rank(k, p);
    else
      out[base + k] = s[k];
  }
}

// Number of keys of the sorted run [run, run + len) below key.
RLENV_D int64_t count_below(const uint64_t* __restrict__ run, int64_t len, uint64_t key) {
  int64_t lo = 0, hi = len;
  while (lo < hi) {
    const int64_t mid = (lo + hi) >> 1;
    if (__ldg(run + mid) < key)
      lo = mid + 1;
    else
      hi = mid;
  }
  return lo;
}

// One merge pass: runs [2r w, 2r w + w) and [2r w + w, 2r w + 2w) of `in`
// become run [2r w, 2r w + 2w) of `out`, or, with `ranks` set, the final ranks.
__global__ void __launch_bounds__(kMergeThreads)
merge_kernel(const uint64_t* __restrict__ in, int64_t p, int64_t w, uint64_t* __restrict__ out,
             float* __restrict__ ranks) {
  const int64_t i = int64_t(blockIdx.x) * kMergeThreads + threadIdx.x;
  if (i >= p) return;
  const int64_t run = i / w;
  const int64_t pair_base = (run & ~int64_t(1)) * w;
  const int64_t sib_lo = (run ^ 1) * w;
  const int64_t sib_len = sib_lo >= p ? 0 : (p - sib_lo < w ? p - sib_lo : w);
  const uint64_t key = __ldg(in + i);
  const int64_t pos = pair_base + (i - run * w) + count_below(in + sib_lo, sib_len, key);
  if (ranks)
    ranks[uint32_t(key)] = centered_rank(pos, p);
  else
    out[pos] = key;
}

int64_t scratch_bytes(int64_t p) { return p <= kTile ? 0 : 2 * p * int64_t(sizeof(uint64_t)); }

}  // namespace

// Sorts p members' keys through `scratch` (16 p bytes, 8-byte aligned, unused
// when p <= kTile) and writes their centred ranks.
int sorted_ranks_launch(const float* fitness, int64_t p, float* ranks, uint64_t* scratch,
                        cudaStream_t s) {
  if (p <= kTile) {
    tile_sort_kernel<<<1, kTileThreads, 0, s>>>(fitness, p, nullptr, ranks);
    return launch_status();
  }
  uint64_t* a = scratch;
  uint64_t* b = scratch + p;
  tile_sort_kernel<<<grid_for(p, kTile), kTileThreads, 0, s>>>(fitness, p, a, nullptr);
  const int grid = grid_for(p, kMergeThreads);
  for (int64_t w = kTile; w < p; w *= 2) {
    const bool last = 2 * w >= p;
    merge_kernel<<<grid, kMergeThreads, 0, s>>>(a, p, w, b, last ? ranks : nullptr);
    uint64_t* t = a;
    a = b;
    b = t;
  }
  return launch_status();
}

int64_t sorted_ranks_scratch_bytes(int64_t p) { return p < 0 ? -1 : scratch_bytes(p); }

}  // namespace rlenv

extern "C" {

int64_t rlenv_es_ranks_scratch_bytes(int64_t p) { return rlenv::sorted_ranks_scratch_bytes(p); }

int rlenv_es_centered_ranks_sorted(const float* fitness, int64_t p, float* ranks, void* scratch,
                                   int64_t scratch_bytes, void* stream) {
  using namespace rlenv;
  if (p < 2 || p > (int64_t(1) << 31) || !fitness || !ranks) return RLENV_EINVAL;
  const int64_t need = sorted_ranks_scratch_bytes(p);
  if (need > 0 && (!scratch || scratch_bytes < need || (reinterpret_cast<uintptr_t>(scratch) & 7u)))
    return RLENV_EINVAL;
  return sorted_ranks_launch(fitness, p, ranks, static_cast<uint64_t*>(scratch), as_stream(stream));
}

}  // extern "C"
