// K-link pendulum step kernels as templates: the mass-matrix form with one
// thread per environment, the same form with K warp lanes per environment, and
// the O(K) articulated-body form. Each pendulum_*.cu instantiates a range of K
// so that the translation units compile in parallel; pendulum.cu holds the
// C ABI entry points and dispatches to them.
#pragma once

#include "pendulum.cuh"

namespace rlenv {
namespace pend {


// Actions are read through a runtime dtype switch, uniform across the grid,
// so each body needs one kernel instance per K rather than three.
RLENV_D int action_at(const void* a, int dtype, int64_t i) {
  switch (dtype) {
    case RLENV_I64: return load_action(static_cast<const int64_t*>(a), i);
    case RLENV_I32: return load_action(static_cast<const int32_t*>(a), i);
    default: return load_action(static_cast<const uint8_t*>(a), i);
  }
}

enum Form { MASS_MATRIX = 0, MASS_MATRIX_PAIRWISE = 1, ARTICULATED = 2 };

// T steps of N environments in one launch, the state in registers (local
// memory above kUnrollLinks) between steps; step t reads actions[t * n + e],
// draws its resets from seed0 + t and writes reward_seq / done_seq row t when
// those are not null. One step is the launch with T = 1, so a chain of single
// steps and one T-step launch run the same code and agree bit for bit.
template <int K, int FORM>
__global__ void __launch_bounds__(128)
pendulum_kernel(const float* __restrict__ state, const void* __restrict__ actions, int dtype,
                uint32_t seed0, int64_t T, int64_t n, int64_t off, float* __restrict__ next,
                float* __restrict__ reward_seq, uint8_t* __restrict__ done_seq) {
  constexpr bool U = K <= kUnrollLinks;  // one indexing style for every per-link array of this K
  const int64_t e = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (e >= n) return;
  float th[K], om[K];
  for_range<K, U>([&](int j) {
    th[j] = __ldg(state + j * n + e);
    om[j] = __ldg(state + (K + j) * n + e);
  });
  // each step's action is loaded one step ahead, off the step's dependency chain
  int act = T > 0 ? action_at(actions, dtype, e) : 0;
  for (int64_t t = 0; t < T; ++t) {
    check_flag(act < 0 || act > 2, kCheckActionRange);
    const float torque = float(act - 1) * pd::TORQUE;
    if (t + 1 < T) act = action_at(actions, dtype, (t + 1) * n + e);
    if constexpr (FORM == ARTICULATED) {
      pendulum_rk4<K, U>(th, om, torque, [](const float* a_t, const float* a_o, float tq, float* a) {
        aba_accel<K>(a_t, a_o, tq, a);
      });
    } else {
      pendulum_rk4<K, U>(th, om, torque,
                         [](const float (&a_t)[K], const float (&a_o)[K], float tq, float (&a)[K]) {
                           mm_accel<K, FORM == MASS_MATRIX_PAIRWISE>(a_t, a_o, tq, a);
                         });
    }
    const bool d = pendulum_terminated<K, U>(th);
    if (d) {
      const uint32_t h = env_hash(seed0 + uint32_t(t), off + e);
      for_range<K, U>([&](int j) {
        th[j] = uniform_pm(pcg_hash(h + uint32_t(j) * kRowStride), pd::RESET_BOUND);
        om[j] = uniform_pm(pcg_hash(h + uint32_t(K + j) * kRowStride), pd::RESET_BOUND);
      });
    }
    if (reward_seq) reward_seq[t * n + e] = d ? 0.0f : -1.0f;
    if (done_seq) done_seq[t * n + e] = d;
  }
  for_range<K, U>([&](int j) {
    check_flag(!(isfinite(th[j]) && isfinite(om[j])), kCheckNonFinite);
    next[j * n + e] = th[j];
    next[(K + j) * n + e] = om[j];
  });
}

// ---- K lanes per environment (pendulum_metal_coop.py:28-149) -----------------
// Lane j of a K-lane segment owns component j: its angle, its velocity, row j
// of the mass matrix and row j of the Cholesky factor. Column c of the factor
// is formed after the diagonal lane c broadcasts its row; forward
// substitution broadcasts each y_i as it is produced; back substitution sums
// the lanes' contributions with a butterfly over the segment. K is a power of
// two no larger than 32, so a segment never straddles a warp.
template <int K>
RLENV_D float seg_sum(float v) {
#pragma unroll
  for (int m = 1; m < K; m <<= 1) v += __shfl_xor_sync(0xffffffffu, v, m, K);
  return v;
}

template <int K>
RLENV_D float coop_accel(float th_j, float om_j, float torque, int j) {
  float sj, cj;
  sincos_fast(th_j, &sj, &cj);
  float Lr[K];
  float r = 0.0f;
#pragma unroll
  for (int p = 0; p < K; ++p) {
    const float cp = __shfl_sync(0xffffffffu, cj, p, K);
    const float sp = __shfl_sync(0xffffffffu, sj, p, K);
    const float op = __shfl_sync(0xffffffffu, om_j, p, K);
    const float mu = float(K - (j > p ? j : p));
    Lr[p] = mu * (cj * cp + sj * sp);
    r += mu * (sj * cp - cj * sp) * (op * op);
  }
  float rhs = -r - (pd::G * float(K - j)) * sj;
  if (j == 0) rhs += torque;
  // The factor's diagonal is used only through its reciprocal, which the hardware's reciprocal
  // square root gives from the broadcast pivot (rsqrt.approx, within two ulp; the pivots of this
  // positive definite matrix are far from zero), so the substitutions multiply instead of
  // divide: 1.6-2.7x on a B200 for K = 2..16 (K = 16, N = 256: 11.8 -> 25.6 M env-steps/s). At
  // K = 32 it measured 20% slower with the batch filling the GPU (38.2 -> 30.7 M at N = 65,536),
  // so K = 32 keeps the square root and the divisions.
  constexpr bool kRsqrt = K < 32;
  float inv_d[kRsqrt ? K : 1];
#pragma unroll
  for (int c = 0; c < K; ++c) {
    float s = Lr[c];
#pragma unroll
    for (int p = 0; p < c; ++p) s -= Lr[p] * __shfl_sync(0xffffffffu, Lr[p], c, K);
    const float pivot = __shfl_sync(0xffffffffu, s, c, K);
    if constexpr (kRsqrt) {
      asm("rsqrt.approx.ftz.f32 %0, %1;" : "=f"(inv_d[c]) : "f"(pivot));
      if (j > c) Lr[c] = s * inv_d[c];
    } else {
      const float dgn = sqrtf(pivot);
      if (j == c) Lr[c] = dgn;
      else if (j > c) Lr[c] = s / dgn;
    }
  }
  float y[K];
#pragma unroll
  for (int i = 0; i < K; ++i) {
    float yi = 0.0f;
    if (j == i) {
      float s = rhs;
#pragma unroll
      for (int p = 0; p < i; ++p) s -= Lr[p] * y[p];
      if constexpr (kRsqrt) yi = s * inv_d[i];
      else yi = s / Lr[i];
    }
    y[i] = __shfl_sync(0xffffffffu, yi, i, K);
  }
  float x = 0.0f;
#pragma unroll
  for (int i = K - 1; i >= 0; --i) {
    const float s = seg_sum<K>(j > i ? Lr[i] * x : 0.0f);
    if (j == i) {
      if constexpr (kRsqrt) x = (y[i] - s) * inv_d[i];
      else x = (y[i] - s) / Lr[i];
    }
  }
  return x;
}

template <int K>
__global__ void __launch_bounds__(256)
pendulum_coop_kernel(const float* __restrict__ state, const void* __restrict__ actions, int dtype,
                     uint32_t seed0, int64_t T, int64_t n, int64_t off, float* __restrict__ next,
                     float* __restrict__ reward_seq, uint8_t* __restrict__ done_seq) {
  const int64_t t_id = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const int j = int(threadIdx.x) & (K - 1);
  const int64_t e_raw = t_id / K;
  const bool valid = e_raw < n;
  const int64_t e = valid ? e_raw : n - 1;  // idle lanes mirror the last env to keep shuffles full
  float th = __ldg(state + j * n + e);
  float om = __ldg(state + (K + j) * n + e);
  int act = T > 0 ? action_at(actions, dtype, e) : 0;  // loaded one step ahead
  for (int64_t t = 0; t < T; ++t) {
    const float torque = float(act - 1) * pd::TORQUE;
    if (t + 1 < T) act = action_at(actions, dtype, (t + 1) * n + e);
    const float a1 = coop_accel<K>(th, om, torque, j);
    float dth = om, dom = a1;
    float ts = th + pd::HALF_DT * om, os = om + pd::HALF_DT * a1;
    const float a2 = coop_accel<K>(ts, os, torque, j);
    dth += 2.0f * os;
    dom += 2.0f * a2;
    ts = th + pd::HALF_DT * os;
    os = om + pd::HALF_DT * a2;
    const float a3 = coop_accel<K>(ts, os, torque, j);
    dth += 2.0f * os;
    dom += 2.0f * a3;
    ts = th + pd::DT * os;
    os = om + pd::DT * a3;
    const float a4 = coop_accel<K>(ts, os, torque, j);
    th = pd_wrap(th + pd::SIXTH_DT * (dth + os));
    om = fminf(fmaxf(om + pd::SIXTH_DT * (dom + a4), -pd::MAX_VEL), pd::MAX_VEL);
    const bool d = -seg_sum<K>(cos_fast(th)) > float(K) * 0.5f;
    if (d) {
      const uint32_t h = env_hash(seed0 + uint32_t(t), off + e);
      th = uniform_pm(pcg_hash(h + uint32_t(j) * kRowStride), pd::RESET_BOUND);
      om = uniform_pm(pcg_hash(h + uint32_t(K + j) * kRowStride), pd::RESET_BOUND);
    }
    if (valid && j == 0) {
      if (reward_seq) reward_seq[t * n + e] = d ? 0.0f : -1.0f;
      if (done_seq) done_seq[t * n + e] = d;
    }
  }
  if (!valid) return;
  next[j * n + e] = th;
  next[(K + j) * n + e] = om;
}

using StepFn = void (*)(const float*, const void*, int, uint32_t, int64_t, int64_t, int64_t, float*, float*,
                        uint8_t*);

// Per-translation-unit pickers: nullptr when the unit does not build this K.
StepFn pick_mm_lo(int k, bool pairwise);    // k in 1..8
StepFn pick_mm_hi(int k, bool pairwise);    // k in 9..16
StepFn pick_aba(int k);                     // k in 1..16
// The articulated body for 2 <= k <= 192 with its per-link arrays in shared memory (pendulum_long.cu).
int launch_aba_long(int k, const float* state, const void* actions, int dtype, uint32_t seed0,
                    int64_t T, int64_t n, int64_t off, float* next, float* reward_seq,
                    uint8_t* done_seq, void* stream);
StepFn pick_coop(int k);                    // k in 2, 4, 8, 16, 32
// The articulated body with one warp per environment, its recurrences along the chain as scans
// over the lanes, for 1 <= k <= kCoopAbaMaxLinks (pendulum_aba_coop.cu).
constexpr int kCoopAbaMaxLinks = 192;
int launch_aba_coop(int k, const float* state, const void* actions, int dtype, uint32_t seed0, int64_t T,
                    int64_t n, int64_t off, float* next, float* reward_seq, uint8_t* done_seq, void* stream);

}  // namespace pend
}  // namespace rlenv
