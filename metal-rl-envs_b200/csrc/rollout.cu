// Fused ES rollouts: one launch runs every member of a population, each with
// its own MLP policy, against its own environment for the whole horizon,
// entirely on chip (cartpole_rollout_metal.py, acrobot_rollout_metal.py,
// legged_rollout_metal.py).
//
// CartPole and Acrobot: a group of G lanes shares one member (G a power of two
// up to H, chosen at launch from the population size: lanes_for below).
// Lane l owns hidden units l, l + G, ...: their first-layer column, bias and
// second-layer row stay in registers for the whole rollout. The hidden
// activations never leave the lane; the logits are a butterfly sum over the
// group, which leaves the same bits in every lane (addition is commutative, and
// every lane adds the same pairs). Every lane of a group then steps the same
// physics on the same inputs, so control flow stays uniform in the group, and
// the group stops at its member's first termination.
//
// Legged: one thread per member; the hidden layer is formed from weights read
// through the read-only cache, then four substeps of the contact dynamics.
#include "classic.cuh"
#include "legged.cuh"

namespace rlenv {
namespace {

constexpr unsigned kFull = 0xffffffffu;

template <int G>
RLENV_D float group_sum(float v) {
#pragma unroll
  for (int m = 1; m < G; m <<= 1) v += __shfl_xor_sync(kFull, v, m, G);
  return v;
}

// First index wins ties (cartpole_rollout_metal.py:56-63, acrobot_rollout_metal.py:40-43).
RLENV_D int argmax3(float l0, float l1, float l2) {
  int a = 0;
  float best = l0;
  if (l1 > best) { a = 1; best = l1; }
  if (l2 > best) a = 2;
  return a;
}

template <int H, int G>
__global__ void __launch_bounds__(256)
cartpole_rollout_kernel(const float* __restrict__ state, const float* __restrict__ theta,
                        int64_t stride, int64_t p, int horizon, float* __restrict__ fitness) {
  static_assert(G <= H && H % G == 0 && G <= 32, "a group owns whole hidden units");
  constexpr int U = H / G;
  const int64_t t = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const int lane = int(threadIdx.x) % G;
  const int64_t m_raw = t / G;
  const bool valid = m_raw < p;
  const int64_t m = valid ? m_raw : p - 1;  // idle lanes mirror the last member
  const float* __restrict__ row = theta + m * stride;
  float w1[4][U], b1[U], w2[2][U];
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int j = lane + u * G;
#pragma unroll
    for (int r = 0; r < 4; ++r) w1[r][u] = __ldg(row + r * H + j);
    b1[u] = __ldg(row + 4 * H + j);
    w2[0][u] = __ldg(row + 5 * H + 2 * j);
    w2[1][u] = __ldg(row + 5 * H + 2 * j + 1);
  }
  const float b2_0 = __ldg(row + 7 * H), b2_1 = __ldg(row + 7 * H + 1);
  CartPole s{__ldg(state + m), __ldg(state + p + m), __ldg(state + 2 * p + m),
             __ldg(state + 3 * p + m)};
  float survived = 0.0f;
  bool alive = true;
  for (int step = 0; step < horizon; ++step) {
    if (!__any_sync(kFull, alive)) break;
    float l0 = 0.0f, l1 = 0.0f;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const float hdn = tanhf(s.x * w1[0][u] + s.xd * w1[1][u] + s.th * w1[2][u] +
                              s.thd * w1[3][u] + b1[u]);
      l0 += hdn * w2[0][u];
      l1 += hdn * w2[1][u];
    }
    l0 = group_sum<G>(l0) + b2_0;
    l1 = group_sum<G>(l1) + b2_1;
    if (alive) {
      s = cartpole_physics(s, l1 > l0 ? cp::FORCE : -cp::FORCE);
      if (cartpole_terminated(s)) alive = false;
      else survived += 1.0f;
    }
  }
  if (valid && lane == 0) fitness[m] = survived;
}

template <int H, int G>
__global__ void __launch_bounds__(256)
acrobot_rollout_kernel(const float* __restrict__ state, const float* __restrict__ theta,
                       int64_t stride, int64_t p, int horizon, float* __restrict__ fitness) {
  static_assert(G <= H && H % G == 0 && G <= 32, "a group owns whole hidden units");
  constexpr int U = H / G;
  const int64_t t = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const int lane = int(threadIdx.x) % G;
  const int64_t m_raw = t / G;
  const bool valid = m_raw < p;
  const int64_t m = valid ? m_raw : p - 1;
  const float* __restrict__ row = theta + m * stride;
  float w1[7][U], w2[3][U];  // rows 0..5 of w1, then b1 in w1[6]
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int j = lane + u * G;
#pragma unroll
    for (int r = 0; r < 7; ++r) w1[r][u] = __ldg(row + r * H + j);
#pragma unroll
    for (int o = 0; o < 3; ++o) w2[o][u] = __ldg(row + 7 * H + 3 * j + o);
  }
  const float b2_0 = __ldg(row + 10 * H), b2_1 = __ldg(row + 10 * H + 1),
              b2_2 = __ldg(row + 10 * H + 2);
  Acrobot s{__ldg(state + m), __ldg(state + p + m), __ldg(state + 2 * p + m),
            __ldg(state + 3 * p + m)};
  float survived = 0.0f;
  bool alive = true;
  // the observation is (cos t1, sin t1, cos t2, sin t2, w1, w2): the state's trig, which the
  // first RK4 stage and the previous step's termination test use too
  AcrobotTrig tr = acrobot_trig(s);
  for (int step = 0; step < horizon; ++step) {
    if (!__any_sync(kFull, alive)) break;
    float l0 = 0.0f, l1 = 0.0f, l2 = 0.0f;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const float hdn = tanhf(tr.c1 * w1[0][u] + tr.s1 * w1[1][u] + tr.c2 * w1[2][u] + tr.s2 * w1[3][u] +
                              s.dth1 * w1[4][u] + s.dth2 * w1[5][u] + w1[6][u]);
      l0 += hdn * w2[0][u];
      l1 += hdn * w2[1][u];
      l2 += hdn * w2[2][u];
    }
    l0 = group_sum<G>(l0) + b2_0;
    l1 = group_sum<G>(l1) + b2_1;
    l2 = group_sum<G>(l2) + b2_2;
    if (alive) {
      s = acrobot_physics(s, tr, float(argmax3(l0, l1, l2) - 1));
      tr = acrobot_trig(s);
      if (acrobot_terminated(tr)) alive = false;
      else survived += 1.0f;
    }
  }
  if (valid && lane == 0) fitness[m] = survived;
}

template <int C, int H>
__global__ void __launch_bounds__(128)
legged_rollout_kernel(const float* __restrict__ state, const float* __restrict__ theta,
                      int64_t stride, int64_t p, int horizon, int iters, float alive_bonus,
                      float fall_penalty, float gate, float assist, float* __restrict__ fitness,
                      float* __restrict__ steps) {
  constexpr int nq = 3 + C, OBS = 5 + 2 * C, OUT = 3 * C;
  constexpr int B1 = OBS * H, W2 = B1 + H, B2 = W2 + H * OUT;
  const int64_t m = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (m >= p) return;
  const float* __restrict__ row = theta + m * stride;
  float q[nq], v[nq];
#pragma unroll
  for (int i = 0; i < nq; ++i) {
    q[i] = __ldg(state + i * p + m);
    v[i] = __ldg(state + (nq + i) * p + m);
  }
  float ret = 0.0f, alive_steps = 0.0f;  // return and steps survived, fall step included
  for (int step = 0; step < horizon; ++step) {
    // observation without x: (y, phi, psi.., x_dot, y_dot, phi_dot, psi_dot..)
    float hdn[H];
#pragma unroll
    for (int j = 0; j < H; ++j) {
      float s = __ldg(row + B1 + j);
#pragma unroll
      for (int k = 1; k < nq; ++k) s += q[k] * __ldg(row + (k - 1) * H + j);
#pragma unroll
      for (int k = 0; k < nq; ++k) s += v[k] * __ldg(row + (nq - 1 + k) * H + j);
      hdn[j] = tanhf(s);
    }
    float tq[C];
#pragma unroll
    for (int leg = 0; leg < C; ++leg) {
      float l[3];
#pragma unroll
      for (int o = 0; o < 3; ++o) {
        float s = __ldg(row + B2 + 3 * leg + o);
#pragma unroll
        for (int j = 0; j < H; ++j) s += hdn[j] * __ldg(row + W2 + j * OUT + 3 * leg + o);
        l[o] = s;
      }
      tq[leg] = float(argmax3(l[0], l[1], l[2]) - 1) * lg::TORQUE;
    }
#pragma unroll 1
    for (int sub = 0; sub < lg::SUBSTEPS; ++sub) legged_substep<C, false>(q, v, tq, assist, iters);
    if (legged_terminated<C>(q)) {
      alive_steps += 1.0f;
      ret -= fall_penalty;
      break;
    }
    ret += (q[1] >= gate ? v[0] : 0.0f) + alive_bonus;
    alive_steps += 1.0f;
  }
  fitness[m] = ret;
  steps[m] = alive_steps;
}

using ClassicRollout = void (*)(const float*, const float*, int64_t, int64_t, int, float*);

// Lanes per member. Every lane of a group steps the same physics, so wide groups repeat it;
// narrow groups leave few warps and long per-lane MLP chains. The group is the widest power of
// two (at most H and kMaxLanes) that keeps the launch within kTargetThreads, chosen on a B200
// at H = 32, horizon 500 (ES generation rollouts; fitness is identical at every width):
//  - CartPole (about 60 instructions of physics a step): 16 lanes at P = 4,096 and 16,384
//    (182 and 199 us; 186 and 212 us at 32 lanes, 664 and 670 us at 1).
//  - Acrobot (about 530): 8 lanes at P = 4,096 (600 us against 1,326 at 32) and 2 at P = 16,384
//    (760 us against 4,267 at 32), about 32K threads in both.
struct LanePolicy {
  int max_lanes;
  int64_t target_threads;
};
constexpr LanePolicy kCartPoleLanes{16, int64_t(1) << 18};
constexpr LanePolicy kAcrobotLanes{32, int64_t(1) << 15};

int lanes_for(const LanePolicy& pol, int h, int64_t p) {
  const int cap = h < pol.max_lanes ? h : pol.max_lanes;
  int g = 1;
  while (2 * g <= cap && p * 2 * g <= pol.target_threads) g *= 2;
  return g;
}

template <template <int, int> class Kern, int H>
ClassicRollout pick_width(int g) {
  switch (g) {
    case 1: return Kern<H, 1>::run;
    case 2: if constexpr (H >= 2) return Kern<H, 2>::run; else return nullptr;
    case 4: if constexpr (H >= 4) return Kern<H, 4>::run; else return nullptr;
    case 8: if constexpr (H >= 8) return Kern<H, 8>::run; else return nullptr;
    case 16: if constexpr (H >= 16) return Kern<H, 16>::run; else return nullptr;
    case 32: if constexpr (H >= 32) return Kern<H, 32>::run; else return nullptr;
    default: return nullptr;
  }
}

template <template <int, int> class Kern>
ClassicRollout pick_classic(int h, int g) {
  switch (h) {
    case 1: return pick_width<Kern, 1>(g);
    case 2: return pick_width<Kern, 2>(g);
    case 4: return pick_width<Kern, 4>(g);
    case 8: return pick_width<Kern, 8>(g);
    case 16: return pick_width<Kern, 16>(g);
    case 32: return pick_width<Kern, 32>(g);
    case 64: return pick_width<Kern, 64>(g);
    default: return nullptr;
  }
}

template <int H, int G>
struct CartPoleRollout {
  static constexpr ClassicRollout run = &cartpole_rollout_kernel<H, G>;
};
template <int H, int G>
struct AcrobotRollout {
  static constexpr ClassicRollout run = &acrobot_rollout_kernel<H, G>;
};

using LeggedRollout = void (*)(const float*, const float*, int64_t, int64_t, int, int, float, float,
                               float, float, float*, float*);

template <int C>
LeggedRollout pick_legged_h(int h) {
  switch (h) {
    case 1: return &legged_rollout_kernel<C, 1>;
    case 2: return &legged_rollout_kernel<C, 2>;
    case 4: return &legged_rollout_kernel<C, 4>;
    case 8: return &legged_rollout_kernel<C, 8>;
    case 16: return &legged_rollout_kernel<C, 16>;
    case 32: return &legged_rollout_kernel<C, 32>;
    default: return nullptr;
  }
}

LeggedRollout pick_legged(int c, int h) {
  switch (c) {
    case 1: return pick_legged_h<1>(h);
    case 2: return pick_legged_h<2>(h);
    case 3: return pick_legged_h<3>(h);
    case 4: return pick_legged_h<4>(h);
    default: return nullptr;
  }
}

int launch_classic(ClassicRollout fn, int g, const float* state, const float* theta,
                   int64_t stride, int64_t p, int horizon, float* fitness, void* stream) {
  if (p < 0 || horizon < 0 || stride < 0) return RLENV_EINVAL;
  if (!fn) return RLENV_EUNSUPPORTED;
  if (p == 0) return RLENV_OK;
  if (!state || !theta || !fitness) return RLENV_EINVAL;
  fn<<<grid_for(p * g, 256), 256, 0, as_stream(stream)>>>(state, theta, stride, p, horizon,
                                                          fitness);
  return launch_status();
}

}  // namespace
}  // namespace rlenv

extern "C" {

int rlenv_cartpole_rollout(const float* state, const float* theta, int64_t theta_stride, int64_t p,
                           int hidden, int horizon, float* fitness, void* stream) {
  using namespace rlenv;
  const int g = lanes_for(kCartPoleLanes, hidden, p);
  return launch_classic(pick_classic<CartPoleRollout>(hidden, g), g, state, theta, theta_stride, p,
                        horizon, fitness, stream);
}

int rlenv_acrobot_rollout(const float* state, const float* theta, int64_t theta_stride, int64_t p,
                          int hidden, int horizon, float* fitness, void* stream) {
  using namespace rlenv;
  const int g = lanes_for(kAcrobotLanes, hidden, p);
  return launch_classic(pick_classic<AcrobotRollout>(hidden, g), g, state, theta, theta_stride, p,
                        horizon, fitness, stream);
}

int rlenv_legged_rollout(int c, int hidden, int horizon, int iters, float alive, float fall,
                         float gate, float assist, const float* state, const float* theta,
                         int64_t theta_stride, int64_t p, float* fitness, float* steps,
                         void* stream) {
  using namespace rlenv;
  if (p < 0 || horizon < 0 || theta_stride < 0 || iters < 1) return RLENV_EINVAL;
  LeggedRollout fn = pick_legged(c, hidden);
  if (!fn) return RLENV_EUNSUPPORTED;
  if (p == 0) return RLENV_OK;
  if (!state || !theta || !fitness || !steps) return RLENV_EINVAL;
  fn<<<grid_for(p, 128), 128, 0, as_stream(stream)>>>(state, theta, theta_stride, p, horizon, iters,
                                                      alive, fall, gate, assist, fitness, steps);
  return launch_status();
}

}  // extern "C"
