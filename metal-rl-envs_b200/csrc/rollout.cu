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
// Legged: a group of 1, 2 or 4 lanes per member, the policy staged once per block in
// shared memory, then four substeps of the contact dynamics per step.
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
  // first RK4 stage and the previous step's termination test use too; taken as the step kernel
  // takes it (acrobot_trig_terminated), so a member steps exactly as rlenv_acrobot_step steps it
  AcrobotTrig tr = acrobot_stage_trig(s);
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
      if (acrobot_trig_terminated(s, tr)) alive = false;
      else survived += 1.0f;
    }
  }
  if (valid && lane == 0) fitness[m] = survived;
}

// Shared-memory image of a legged member's policy for one lane of its group of G lanes.
// es.unflatten's row (w1 (OBS, H), b1 (H), w2 (H, OUT), b2 (OUT)) is cut into the slices the
// lanes use: lane gl forms hidden units [gl U, (gl + 1) U) and the logits of legs
// [gl CL, (gl + 1) CL), so its slice holds those columns of w1 and b1 ((OBS, U) and U),
// those outputs' rows of w2, transposed ((3 CL, H)), and their biases. A lane reads only its
// own slice. The slice stride SL keeps a warp's loads conflict-free: with 128-bit loads a
// quarter-warp's eight slices start SL / 4 (odd) chunks of 16 bytes apart, eight distinct
// chunks modulo eight; with scalar loads only, SL is odd. The group's exchange areas
// (legged.cuh) follow the slices.
template <int C, int H, int G>
struct LeggedSlice {
  static constexpr int OBS = 5 + 2 * C, OUT = 3 * C;
  static constexpr int B1g = OBS * H, W2g = B1g + H, B2g = W2g + H * OUT;  // in the global row
  static constexpr int U = H / G, CL = C / G, NO = 3 * CL;
  static constexpr bool kVec1 = U % 4 == 0, kVec2 = H % 4 == 0;
  static constexpr int W1 = 0, B1 = OBS * U, W2 = (B1 + U + 3) / 4 * 4, B2 = W2 + NO * H;
  static constexpr int SL0 = B2 + NO;
  static constexpr int SL4 = (SL0 + 3) / 4 * 4;
  static constexpr int SL = (kVec1 || kVec2) ? ((SL4 / 4) % 2 ? SL4 : SL4 + 4) : (SL0 % 2 ? SL0 : SL0 + 1);
  static constexpr int kMembers = 32 / G;  // one warp per block
  static constexpr int XS = G > 1 ? lgx::xch_floats<C, H>() : 0;  // exchange floats per member
  static constexpr size_t kSmem = (size_t(32) * SL + size_t(kMembers) * XS) * sizeof(float);
};

// A group of G lanes per member (G divides C and H): lane gl owns C / G contacts and legs
// (legged_substep) and H / G hidden units. A block is one warp of 32 / G members whose
// policy slices are staged once into shared memory (LeggedSlice), so that the per-step
// weight reads are conflict-free shared loads rather than 32-row gathers through L1. Each
// step: the MLP on the state without x (legged_rollout_metal.py:36-51: bias first, then the
// inputs in order; each lane forms its hidden units whole and its legs' logits whole from
// the gathered hidden layer, so no sum depends on G), one three-way head per leg with the
// first index winning ties, four contact substeps, termination, and the shaped reward
// (legged_rollout_metal.py:52-55). Every lane stays in the loop until the last member of its
// warp has fallen (finished members keep stepping, unrecorded), so the exchanges and the
// warp-wide votes of the substep's contact skipping always see 32 lanes.
template <int C, int H, int G, int kIters>
__global__ void __launch_bounds__(32)
legged_rollout_kernel(const float* __restrict__ state, const float* __restrict__ theta,
                      int64_t stride, int64_t p, int horizon, int iters, float alive_bonus,
                      float fall_penalty, float gate, float assist, float* __restrict__ fitness,
                      float* __restrict__ steps) {
  using R = LeggedSlice<C, H, G>;
  using namespace lgx;
  constexpr int nq = 3 + C, OBS = R::OBS, U = R::U, CL = R::CL, NO = R::NO;
  extern __shared__ float4 smem4[];
  float* __restrict__ my = reinterpret_cast<float*>(smem4) + threadIdx.x * R::SL;
  const int lane = int(threadIdx.x), gl = lane % G;
  float* xch = G > 1 ? reinterpret_cast<float*>(smem4) + 32 * R::SL + (lane / G) * R::XS : nullptr;
  const int64_t m_raw = int64_t(blockIdx.x) * R::kMembers + lane / G;
  const bool valid = m_raw < p;
  const int64_t m = valid ? m_raw : p - 1;  // lanes past p shadow the last member, unrecorded
  {
    const float* __restrict__ row = theta + m * stride;
#pragma unroll 1
    for (int k = 0; k < OBS; ++k) {
#pragma unroll
      for (int u = 0; u < U; ++u) my[R::W1 + k * U + u] = __ldg(row + k * H + gl * U + u);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) my[R::B1 + u] = __ldg(row + R::B1g + gl * U + u);
#pragma unroll 1
    for (int j = 0; j < H; ++j) {
#pragma unroll
      for (int o = 0; o < NO; ++o) my[R::W2 + o * H + j] = __ldg(row + R::W2g + j * R::OUT + gl * NO + o);
    }
#pragma unroll
    for (int o = 0; o < NO; ++o) my[R::B2 + o] = __ldg(row + R::B2g + gl * NO + o);
  }
  float qt[3], vt[3], ql[CL], vl[CL];
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    qt[i] = __ldg(state + i * p + m);
    vt[i] = __ldg(state + (nq + i) * p + m);
  }
#pragma unroll
  for (int c = 0; c < CL; ++c) {
    ql[c] = __ldg(state + (3 + gl * CL + c) * p + m);
    vl[c] = __ldg(state + (nq + 3 + gl * CL + c) * p + m);
  }
  bool alive = valid;
  float ret = 0.0f, taken = 0.0f;  // return and steps taken, fall step included
  for (int step = 0; step < horizon; ++step) {
    if (!__any_sync(kFull, alive)) break;
    // The weights do not change inside the loop, and without this barrier the compiler hoists
    // all of their loads out of it, into far more registers than a thread has.
    asm volatile("" ::: "memory");
    // observation without x: (y, phi, psi.., x_dot, y_dot, phi_dot, psi_dot..)
    float obs[OBS];
    {
      float own[2][CL], all[2][C];
#pragma unroll
      for (int c = 0; c < CL; ++c) {
        own[0][c] = ql[c];
        own[1][c] = vl[c];
      }
      contact_exchange<C, G, 2>(own, all, xch + kXchObs * C, gl);
      obs[0] = qt[1];
      obs[1] = qt[2];
#pragma unroll
      for (int k = 0; k < C; ++k) obs[2 + k] = all[0][k];
#pragma unroll
      for (int i = 0; i < 3; ++i) obs[2 + C + i] = vt[i];
#pragma unroll
      for (int k = 0; k < C; ++k) obs[5 + C + k] = all[1][k];
    }
    float hown[U];
    if constexpr (R::kVec1) {
#pragma unroll
      for (int u = 0; u < U; u += 4) {
        const float4 b = *reinterpret_cast<const float4*>(my + R::B1 + u);
        float acc[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
        for (int k = 0; k < OBS; ++k) {
          const float4 w = *reinterpret_cast<const float4*>(my + R::W1 + k * U + u);
          acc[0] = fmaf(obs[k], w.x, acc[0]);
          acc[1] = fmaf(obs[k], w.y, acc[1]);
          acc[2] = fmaf(obs[k], w.z, acc[2]);
          acc[3] = fmaf(obs[k], w.w, acc[3]);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) hown[u + i] = tanhf(acc[i]);
      }
    } else {
#pragma unroll
      for (int u = 0; u < U; ++u) {
        float acc = my[R::B1 + u];
#pragma unroll
        for (int k = 0; k < OBS; ++k) acc = fmaf(obs[k], my[R::W1 + k * U + u], acc);
        hown[u] = tanhf(acc);
      }
    }
    float hdn[H];
    if constexpr (G == 1) {
#pragma unroll
      for (int j = 0; j < H; ++j) hdn[j] = hown[j];
    } else {
      float* hx = xch + xch_hidden<C>();
#pragma unroll
      for (int u = 0; u < U; ++u) hx[gl * U + u] = hown[u];
      __syncwarp();
#pragma unroll
      for (int j = 0; j < H; ++j) hdn[j] = hx[j];
    }
    float tq[CL];
#pragma unroll
    for (int c = 0; c < CL; ++c) {
      float l[3];
#pragma unroll
      for (int o = 0; o < 3; ++o) {
        const float* __restrict__ w2 = my + R::W2 + (3 * c + o) * H;
        float acc = my[R::B2 + 3 * c + o];
        if constexpr (R::kVec2) {
#pragma unroll
          for (int j = 0; j < H; j += 4) {
            const float4 w = *reinterpret_cast<const float4*>(w2 + j);
            acc = fmaf(hdn[j], w.x, acc);
            acc = fmaf(hdn[j + 1], w.y, acc);
            acc = fmaf(hdn[j + 2], w.z, acc);
            acc = fmaf(hdn[j + 3], w.w, acc);
          }
        } else {
#pragma unroll
          for (int j = 0; j < H; ++j) acc = fmaf(hdn[j], w2[j], acc);
        }
        l[o] = acc;
      }
      tq[c] = float(argmax3(l[0], l[1], l[2]) - 1) * lg::TORQUE;
    }
#pragma unroll 1
    for (int ss = 0; ss < lg::SUBSTEPS; ++ss)
      legged_substep<C, G, false, false, true, kIters>(qt, vt, ql, vl, tq, assist, iters, xch, gl, alive);
    if (alive) {
      taken += 1.0f;
      if (legged_terminated(qt)) {
        ret = sub(ret, fall_penalty);
        alive = false;
      } else {
        ret = add(ret, add(qt[1] >= gate ? vt[0] : 0.0f, alive_bonus));
      }
    }
  }
  if (valid && gl == 0) {
    check_flag(!isfinite(ret), kCheckNonFinite);
    fitness[m] = ret;
    steps[m] = taken;
  }
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

struct LeggedLaunch {
  LeggedRollout fn;
  size_t smem;
  int lanes;
};

// kIters = 8 (legged_rollout_metal.py's ITERS, the sweeps of every legged task) has its own
// instances for the tasks' two and four legs, with the sweeps unrolled; other counts loop.
template <int C, int H, int G, int kIters>
LeggedLaunch legged_instance() {
  if constexpr (C % G == 0 && H % G == 0 && (G == 1 || C % 2 == 0))
    return LeggedLaunch{&legged_rollout_kernel<C, H, G, kIters>, LeggedSlice<C, H, G>::kSmem, G};
  else
    return LeggedLaunch{nullptr, 0, G};
}

template <int C, int H, int kIters>
LeggedLaunch pick_legged_g(int g) {
  switch (g) {
    case 1: return legged_instance<C, H, 1, kIters>();
    case 2: return legged_instance<C, H, 2, kIters>();
    case 4: return legged_instance<C, H, 4, kIters>();
    default: return LeggedLaunch{nullptr, 0, g};
  }
}

template <int C, int kIters = 0>
LeggedLaunch pick_legged_h(int h, int g) {
  switch (h) {
    case 1: return pick_legged_g<C, 1, kIters>(g);
    case 2: return pick_legged_g<C, 2, kIters>(g);
    case 4: return pick_legged_g<C, 4, kIters>(g);
    case 8: return pick_legged_g<C, 8, kIters>(g);
    case 16: return pick_legged_g<C, 16, kIters>(g);
    case 32: return pick_legged_g<C, 32, kIters>(g);
    default: return LeggedLaunch{nullptr, 0, g};
  }
}

LeggedLaunch pick_legged(int c, int h, int g, int iters) {
  const bool eight = iters == 8;
  switch (c) {
    case 1: return pick_legged_h<1>(h, g);
    case 2: return eight ? pick_legged_h<2, 8>(h, g) : pick_legged_h<2>(h, g);
    case 3: return pick_legged_h<3>(h, g);
    case 4: return eight ? pick_legged_h<4, 8>(h, g) : pick_legged_h<4>(h, g);
    default: return LeggedLaunch{nullptr, 0, g};
  }
}

// Opt a kernel in to its dynamic shared memory on the current device. The attribute is per
// function and device, and setting it again is harmless, so each launch sets it (a few
// microseconds against a rollout of milliseconds) instead of caching it per device.
int prepare_smem(const void* fn, size_t smem) {
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout,
                             int(cudaSharedmemCarveoutMaxShared));
  return e == cudaSuccess ? RLENV_OK : int(e);
}

// Lanes per legged member when the caller leaves it open. Measured on a B200 (legged4, H = 16,
// horizon 1,000, an ES population after five generations): a member's time is the latency of
// its warp's serial chain of steps, and 4 lanes shorten it only while each SM sub-partition
// holds at most one such warp; 2 lanes never paid.
//   P = 32:     1 lane 5.18 ms, 2 lanes 5.72, 4 lanes 4.62
//   P = 2,048:  5.62, 6.27, 5.11          P = 4,096: 5.62, 6.28, 5.13
//   P = 16,384: 5.71, 8.37, 7.55 (all standing: 5.36, 11.6, 11.7)
// So 4 lanes when C and H allow it and P * 4 lanes fill at most one warp per sub-partition
// (P <= 32 x SMs), else one.
int legged_lanes(int c, int h, int64_t p) {
  int dev = 0, sms = 0;
  if (c % 4 || h % 4) return 1;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
    return 1;
  return p <= int64_t(32) * sms ? 4 : 1;
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

int rlenv_legged_rollout_lanes(int lanes, int c, int hidden, int horizon, int iters, float alive,
                               float fall, float gate, float assist, const float* state,
                               const float* theta, int64_t theta_stride, int64_t p, float* fitness,
                               float* steps, void* stream) {
  using namespace rlenv;
  if (p < 0 || horizon < 0 || theta_stride < 0 || iters < 1) return RLENV_EINVAL;
  if (pick_legged(c, hidden, 1, iters).fn == nullptr) return RLENV_EUNSUPPORTED;
  if (lanes == 0) lanes = legged_lanes(c, hidden, p);
  const LeggedLaunch L = pick_legged(c, hidden, lanes, iters);
  if (!L.fn) return RLENV_EUNSUPPORTED;
  if (p == 0) return RLENV_OK;
  if (!state || !theta || !fitness || !steps) return RLENV_EINVAL;
  const int st = prepare_smem(reinterpret_cast<const void*>(L.fn), L.smem);
  if (st != RLENV_OK) return st;
  const int64_t members = 32 / L.lanes;
  const int64_t blocks = (p + members - 1) / members;
  if (blocks > int64_t(0x7fffffff)) return RLENV_EINVAL;
  L.fn<<<int(blocks), 32, L.smem, as_stream(stream)>>>(state, theta, theta_stride, p, horizon, iters,
                                                       alive, fall, gate, assist, fitness, steps);
  return launch_status();
}

int rlenv_legged_rollout(int c, int hidden, int horizon, int iters, float alive, float fall,
                         float gate, float assist, const float* state, const float* theta,
                         int64_t theta_stride, int64_t p, float* fitness, float* steps,
                         void* stream) {
  return rlenv_legged_rollout_lanes(0, c, hidden, horizon, iters, alive, fall, gate, assist, state,
                                    theta, theta_stride, p, fitness, steps, stream);
}

}  // extern "C"
