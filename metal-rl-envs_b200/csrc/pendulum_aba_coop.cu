// The articulated-body pendulum with a warp, or a segment of one, per environment: the
// warp-cooperative form for batches too small to fill the GPU with one thread per environment
// (BASELINE's N = 256 configurations). Up to 32 links, an environment takes a segment of the next
// power of two of lanes, one link each (a warp holds 32 / SEG environments); above, a whole warp,
// lane l owning links l L .. l L + L - 1 (L = 2, 4 or 6 for K up to 64, 128, 192). The algorithm is the rank-one articulated body of pendulum.cuh (aba_accel_unrolled;
// pendulum_aba_np.py:30-99), with every recurrence along the chain written as a scan over the
// lanes, so a derivative evaluation takes a few levels of shuffles instead of K dependent steps:
//  - link velocities: in the world frame the velocity of link i's joint is the exclusive prefix
//    sum of om_j (-sin th_j, cos th_j) over j < i, rotated into link i's frame;
//  - the articulated mass m_i the subtree at link i hands its parent obeys
//    m_i = (1 + m_{i+1}) / (1 + s_{i+1}^2 m_{i+1}) (s the joint sine; m = 1 at the last link):
//    a linear fractional map, so m_i is the ratio of a suffix product of 2 x 2 matrices
//    [[1, 1], [s^2, 1]] applied to (1, 1);
//  - the bias the subtree hands its parent obeys pa1_i = alpha_i + beta_i pa1_{i+1}, with
//    beta_i = c_{i+1} / (1 + m_{i+1} s_{i+1}^2): a suffix scan of affine maps;
//  - the outward accelerations keep two numbers per link, ax and z = ay + aw, and
//    (ax, z) -> (c ax + s z + c1, g - U1 (c ax + s z + c1)) is affine: a prefix scan of 2 x 2
//    affine maps; each link's absolute angular acceleration is z - ay.
// The scan form equals the sequential recurrences in exact arithmetic (tests/test_aba_scan_form.py
// restates it in float64 and checks it against the oracle's articulated body); in float32 the sums are
// associated differently, so it agrees with the one-thread kernels to rounding, not bit for bit.
#include "pendulum_kernels.cuh"

namespace rlenv {
namespace pend {
namespace {

constexpr unsigned kWarp = 0xffffffffu;

// The hardware reciprocal (rcp.approx.ftz, within one ulp): every denominator here is at least
// one (1 + m s^2, and the sums of a product's non-negative entries after rescaling), where the
// correctly rounded reciprocal and division carry slow-path branches that a lone warp waits on.
RLENV_D float rcp_fast(float a) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(a));
  return r;
}

// v -> M v + b on (ax, z)
struct Aff2 {
  float m00, m01, m10, m11, b0, b1;
};

RLENV_D Aff2 aff2_identity() { return Aff2{1.0f, 0.0f, 0.0f, 1.0f, 0.0f, 0.0f}; }

// f then g (f applied first)
RLENV_D Aff2 aff2_then(const Aff2& f, const Aff2& g) {
  return Aff2{fmaf(g.m00, f.m00, g.m01 * f.m10), fmaf(g.m00, f.m01, g.m01 * f.m11),
              fmaf(g.m10, f.m00, g.m11 * f.m10), fmaf(g.m10, f.m01, g.m11 * f.m11),
              fmaf(g.m00, f.b0, fmaf(g.m01, f.b1, g.b0)), fmaf(g.m10, f.b0, fmaf(g.m11, f.b1, g.b1))};
}

RLENV_D Aff2 aff2_shfl_up(const Aff2& a, int d, int w) {
  return Aff2{__shfl_up_sync(kWarp, a.m00, d, w), __shfl_up_sync(kWarp, a.m01, d, w),
              __shfl_up_sync(kWarp, a.m10, d, w), __shfl_up_sync(kWarp, a.m11, d, w),
              __shfl_up_sync(kWarp, a.b0, d, w), __shfl_up_sync(kWarp, a.b1, d, w)};
}

// a 2 x 2 matrix with non-negative entries, kept near unit size (its action on a ratio does not
// depend on the scale, and a product of K factors would otherwise overflow)
struct Mat2 {
  float a, b, c, d;
};

RLENV_D Mat2 mat2_identity() { return Mat2{1.0f, 0.0f, 0.0f, 1.0f}; }

RLENV_D Mat2 mat2_mul(const Mat2& p, const Mat2& q) {
  const Mat2 r{fmaf(p.a, q.a, p.b * q.c), fmaf(p.a, q.b, p.b * q.d), fmaf(p.c, q.a, p.d * q.c),
               fmaf(p.c, q.b, p.d * q.d)};
  const float sc = rcp_fast(r.a + r.b + r.c + r.d);
  return Mat2{r.a * sc, r.b * sc, r.c * sc, r.d * sc};
}

RLENV_D Mat2 mat2_shfl_down(const Mat2& p, int d, int w) {
  return Mat2{__shfl_down_sync(kWarp, p.a, d, w), __shfl_down_sync(kWarp, p.b, d, w),
              __shfl_down_sync(kWarp, p.c, d, w), __shfl_down_sync(kWarp, p.d, d, w)};
}

// the ratio a subtree's product hands on: P applied to (1, 1)
RLENV_D float mat2_ratio(const Mat2& p) { return (p.a + p.b) * rcp_fast(p.c + p.d); }

// Absolute angular accelerations of this lane's links j = lane L + t (t < L) of a k-link chain,
// lane being the lane's place in its environment's segment of SEG lanes (SEG a power of two up to
// 32: every scan and shuffle stays inside the segment); links past the chain are padding and
// read as zero angles and rates.
template <int L, int SEG>
RLENV_D void coop_aba_accel(const float (&th)[L], const float (&om)[L], float torque, int k, int lane,
                            float (&acc)[L]) {
  const int j0 = lane * L;
  // joint (relative) trig and rates, absolute trig; the previous link of the lane's first link is
  // the last link of the lane before
  const float th_prev = __shfl_up_sync(kWarp, th[L - 1], 1, SEG);
  const float om_prev = __shfl_up_sync(kWarp, om[L - 1], 1, SEG);
  float sn[L], cs[L], sa[L], ca[L], qd[L];
#pragma unroll
  for (int t = 0; t < L; ++t) {
    const int j = j0 + t;
    const float tp = t == 0 ? (lane == 0 ? 0.0f : th_prev) : th[t - 1];
    const float op = t == 0 ? (lane == 0 ? 0.0f : om_prev) : om[t - 1];
    sincos_sfu_near(th[t] - tp, &sn[t], &cs[t]);
    sincos_sfu_near(th[t], &sa[t], &ca[t]);
    qd[t] = om[t] - op;
    if (j >= k) {  // padding: no joint
      sn[t] = 0.0f;
      cs[t] = 0.0f;
    }
  }
  // ---- velocities: exclusive prefix sum of om_j (-sin th_j, cos th_j) in the world frame
  float vx[L], vy[L];
  {
    float s0 = 0.0f, s1 = 0.0f;  // this lane's links' sum
#pragma unroll
    for (int t = 0; t < L; ++t) {
      s0 = fmaf(-om[t], sa[t], s0);
      s1 = fmaf(om[t], ca[t], s1);
    }
    float i0 = s0, i1 = s1;  // inclusive over lanes
#pragma unroll
    for (int d = 1; d < SEG; d <<= 1) {
      const float u0 = __shfl_up_sync(kWarp, i0, d, SEG), u1 = __shfl_up_sync(kWarp, i1, d, SEG);
      const bool in = lane >= d;  // every combine below is computed and selected, not branched
      i0 += in ? u0 : 0.0f;
      i1 += in ? u1 : 0.0f;
    }
    float e0 = i0 - s0, e1 = i1 - s1;  // exclusive: the links before this lane
#pragma unroll
    for (int t = 0; t < L; ++t) {
      vx[t] = fmaf(ca[t], e0, sa[t] * e1);
      vy[t] = fmaf(-sa[t], e0, ca[t] * e1);
      e0 = fmaf(-om[t], sa[t], e0);
      e1 = fmaf(om[t], ca[t], e1);
    }
  }
  // ---- articulated masses: m_j = ratio of M_{j+1} ... M_{k-1}, M_j = [[1, 1], [s_j^2, 1]] for
  // 1 <= j < k and the identity elsewhere
  float m[L];
  {
    Mat2 own = mat2_identity();
#pragma unroll
    for (int t = 0; t < L; ++t) {
      const int j = j0 + t;
      const Mat2 next = mat2_mul(own, Mat2{1.0f, 1.0f, sn[t] * sn[t], 1.0f});
      own = j >= 1 && j < k ? next : own;
    }
    Mat2 sfx = own;  // inclusive suffix over lanes: this lane's links and every later one
#pragma unroll
    for (int d = 1; d < SEG; d <<= 1) {
      const Mat2 later = mat2_shfl_down(sfx, d, SEG);
      const Mat2 both = mat2_mul(sfx, later);
      sfx = lane + d < SEG ? both : sfx;
    }
    const Mat2 next_lanes = mat2_shfl_down(sfx, 1, SEG);  // the links after this lane
    Mat2 after = lane == SEG - 1 ? mat2_identity() : next_lanes;
#pragma unroll
    for (int t = L - 1; t >= 0; --t) {
      const int j = j0 + t;
      m[t] = mat2_ratio(after);
      const Mat2 next = mat2_mul(Mat2{1.0f, 1.0f, sn[t] * sn[t], 1.0f}, after);
      after = j >= 1 && j < k ? next : after;
    }
  }
  // the next link's joint trig and mass (zero joint trig past the chain: no child)
  float sn1[L], cs1[L], m1[L];
  {
    const float sn_next = __shfl_down_sync(kWarp, sn[0], 1, SEG), cs_next = __shfl_down_sync(kWarp, cs[0], 1, SEG);
    const float m_next = __shfl_down_sync(kWarp, m[0], 1, SEG);
#pragma unroll
    for (int t = 0; t < L; ++t) {
      const bool last = t == L - 1;
      sn1[t] = last ? (lane == SEG - 1 ? 0.0f : sn_next) : sn[t + 1];
      cs1[t] = last ? (lane == SEG - 1 ? 0.0f : cs_next) : cs[t + 1];
      m1[t] = last ? (lane == SEG - 1 ? 0.0f : m_next) : m[t + 1];
    }
  }
  // ---- per link: the articulated inertia seen from its joint and the velocity-product terms
  float r[L], u1[L], c1[L], c2[L], alpha[L], beta[L];
  float root_a00 = 1.0f, root_a01 = 0.0f;  // link 0's, for the root
#pragma unroll
  for (int t = 0; t < L; ++t) {
    const float a00 = fmaf(m1[t] * sn1[t], sn1[t], 1.0f);
    const float a01 = (m1[t] * sn1[t]) * cs1[t];
    if (t == 0) {
      root_a00 = a00;
      root_a01 = a01;
    }
    r[t] = rcp_fast(a00);
    u1[t] = a01 * r[t];
    const float w = om[t], x = vx[t], y = vy[t];
    c1[t] = qd[t] * y;
    c2[t] = -qd[t] * x;
    alpha[t] = fmaf(-w, w + y, fmaf(m[t], c1[t], -u1[t] * (x * w)));
    beta[t] = cs1[t] * r[t];
  }
  // ---- bias: pa1_j = alpha_j + beta_j pa1_{j+1} for 1 <= j < k, pa1 past the chain zero; a
  // lane's links compose to pa1_first = A + B pa1_after
  float pa1_next[L];  // pa1_{j+1}
  {
    float B = 1.0f, A = 0.0f;
#pragma unroll
    for (int t = L - 1; t >= 0; --t) {
      const bool in = j0 + t >= 1 && j0 + t < k;  // outside the chain: the identity map
      A = fmaf(in ? beta[t] : 1.0f, A, in ? alpha[t] : 0.0f);
      B = (in ? beta[t] : 1.0f) * B;
    }
    float SB = B, SA = A;  // inclusive suffix over lanes
#pragma unroll
    for (int d = 1; d < SEG; d <<= 1) {
      const float lb = __shfl_down_sync(kWarp, SB, d, SEG), la = __shfl_down_sync(kWarp, SA, d, SEG);
      const bool in = lane + d < SEG;
      SA = fmaf(SB, in ? la : 0.0f, SA);
      SB = SB * (in ? lb : 1.0f);
    }
    const float pa_next_lane = __shfl_down_sync(kWarp, SA, 1, SEG);  // pa1 of the next lane's first link
    float pa = lane == SEG - 1 ? 0.0f : pa_next_lane;
#pragma unroll
    for (int t = L - 1; t >= 0; --t) {
      const bool in = j0 + t >= 1 && j0 + t < k;
      pa1_next[t] = pa;
      pa = fmaf(in ? beta[t] : 1.0f, pa, in ? alpha[t] : 0.0f);
    }
  }
  float g[L];
#pragma unroll
  for (int t = 0; t < L; ++t) g[t] = -fmaf(vx[t], om[t], sn1[t] * pa1_next[t]) * r[t];
  // ---- the root (lane 0's first link), the base accelerating at -G
  // every lane evaluates it on its own first link and lane 0's result is broadcast (no branch)
  float ax0, z0, qdd0;
  {
    const float U0 = root_a00, U1_0 = root_a01;  // U0 = 1 + m_1 s_1^2 >= 1
    const float uu0 = torque - sn1[0] * pa1_next[0];
    const float ax = ca[0] * -pd::G;
    const float ay = -sa[0] * -pd::G;
    const float q = (uu0 - fmaf(U1_0, ax, U0 * ay)) * rcp_fast(U0);
    ax0 = __shfl_sync(kWarp, ax, 0, SEG);
    z0 = __shfl_sync(kWarp, ay + q, 0, SEG);
    qdd0 = __shfl_sync(kWarp, q, 0, SEG);
  }
  // ---- outward accelerations: (ax, z) through each link's affine map, prefix over the lanes
  {
    Aff2 own = aff2_identity();
#pragma unroll
    for (int t = 0; t < L; ++t) {
      const int j = j0 + t;
      const Aff2 f{cs[t], sn[t], -u1[t] * cs[t], -u1[t] * sn[t], c1[t], fmaf(-u1[t], c1[t], g[t])};
      const Aff2 next = aff2_then(own, f);
      own = j >= 1 && j < k ? next : own;
    }
    Aff2 pre = own;  // inclusive prefix over lanes
#pragma unroll
    for (int d = 1; d < SEG; d <<= 1) {
      const Aff2 earlier = aff2_shfl_up(pre, d, SEG);
      const Aff2 both = aff2_then(earlier, pre);
      pre = lane >= d ? both : pre;
    }
    const Aff2 earlier_lanes = aff2_shfl_up(pre, 1, SEG);  // the links before this lane
    const Aff2 before = lane == 0 ? aff2_identity() : earlier_lanes;
    float ax = fmaf(before.m00, ax0, fmaf(before.m01, z0, before.b0));
    float z = fmaf(before.m10, ax0, fmaf(before.m11, z0, before.b1));
#pragma unroll
    for (int t = 0; t < L; ++t) {
      const int j = j0 + t;
      if (j == 0) {
        acc[t] = qdd0;
      } else if (j >= k) {
        acc[t] = 0.0f;  // padding stays at rest
      } else {
        const float ap1 = fmaf(cs[t], ax, fmaf(sn[t], z, c1[t]));
        const float ay = fmaf(-sn[t], ax, fmaf(cs[t], z, c2[t]));
        z = fmaf(-u1[t], ap1, g[t]);
        ax = ap1;
        acc[t] = z - ay;
      }
    }
  }
}

// T steps of N environments, a segment of SEG lanes per environment (a warp holds 32 / SEG of
// them; blocks of 128 threads), the lane's links' state in registers between steps; step t reads
// actions[t * n + e], draws its resets from seed0 + t and writes reward_seq / done_seq row t when
// those are not null. One step is the launch with T = 1, so a chain of single steps and one
// T-step launch agree bit for bit. Segments past the last environment mirror it (every lane of a
// warp takes part in its shuffles) and store nothing.
template <int L, int SEG>
__global__ void __launch_bounds__(128)
pendulum_aba_coop_kernel(const float* __restrict__ state, const void* __restrict__ actions, int dtype,
                         uint32_t seed0, int k, int64_t T, int64_t n, int64_t off, float* __restrict__ next,
                         float* __restrict__ reward_seq, uint8_t* __restrict__ done_seq) {
  const int64_t gt = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if ((gt & ~int64_t(31)) / SEG >= n) return;  // a whole warp past the batch
  const int lane = int(threadIdx.x) & (SEG - 1);
  const int64_t e_raw = gt / SEG;
  const bool valid = e_raw < n;
  const int64_t e = valid ? e_raw : n - 1;
  float th[L], om[L];
#pragma unroll
  for (int t = 0; t < L; ++t) {
    const int j = lane * L + t;
    th[t] = j < k ? __ldg(state + int64_t(j) * n + e) : 0.0f;
    om[t] = j < k ? __ldg(state + int64_t(k + j) * n + e) : 0.0f;
  }
  int act = T > 0 ? action_at(actions, dtype, e) : 0;  // loaded one step ahead
  for (int64_t t = 0; t < T; ++t) {
    check_flag(act < 0 || act > 2, kCheckActionRange);
    const float torque = float(act - 1) * pd::TORQUE;
    if (t + 1 < T) act = action_at(actions, dtype, (t + 1) * n + e);
    pendulum_rk4<L, true>(th, om, torque, [&](const float (&a_t)[L], const float (&a_o)[L], float tq, float (&a)[L]) {
      coop_aba_accel<L, SEG>(a_t, a_o, tq, k, lane, a);
    });
    // the tip above half the chain's length: -sum cos th > k / 2, summed over the segment
    float h = 0.0f;
#pragma unroll
    for (int u = 0; u < L; ++u)
      h += lane * L + u < k ? cos_fast(th[u]) : 0.0f;
#pragma unroll
    for (int d = SEG / 2; d >= 1; d >>= 1) h += __shfl_xor_sync(kWarp, h, d, SEG);
    const bool dn = -h > float(k) * 0.5f;
    if (dn) {
      const uint32_t hs = env_hash(seed0 + uint32_t(t), off + e);
#pragma unroll
      for (int u = 0; u < L; ++u) {
        const int j = lane * L + u;
        if (j < k) {
          th[u] = uniform_pm(pcg_hash(hs + uint32_t(j) * kRowStride), pd::RESET_BOUND);
          om[u] = uniform_pm(pcg_hash(hs + uint32_t(k + j) * kRowStride), pd::RESET_BOUND);
        }
      }
    }
    if (lane == 0 && valid) {
      if (reward_seq) reward_seq[t * n + e] = dn ? 0.0f : -1.0f;
      if (done_seq) done_seq[t * n + e] = dn;
    }
  }
  if (!valid) return;
#pragma unroll
  for (int u = 0; u < L; ++u) {
    const int j = lane * L + u;
    if (j < k) {
      check_flag(!(isfinite(th[u]) && isfinite(om[u])), kCheckNonFinite);
      next[int64_t(j) * n + e] = th[u];
      next[int64_t(k + j) * n + e] = om[u];
    }
  }
}

template <int L, int SEG>
int launch_seg(int k, const float* state, const void* actions, int dtype, uint32_t seed0, int64_t T, int64_t n,
               int64_t off, float* next, float* reward_seq, uint8_t* done_seq, cudaStream_t s) {
  const int64_t threads = n * SEG;
  const unsigned blocks = unsigned((threads + 127) / 128);
  pendulum_aba_coop_kernel<L, SEG><<<blocks, 128, 0, s>>>(state, actions, dtype, seed0, k, T, n, off, next,
                                                          reward_seq, done_seq);
  return launch_status();
}

}  // namespace

int launch_aba_coop(int k, const float* state, const void* actions, int dtype, uint32_t seed0, int64_t T,
                    int64_t n, int64_t off, float* next, float* reward_seq, uint8_t* done_seq, void* stream) {
  if (k < 1 || k > kCoopAbaMaxLinks) return RLENV_EUNSUPPORTED;
  cudaStream_t s = as_stream(stream);
  // one link per lane in a segment of the next power of two up to 32 lanes, then a whole warp
  // with 2, 4 or 6 links per lane
  if (k <= 1) return launch_seg<1, 1>(k, state, actions, dtype, seed0, T, n, off, next, reward_seq, done_seq, s);
  if (k <= 2) return launch_seg<1, 2>(k, state, actions, dtype, seed0, T, n, off, next, reward_seq, done_seq, s);
  if (k <= 4) return launch_seg<1, 4>(k, state, actions, dtype, seed0, T, n, off, next, reward_seq, done_seq, s);
  if (k <= 8) return launch_seg<1, 8>(k, state, actions, dtype, seed0, T, n, off, next, reward_seq, done_seq, s);
  if (k <= 16) return launch_seg<1, 16>(k, state, actions, dtype, seed0, T, n, off, next, reward_seq, done_seq, s);
  if (k <= 32) return launch_seg<1, 32>(k, state, actions, dtype, seed0, T, n, off, next, reward_seq, done_seq, s);
  if (k <= 64) return launch_seg<2, 32>(k, state, actions, dtype, seed0, T, n, off, next, reward_seq, done_seq, s);
  if (k <= 128) return launch_seg<4, 32>(k, state, actions, dtype, seed0, T, n, off, next, reward_seq, done_seq, s);
  return launch_seg<6, 32>(k, state, actions, dtype, seed0, T, n, off, next, reward_seq, done_seq, s);
}

}  // namespace pend
}  // namespace rlenv
