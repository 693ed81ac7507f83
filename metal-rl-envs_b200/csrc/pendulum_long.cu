// Articulated-body pendulum for long chains (pendulum_aba_np.py:30-132): one thread per
// environment, any K from 2 to kMaxLongLinks chosen at run time, every per-link array in
// shared memory.
//
// A thread keeps eight arrays of K floats: the state (theta, omega), the RK4 stage state,
// the RK4 sums, and the two values the articulated-body inward pass hands to the last pass
// (u / D, U1 / D; U0 / D and U2 / D are 1: the rank-one form of pendulum.cuh's
// aba_accel_unrolled, which this kernel follows). Kept in local memory, 4 KB per
// environment at K = 64 missed L1 and L2 and the kernel waited on memory. Two things keep
// the count at eight:
// - link velocities are not stored: the inward pass starts from the last link's velocity and
//   walks them back link by link through the inverse joint transform (a rotation and a
//   shift), and the last pass recomputes them forward;
// - each joint's sine and cosine come from the special function unit in every pass instead
//   of being stored.
// The last pass applies the RK4 stage update to each link as soon as its acceleration is
// known, so no acceleration array is kept, and it walks the velocities of the state it
// writes forward as it writes them: the last link's velocity, which the next stage's inward
// pass starts from, needs no pass of its own except at a launch's first step and after a
// reset. The last pass of a step's final stage also sums the termination height. The arrays
// are laid out (link, array, thread): the 32 threads of a block touch 32 consecutive words
// (no bank conflicts), and one pointer per link reaches all eight.
#include "pendulum_kernels.cuh"

namespace rlenv {
namespace pend {

constexpr int kLongBlock = 32;
constexpr int kLongArrays = 8;
constexpr int kMaxLongLinks = 192;  // 8 K floats x 32 threads within 227 KB of shared memory
enum LongArray { kTh = 0, kOm, kTs, kOs, kDth, kDom, kGu, kU1 };

size_t long_smem_bytes(int k) { return size_t(kLongArrays) * k * kLongBlock * sizeof(float); }

// The hardware reciprocal (within one ulp): on the inward pass's serial chain, where the
// correctly rounded division would add its slow-path sequence to every link.
RLENV_D float rcp_approx(float a) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(a));
  return r;
}

// Link-major: the eight values of link i sit together, (link, array, thread), so a pass over the
// links advances one pointer and reaches every array at a fixed offset from it.
struct LongLinks {
  float* base;  // link 0, array 0 of this thread
  int k;
  RLENV_D float& at(int a, int i) const { return base[(i * kLongArrays + a) * kLongBlock]; }
};

// A link's velocity: angular w, then linear (x, y) in the link's frame.
struct LinkVel {
  float w, x, y;
};

// The sine and cosine of a joint angle (the difference of two stage angles, or the root's stage
// angle), from the special function unit without a 2 pi reduction (sincos_sfu_near). Stage angles
// are wrapped angles plus at most dt times a clipped rate (0.63), so a joint angle lies within
// 2 pi + 1.3 < 8 of zero, where the unit is within 1.21e-6 of sin and cos; the accelerations
// enter the step weighted by dt / 6 and dt / 3.
RLENV_D void joint_sincos(float x, float* s, float* c) { sincos_sfu_near(x, s, c); }

// v_i = X_i v_{i-1} + S qd_i: the velocity of link i from its parent's, given the joint's sine,
// cosine and rate qd (the joint sits at (1, 0) of the parent). Explicit operations: the pass of
// its own and the last pass of the stage before form the same bits.
RLENV_D void outward_link(float s, float c, float qd, LinkVel& v) {
  const float xy = __fadd_rn(v.y, v.w);
  const float nx = fmaf(c, v.x, __fmul_rn(s, xy));
  const float ny = fmaf(-s, v.x, __fmul_rn(c, xy));
  v.w = __fadd_rn(v.w, qd);
  v.x = nx;
  v.y = ny;
}

// The last link's velocity for the angles and rates of arrays (ia, io).
RLENV_D LinkVel last_link_velocity(const LongLinks& L, int ia, int io) {
  LinkVel v{L.at(io, 0), 0.0f, 0.0f};
  float pth = L.at(ia, 0), pom = v.w;
#pragma unroll 4
  for (int i = 1; i < L.k; ++i) {
    const float th = L.at(ia, i), om = L.at(io, i);
    float s, c;
    joint_sincos(__fsub_rn(th, pth), &s, &c);
    outward_link(s, c, __fsub_rn(om, pom), v);
    pth = th;
    pom = om;
  }
  return v;
}

// Accelerations of the stage whose angles and velocities are arrays (ia, io) and whose last
// link's velocity is tip, applied at once as RK4 stage `stage` (0..3): pendulum_rk4's update
// for link i, written into the stage, sum and state arrays (pendulum_np.py:60-66). Returns the
// last link's velocity of the state written: the next stage's, or with stage 3 the next step's,
// whose sum of cos theta_j over the links, from the special function unit, goes to height.
RLENV_D LinkVel aba_stage(const LongLinks& L, int ia, int io, float torque, int stage, LinkVel tip,
                          float& height) {
  const int k = L.k;
  // ---- inward: the subtree's articulated inertia (I00, I01, I11) and bias (p0, p1), carried to
  // the parent in the rank-one form; the link velocities walked back from the last
  // (x_{i-1} = c x_i - s y_i, y_{i-1} = s x_i + c y_i - w_{i-1})
  float cI00 = 0.0f, cI01 = 0.0f, cI11 = 0.0f, cp0 = 0.0f, cp1 = 0.0f;
  {
    float vw = tip.w, vx = tip.x, vy = tip.y;
    float th = L.at(ia, k - 1), om = L.at(io, k - 1);
#pragma unroll 2
    for (int i = k - 1; i >= 1; --i) {
      const float pth = L.at(ia, i - 1), pom = L.at(io, i - 1);
      const float qd = om - pom;
      float s, c;
      joint_sincos(__fsub_rn(th, pth), &s, &c);
      const float w = vw, x = vx, y = vy;
      // own bias v x* (I v) of a unit mass at (1, 0): (x w, -w (w + y), x w)
      const float p0 = x * w + cp0;
      const float p1 = -w * (w + y) + cp1;
      const float a00 = 1.0f + cI00, a01 = cI01, a11 = 1.0f + cI11;
      const float r = rcp_approx(a00);
      const float g = -p0 * r;
      const float u1 = a01 * r;
      const float m = a11 - a01 * u1;
      L.at(kGu, i) = g;
      L.at(kU1, i) = u1;
      const float pa1 = p1 + m * (qd * y) + a01 * g;
      const float ms = m * s;
      cI00 = ms * s;
      cI01 = ms * c;
      cI11 = (m * c) * c;
      cp0 = s * pa1;
      cp1 = c * pa1;
      // the parent's velocity
      const float pw = w - qd;
      vx = c * x - s * y;
      vy = (s * x + c * y) - pw;
      vw = pw;
      th = pth;
      om = pom;
    }
  }
  // ---- last pass: accelerations outward from the root (gravity as a base acceleration -G),
  // each link's RK4 stage update applied as soon as its acceleration is known
  const float th0 = L.at(ia, 0), om0 = L.at(io, 0);
  float ax, ay, aw, run;
  {
    const float U0_0 = 1.0f + cI00, U1_0 = cI01;  // U2 = U0
    const float uu0 = torque - cp0;  // the root's own bias is zero: v_0 = (qd_0, 0, 0)
    float sn0, cs0;
    joint_sincos(th0, &sn0, &cs0);
    ax = cs0 * -pd::G;
    ay = -sn0 * -pd::G;
    const float qdd = (uu0 - (U1_0 * ax + U0_0 * ay)) * rcp_approx(U0_0);
    aw = qdd;
    run = qdd;
  }
  // link i's update; (nth, nom) receive what it writes for the next stage (the next step's state
  // at stage 3)
  auto update = [&](int i, float a, float& nth, float& nom) {
    float& th = L.at(kTh, i);
    float& om = L.at(kOm, i);
    const float om_in = L.at(io, i);
    switch (stage) {
      case 0:
        L.at(kDth, i) = om_in;
        L.at(kDom, i) = a;
        nth = th + pd::HALF_DT * om_in;
        nom = om + pd::HALF_DT * a;
        L.at(kTs, i) = nth;
        L.at(kOs, i) = nom;
        break;
      case 1:
      case 2:
        L.at(kDth, i) += 2.0f * om_in;
        L.at(kDom, i) += 2.0f * a;
        nth = th + (stage == 1 ? pd::HALF_DT : pd::DT) * om_in;
        nom = om + (stage == 1 ? pd::HALF_DT : pd::DT) * a;
        L.at(kTs, i) = nth;
        L.at(kOs, i) = nom;
        break;
      default:
        nth = pd_wrap(th + pd::SIXTH_DT * (L.at(kDth, i) + om_in));
        nom = fminf(fmaxf(om + pd::SIXTH_DT * (L.at(kDom, i) + a), -pd::MAX_VEL), pd::MAX_VEL);
        th = nth;
        om = nom;
        break;
    }
  };
  float nth, nom;
  update(0, run, nth, nom);
  LinkVel next{nom, 0.0f, 0.0f};  // the written state's link velocities, forward
  float hq = stage == 3 ? __cosf(nth) : 0.0f;
  {
    float pth = th0, pom = om0, pnth = nth, pnom = nom;
    LinkVel v{om0, 0.0f, 0.0f};  // this stage's link velocities, forward again
#pragma unroll 4
    for (int i = 1; i < k; ++i) {
      const float th = L.at(ia, i), om = L.at(io, i);  // read before this link's update rewrites them
      const float qd = __fsub_rn(om, pom);
      float s, c;
      joint_sincos(__fsub_rn(th, pth), &s, &c);
      outward_link(s, c, qd, v);
      const float c1 = qd * v.y, c2 = -qd * v.x;
      const float xy = ay + aw;
      const float ap1 = c * ax + s * xy + c1;
      const float ap2 = -s * ax + c * xy + c2;
      const float q2 = L.at(kGu, i) - aw - L.at(kU1, i) * ap1 - ap2;
      aw = aw + q2;
      ax = ap1;
      ay = ap2;
      run += q2;
      update(i, run, nth, nom);
      float sn, cn;
      joint_sincos(__fsub_rn(nth, pnth), &sn, &cn);
      outward_link(sn, cn, __fsub_rn(nom, pnom), next);
      if (stage == 3) hq += __cosf(nth);
      pth = th;
      pom = om;
      pnth = nth;
      pnom = nom;
    }
  }
  height = hq;
  return next;
}

// T steps per launch for N environments; step t reads actions[t * n + e], draws its resets
// from seed0 + t and writes reward_seq / done_seq row t when those are not null.
__global__ void __launch_bounds__(kLongBlock)
pendulum_aba_long_kernel(int k, const float* __restrict__ state, const void* __restrict__ actions,
                         int dtype, uint32_t seed0, int64_t T, int64_t n, int64_t off,
                         float* __restrict__ next, float* __restrict__ reward_seq,
                         uint8_t* __restrict__ done_seq) {
  extern __shared__ float links[];
  const int64_t e = int64_t(blockIdx.x) * kLongBlock + threadIdx.x;
  if (e >= n) return;
  const LongLinks L{links + threadIdx.x, k};
  for (int j = 0; j < k; ++j) {
    L.at(kTh, j) = __ldg(state + j * n + e);
    L.at(kOm, j) = __ldg(state + (k + j) * n + e);
  }
  int act = T > 0 ? action_at(actions, dtype, e) : 0;
  // The tip above half the chain's length, -sum_j cos t_j > K / 2, is decided on cos_fast's
  // terms (within 1.6 ulp). The special function unit's sum, hq, of the same wrapped angles
  // (each term within 6.5e-7 of cos, measured on a B200 for |x| <= 4) is within K 1e-6 +
  // K^2 2^-23 of it: the terms' errors, plus at most one ulp of a partial sum (|partial| <= K)
  // per addition between the two sums' roundings. Outside twice that band of the threshold
  // both decide alike; inside it the cos_fast sum decides.
  const float half = float(k) * 0.5f;
  const float band = 2.0f * (float(k) * 1e-6f + float(k) * float(k) * 1.1920929e-7f);
  LinkVel tip = last_link_velocity(L, kTh, kOm);
  for (int64_t t = 0; t < T; ++t) {
    check_flag(act < 0 || act > 2, kCheckActionRange);
    const float torque = float(act - 1) * pd::TORQUE;
    if (t + 1 < T) act = action_at(actions, dtype, (t + 1) * n + e);
    float hq;
    tip = aba_stage(L, kTh, kOm, torque, 0, tip, hq);
    tip = aba_stage(L, kTs, kOs, torque, 1, tip, hq);
    tip = aba_stage(L, kTs, kOs, torque, 2, tip, hq);
    tip = aba_stage(L, kTs, kOs, torque, 3, tip, hq);
    bool d;
    if (fabsf(-hq - half) <= band) {
      float h = 0.0f;
      for (int j = 0; j < k; ++j) h += cos_fast(L.at(kTh, j));
      d = -h > half;
    } else {
      d = -hq > half;
    }
    if (d) {
      const uint32_t hs = env_hash(seed0 + uint32_t(t), off + e);
      for (int j = 0; j < k; ++j) {
        L.at(kTh, j) = uniform_pm(pcg_hash(hs + uint32_t(j) * kRowStride), pd::RESET_BOUND);
        L.at(kOm, j) = uniform_pm(pcg_hash(hs + uint32_t(k + j) * kRowStride), pd::RESET_BOUND);
      }
      tip = last_link_velocity(L, kTh, kOm);
    }
    if (reward_seq) reward_seq[t * n + e] = d ? 0.0f : -1.0f;
    if (done_seq) done_seq[t * n + e] = d;
  }
  for (int j = 0; j < k; ++j) {
    check_flag(!(isfinite(L.at(kTh, j)) && isfinite(L.at(kOm, j))), kCheckNonFinite);
    next[j * n + e] = L.at(kTh, j);
    next[(k + j) * n + e] = L.at(kOm, j);
  }
}

int launch_aba_long(int k, const float* state, const void* actions, int dtype, uint32_t seed0,
                    int64_t T, int64_t n, int64_t off, float* next, float* reward_seq,
                    uint8_t* done_seq, void* stream) {
  if (k < 2 || k > kMaxLongLinks) return RLENV_EUNSUPPORTED;
  if (n == 0) return RLENV_OK;
  const size_t smem = long_smem_bytes(k);
  cudaError_t e = cudaFuncSetAttribute(pendulum_aba_long_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(pendulum_aba_long_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                             int(cudaSharedmemCarveoutMaxShared));
  if (e != cudaSuccess) return int(e);
  const int64_t blocks = (n + kLongBlock - 1) / kLongBlock;
  if (blocks > int64_t(0x7fffffff)) return RLENV_EINVAL;
  pendulum_aba_long_kernel<<<int(blocks), kLongBlock, smem, as_stream(stream)>>>(
      k, state, actions, dtype, seed0, T, n, off, next, reward_seq, done_seq);
  return launch_status();
}

}  // namespace pend
}  // namespace rlenv
