// K-link planar pendulum dynamics: the mass-matrix form (pendulum_np.py) and
// Featherstone's articulated-body form (pendulum_aba_np.py), plus the shared
// RK4 driver. Unit point masses on unit massless rods, absolute angles from
// the downward vertical, torque at the root joint.
#pragma once

#include "common.cuh"

namespace rlenv {
namespace pd {
constexpr float G = 9.8f;
constexpr float DT = 0.02f;
constexpr float HALF_DT = 0.01f;
constexpr float SIXTH_DT = 0.0033333333333333335f;
constexpr float TORQUE = 1.0f;
constexpr float MAX_VEL = 31.41592653589793f;  // 10 pi
constexpr float PI = 3.141592653589793f;
constexpr float TWO_PI = 6.283185307179586f;
constexpr float RESET_BOUND = 0.1f;
}  // namespace pd

RLENV_D float pd_wrap(float x) { return wrap_to_pi(x); }  // pendulum_np.py wrap

// Calls f(i) for i = 0 .. N-1, fully unrolled when UNROLL, as a plain loop
// otherwise. A per-environment array is either always indexed by constants
// (unrolled: it lives in registers) or always by the loop variable (local
// memory): every loop that touches the arrays of one K uses the same UNROLL,
// never a mix of the two.
template <int N, bool UNROLL, typename F>
RLENV_D void for_range(F&& f) {
  if constexpr (UNROLL) {
#pragma unroll
    for (int i = 0; i < N; ++i) f(i);
  } else {
    // partly unrolled: the local-memory loads of eight iterations are independent of one another
    // and issue together, where one at a time each waited for its own round trip
#pragma unroll 8
    for (int i = 0; i < N; ++i) f(i);
  }
}

// K-link arrays stay in registers (fully unrolled loops) up to this size.
constexpr int kUnrollLinks = 16;

// Every acceleration evaluation (the four RK4 stages) takes its sines and cosines from
// the special function unit (the mass matrix through sincos_sfu, within 5.9e-7 absolute; the
// articulated body without the 2 pi reduction, sincos_sfu_near, within 1.21e-6 over the
// |x| < 8 that a joint angle of two stage angles spans); the derivatives enter the step
// weighted by dt / 6 and dt / 3. Termination, which the done flags must get
// exactly right, uses cos_fast (within 1.6 ulp). The reference's Metal kernels call
// Metal's default fast-math sin and cos (pendulum_metal.py:27, 98-102;
// pendulum_aba_metal.py:34, 61, 74).

// ---- mass-matrix accelerations (pendulum_np.py:68-111) ---------------------
// M_ij = mu_ij cos(t_i - t_j), mu_ij = K - max(i, j); rhs_i = -sum_j mu_ij
// sin(t_i - t_j) w_j^2 - G mu_ii sin t_i (+ torque at the root); M acc = rhs by
// Cholesky. The lower triangle is stored packed. The angle-difference
// cosines and sines come from K cosines and sines by the addition formulas,
// or, with PAIRWISE, are evaluated directly (the v9 variant,
// pendulum_metal.py:96-103).
template <int K, bool PAIRWISE>
RLENV_D void mm_accel(const float (&th)[K], const float (&om)[K], float torque, float (&acc)[K]) {
  float c[K], s[K];
#pragma unroll
  for (int i = 0; i < K; ++i) sincos_sfu(th[i], &s[i], &c[i]);
  float L[K * (K + 1) / 2];
  float rhs[K];
#pragma unroll
  for (int i = 0; i < K; ++i) {
    float r = 0.0f;
#pragma unroll
    for (int j = 0; j < K; ++j) {
      const float mu = float(K - (i > j ? i : j));
      float cd, sd;
      if (PAIRWISE) {
        sincos_sfu(th[i] - th[j], &sd, &cd);
      } else {
        cd = c[i] * c[j] + s[i] * s[j];
        sd = s[i] * c[j] - c[i] * s[j];
      }
      if (j <= i) L[tri(i, j)] = mu * cd;
      r += mu * sd * (om[j] * om[j]);
    }
    rhs[i] = -r - (pd::G * float(K - i)) * s[i];
  }
  rhs[0] += torque;
  // Cholesky in place with the reciprocals of the diagonal, then forward and back
  // substitution. The diagonal itself is needed only through its reciprocal, which the
  // hardware's reciprocal square root gives directly from the pivot (rsqrt.approx, within two
  // ulp; the pivots of this positive definite matrix are far from zero): no square root and no
  // division, each a multi-instruction sequence with a slow path.
  float inv_d[K];
#pragma unroll
  for (int i = 0; i < K; ++i) {
#pragma unroll
    for (int j = 0; j <= i; ++j) {
      float v = L[tri(i, j)];
#pragma unroll
      for (int p = 0; p < j; ++p) v -= L[tri(i, p)] * L[tri(j, p)];
      if (i == j) {
        asm("rsqrt.approx.ftz.f32 %0, %1;" : "=f"(inv_d[i]) : "f"(v));
      } else {
        L[tri(i, j)] = v * inv_d[j];
      }
    }
  }
#pragma unroll
  for (int i = 0; i < K; ++i) {
    float v = rhs[i];
#pragma unroll
    for (int p = 0; p < i; ++p) v -= L[tri(i, p)] * acc[p];
    acc[i] = v * inv_d[i];
  }
#pragma unroll
  for (int i = K - 1; i >= 0; --i) {
    float v = acc[i];
#pragma unroll
    for (int p = i + 1; p < K; ++p) v -= L[tri(p, i)] * acc[p];
    acc[i] = v * inv_d[i];
  }
}

// ---- articulated-body accelerations (pendulum_aba_np.py:30-99) -------------
// Planar spatial algebra: motion vectors (w, vx, vy), force vectors (n, fx,
// fy), symmetric 3x3 inertias stored as (00, 01, 02, 11, 12, 22). Link i's
// frame is rotated by its absolute angle; the joint coordinate is
// q_i = t_i - t_{i-1}; each unit mass sits at (1, 0) of its link frame and
// the next joint at (1, 0) too. Gravity enters as a base acceleration of -G.
// Per link only the link velocity, U = I^A S and u are kept; the bias force
// and the transform are recomputed. The root link (joint at the base origin,
// r = 0) is peeled out of every pass, so the loops over links 1..K-1 have no
// special cases; they are fully unrolled up to K = 16 and left as loops above.

// Calls f(i) for i = LO .. HI-1 (UP) or HI-1 down to LO, unrolled as for_range.
template <int LO, int HI, bool UP, bool UNROLL, typename F>
RLENV_D void for_links(F&& f) {
  for_range<HI - LO, UNROLL>([&](int t) { f(UP ? LO + t : HI - 1 - t); });
}

// The hardware reciprocal (rcp.approx.ftz, within one ulp) for the articulated inertias' D = a00
// and the root's U0, both at least one: the correctly rounded division is a multi-instruction
// sequence with a slow-path branch.
RLENV_D float aba_rcp(float a) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(a));
  return r;
}

// The three passes fully unrolled, every per-link array in registers (K <= kUnrollLinks).
//
// Every link is a unit point mass at (1, 0) of its frame, and every child's joint sits at that
// point. The articulated-body algebra then collapses, exactly (checked in float64 against the
// full 3x3 form to 1e-14): a subtree's articulated inertia, seen from its joint, has the
// pattern I00 = I02 = I22 of a mass at the joint's point, so U2 / D is 1; its projection
// Ia = I - U U^T / D keeps one nonzero entry, m = Ia11, and so what a subtree hands to its
// parent is rank one, m (s^2, s c, c^2) in (I00, I01, I11) and pa1 (s, c) in the bias (s, c the
// joint's sine and cosine), with pa0 = pa2 = 0. An inward step is then about 20 flops where the
// full 3x3 form takes about 80, and a link keeps u / D and U1 / D only.
template <int K>
RLENV_D void aba_accel_unrolled(const float* th, const float* om, float torque, float* acc) {
  // per link: velocity, the joint rotation's sine and cosine (evaluated once, used by all three
  // passes); the inward pass then overwrites the velocity with what the last pass needs
  // (u / D and the velocity-product terms c2 = -qd vx, c1 = qd vy) and keeps U1 / D
  float vw[K], vx[K], vy[K], sn[K], cs[K], U1r[K];
  // outward: link velocities v_i = X_i v_{i-1} + S qd_i; the root has v_0 = (qd_0, 0, 0)
  vw[0] = om[0];
  vx[0] = 0.0f;
  vy[0] = 0.0f;
  for_links<1, K, true, true>([&](int i) {
    const float qd = om[i] - om[i - 1];
    sincos_sfu_near(th[i] - th[i - 1], &sn[i], &cs[i]);
    const float pw = vw[i - 1], px = vx[i - 1], xy = vy[i - 1] + pw;  // joint at (1, 0)
    vw[i] = pw + qd;
    vx[i] = cs[i] * px + sn[i] * xy;
    vy[i] = -sn[i] * px + cs[i] * xy;
  });
  // inward: the subtree's articulated inertia (I00, I01, I11) and bias (p0, p1) carried to the
  // parent as the child's contribution; zero below the last link
  float cI00 = 0.0f, cI01 = 0.0f, cI11 = 0.0f, cp0 = 0.0f, cp1 = 0.0f;
  for_links<1, K, false, true>([&](int i) {
    const float w = vw[i], x = vx[i], y = vy[i];
    const float qd = om[i] - om[i - 1];
    // own bias v x* (I v) of a unit mass at (1, 0): (x w, -w (w + y), x w)
    const float p0 = x * w + cp0;
    const float p1 = -w * (w + y) + cp1;
    const float a00 = 1.0f + cI00, a01 = cI01, a11 = 1.0f + cI11;
    const float r = aba_rcp(a00);  // D = a00 >= 1
    const float g = -p0 * r;     // u / D, u = -p0
    const float u1 = a01 * r;
    const float m = a11 - a01 * u1;
    const float c1 = qd * y, c2 = -qd * x;  // c_i = v_i x S qd
    const float pa1 = p1 + m * c1 + a01 * g;
    vw[i] = g;
    vx[i] = c2;
    vy[i] = c1;
    U1r[i] = u1;
    const float s = sn[i], c = cs[i];
    const float ms = m * s;
    cI00 = ms * s;
    cI01 = ms * c;
    cI11 = (m * c) * c;
    cp0 = s * pa1;
    cp1 = c * pa1;
  });
  // root link: its inertia and bias with the whole chain's contribution (U2 = U0; the root's own
  // bias is zero, v_0 = (qd_0, 0, 0))
  const float U0_0 = 1.0f + cI00, U1_0 = cI01;
  const float uu0 = torque - cp0;
  // outward: accelerations, the base accelerating at -G; the absolute angular
  // accelerations are the running sum of the joint accelerations
  float sn0, cs0;
  sincos_sfu_near(th[0], &sn0, &cs0);
  // root: X_0 maps the base acceleration (0, -G, 0)
  float ax = cs0 * -pd::G;
  float ay = -sn0 * -pd::G;
  const float qdd = (uu0 - (U1_0 * ax + U0_0 * ay)) * aba_rcp(U0_0);
  float aw = qdd;
  float run = qdd;
  acc[0] = run;
  for_links<1, K, true, true>([&](int i) {
    const float xy = ay + aw;
    const float ap1 = cs[i] * ax + sn[i] * xy + vy[i];
    const float ap2 = -sn[i] * ax + cs[i] * xy + vx[i];
    const float q2 = vw[i] - aw - U1r[i] * ap1 - ap2;
    aw = aw + q2;
    ax = ap1;
    ay = ap2;
    run += q2;
    acc[i] = run;
  });
}

template <int K>
RLENV_D void aba_accel(const float* th, const float* om, float torque, float* acc) {
  static_assert(K <= kUnrollLinks, "longer chains run in pendulum_long.cu");
  aba_accel_unrolled<K>(th, om, torque, acc);
}

// ---- RK4 step on (theta, omega) (pendulum_np.py:60-66) -----------------------
// The angle derivative is omega itself, so only the accelerations need the
// dynamics. Returns wrapped angles and clipped velocities in th, om.
template <int K, bool UNROLL, typename Accel>
RLENV_D void pendulum_rk4(float (&th)[K], float (&om)[K], float torque, Accel accel) {
  float ts[K], os[K], a[K], dth[K], dom[K];
  accel(th, om, torque, a);  // k1 = (om, a1)
  for_range<K, UNROLL>([&](int j) {
    dth[j] = om[j];
    dom[j] = a[j];
    ts[j] = th[j] + pd::HALF_DT * om[j];
    os[j] = om[j] + pd::HALF_DT * a[j];
  });
  accel(ts, os, torque, a);  // k2 = (os, a2)
  for_range<K, UNROLL>([&](int j) {
    dth[j] += 2.0f * os[j];
    dom[j] += 2.0f * a[j];
    ts[j] = th[j] + pd::HALF_DT * os[j];
    os[j] = om[j] + pd::HALF_DT * a[j];
  });
  accel(ts, os, torque, a);  // k3
  for_range<K, UNROLL>([&](int j) {
    dth[j] += 2.0f * os[j];
    dom[j] += 2.0f * a[j];
    ts[j] = th[j] + pd::DT * os[j];
    os[j] = om[j] + pd::DT * a[j];
  });
  accel(ts, os, torque, a);  // k4
  for_range<K, UNROLL>([&](int j) {
    th[j] = pd_wrap(th[j] + pd::SIXTH_DT * (dth[j] + os[j]));
    om[j] = fminf(fmaxf(om[j] + pd::SIXTH_DT * (dom[j] + a[j]), -pd::MAX_VEL), pd::MAX_VEL);
  });
}

// The tip above half the chain's length: -sum_j cos t_j > K / 2.
template <int K, bool UNROLL>
RLENV_D bool pendulum_terminated(const float (&th)[K]) {
  float h = 0.0f;
  for_range<K, UNROLL>([&](int j) { h += cos_fast(th[j]); });
  return -h > float(K) * 0.5f;
}

}  // namespace rlenv
