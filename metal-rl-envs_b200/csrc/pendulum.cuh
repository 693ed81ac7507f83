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
    // and issue together, where one at a time each waited for its own round trip (measured on a
    // B200 at K = 64, N = 65,536, with aba_accel_loops below: 60 -> 105 M env-steps/s)
#pragma unroll 8
    for (int i = 0; i < N; ++i) f(i);
  }
}

// K-link arrays stay in registers (fully unrolled loops) up to this size.
constexpr int kUnrollLinks = 16;

// Every acceleration evaluation (the four RK4 stages) takes its sines and cosines from
// the special function unit (sincos_sfu, within 5.9e-7 absolute); the derivatives enter
// the step weighted by dt / 6 and dt / 3. Termination, which the done flags must get
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
  // Cholesky in place with the reciprocals of the diagonal, then forward and
  // back substitution: K divisions instead of K (K + 3) / 2.
  float inv_d[K];
#pragma unroll
  for (int i = 0; i < K; ++i) {
#pragma unroll
    for (int j = 0; j <= i; ++j) {
      float v = L[tri(i, j)];
#pragma unroll
      for (int p = 0; p < j; ++p) v -= L[tri(i, p)] * L[tri(j, p)];
      if (i == j) {
        L[tri(i, i)] = sqrtf(v);
        inv_d[i] = 1.0f / L[tri(i, i)];
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

// The same three passes as loops over per-link arrays in local memory, for
// chains too long to unroll fully (K > kUnrollLinks), unrolled by 8 so that the
// per-link loads of several links are in flight together. It is kept out of line: when
// nvcc inlined these loops into the RK4 driver, whose stage arrays they index
// by the loop variable, the optimised device code returned wrong accelerations
// for K >= 24 although every single evaluation was right; the same source is
// correct out of line, without NVVM optimisation (-Xcicc -O0), under -G, and
// compiled for the host.
template <int K>
__device__ __noinline__ void aba_accel_loops(const float* th, const float* om, float torque,
                                             float* acc) {
  // Seven per-link arrays in local memory. The inward pass overwrites what the last pass no
  // longer needs: vw becomes u / D, vx and vy the velocity-product terms -qd vx and qd vy,
  // and U1r, U2r hold U1 / D and U2 / D (U0 / D is 1: D = U0).
  float vw[K], vx[K], vy[K], sn[K], cs[K], U1r[K], U2r[K];
  vw[0] = om[0];
  vx[0] = 0.0f;
  vy[0] = 0.0f;
#pragma unroll 8
  for (int i = 1; i < K; ++i) {
    const float qd = om[i] - om[i - 1];
    float s, c;
    sincos_sfu(th[i] - th[i - 1], &s, &c);
    sn[i] = s;
    cs[i] = c;
    const float pw = vw[i - 1], px = vx[i - 1], xy = vy[i - 1] + pw;
    vw[i] = pw + qd;
    vx[i] = c * px + s * xy;
    vy[i] = -s * px + c * xy;
  }
  // Articulated inertia (symmetric 3x3, upper half) and bias force that the child link hands to
  // its parent in the inward pass; zero below the last link.
  float carry_I00 = 0.0f, carry_I01 = 0.0f, carry_I02 = 0.0f;
  float carry_I11 = 0.0f, carry_I12 = 0.0f, carry_I22 = 0.0f;
  float carry_p0 = 0.0f, carry_p1 = 0.0f, carry_p2 = 0.0f;
#pragma unroll 8
  for (int i = K - 1; i >= 1; --i) {
    const float w = vw[i], x = vx[i], y = vy[i];
    const float qd = om[i] - om[i - 1];
    const float fy = w + y;
    const float p0 = (x * fy - y * x) + carry_p0, p1 = (-w * fy) + carry_p1, p2 = (w * x) + carry_p2;
    const float a00 = 1.0f + carry_I00, a01 = carry_I01, a02 = 1.0f + carry_I02;
    const float a11 = 1.0f + carry_I11, a12 = carry_I12, a22 = 1.0f + carry_I22;
    const float r = 1.0f / a00;
    const float Ia00 = a00 - a00 * a00 * r, Ia01 = a01 - a00 * a01 * r, Ia02 = a02 - a00 * a02 * r;
    const float Ia11 = a11 - a01 * a01 * r, Ia12 = a12 - a01 * a02 * r, Ia22 = a22 - a02 * a02 * r;
    const float c1 = qd * y, c2 = -qd * x;
    const float g = -p0 * r;
    vw[i] = g;
    vx[i] = c2;
    vy[i] = c1;
    U1r[i] = a01 * r;
    U2r[i] = a02 * r;
    const float pa0 = p0 + (Ia01 * c1 + Ia02 * c2) + a00 * g;
    const float pa1 = p1 + (Ia11 * c1 + Ia12 * c2) + a01 * g;
    const float pa2 = p2 + (Ia12 * c1 + Ia22 * c2) + a02 * g;
    const float s = sn[i], c = cs[i];
    const float B00 = Ia00 + Ia01 * s + Ia02 * c, B01 = Ia01 * c - Ia02 * s, B02 = Ia01 * s + Ia02 * c;
    const float B10 = Ia01 + Ia11 * s + Ia12 * c, B11 = Ia11 * c - Ia12 * s, B12 = Ia11 * s + Ia12 * c;
    const float B20 = Ia02 + Ia12 * s + Ia22 * c, B21 = Ia12 * c - Ia22 * s, B22 = Ia12 * s + Ia22 * c;
    carry_I00 = B00 + s * B10 + c * B20;
    carry_I01 = B01 + s * B11 + c * B21;
    carry_I02 = B02 + s * B12 + c * B22;
    carry_I11 = c * B11 - s * B21;
    carry_I12 = c * B12 - s * B22;
    carry_I22 = s * B12 + c * B22;
    carry_p0 = pa0 + s * pa1 + c * pa2;
    carry_p1 = c * pa1 - s * pa2;
    carry_p2 = s * pa1 + c * pa2;
  }
  const float w0 = vw[0], x0 = vx[0], y0 = vy[0], fy0 = w0 + y0;
  const float U0_0 = 1.0f + carry_I00, U1_0 = carry_I01, U2_0 = 1.0f + carry_I02;
  const float uu0 = torque - ((x0 * fy0 - y0 * x0) + carry_p0);
  float sn0, cs0;
  sincos_sfu(th[0], &sn0, &cs0);
  float ax = cs0 * -pd::G + om[0] * y0;
  float ay = -sn0 * -pd::G - om[0] * x0;
  const float qdd = (uu0 - (U0_0 * 0.0f + U1_0 * ax + U2_0 * ay)) / U0_0;
  float aw = 0.0f + qdd, run = qdd;
  acc[0] = run;
#pragma unroll 8
  for (int i = 1; i < K; ++i) {
    const float xy = ay + aw;
    const float ap1 = cs[i] * ax + sn[i] * xy + vy[i];
    const float ap2 = -sn[i] * ax + cs[i] * xy + vx[i];
    const float q2 = vw[i] - aw - U1r[i] * ap1 - U2r[i] * ap2;
    aw = aw + q2;
    ax = ap1;
    ay = ap2;
    run += q2;
    acc[i] = run;
  }
}

// The three passes fully unrolled, every per-link array in registers (K <= kUnrollLinks).
template <int K>
RLENV_D void aba_accel_unrolled(const float* th, const float* om, float torque, float* acc) {
  // per link: velocity, the joint rotation's sine and cosine (evaluated once, used by all three
  // passes); the inward pass then overwrites the velocity with what the last pass needs
  // (u / D and the velocity-product terms c2 = -qd vx, c1 = qd vy) and keeps U1 / D, U2 / D
  // (U0 / D is 1: D = U0)
  float vw[K], vx[K], vy[K], sn[K], cs[K], U1r[K], U2r[K];
  // outward: link velocities v_i = X_i v_{i-1} + S qd_i; the root has v_0 = (qd_0, 0, 0)
  vw[0] = om[0];
  vx[0] = 0.0f;
  vy[0] = 0.0f;
  for_links<1, K, true, true>([&](int i) {
    const float qd = om[i] - om[i - 1];
    sincos_sfu(th[i] - th[i - 1], &sn[i], &cs[i]);
    const float pw = vw[i - 1], px = vx[i - 1], xy = vy[i - 1] + pw;  // joint at (1, 0)
    vw[i] = pw + qd;
    vx[i] = cs[i] * px + sn[i] * xy;
    vy[i] = -sn[i] * px + cs[i] * xy;
  });
  // inward: articulated inertia (symmetric 3x3, upper half) and bias force of the subtree,
  // carried to the parent as the child's contribution; zero below the last link
  float carry_I00 = 0.0f, carry_I01 = 0.0f, carry_I02 = 0.0f;
  float carry_I11 = 0.0f, carry_I12 = 0.0f, carry_I22 = 0.0f;
  float carry_p0 = 0.0f, carry_p1 = 0.0f, carry_p2 = 0.0f;
  for_links<1, K, false, true>([&](int i) {
    const float w = vw[i], x = vx[i], y = vy[i];
    const float qd = om[i] - om[i - 1];
    // own bias p = v x* (I v), I of a unit mass at (1, 0) = [[1,0,1],[0,1,0],[1,0,1]]
    const float fy = w + y;
    const float p0 = (x * fy - y * x) + carry_p0;
    const float p1 = (-w * fy) + carry_p1;
    const float p2 = (w * x) + carry_p2;
    const float a00 = 1.0f + carry_I00, a01 = carry_I01, a02 = 1.0f + carry_I02;
    const float a11 = 1.0f + carry_I11, a12 = carry_I12, a22 = 1.0f + carry_I22;
    const float r = 1.0f / a00;  // D = a00
    const float Ia00 = a00 - a00 * a00 * r, Ia01 = a01 - a00 * a01 * r, Ia02 = a02 - a00 * a02 * r;
    const float Ia11 = a11 - a01 * a01 * r, Ia12 = a12 - a01 * a02 * r, Ia22 = a22 - a02 * a02 * r;
    const float c1 = qd * y, c2 = -qd * x;  // c_i = v_i x S qd
    const float g = -p0 * r;                 // u / D, u = -p0
    vw[i] = g;
    vx[i] = c2;
    vy[i] = c1;
    U1r[i] = a01 * r;
    U2r[i] = a02 * r;
    const float pa0 = p0 + (Ia01 * c1 + Ia02 * c2) + a00 * g;
    const float pa1 = p1 + (Ia11 * c1 + Ia12 * c2) + a01 * g;
    const float pa2 = p2 + (Ia12 * c1 + Ia22 * c2) + a02 * g;
    const float s = sn[i], c = cs[i];
    // B = Ia X with X = [[1,0,0],[s,c,s],[c,-s,c]] (r = 1); parent gets X^T B and X^T pa
    const float B00 = Ia00 + Ia01 * s + Ia02 * c, B01 = Ia01 * c - Ia02 * s, B02 = Ia01 * s + Ia02 * c;
    const float B10 = Ia01 + Ia11 * s + Ia12 * c, B11 = Ia11 * c - Ia12 * s, B12 = Ia11 * s + Ia12 * c;
    const float B20 = Ia02 + Ia12 * s + Ia22 * c, B21 = Ia12 * c - Ia22 * s, B22 = Ia12 * s + Ia22 * c;
    carry_I00 = B00 + s * B10 + c * B20;
    carry_I01 = B01 + s * B11 + c * B21;
    carry_I02 = B02 + s * B12 + c * B22;
    carry_I11 = c * B11 - s * B21;
    carry_I12 = c * B12 - s * B22;
    carry_I22 = s * B12 + c * B22;
    carry_p0 = pa0 + s * pa1 + c * pa2;
    carry_p1 = c * pa1 - s * pa2;
    carry_p2 = s * pa1 + c * pa2;
  });
  // root link: its inertia and bias with the whole chain's contribution
  const float w0 = vw[0], x0 = vx[0], y0 = vy[0], fy0 = w0 + y0;
  const float U0_0 = 1.0f + carry_I00, U1_0 = carry_I01, U2_0 = 1.0f + carry_I02;
  const float uu0 = torque - ((x0 * fy0 - y0 * x0) + carry_p0);
  // outward: accelerations, the base accelerating at -G; the absolute angular
  // accelerations are the running sum of the joint accelerations
  float sn0, cs0;
  sincos_sfu(th[0], &sn0, &cs0);
  const float qd0 = om[0];
  // root: X_0 maps the base acceleration (0, -G, 0); r = 0
  float ax = cs0 * -pd::G + qd0 * y0;
  float ay = -sn0 * -pd::G - qd0 * x0;
  const float qdd = (uu0 - (U0_0 * 0.0f + U1_0 * ax + U2_0 * ay)) / U0_0;
  float aw = 0.0f + qdd;
  float run = qdd;
  acc[0] = run;
  for_links<1, K, true, true>([&](int i) {
    const float xy = ay + aw;
    const float ap1 = cs[i] * ax + sn[i] * xy + vy[i];
    const float ap2 = -sn[i] * ax + cs[i] * xy + vx[i];
    const float q2 = vw[i] - aw - U1r[i] * ap1 - U2r[i] * ap2;
    aw = aw + q2;
    ax = ap1;
    ay = ap2;
    run += q2;
    acc[i] = run;
  });
}

template <int K>
RLENV_D void aba_accel(const float* th, const float* om, float torque, float* acc) {
  if constexpr (K > kUnrollLinks) {
    aba_accel_loops<K>(th, om, torque, acc);
  } else {
    aba_accel_unrolled<K>(th, om, torque, acc);
  }
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
