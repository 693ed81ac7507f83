// CartPole and Acrobot dynamics as device functions, shared by the single-step
// kernels, the T-step kernels and the fused ES rollouts so that all of them run
// the same arithmetic.
#pragma once

#include "common.cuh"

namespace rlenv {

// ---- CartPole: Gym CartPole-v1, explicit Euler with tau = 0.02 -------------
// Constants and formulas follow cartpole_np.py:20-31 and 58-77: the float32
// values of the reference's Python constants.
namespace cp {
constexpr float G = 9.8f;
constexpr float POLE_MASS = 0.1f;
constexpr float TOTAL_MASS = 1.1f;         // 1.0 + 0.1
constexpr float HALF_POLE = 0.5f;
constexpr float POLE_MASS_LENGTH = 0.05f;  // 0.1 * 0.5
constexpr float FORCE = 10.0f;
constexpr float TAU = 0.02f;
constexpr float X_LIMIT = 2.4f;
constexpr float THETA_LIMIT = 0.20943951023931953f;  // 12 * 2 * pi / 360
constexpr float FOUR_THIRDS = 1.3333333333333333f;
constexpr float RESET_BOUND = 0.05f;
}  // namespace cp

struct CartPole {
  float x, xd, th, thd;
};

// The hardware reciprocal (rcp.approx, within one ulp) for denominators known to be normal.
RLENV_D float rcp_hw(float a) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(a));
  return r;
}

// One Euler step for a push of `force` (cartpole_np.py:58-77), with the divisions by the
// total mass M folded into constants (m l / M and 1 / M, each the float32 of the exact
// quotient):
//   temp = force / M + (m l / M) thd^2 sin,
//   th_acc = (G sin - cos temp) / (l (4/3 - m cos^2 / M)) = (G sin - cos temp) / (2/3 - (m l / M) cos^2),
//   x_acc = temp - (m l / M) th_acc cos,
// the pole's denominator, in [0.62, 0.67], through the hardware reciprocal. The sine and cosine
// come from the special function unit on the angle as given (sincos_sfu_near): a live pole is
// within 12 degrees of upright and a fresh one within 0.05 rad, where the unit is within
// 4.1e-7. The step's done flag depends on the state stepped from only (explicit Euler moves x
// and theta by the old rates), so the flags are the reference's whatever the rounding here;
// the rates move by a few 1e-8 against the reference's step.
RLENV_D CartPole cartpole_physics(CartPole s, float force) {
  constexpr float kInvM = float(1.0 / 1.1);
  constexpr float kMlOverM = float(0.05 / 1.1);
  constexpr float kTwoThirds = float(2.0 / 3.0);
  float sn, c;
  sincos_sfu_near(s.th, &sn, &c);
  const float temp = fmaf(kMlOverM * (s.thd * s.thd), sn, force * kInvM);
  const float th_acc = (cp::G * sn - c * temp) * rcp_hw(fmaf(-kMlOverM * c, c, kTwoThirds));
  const float x_acc = fmaf(-kMlOverM * th_acc, c, temp);
  CartPole n;
  n.x = s.x + cp::TAU * s.xd;
  n.xd = s.xd + cp::TAU * x_acc;
  n.th = s.th + cp::TAU * s.thd;
  n.thd = s.thd + cp::TAU * th_acc;
  return n;
}

RLENV_D bool cartpole_terminated(const CartPole& s) {
  return fabsf(s.x) > cp::X_LIMIT || fabsf(s.th) > cp::THETA_LIMIT;
}

RLENV_D float cartpole_force(int action) { return action == 1 ? cp::FORCE : -cp::FORCE; }

// ---- Acrobot: Gym's book dynamics, RK4 with dt = 0.2 -----------------------
// acrobot_np.py:19-30 and 47-93.
namespace ac {
constexpr float DT = 0.2f;
constexpr float HALF_DT = 0.1f;
constexpr float SIXTH_DT = 0.03333333333333333f;
constexpr float MAX_VEL_1 = 12.566370614359172f;  // 4 pi
constexpr float MAX_VEL_2 = 28.274333882308138f;  // 9 pi
constexpr float PI = 3.141592653589793f;
constexpr float TWO_PI = 6.283185307179586f;
constexpr float HALF_PI = 1.5707963267948966f;
constexpr float RESET_BOUND = 0.1f;
// Products of the unit link constants, as the reference's Python evaluates them.
constexpr float PHI2_K = 4.9f;      // m2 lc2 g
constexpr float PHI1_K = 14.700000000000001f;  // (m1 lc1 + m2 l1) g
}  // namespace ac

struct Acrobot {
  float th1, th2, dth1, dth2;
};

// Sines and cosines of both angles of an Acrobot state. Every derivative
// evaluation needs exactly these: the reference's cos(theta1 + theta2 - pi/2)
// and cos(theta1 - pi/2) are sin(theta1 + theta2) and sin(theta1), and the
// former comes from the addition formula. The termination test of a stepped
// state needs them too, and they are then the first RK4 stage's of the next
// step, so a chain of steps evaluates them once per state.
struct AcrobotTrig {
  float s1, c1, s2, c2;
};

RLENV_D AcrobotTrig acrobot_trig(const Acrobot& s) {
  AcrobotTrig t;
  sincos_fast(s.th1, &t.s1, &t.c1);
  sincos_fast(s.th2, &t.s2, &t.c2);
  return t;
}

// The trig of an Acrobot state from the special function unit, with no 2 pi reduction
// (sincos_sfu_near), for every state a step evaluates: a wrapped stepped state (|angle| <=
// 3.1415968: within 4.1e-7 of sin and cos, measured on a B200), a fresh one, a state read from
// memory (a launch's first step), and the second to fourth RK4 stage states, whose angles are a
// wrapped angle plus dt / 2 or dt times a stage rate, within 8 of zero but for extreme rates
// (within 1.21e-6). The stage derivatives enter the step weighted by dt / 3 and dt / 6, and the
// stepped state stays within the 1e-5 single-step gate of the reference's. It is one function
// of the state alone, so a chain of steps gives the same bits whether the state stays in
// registers or goes through memory. Against a 2 pi reduction first (sincos_sfu) it saves four
// instructions per angle, 32 per environment-step. The reference's Metal kernel evaluates
// every sine and cosine with Metal's default fast-math sin and cos (acrobot_metal.py:42-47, 75).
RLENV_D AcrobotTrig acrobot_stage_trig(const Acrobot& s) {
  AcrobotTrig t;
  sincos_sfu_near(s.th1, &t.s1, &t.c1);
  sincos_sfu_near(s.th2, &t.s2, &t.c2);
  return t;
}

// Gym AcrobotEnv._dsdt with the torque passed alongside (acrobot_np.py:64-86), with the unit
// link constants folded (m1 = m2 = l1 = I1 = I2 = 1, lc1 = lc2 = 1/2, g = 9.8):
//   d1 = m1 lc1^2 + m2 (l1^2 + lc2^2 + 2 l1 lc2 c2) + I1 + I2 = 3.5 + c2,
//   d2 = m2 (lc2^2 + l1 lc2 c2) + I2 = 1.25 + c2 / 2,
//   phi1 = -(1/2) w2^2 s2 - w2 w1 s2 + 14.7 s1 + phi2 = -(w2 s2)(w2 / 2 + w1) + 14.7 s1 + phi2,
//   dd2 = (torque + d2/d1 phi1 - (1/2) w1^2 s2 - phi2) / (1.25 - d2^2/d1), multiplied through by
//   d1: its denominator 1.25 d1 - d2^2 = 2.8125 - c2^2 / 4,
//   dd1 = -(d2 dd2 + phi1) / d1;
// both 1/d1 and 1/(2.8125 - c2^2/4) come from one reciprocal of their product, which lies in
// [6.4, 12.7] for every angle. The same dynamics as the reference term by term; each folded
// constant is exact, so only the rounding of the sums differs (the single-step gate is 1e-5).
// The reciprocal is the hardware approximation (rcp.approx, within one ulp): against a
// correctly rounded division it saves 5% of the T-step kernel's time at the same one-step
// error against the reference.
RLENV_D Acrobot acrobot_dsdt(const Acrobot& s, const AcrobotTrig& t, float torque) {
  const float d1 = 3.5f + t.c2;
  const float d2 = fmaf(0.5f, t.c2, 1.25f);
  const float phi2 = ac::PHI2_K * fmaf(t.s1, t.c2, t.c1 * t.s2);  // 4.9 sin(t1 + t2)
  const float phi1 = fmaf(-(s.dth2 * t.s2), fmaf(0.5f, s.dth2, s.dth1), fmaf(ac::PHI1_K, t.s1, phi2));
  const float num = fmaf(d1, fmaf(-0.5f * s.dth1, s.dth1 * t.s2, torque - phi2), d2 * phi1);
  const float den = fmaf(-0.25f * t.c2, t.c2, 2.8125f);
  const float r = rcp_hw(d1 * den);
  const float dd2 = num * (d1 * r);
  const float dd1 = -fmaf(d2, dd2, phi1) * (den * r);
  return Acrobot{s.dth1, s.dth2, dd1, dd2};
}

// Angle to [-pi, pi) (acrobot_np.py:87-89).
RLENV_D float wrap_angle(float x) { return wrap_to_pi(x); }

RLENV_D Acrobot acrobot_stage(const Acrobot& s, const Acrobot& k, float h) {
  return Acrobot{s.th1 + h * k.th1, s.th2 + h * k.th2, s.dth1 + h * k.dth1, s.dth2 + h * k.dth2};
}

// One RK4 step of dt 0.2, then wrap and clip (acrobot_np.py:47-61). t0 is the
// trig of s.
RLENV_D Acrobot acrobot_physics(const Acrobot& s, const AcrobotTrig& t0, float torque) {
  const Acrobot k1 = acrobot_dsdt(s, t0, torque);
  const Acrobot s2 = acrobot_stage(s, k1, ac::HALF_DT);
  const Acrobot k2 = acrobot_dsdt(s2, acrobot_stage_trig(s2), torque);
  const Acrobot s3 = acrobot_stage(s, k2, ac::HALF_DT);
  const Acrobot k3 = acrobot_dsdt(s3, acrobot_stage_trig(s3), torque);
  const Acrobot s4 = acrobot_stage(s, k3, ac::DT);
  const Acrobot k4 = acrobot_dsdt(s4, acrobot_stage_trig(s4), torque);
  Acrobot n;
  n.th1 = wrap_angle(s.th1 + ac::SIXTH_DT * (k1.th1 + 2.0f * k2.th1 + 2.0f * k3.th1 + k4.th1));
  n.th2 = wrap_angle(s.th2 + ac::SIXTH_DT * (k1.th2 + 2.0f * k2.th2 + 2.0f * k3.th2 + k4.th2));
  n.dth1 = fminf(fmaxf(s.dth1 + ac::SIXTH_DT * (k1.dth1 + 2.0f * k2.dth1 + 2.0f * k3.dth1 + k4.dth1),
                       -ac::MAX_VEL_1), ac::MAX_VEL_1);
  n.dth2 = fminf(fmaxf(s.dth2 + ac::SIXTH_DT * (k1.dth2 + 2.0f * k2.dth2 + 2.0f * k3.dth2 + k4.dth2),
                       -ac::MAX_VEL_2), ac::MAX_VEL_2);
  return n;
}

// The tip above height 1: -cos t1 - cos(t1 + t2) > 1 (acrobot_np.py:92-93),
// from the state's trig.
RLENV_D float acrobot_height(const AcrobotTrig& t) { return -t.c1 - (t.c1 * t.c2 - t.s1 * t.s2); }
RLENV_D bool acrobot_terminated(const AcrobotTrig& t) { return acrobot_height(t) > 1.0f; }

// A stepped state's trig and termination for the step kernels. The trig is acrobot_stage_trig's;
// the height it gives is within 4e-6 of the height from sincos_fast's values (each sine and
// cosine within 6e-7 of the other's, two products and a sum), so more than 1e-5 from the
// threshold the decision is the same, and closer than that the decision is taken from
// sincos_fast's values: termination is decided exactly as acrobot_terminated(acrobot_trig(s))
// decides it. The trig returned starts the next step (its first RK4 stage, weighted dt / 6).
RLENV_D bool acrobot_trig_terminated(const Acrobot& s, AcrobotTrig& t) {
  t = acrobot_stage_trig(s);
  const float h = acrobot_height(t);
  if (fabsf(h - 1.0f) < 1e-5f) return acrobot_terminated(acrobot_trig(s));
  return h > 1.0f;
}

}  // namespace rlenv
