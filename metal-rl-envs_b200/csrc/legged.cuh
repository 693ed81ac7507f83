// Planar legged bodies with hard ground contacts (hopper_np.py, legged_np.py):
// a torso disk at the hip (x, y, phi) and C massless legs at relative angles
// psi_k, each with a point mass at its foot. C = 1 with one sweep is the
// hopper. One substep is semi-implicit Euler with exact single-contact
// impulses combined by block projected Gauss-Seidel over the feet.
#pragma once

#include "common.cuh"

namespace rlenv {
namespace lg {
constexpr float M_T = 1.0f;
constexpr float I_T = 0.1f;
constexpr float M_F = 0.2f;
constexpr float L = 1.0f;
constexpr float G = 9.8f;
constexpr float TORQUE = 2.0f;
constexpr float MU = 0.7f;
constexpr float H = 0.01f;
constexpr int SUBSTEPS = 4;
constexpr float BAUMGARTE_OVER_H = 20.0f;  // 0.2 / 0.01
constexpr float FALL_HEIGHT = 0.6f;
constexpr float FALL_ANGLE = 1.0f;
constexpr float RESET_BOUND = 0.05f;
constexpr float ASSIST_DAMPING = 0.1f;
}  // namespace lg

// Exact impulse (lt, ln) of one contact with Delassus block [[Att, Atn],
// [Atn, Ann]], free relative velocity (wt, wn) and penetration depth
// (hopper_np.py:80-109): inelastic normal with Baumgarte push-out, Coulomb
// friction (stick inside the cone, else slide on its edge), nothing for a
// contact above the floor, one that would pull, or one already separating.
// inv_det, inv_dp and inv_dm are 1 / det, 1 / (Ann + mu Atn) and
// 1 / (Ann - mu Atn), and slip is Att mu + Atn: they depend on the block only
// and so are computed once per substep. A sliding direction whose denominator is
// not positive has a zero reciprocal, so its normal impulse is zero (the
// reference's Painleve guard). target is the Baumgarte velocity
// (0.2 / H) max(depth, 0) of a touching foot and -infinity for one above the
// floor, so that "touching and wn < target" is one comparison. The reference
// clamps the sliding normal impulses at zero; here they are not clamped, which
// changes nothing: a result counts only when target - wn > 0, and then both are
// already non-negative. BRANCHY skips the solve of an airborne contact with a
// branch (the variant of hopper_metal.py:110) instead of computing it and
// selecting zero.
struct ContactConsts {
  float inv_det, inv_dp, inv_dm, slip, target;
};

RLENV_D ContactConsts contact_consts(float Att, float Atn, float Ann, float depth) {
  const float den_p = Ann + lg::MU * Atn, den_m = Ann - lg::MU * Atn;
  return ContactConsts{1.0f / (Att * Ann - Atn * Atn), den_p > 0.0f ? 1.0f / den_p : 0.0f,
                       den_m > 0.0f ? 1.0f / den_m : 0.0f, Att * lg::MU + Atn,
                       depth >= 0.0f ? lg::BAUMGARTE_OVER_H * depth : -INFINITY};
}

template <bool BRANCHY>
RLENV_D void contact_impulse(float Att, float Atn, float Ann, const ContactConsts& k, float wt,
                             float wn, float& lt, float& ln) {
  if (BRANCHY && k.target == -INFINITY) {
    lt = 0.0f;
    ln = 0.0f;
    return;
  }
  const float gap = k.target - wn;
  const float ln_stick = (Att * gap + Atn * wt) * k.inv_det;
  const float lt_stick = (-Ann * wt - Atn * gap) * k.inv_det;
  const bool sticks = fabsf(lt_stick) <= lg::MU * ln_stick;
  const float ln_p = gap * k.inv_dp;
  const float ln_m = gap * k.inv_dm;
  const float slip_p = wt + k.slip * ln_p;
  const float sgn = slip_p <= 0.0f ? 1.0f : -1.0f;
  const float ln_slide = slip_p <= 0.0f ? ln_p : ln_m;
  const float lt_slide = (lg::MU * sgn) * ln_slide;
  const float l_n = sticks ? ln_stick : ln_slide;
  const float l_t = sticks ? lt_stick : lt_slide;
  const bool active = gap > 0.0f && l_n > 0.0f;
  ln = active ? l_n : 0.0f;
  lt = active ? l_t : 0.0f;
}

// Non-zero pattern of foot k's Jacobian rows: the tangent row is
// (1, 0, L cos a, 0.., L cos a at 3+k, 0..), the normal row
// (0, 1, L sin a, 0.., L sin a at 3+k, 0..), a = phi + psi_k. After unrolling
// these tests are compile-time, so zero entries are skipped; skipping an
// exact zero leaves every product and sum unchanged.
RLENV_HD constexpr bool jt_nz(int k, int i) { return i == 0 || i == 2 || i == 3 + k; }
RLENV_HD constexpr bool jn_nz(int k, int i) { return i == 1 || i == 2 || i == 3 + k; }
RLENV_D float jt_at(int i, float lca) { return i == 0 ? 1.0f : lca; }
RLENV_D float jn_at(int i, float lsa) { return i == 1 ? 1.0f : lsa; }

// ---- the mass matrix in closed form ----------------------------------------
// M = diag(M_T, M_T, I_T, 0..) + M_F sum_k (Jt_k^T Jt_k + Jn_k^T Jn_k) (legged_np.py:67-72)
// is an arrowhead matrix: each leg coordinate 3+k couples only to the torso
// (x, y, phi), never to another leg, and its diagonal is D = M_F (lca^2 + lsa^2)
// = M_F L^2. Eliminating the legs first leaves the torso's Schur complement
//   S = [[M_T + (M_F/L^2) sum lsa^2, -(M_F/L^2) sum lca lsa, 0],
//        [-(M_F/L^2) sum lca lsa, M_T + (M_F/L^2) sum lca^2, 0],
//        [0, 0, I_T]]
// (the phi row and column reduce exactly: a leg's own rotation carries the
// torso's), so M x = b is solved by the 2x2 inverse of S's upper block and a
// few products per leg: no Cholesky factor and no square roots. The solution
// is the reference's dense Cholesky solution in exact arithmetic; in float32
// it differs by rounding only.
template <int C>
struct MassInverse {
  float lca[C], lsa[C];  // L cos a_k, L sin a_k of every foot
  float s00, s01, s11;   // inverse of S's upper 2x2 block
};

template <int C>
RLENV_D void mass_inverse_init(MassInverse<C>& m) {
  constexpr float kScale = lg::M_F / (lg::L * lg::L);
  float sss = 0.0f, scc = 0.0f, scs = 0.0f;
#pragma unroll
  for (int k = 0; k < C; ++k) {
    sss += m.lsa[k] * m.lsa[k];
    scc += m.lca[k] * m.lca[k];
    scs += m.lca[k] * m.lsa[k];
  }
  const float a = lg::M_T + kScale * sss, d = lg::M_T + kScale * scc, b = -kScale * scs;
  const float inv_det = 1.0f / (a * d - b * b);
  m.s00 = d * inv_det;
  m.s01 = -b * inv_det;
  m.s11 = a * inv_det;
}

// b <- M^-1 b.
template <int C>
RLENV_D void mass_solve(const MassInverse<C>& m, float (&b)[3 + C]) {
  constexpr float kInvD = 1.0f / (lg::M_F * lg::L * lg::L);
  constexpr float kInvL2 = 1.0f / (lg::L * lg::L);
  float r0 = b[0], r1 = b[1], r2 = b[2], t[C];
#pragma unroll
  for (int k = 0; k < C; ++k) {
    t[k] = b[3 + k] * kInvD;
    r0 -= (m.lca[k] * kInvL2) * b[3 + k];
    r1 -= (m.lsa[k] * kInvL2) * b[3 + k];
    r2 -= b[3 + k];
  }
  const float x0 = m.s00 * r0 + m.s01 * r1;
  const float x1 = m.s01 * r0 + m.s11 * r1;
  const float x2 = r2 * (1.0f / lg::I_T);
#pragma unroll
  for (int k = 0; k < C; ++k) b[3 + k] = t[k] - (m.lca[k] * x0 + m.lsa[k] * x1) * kInvL2 - x2;
  b[0] = x0;
  b[1] = x1;
  b[2] = x2;
}

// One substep of H for C legs (legged_np.py:57-97), in place on q and v. With
// IMPULSES, each contact's final (lt, ln) of the substep is added to imp[2k],
// imp[2k + 1].
template <int C, bool BRANCHY, bool IMPULSES = false>
RLENV_D void legged_substep(float (&q)[3 + C], float (&v)[3 + C], const float (&tq)[C],
                            float assist, int iters, float* imp = nullptr) {
  constexpr int n = 3 + C;
  MassInverse<C> mi;
  float dx[C], dy[C], depth[C];
#pragma unroll
  for (int k = 0; k < C; ++k) {
    float sa, ca;
    sincos_fast<TrigFar::kInline>(q[2] + q[3 + k], &sa, &ca);
    const float ad = v[2] + v[3 + k];
    mi.lca[k] = lg::L * ca;
    mi.lsa[k] = lg::L * sa;
    dx[k] = -lg::L * sa * ad * ad;  // foot acceleration at zero joint acceleration
    dy[k] = lg::L * ca * ad * ad;
    depth[k] = -(q[1] - lg::L * ca);
  }
  const float (&lca)[C] = mi.lca;
  const float (&lsa)[C] = mi.lsa;
  mass_inverse_init<C>(mi);
  // generalised forces, then the free velocity v + H M^-1 f
  float f[n];
#pragma unroll
  for (int i = 0; i < n; ++i) {
    float drift = 0.0f, jn_sum = 0.0f;
#pragma unroll
    for (int k = 0; k < C; ++k) {
      if (jt_nz(k, i) && jn_nz(k, i)) drift += jt_at(i, lca[k]) * dx[k] + jn_at(i, lsa[k]) * dy[k];
      else if (jt_nz(k, i)) drift += jt_at(i, lca[k]) * dx[k];
      else if (jn_nz(k, i)) drift += jn_at(i, lsa[k]) * dy[k];
      if (jn_nz(k, i)) jn_sum += jn_at(i, lsa[k]);
    }
    f[i] = -lg::M_F * drift - lg::G * (lg::M_F * jn_sum + (i == 1 ? lg::M_T : 0.0f));
    if (i >= 3) f[i] += tq[i - 3];
  }
  f[2] = f[2] - assist * q[2] - (lg::ASSIST_DAMPING * assist) * v[2];
  mass_solve<C>(mi, f);
  float vf[n];
#pragma unroll
  for (int i = 0; i < n; ++i) vf[i] = v[i] + lg::H * f[i];

  // Delassus matrix J M^-1 J^T in closed form: with g_k = (lsa_k, -lca_k) / L^2
  // and G[k][l] = g_k . S^-1 g_l (S's upper block), the blocks of contacts k, l are
  //   Att = lsa_k lsa_l G + [k = l] lca_k^2 / D,  Atn = -lsa_k lca_l G + [k = l] lca_k lsa_k / D,
  //   Ann = lca_k lca_l G + [k = l] lsa_k^2 / D   (Atn[k][l] pairs k's tangent with l's normal).
  // Off the diagonal a block is rank one: contact l's impulse (lt_l, ln_l) adds
  // (lsa_k, -lca_k) G[k][l] P_l to contact k's relative velocity, where
  // P_l = lsa_l lt_l - lca_l ln_l. So the sweeps keep G below the diagonal (packed,
  // G[k][l] at tri(k - 1, l)), the running P_l and the diagonal blocks.
  constexpr float kInvD = 1.0f / (lg::M_F * lg::L * lg::L);
  constexpr float kInvL2 = 1.0f / (lg::L * lg::L);
  float gkl[C * (C - 1) / 2 + 1];
  float dtt[C], dtn[C], dnn[C];
  {
    float h0[C], h1[C];  // S^-1 g_l
#pragma unroll
    for (int l = 0; l < C; ++l) {
      const float g0 = lsa[l] * kInvL2, g1 = -lca[l] * kInvL2;
      h0[l] = mi.s00 * g0 + mi.s01 * g1;
      h1[l] = mi.s01 * g0 + mi.s11 * g1;
    }
#pragma unroll
    for (int k = 0; k < C; ++k) {
      const float g0 = lsa[k] * kInvL2, g1 = -lca[k] * kInvL2;
#pragma unroll
      for (int l = 0; l <= k; ++l) {
        const float gam = g0 * h0[l] + g1 * h1[l];
        if (l < k) {
          gkl[tri(k - 1, l)] = gam;
        } else {
          dtt[k] = lsa[k] * lsa[k] * gam + lca[k] * lca[k] * kInvD;
          dtn[k] = -lsa[k] * lca[k] * gam + lca[k] * lsa[k] * kInvD;
          dnn[k] = lca[k] * lca[k] * gam + lsa[k] * lsa[k] * kInvD;
        }
      }
    }
  }
  // free relative velocities J_k v_free and the per-contact constants
  float w0t[C], w0n[C];
  ContactConsts cc[C];
#pragma unroll
  for (int k = 0; k < C; ++k) {
    float wt = 0.0f, wn = 0.0f;
#pragma unroll
    for (int i = 0; i < n; ++i) {
      if (jt_nz(k, i)) wt += jt_at(i, lca[k]) * vf[i];
      if (jn_nz(k, i)) wn += jn_at(i, lsa[k]) * vf[i];
    }
    w0t[k] = wt;
    w0n[k] = wn;
    cc[k] = contact_consts(dtt[k], dtn[k], dnn[k], depth[k]);
  }
  // block projected Gauss-Seidel: each contact solved exactly given the others
  float lt[C], ln[C], pl[C];
#pragma unroll
  for (int k = 0; k < C; ++k) {
    lt[k] = 0.0f;
    ln[k] = 0.0f;
    pl[k] = 0.0f;
  }
  for (int it = 0; it < iters; ++it) {
#pragma unroll
    for (int k = 0; k < C; ++k) {
      // the free velocity plus the other contacts' contribution (legged_np.py:91-94)
      float wt = w0t[k], wn = w0n[k];
      if constexpr (C > 1) {
        float sum = 0.0f;
#pragma unroll
        for (int l = 0; l < C; ++l) {
          if (l != k) sum += gkl[k > l ? tri(k - 1, l) : tri(l - 1, k)] * pl[l];
        }
        wt = fmaf(lsa[k], sum, wt);
        wn = fmaf(-lca[k], sum, wn);
      }
      contact_impulse<BRANCHY>(dtt[k], dtn[k], dnn[k], cc[k], wt, wn, lt[k], ln[k]);
      if constexpr (C > 1) pl[k] = lsa[k] * lt[k] - lca[k] * ln[k];
    }
  }
  // v = v_free + M^-1 J^T lambda
  float r[n];
#pragma unroll
  for (int i = 0; i < n; ++i) {
    float ri = 0.0f;
#pragma unroll
    for (int k = 0; k < C; ++k) {
      if (jt_nz(k, i)) ri += jt_at(i, lca[k]) * lt[k];
      if (jn_nz(k, i)) ri += jn_at(i, lsa[k]) * ln[k];
    }
    r[i] = ri;
  }
  mass_solve<C>(mi, r);
#pragma unroll
  for (int i = 0; i < n; ++i) {
    v[i] = vf[i] + r[i];
    q[i] += lg::H * v[i];
  }
  if constexpr (IMPULSES) {
#pragma unroll
    for (int k = 0; k < C; ++k) {
      imp[2 * k] += lt[k];
      imp[2 * k + 1] += ln[k];
    }
  }
}

template <int C>
RLENV_D bool legged_terminated(const float (&q)[3 + C]) {
  return q[1] < lg::FALL_HEIGHT || fabsf(q[2]) > lg::FALL_ANGLE;
}

}  // namespace rlenv
