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
// 1 / (Ann - mu Atn), which depend on the block only and so are computed once
// per substep; a sliding direction whose denominator is not positive has a
// zero reciprocal, so its normal impulse is zero (the reference's Painleve
// guard). BRANCHY skips the solve of an airborne contact with a branch (the
// variant of hopper_metal.py:110) instead of computing it and selecting zero.
struct ContactConsts {
  float inv_det, inv_dp, inv_dm;
};

RLENV_D ContactConsts contact_consts(float Att, float Atn, float Ann) {
  const float den_p = Ann + lg::MU * Atn, den_m = Ann - lg::MU * Atn;
  return ContactConsts{1.0f / (Att * Ann - Atn * Atn), den_p > 0.0f ? 1.0f / den_p : 0.0f,
                       den_m > 0.0f ? 1.0f / den_m : 0.0f};
}

template <bool BRANCHY>
RLENV_D void contact_impulse(float Att, float Atn, float Ann, const ContactConsts& k, float wt,
                             float wn, float depth, float& lt, float& ln) {
  const bool touching = depth >= 0.0f;
  if (BRANCHY && !touching) {
    lt = 0.0f;
    ln = 0.0f;
    return;
  }
  const float target = lg::BAUMGARTE_OVER_H * fmaxf(depth, 0.0f);
  const float gap = target - wn;
  const float ln_stick = (Att * gap + Atn * wt) * k.inv_det;
  const float lt_stick = (-Ann * wt - Atn * gap) * k.inv_det;
  const bool sticks = fabsf(lt_stick) <= lg::MU * ln_stick;
  const float ln_p = fmaxf(gap * k.inv_dp, 0.0f);
  const float ln_m = fmaxf(gap * k.inv_dm, 0.0f);
  const float slip_p = wt + (Att * lg::MU + Atn) * ln_p;
  const float sgn = slip_p <= 0.0f ? 1.0f : -1.0f;
  const float ln_slide = slip_p <= 0.0f ? ln_p : ln_m;
  const float lt_slide = (lg::MU * sgn) * ln_slide;
  const float l_n = sticks ? ln_stick : ln_slide;
  const float l_t = sticks ? lt_stick : lt_slide;
  const bool active = touching && l_n > 0.0f && wn < target;
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

template <int n>
RLENV_D void cholesky_packed(float (&Lm)[n * (n + 1) / 2], float (&inv_diag)[n]) {
#pragma unroll
  for (int i = 0; i < n; ++i) {
#pragma unroll
    for (int j = 0; j <= i; ++j) {
      float v = Lm[tri(i, j)];
#pragma unroll
      for (int p = 0; p < j; ++p) v -= Lm[tri(i, p)] * Lm[tri(j, p)];
      if (i == j) {
        const float d = sqrtf(v);
        Lm[tri(i, i)] = d;
        inv_diag[i] = 1.0f / d;
      } else {
        Lm[tri(i, j)] = v * inv_diag[j];
      }
    }
  }
}

// L y = b in place, for a b whose first LEAD entries are exactly zero (they
// stay zero and are skipped).
template <int n, int LEAD = 0>
RLENV_D void forward_solve(const float (&Lm)[n * (n + 1) / 2], const float (&inv_diag)[n],
                           float (&b)[n]) {
#pragma unroll
  for (int i = 0; i < n; ++i) {
    if (i < LEAD) {
      b[i] = 0.0f;
      continue;
    }
    float v = b[i];
#pragma unroll
    for (int p = LEAD; p < i; ++p) v -= Lm[tri(i, p)] * b[p];
    b[i] = v * inv_diag[i];
  }
}

// L^T x = y in place.
template <int n>
RLENV_D void back_solve(const float (&Lm)[n * (n + 1) / 2], const float (&inv_diag)[n],
                        float (&b)[n]) {
#pragma unroll
  for (int i = n - 1; i >= 0; --i) {
    float v = b[i];
#pragma unroll
    for (int p = i + 1; p < n; ++p) v -= Lm[tri(p, i)] * b[p];
    b[i] = v * inv_diag[i];
  }
}

template <int n>
RLENV_D void cholesky_solve(const float (&Lm)[n * (n + 1) / 2], const float (&inv_diag)[n],
                            float (&b)[n]) {
  forward_solve<n>(Lm, inv_diag, b);
  back_solve<n>(Lm, inv_diag, b);
}

// Dot product of two length-n vectors from index LEAD on.
template <int n, int LEAD = 0>
RLENV_D float dot_from(const float (&a)[n], const float (&b)[n]) {
  float s = 0.0f;
#pragma unroll
  for (int i = LEAD; i < n; ++i) s += a[i] * b[i];
  return s;
}

// One substep of H for C legs (legged_np.py:57-97), in place on q and v. With
// IMPULSES, each contact's final (lt, ln) of the substep is added to imp[2k],
// imp[2k + 1].
template <int C, bool BRANCHY, bool IMPULSES = false>
RLENV_D void legged_substep(float (&q)[3 + C], float (&v)[3 + C], const float (&tq)[C],
                            float assist, int iters, float* imp = nullptr) {
  constexpr int n = 3 + C;
  float lca[C], lsa[C], dx[C], dy[C], depth[C];
#pragma unroll
  for (int k = 0; k < C; ++k) {
    float sa, ca;
    sincosf(q[2] + q[3 + k], &sa, &ca);
    const float ad = v[2] + v[3 + k];
    lca[k] = lg::L * ca;
    lsa[k] = lg::L * sa;
    dx[k] = -lg::L * sa * ad * ad;  // foot acceleration at zero joint acceleration
    dy[k] = lg::L * ca * ad * ad;
    depth[k] = -(q[1] - lg::L * ca);
  }
  // mass matrix M = M_T diag(1,1,0..) + I_T e_phi e_phi^T + M_F sum_k J_k^T J_k,
  // lower triangle packed, and the generalised forces
  float Lm[n * (n + 1) / 2];
  float f[n];
#pragma unroll
  for (int i = 0; i < n; ++i) {
#pragma unroll
    for (int j = 0; j <= i; ++j) {
      float s = 0.0f;
#pragma unroll
      for (int k = 0; k < C; ++k) {
        const bool tt = jt_nz(k, i) && jt_nz(k, j);
        const bool nn = jn_nz(k, i) && jn_nz(k, j);
        if (tt && nn) s += jt_at(i, lca[k]) * jt_at(j, lca[k]) + jn_at(i, lsa[k]) * jn_at(j, lsa[k]);
        else if (tt) s += jt_at(i, lca[k]) * jt_at(j, lca[k]);
        else if (nn) s += jn_at(i, lsa[k]) * jn_at(j, lsa[k]);
      }
      const float base = (i == j) ? (i < 2 ? lg::M_T : (i == 2 ? lg::I_T : 0.0f)) : 0.0f;
      Lm[tri(i, j)] = base + lg::M_F * s;
    }
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

  float inv_diag[n];
  cholesky_packed<n>(Lm, inv_diag);
  cholesky_solve<n>(Lm, inv_diag, f);
  float vf[n];
#pragma unroll
  for (int i = 0; i < n; ++i) vf[i] = v[i] + lg::H * f[i];

  // W = L^-1 J^T, one column per contact row (the normal rows start with a zero),
  // so the Delassus matrix J M^-1 J^T = W^T W is a table of dot products. It is
  // symmetric: Att and Ann are kept as packed lower triangles over the contacts,
  // and the tangent-normal block in full (Ant[k][l] = Atn[l][k]).
  float att[C * (C + 1) / 2], ann[C * (C + 1) / 2], atn[C][C];
  {
    float Wt[C][n], Wn[C][n];
#pragma unroll
    for (int k = 0; k < C; ++k) {
#pragma unroll
      for (int i = 0; i < n; ++i) {
        Wt[k][i] = jt_nz(k, i) ? jt_at(i, lca[k]) : 0.0f;
        Wn[k][i] = jn_nz(k, i) ? jn_at(i, lsa[k]) : 0.0f;
      }
      forward_solve<n, 0>(Lm, inv_diag, Wt[k]);
      forward_solve<n, 1>(Lm, inv_diag, Wn[k]);
    }
#pragma unroll
    for (int k = 0; k < C; ++k) {
#pragma unroll
      for (int l = 0; l <= k; ++l) {
        att[tri(k, l)] = dot_from<n, 0>(Wt[k], Wt[l]);
        ann[tri(k, l)] = dot_from<n, 1>(Wn[k], Wn[l]);
      }
#pragma unroll
      for (int l = 0; l < C; ++l) atn[k][l] = dot_from<n, 1>(Wt[k], Wn[l]);
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
    cc[k] = contact_consts(att[tri(k, k)], atn[k][k], ann[tri(k, k)]);
  }
  // block projected Gauss-Seidel: each contact solved exactly given the others
  float lt[C], ln[C];
#pragma unroll
  for (int k = 0; k < C; ++k) {
    lt[k] = 0.0f;
    ln[k] = 0.0f;
  }
  for (int it = 0; it < iters; ++it) {
#pragma unroll
    for (int k = 0; k < C; ++k) {
      // the other contacts' contribution first, then the free velocity (legged_np.py:91-94)
      float st = 0.0f, sn = 0.0f;
#pragma unroll
      for (int l = 0; l < C; ++l) {
        if (l == k) continue;
        const int kl = k > l ? tri(k, l) : tri(l, k);
        st += att[kl] * lt[l] + atn[k][l] * ln[l];
        sn += atn[l][k] * lt[l] + ann[kl] * ln[l];
      }
      contact_impulse<BRANCHY>(att[tri(k, k)], atn[k][k], ann[tri(k, k)], cc[k], w0t[k] + st,
                               w0n[k] + sn, depth[k], lt[k], ln[k]);
    }
  }
  // v = v_free + M^-1 J^T lambda, one solve with the factor of M
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
  cholesky_solve<n>(Lm, inv_diag, r);
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
