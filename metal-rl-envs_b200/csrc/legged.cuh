// Planar legged bodies with hard ground contacts (hopper_np.py, legged_np.py):
// a torso disk at the hip (x, y, phi) and C massless legs at relative angles
// psi_k, each with a point mass at its foot. C = 1 with one sweep is the
// hopper. One substep is semi-implicit Euler with exact single-contact
// impulses combined by block projected Gauss-Seidel over the feet.
//
// One substep is written once for a group of G lanes per body (G divides C): lane gl
// of the group owns contacts [gl C/G, (gl + 1) C/G) and the leg coordinates that go
// with them, and every lane holds the torso. The step kernels run G = 1; the ES rollout
// picks G per launch. Every floating-point operation below is one explicit operation
// (fmaf, __fmul_rn, __fadd_rn, __fsub_rn, the hardware reciprocal, the special function
// unit's sine and cosine), so the compiler cannot contract or reorder any of them
// differently in different kernels; sums over contacts follow one fixed pairwise tree,
// which a lane group evaluates from values exchanged through shared memory. Every G
// therefore gives the same bits, and the fused rollout steps a body exactly as the step
// kernel does.
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
constexpr float INV_D = 1.0f / (M_F * L * L);  // inverse mass of a leg coordinate
constexpr float INV_L2 = 1.0f / (L * L);
constexpr float INV_I_T = 1.0f / I_T;
}  // namespace lg

namespace lgx {
constexpr unsigned kFull = 0xffffffffu;
RLENV_D float mul(float a, float b) { return __fmul_rn(a, b); }
// Products with the leg length L and with 1 / L^2 (both 1 in the reference's model,
// legged_np.py:26): an explicit multiply by one is still an instruction, and a substep has
// about fifty of them at C = 4. Skipping them changes no bit.
RLENV_D float times_l(float x) {
  if constexpr (lg::L == 1.0f) return x;
  else return __fmul_rn(lg::L, x);
}
RLENV_D float times_inv_l2(float x) {
  if constexpr (lg::INV_L2 == 1.0f) return x;
  else return __fmul_rn(x, lg::INV_L2);
}
RLENV_D float add(float a, float b) { return __fadd_rn(a, b); }
RLENV_D float sub(float a, float b) { return __fsub_rn(a, b); }

// The hardware reciprocal (rcp.approx.ftz.f32, within one ulp; no denominator here is
// subnormal). The correctly rounded reciprocal is a multi-instruction sequence with a slow
// path, and a substep takes 13 of them at C = 4: on a B200 it made the legged step kernel
// 22% slower and the one-thread rollout 37% slower.
RLENV_D float rcp(float a) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(a));
  return r;
}

// Sum over the C contacts in one fixed pairwise order: ((x0 + x1) + (x2 + x3)) for C = 4,
// (x0 + x1) + x2 for C = 3.
template <int C>
RLENV_D float tree_sum(const float (&x)[C]) {
  if constexpr (C == 1) return x[0];
  else if constexpr (C == 2) return add(x[0], x[1]);
  else if constexpr (C == 3) return add(add(x[0], x[1]), x[2]);
  else return add(add(x[0], x[1]), add(x[2], x[3]));
}

// Shared-memory exchange area of one body's lane group (G > 1), in floats. Fields are C
// floats each (one per contact): 11 for the first exchange of a substep, 14 for the
// second, 5 for the third, 2 for the policy's leg coordinates, then H floats of hidden
// activations. The size is padded so that consecutive groups sit an odd number of 16-byte
// chunks apart, which keeps a warp's vector loads in distinct bank groups.
constexpr int kXch1 = 0, kXch1Fields = 11;
constexpr int kXch2 = 11, kXch2Fields = 14;
constexpr int kXch3 = 25, kXch3Fields = 5;
constexpr int kXchObs = 30;
template <int C, int H>
constexpr int xch_floats() {
  constexpr int n = 32 * C + H;
  constexpr int n4 = (n + 3) / 4 * 4;
  return (n4 / 4) % 2 ? n4 : n4 + 4;
}
template <int C>
constexpr int xch_hidden() {
  return 32 * C;
}

// Every contact's value of NF fields in every lane of the group; lane gl holds own[f][c]
// for its contacts gl C/G + c. With G > 1 each lane writes its values into the group's
// area x (field f at x + f C), and after __syncwarp reads each field's C values back with
// one vector load; all 32 lanes of the warp must call together. Each call site has its own
// fields, so an area is rewritten only after every lane has passed a later exchange, and
// with it a later __syncwarp.
template <int C, int G, int NF>
RLENV_D void contact_exchange(const float (&own)[NF][C / G], float (&all)[NF][C], float* x, int gl) {
  constexpr int CL = C / G;
  if constexpr (G == 1) {
#pragma unroll
    for (int f = 0; f < NF; ++f)
#pragma unroll
      for (int k = 0; k < C; ++k) all[f][k] = own[f][k];
  } else {
    static_assert(C == 2 || C == 4, "lane groups exchange two or four contacts");
#pragma unroll
    for (int f = 0; f < NF; ++f)
#pragma unroll
      for (int c = 0; c < CL; ++c) x[f * C + gl * CL + c] = own[f][c];
    __syncwarp();
#pragma unroll
    for (int f = 0; f < NF; ++f) {
      if constexpr (C == 4) {
        const float4 v = *reinterpret_cast<const float4*>(x + f * 4);
        all[f][0] = v.x;
        all[f][1] = v.y;
        all[f][2] = v.z;
        all[f][3] = v.w;
      } else {
        const float2 v = *reinterpret_cast<const float2*>(x + f * 2);
        all[f][0] = v.x;
        all[f][1] = v.y;
      }
    }
  }
}
}  // namespace lgx

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
  using namespace lgx;
  const float den_p = fmaf(lg::MU, Atn, Ann), den_m = fmaf(-lg::MU, Atn, Ann);
  return ContactConsts{rcp(fmaf(Att, Ann, -mul(Atn, Atn))), den_p > 0.0f ? rcp(den_p) : 0.0f,
                       den_m > 0.0f ? rcp(den_m) : 0.0f, fmaf(Att, lg::MU, Atn),
                       depth >= 0.0f ? mul(lg::BAUMGARTE_OVER_H, depth) : -INFINITY};
}

template <bool BRANCHY>
RLENV_D void contact_impulse(float Att, float Atn, float Ann, const ContactConsts& k, float wt,
                             float wn, float& lt, float& ln) {
  using namespace lgx;
  if (BRANCHY && k.target == -INFINITY) {
    lt = 0.0f;
    ln = 0.0f;
    return;
  }
  const float gap = sub(k.target, wn);
  const float ln_stick = mul(fmaf(Att, gap, mul(Atn, wt)), k.inv_det);
  const float lt_stick = mul(fmaf(-Ann, wt, -mul(Atn, gap)), k.inv_det);
  const bool sticks = fabsf(lt_stick) <= mul(lg::MU, ln_stick);
  const float ln_p = mul(gap, k.inv_dp);
  const float ln_m = mul(gap, k.inv_dm);
  const float slip_p = fmaf(k.slip, ln_p, wt);
  const float sgn = slip_p <= 0.0f ? 1.0f : -1.0f;
  const float ln_slide = slip_p <= 0.0f ? ln_p : ln_m;
  const float lt_slide = mul(lg::MU * sgn, ln_slide);
  const float l_n = sticks ? ln_stick : ln_slide;
  const float l_t = sticks ? lt_stick : lt_slide;
  const bool active = gap > 0.0f && l_n > 0.0f;
  ln = active ? l_n : 0.0f;
  lt = active ? l_t : 0.0f;
}

// One contact's Gauss-Seidel solve as affine functions of its coupling
// s = sum_{l != k} G[k][l] P_l (legged_substep): gap = g0 + lca s, and lt_stick,
// mu ln_stick, slip_p, P_stick, P_plus and P_minus each a + b s.
struct ContactAffine {
  float g0, lca, a_lt, b_lt, a_mln, b_mln, a_sl, b_sl, a_ps, b_ps, a_pp, b_pp, a_pm, b_pm;
};
static_assert(sizeof(ContactAffine) == lgx::kXch2Fields * sizeof(float), "one exchange field each");

RLENV_D ContactAffine contact_affine(float Att, float Atn, float Ann, const ContactConsts& k,
                                     float w0t, float w0n, float lca, float lsa) {
  using namespace lgx;
  const float g0 = sub(k.target, w0n);
  const float a_ln = mul(fmaf(Att, g0, mul(Atn, w0t)), k.inv_det);
  const float b_ln = mul(fmaf(Att, lca, mul(Atn, lsa)), k.inv_det);
  const float a_lt = mul(fmaf(-Ann, w0t, -mul(Atn, g0)), k.inv_det);
  const float b_lt = mul(fmaf(-Ann, lsa, -mul(Atn, lca)), k.inv_det);
  const float a_p = mul(g0, k.inv_dp), b_p = mul(lca, k.inv_dp);
  const float a_m = mul(g0, k.inv_dm), b_m = mul(lca, k.inv_dm);
  const float kp = fmaf(lg::MU, lsa, -lca), km = fmaf(-lg::MU, lsa, -lca);
  return ContactAffine{g0,
                       lca,
                       a_lt,
                       b_lt,
                       mul(lg::MU, a_ln),
                       mul(lg::MU, b_ln),
                       fmaf(k.slip, a_p, w0t),
                       fmaf(k.slip, b_p, lsa),
                       fmaf(lsa, a_lt, -mul(lca, a_ln)),
                       fmaf(lsa, b_lt, -mul(lca, b_ln)),
                       mul(kp, a_p),
                       mul(kp, b_p),
                       mul(km, a_m),
                       mul(km, b_m)};
}

// P_k of one solve at coupling s: seven multiply-adds side by side, three comparisons and
// three selects.
RLENV_D float contact_solve(const ContactAffine& a, float s) {
  const float gap = fmaf(a.lca, s, a.g0);
  const float lts = fmaf(a.b_lt, s, a.a_lt);
  const float mln = fmaf(a.b_mln, s, a.a_mln);
  const float slip = fmaf(a.b_sl, s, a.a_sl);
  const float ps = fmaf(a.b_ps, s, a.a_ps);
  const float pp = fmaf(a.b_pp, s, a.a_pp);
  const float pm = fmaf(a.b_pm, s, a.a_pm);
  const float slide = slip <= 0.0f ? pp : pm;
  const float pk = fabsf(lts) <= mln ? ps : slide;
  return gap > 0.0f ? pk : 0.0f;
}

// Gauss-Seidel sweeps over the contacts whose bit is set in `act` (every contact with
// kAll), in contact order, the P of every other contact zero throughout; sk receives each
// visited contact's coupling in the last sweep. A coupling adds the other contacts' terms
// least recently updated first, so that only its last multiply-add waits for the contact
// solved just before (legged_np.py:91-94).

template <int C, bool kAll, int kSweeps = 0>
RLENV_D void gauss_seidel(const ContactAffine (&af)[C], const float (&gkl)[C * (C - 1) / 2 + 1],
                          unsigned act, int sweeps, float (&sk)[C]) {
  float pl[C];
#pragma unroll
  for (int k = 0; k < C; ++k) pl[k] = 0.0f;
  auto sweep = [&]() {
#pragma unroll
    for (int k = 0; k < C; ++k) {
      if (!kAll && !(act & (1u << k))) continue;
      float s = 0.0f;
#pragma unroll
      for (int d = 1; d < C; ++d) {
        const int l = (k + d) % C;
        if (!kAll && !(act & (1u << l))) continue;
        s = fmaf(gkl[k > l ? tri(k - 1, l) : tri(l - 1, k)], pl[l], s);
      }
      pl[k] = contact_solve(af[k], s);
      sk[k] = s;
    }
  };
  if constexpr (kSweeps > 0) {
    // a sweep count known at compile time: the sweeps unrolled, the same operations in the same
    // order as the loop below
#pragma unroll
    for (int it = 0; it < kSweeps; ++it) sweep();
  } else {
    for (int it = 0; it < sweeps; ++it) sweep();
  }
}

// One substep of H for C legs (legged_np.py:57-97), in place on the torso (qt, vt: x, y,
// phi and their rates, held by every lane of the group) and this lane's legs (ql, vl: psi
// and its rate for contacts gl C/G ..). tq holds this lane's legs' torques. xch is the
// group's shared exchange area (unused for G = 1), gl the lane's index in its group. With
// IMPULSES, each own contact's final (lt, ln) of the substep is added to imp[2c],
// imp[2c + 1]. With SKIP (all 32 lanes of the warp call together), contacts that no lane
// with `alive` set touches are left out of the sweeps: their impulse is zero in every
// sweep, and a zero term changes no sum, so the results are the same; with one contact
// left, one sweep already gives the result of all of them.
template <int C, int G, bool BRANCHY, bool IMPULSES = false, bool SKIP = false, int kIters = 0>
RLENV_D void legged_substep(float (&qt)[3], float (&vt)[3], float (&ql)[C / G], float (&vl)[C / G],
                            const float (&tq)[C / G], float assist, int iters, float* xch = nullptr,
                            int gl = 0, bool alive = true, float* imp = nullptr) {
  using namespace lgx;
  static_assert(C % G == 0, "a lane owns whole contacts");
  constexpr int CL = C / G;
  // ---- foot kinematics of the own contacts. The leg angles' sine and cosine come from the
  // special function unit (sincos_sfu: within 6e-7 absolute after its 2 pi reduction,
  // against 1.6 ulp for sincos_fast, at about a third of the instructions).
  float lca[CL], lsa[CL];
  float e1[kXch1Fields][CL];  // this lane's share of the first exchange
  float fl[CL], depth[CL];
#pragma unroll
  for (int c = 0; c < CL; ++c) {
    float sa, ca;
    sincos_sfu(add(qt[2], ql[c]), &sa, &ca);
    const float ad = add(vt[2], vl[c]);
    const float ad2 = mul(ad, ad);
    lca[c] = times_l(ca);
    lsa[c] = times_l(sa);
    const float dx = -mul(lsa[c], ad2);  // foot acceleration at zero joint acceleration
    const float dy = mul(lca[c], ad2);
    depth[c] = sub(lca[c], qt[1]);
    // Jt . drift_x + Jn . drift_y on phi and on psi_k; the leg's generalised force
    const float t_dr = fmaf(lca[c], dx, mul(lsa[c], dy));
    fl[c] = add(fmaf(-lg::M_F, t_dr, -mul(lg::G, mul(lg::M_F, lsa[c]))), tq[c]);
    e1[0][c] = mul(lsa[c], lsa[c]);
    e1[1][c] = mul(lca[c], lca[c]);
    e1[2][c] = mul(lca[c], lsa[c]);
    e1[3][c] = dx;
    e1[4][c] = dy;
    e1[5][c] = t_dr;
    e1[6][c] = lsa[c];
    e1[7][c] = mul(times_inv_l2(lca[c]), fl[c]);
    e1[8][c] = mul(times_inv_l2(lsa[c]), fl[c]);
    e1[9][c] = fl[c];
    e1[10][c] = lca[c];
  }
  float a1[kXch1Fields][C];
  contact_exchange<C, G, kXch1Fields>(e1, a1, xch + kXch1 * C, gl);

  // ---- the mass matrix in closed form
  // M = diag(M_T, M_T, I_T, 0..) + M_F sum_k (Jt_k^T Jt_k + Jn_k^T Jn_k) (legged_np.py:67-72)
  // is an arrowhead matrix: each leg coordinate couples only to the torso (x, y, phi),
  // never to another leg, and its diagonal is M_F (lca^2 + lsa^2) = M_F L^2. Eliminating the
  // legs first leaves the torso's Schur complement
  //   S = [[M_T + (M_F/L^2) sum lsa^2, -(M_F/L^2) sum lca lsa, 0],
  //        [-(M_F/L^2) sum lca lsa, M_T + (M_F/L^2) sum lca^2, 0],
  //        [0, 0, I_T]]
  // (the phi row and column reduce exactly: a leg's own rotation carries the torso's), so
  // M x = b is solved by the 2x2 inverse of S's upper block and a few products per leg: no
  // Cholesky factor and no square roots. The solution is the reference's dense Cholesky
  // solution in exact arithmetic; in float32 it differs by rounding only.
  float s00, s01, s11;
  {
    constexpr float kScale = lg::M_F / (lg::L * lg::L);
    const float a = fmaf(kScale, tree_sum<C>(a1[0]), lg::M_T);
    const float d = fmaf(kScale, tree_sum<C>(a1[1]), lg::M_T);
    const float b = -mul(kScale, tree_sum<C>(a1[2]));
    const float inv_det = rcp(fmaf(a, d, -mul(b, b)));
    s00 = mul(d, inv_det);
    s01 = -mul(b, inv_det);
    s11 = mul(a, inv_det);
  }
  // x = M^-1 b for a torso part (b0, b1, b2) and this lane's leg part bl, given the sums over
  // contacts of (lca / L^2) bl, (lsa / L^2) bl and bl; bl becomes the leg part of x
  auto mass_solve = [&](float& b0, float& b1, float& b2, float (&bl)[CL], float su0, float su1,
                        float sbl) {
    const float r0 = sub(b0, su0), r1 = sub(b1, su1), r2 = sub(b2, sbl);
    const float x0 = fmaf(s00, r0, mul(s01, r1));
    const float x1 = fmaf(s01, r0, mul(s11, r1));
    const float x2 = mul(r2, lg::INV_I_T);
#pragma unroll
    for (int c = 0; c < CL; ++c)
      bl[c] = sub(sub(mul(bl[c], lg::INV_D), times_inv_l2(fmaf(lca[c], x0, mul(lsa[c], x1)))), x2);
    b0 = x0;
    b1 = x1;
    b2 = x2;
  };
  // ---- generalised forces (gravity on the torso and the feet, the feet's velocity-product
  // terms, the joint torques, the torso assist spring), then the free velocity v + H M^-1 f
  float f0 = -mul(lg::M_F, tree_sum<C>(a1[3]));
  float f1 = fmaf(-lg::M_F, tree_sum<C>(a1[4]), -mul(lg::G, fmaf(lg::M_F, float(C), lg::M_T)));
  float f2 = fmaf(-lg::M_F, tree_sum<C>(a1[5]), -mul(lg::G, mul(lg::M_F, tree_sum<C>(a1[6]))));
  f2 = sub(sub(f2, mul(assist, qt[2])), mul(mul(lg::ASSIST_DAMPING, assist), vt[2]));
  mass_solve(f0, f1, f2, fl, tree_sum<C>(a1[7]), tree_sum<C>(a1[8]), tree_sum<C>(a1[9]));
  const float vf0 = fmaf(lg::H, f0, vt[0]), vf1 = fmaf(lg::H, f1, vt[1]), vf2 = fmaf(lg::H, f2, vt[2]);
  float vfl[CL];
#pragma unroll
  for (int c = 0; c < CL; ++c) vfl[c] = fmaf(lg::H, fl[c], vl[c]);

  // ---- the Delassus matrix J M^-1 J^T in closed form: with g_k = (lsa_k, -lca_k) / L^2 and
  // G[k][l] = g_k . S^-1 g_l (S's upper block), the blocks of contacts k, l are
  //   Att = lsa_k lsa_l G + [k = l] lca_k^2 / D,  Atn = -lsa_k lca_l G + [k = l] lca_k lsa_k / D,
  //   Ann = lca_k lca_l G + [k = l] lsa_k^2 / D   (Atn[k][l] pairs k's tangent with l's normal).
  // Off the diagonal a block is rank one: contact l's impulse (lt_l, ln_l) adds
  // (lsa_k, -lca_k) G[k][l] P_l to contact k's relative velocity, where
  // P_l = lsa_l lt_l - lca_l ln_l. So the sweeps keep G below the diagonal (packed,
  // G[k][l] at tri(k - 1, l)), the running P_l and the diagonal blocks.
  auto g_of = [](float la, float ls, float& g0, float& g1) {
    g0 = times_inv_l2(ls);
    g1 = -times_inv_l2(la);
  };
  auto h_of = [&](float g0, float g1, float& h0, float& h1) {
    h0 = fmaf(s00, g0, mul(s01, g1));
    h1 = fmaf(s01, g0, mul(s11, g1));
  };
  float dtt[CL], dtn[CL], dnn[CL];
#pragma unroll
  for (int c = 0; c < CL; ++c) {
    float g0, g1, h0, h1;
    g_of(lca[c], lsa[c], g0, g1);
    h_of(g0, g1, h0, h1);
    const float gam = fmaf(g0, h0, mul(g1, h1));
    dtt[c] = fmaf(mul(lsa[c], lsa[c]), gam, mul(mul(lca[c], lca[c]), lg::INV_D));
    dtn[c] = fmaf(-mul(lsa[c], lca[c]), gam, mul(mul(lca[c], lsa[c]), lg::INV_D));
    dnn[c] = fmaf(mul(lca[c], lca[c]), gam, mul(mul(lsa[c], lsa[c]), lg::INV_D));
  }
  float gkl[C * (C - 1) / 2 + 1];
  if constexpr (C > 1) {
    float g0a[C], g1a[C], h0a[C], h1a[C];
#pragma unroll
    for (int k = 0; k < C; ++k) {
      g_of(a1[10][k], a1[6][k], g0a[k], g1a[k]);
      h_of(g0a[k], g1a[k], h0a[k], h1a[k]);
    }
#pragma unroll
    for (int k = 1; k < C; ++k)
#pragma unroll
      for (int l = 0; l < k; ++l) gkl[tri(k - 1, l)] = fmaf(g0a[k], h0a[l], mul(g1a[k], h1a[l]));
  }
  // ---- free relative velocities J_k v_free and the per-contact constants
  float w0t[CL], w0n[CL];
  ContactConsts cc[CL];
#pragma unroll
  for (int c = 0; c < CL; ++c) {
    w0t[c] = fmaf(lca[c], vfl[c], fmaf(lca[c], vf2, vf0));
    w0n[c] = fmaf(lsa[c], vfl[c], fmaf(lsa[c], vf2, vf1));
    cc[c] = contact_consts(dtt[c], dtn[c], dnn[c], depth[c]);
  }
  // ---- block projected Gauss-Seidel: each contact solved exactly given the others
  float lt[CL], ln[CL];
  if constexpr (C == 1) {
    // a single contact has no coupling: every sweep solves the same block
    contact_impulse<BRANCHY>(dtt[0], dtn[0], dnn[0], cc[0], w0t[0], w0n[0], lt[0], ln[0]);
  } else {
    // Contact k sees the others only through the scalar s_k = sum_{l != k} G[k][l] P_l:
    // (wt, wn) = (w0t + lsa s, w0n - lca s). Every quantity the exact block solve forms
    // from (wt, wn) is then affine in s, and so is P_k = lsa lt - lca ln in each regime
    // (stick, slide either way). The coefficients are formed once per substep, so a solve
    // in the sweep is
    //   P_k = gap > 0 ? (|lt_stick| <= mu ln_stick ? P_stick : (slip_p <= 0 ? P_plus : P_minus)) : 0.
    // A sliding direction with a zero reciprocal has zero coefficients (no impulse). The
    // exact solve's test ln > 0 is gap > 0 for a slide (ln = gap / den there), and for a
    // stick it follows from |lt| <= mu ln except at ln = 0, where P is zero either way. A
    // contact above the floor has gap = -infinity, so its P is zero whatever its
    // coefficients hold. The sweeps carry only P; each contact's final (lt, ln) is the
    // exact solve at its last coupling.
    ContactAffine af[C];
    {
      float e2[kXch2Fields][CL], a2[kXch2Fields][C];
#pragma unroll
      for (int c = 0; c < CL; ++c) {
        const ContactAffine o = contact_affine(dtt[c], dtn[c], dnn[c], cc[c], w0t[c], w0n[c], lca[c], lsa[c]);
#pragma unroll
        for (int f = 0; f < kXch2Fields; ++f) e2[f][c] = reinterpret_cast<const float*>(&o)[f];
      }
      contact_exchange<C, G, kXch2Fields>(e2, a2, xch + kXch2 * C, gl);
#pragma unroll
      for (int k = 0; k < C; ++k)
#pragma unroll
        for (int f = 0; f < kXch2Fields; ++f) reinterpret_cast<float*>(&af[k])[f] = a2[f][k];
    }
    float sk[C];
#pragma unroll
    for (int k = 0; k < C; ++k) sk[k] = 0.0f;
    constexpr unsigned kAllMask = (1u << C) - 1u;
    unsigned act = kAllMask;
    if constexpr (SKIP) {
      act = 0u;
#pragma unroll
      for (int k = 0; k < C; ++k)
        if (__any_sync(kFull, alive && af[k].g0 > -INFINITY)) act |= 1u << k;
    }
    if (act == kAllMask) gauss_seidel<C, true, kIters>(af, gkl, act, iters, sk);
    else if (act != 0u) gauss_seidel<C, false>(af, gkl, act, __popc(act) == 1 ? 1 : iters, sk);
#pragma unroll
    for (int c = 0; c < CL; ++c) {
      // the coupling of own contact gl CL + c in the last sweep
      float sc = sk[c];
      if constexpr (G > 1) {
#pragma unroll
        for (int k = 0; k < C; ++k) sc = k == gl * CL + c ? sk[k] : sc;
      }
      contact_impulse<BRANCHY>(dtt[c], dtn[c], dnn[c], cc[c], fmaf(lsa[c], sc, w0t[c]),
                               fmaf(-lca[c], sc, w0n[c]), lt[c], ln[c]);
    }
  }
  // ---- v = v_free + M^-1 J^T lambda: J^T lambda is (sum lt, sum ln, sum t2) on the torso and
  // t2 = lca lt + lsa ln on each leg
  float rl[CL], a3[kXch3Fields][C];
  {
    float e3[kXch3Fields][CL];
#pragma unroll
    for (int c = 0; c < CL; ++c) {
      rl[c] = fmaf(lca[c], lt[c], mul(lsa[c], ln[c]));
      e3[0][c] = lt[c];
      e3[1][c] = ln[c];
      e3[2][c] = rl[c];
      e3[3][c] = mul(times_inv_l2(lca[c]), rl[c]);
      e3[4][c] = mul(times_inv_l2(lsa[c]), rl[c]);
    }
    contact_exchange<C, G, kXch3Fields>(e3, a3, xch + kXch3 * C, gl);
  }
  float r0 = tree_sum<C>(a3[0]), r1 = tree_sum<C>(a3[1]), r2 = tree_sum<C>(a3[2]);
  mass_solve(r0, r1, r2, rl, tree_sum<C>(a3[3]), tree_sum<C>(a3[4]), tree_sum<C>(a3[2]));
  vt[0] = add(vf0, r0);
  vt[1] = add(vf1, r1);
  vt[2] = add(vf2, r2);
#pragma unroll
  for (int i = 0; i < 3; ++i) qt[i] = fmaf(lg::H, vt[i], qt[i]);
#pragma unroll
  for (int c = 0; c < CL; ++c) {
    vl[c] = add(vfl[c], rl[c]);
    ql[c] = fmaf(lg::H, vl[c], ql[c]);
  }
  if constexpr (IMPULSES) {
#pragma unroll
    for (int c = 0; c < CL; ++c) {
      imp[2 * c] = add(imp[2 * c], lt[c]);
      imp[2 * c + 1] = add(imp[2 * c + 1], ln[c]);
    }
  }
}

RLENV_D bool legged_terminated(const float (&qt)[3]) {
  return qt[1] < lg::FALL_HEIGHT || fabsf(qt[2]) > lg::FALL_ANGLE;
}

}  // namespace rlenv
