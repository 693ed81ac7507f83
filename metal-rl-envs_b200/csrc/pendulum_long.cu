// Articulated-body pendulum for long chains (pendulum_aba_np.py:30-132): one thread per
// environment, any K from 17 to kMaxLongLinks chosen at run time.
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
// reset. The last pass of a step's final stage also sums the termination height.
//
// Where the arrays live. Shared memory holds 227 KB per block, 8 K floats per environment:
// at K = 64 three one-warp blocks per SM, one of the four sub-partitions idle. Tensor memory
// (256 KB per SM, 128 lanes of 512 32-bit columns, each quarter of lanes reachable by the warps
// of one sub-partition) holds a whole environment of up to 64 links in one lane: eight columns
// per link. So for 32 <= K <= 64, when the batch fills the GPU, a block runs four
// tensor-memory warps, one per sub-partition, whose environments live in tensor memory, beside
// up to four shared-memory warps: at K = 64 seven warps per SM where shared memory alone fits
// three (mixed_shared_warps has the measured rule). A dependent tensor-memory load and wait
// takes about 6 cycles (measured on a B200). Both kernels run the same per-link arithmetic,
// written one explicit operation at a time, so an environment's results depend neither on the
// kind of warp that stepped it nor on the kernel its batch size chose.
#include <algorithm>

#include "pendulum_kernels.cuh"

namespace rlenv {
namespace pend {

constexpr int kLongBlock = 32;
constexpr int kLongArrays = 8;
constexpr int kMaxLongLinks = 192;  // 8 K floats x 32 threads within 227 KB of shared memory
enum LongArray { kTh = 0, kOm, kTs, kOs, kDth, kDom, kGu, kU1 };

constexpr int kTensorWarps = 4;        // one per sub-partition, each with its quarter of the lanes
constexpr int kTensorMaxLinks = 64;    // eight 32-bit columns per link in a lane's 512
constexpr int kTensorColumns = 512;
constexpr int kMaxSharedWarps = 4;     // beside the four tensor-memory warps
constexpr int kMixedMaxThreads = 32 * (kTensorWarps + kMaxSharedWarps);
constexpr int kMaxDynamicSmem = 227 * 1024;
// a block whose dynamic shared memory is above half the SM's 228 KB is the only one on its SM,
// so its allocation of all 512 tensor-memory columns never waits for another block's
constexpr int kOneBlockPerSmSmem = 115 * 1024;
// columns of link i's record in a tensor-memory lane: 8 i + field
enum TensorField { tTs = 0, tOs = 1, tTh = 2, tOm = 3, tGu = 4, tU1 = 5, tDth = 6, tDom = 7 };

size_t long_smem_bytes(int k) { return size_t(kLongArrays) * k * kLongBlock * sizeof(float); }

// The hardware reciprocal (within one ulp): on the inward pass's serial chain, where the
// correctly rounded division would add its slow-path sequence to every link.
RLENV_D float rcp_approx(float a) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(a));
  return r;
}

RLENV_D float mul(float a, float b) { return __fmul_rn(a, b); }
RLENV_D float add(float a, float b) { return __fadd_rn(a, b); }
RLENV_D float sub(float a, float b) { return __fsub_rn(a, b); }

// Link-major shared memory: the eight values of link i sit together, (link, array, thread), so a
// pass over the links advances one pointer and reaches every array at a fixed offset from it; the
// 32 threads of a warp touch 32 consecutive words (no bank conflicts).
struct LongLinks {
  float* base;  // link 0, array 0 of this thread
  int k;
  RLENV_D float& at(int a, int i) const { return base[(i * kLongArrays + a) * kLongBlock]; }
};

// A link's velocity: angular w, then linear (x, y) in the link's frame.
struct LinkVel {
  float w, x, y;
};

// The base acceleration carried outward in the last pass, in the same order.
struct LinkAcc {
  float w, x, y;
};

// What a subtree hands to its parent in the inward pass, in the rank-one form: its articulated
// inertia (I00, I01, I11) and bias (p0, p1) in the parent's frame.
struct Carry {
  float I00, I01, I11, p0, p1;
};

// The sine and cosine of a joint angle (the difference of two stage angles, or the root's stage
// angle), from the special function unit without a 2 pi reduction (sincos_sfu_near). Stage angles
// are wrapped angles plus at most dt times a clipped rate (0.63), so a joint angle lies within
// 2 pi + 1.3 < 8 of zero, where the unit is within 1.21e-6 of sin and cos; the accelerations
// enter the step weighted by dt / 6 and dt / 3.
RLENV_D void joint_sincos(float x, float* s, float* c) { sincos_sfu_near(x, s, c); }

// v_i = X_i v_{i-1} + S qd_i: the velocity of link i from its parent's, given the joint's sine,
// cosine and rate qd (the joint sits at (1, 0) of the parent).
RLENV_D void outward_link(float s, float c, float qd, LinkVel& v) {
  const float xy = add(v.y, v.w);
  const float nx = fmaf(c, v.x, mul(s, xy));
  const float ny = fmaf(-s, v.x, mul(c, xy));
  v.w = add(v.w, qd);
  v.x = nx;
  v.y = ny;
}

// The inward step of link i, stage angle and rate (th, om), parent's (pth, pom): the values the
// last pass needs (g = u / D, u1 = U1 / D), C carried to the parent, v walked back to the
// parent's velocity (x_{i-1} = c x_i - s y_i, y_{i-1} = s x_i + c y_i - w_{i-1}).
RLENV_D void inward_link(float th, float om, float pth, float pom, LinkVel& v, Carry& C, float& g,
                         float& u1) {
  const float qd = sub(om, pom);
  float s, c;
  joint_sincos(sub(th, pth), &s, &c);
  const float w = v.w, x = v.x, y = v.y;
  // own bias v x* (I v) of a unit mass at (1, 0): (x w, -w (w + y), x w)
  const float p0 = fmaf(x, w, C.p0);
  const float p1 = fmaf(-w, add(w, y), C.p1);
  const float a00 = add(1.0f, C.I00), a01 = C.I01, a11 = add(1.0f, C.I11);
  const float r = rcp_approx(a00);
  g = -mul(p0, r);
  u1 = mul(a01, r);
  const float m = fmaf(-a01, u1, a11);
  const float pa1 = fmaf(a01, g, fmaf(m, mul(qd, y), p1));
  const float ms = mul(m, s);
  C.I00 = mul(ms, s);
  C.I01 = mul(ms, c);
  C.I11 = mul(mul(m, c), c);
  C.p0 = mul(s, pa1);
  C.p1 = mul(c, pa1);
  const float pw = sub(w, qd);
  v.x = fmaf(c, x, -mul(s, y));
  v.y = sub(fmaf(s, x, mul(c, y)), pw);
  v.w = pw;
}

// The root's joint acceleration (gravity as a base acceleration -G; the root's own bias is zero,
// v_0 = (qd_0, 0, 0); U2 = U0), and the root link's acceleration in a.
RLENV_D float root_accel(float th0, float torque, const Carry& C, LinkAcc& a) {
  const float U0 = add(1.0f, C.I00), U1 = C.I01;
  float sn0, cs0;
  joint_sincos(th0, &sn0, &cs0);
  a.x = mul(cs0, -pd::G);
  a.y = mul(sn0, pd::G);
  const float qdd = mul(sub(sub(torque, C.p0), fmaf(U1, a.x, mul(U0, a.y))), rcp_approx(U0));
  a.w = qdd;
  return qdd;
}

// The last pass at link i >= 1: v walks this stage's velocities forward, a the accelerations;
// returns the joint acceleration q2 of link i.
RLENV_D float last_link(float th, float om, float pth, float pom, float gu, float u1, LinkVel& v,
                        LinkAcc& a) {
  const float qd = sub(om, pom);
  float s, c;
  joint_sincos(sub(th, pth), &s, &c);
  outward_link(s, c, qd, v);
  const float c1 = mul(qd, v.y), c2 = -mul(qd, v.x);
  const float xy = add(a.y, a.w);
  const float ap1 = add(fmaf(c, a.x, mul(s, xy)), c1);
  const float ap2 = add(fmaf(-s, a.x, mul(c, xy)), c2);
  const float q2 = sub(fmaf(-u1, ap1, sub(gu, a.w)), ap2);
  a.w = add(a.w, q2);
  a.x = ap1;
  a.y = ap2;
  return q2;
}

// pendulum_rk4's update of one link at stage `stage` (pendulum_np.py:60-66): from the state
// (th, om), the stage's rate om_in and acceleration acc, the sums (dth, dom) and the next stage's
// angle and rate (nth, nom); at stage 3 the next step's state, wrapped and clipped.
RLENV_D void stage_update(int stage, float th, float om, float om_in, float acc, float& dth, float& dom,
                          float& nth, float& nom) {
  switch (stage) {
    case 0:
      dth = om_in;
      dom = acc;
      nth = fmaf(pd::HALF_DT, om_in, th);
      nom = fmaf(pd::HALF_DT, acc, om);
      break;
    case 1:
    case 2: {
      const float h = stage == 1 ? pd::HALF_DT : pd::DT;
      dth = fmaf(2.0f, om_in, dth);
      dom = fmaf(2.0f, acc, dom);
      nth = fmaf(h, om_in, th);
      nom = fmaf(h, acc, om);
      break;
    }
    default:
      nth = pd_wrap(fmaf(pd::SIXTH_DT, add(dth, om_in), th));
      nom = fminf(fmaxf(fmaf(pd::SIXTH_DT, add(dom, acc), om), -pd::MAX_VEL), pd::MAX_VEL);
      break;
  }
}

// The tip above half the chain's length, -sum_j cos t_j > K / 2, is decided on cos_fast's terms
// (within 1.6 ulp). The special function unit's sum, hq, of the same wrapped angles (each term
// within 6.5e-7 of cos, measured on a B200 for |x| <= 4) is within K 1e-6 + K^2 2^-23 of it: the
// terms' errors, plus at most one ulp of a partial sum (|partial| <= K) per addition between the
// two sums' roundings. Outside twice that band of the threshold both decide alike; inside it the
// cos_fast sum decides.
RLENV_D float height_band(int k) {
  return 2.0f * (float(k) * 1e-6f + float(k) * float(k) * 1.1920929e-7f);
}

// What a launch hands every thread.
struct LongArgs {
  int k;
  const float* state;
  const void* actions;
  int dtype;
  uint32_t seed0;
  int64_t T, n, off;
  float* next;
  float* reward_seq;
  uint8_t* done_seq;
};

// ============================== shared-memory warps ==============================

// The last link's velocity for the angles and rates of arrays (ia, io).
RLENV_D LinkVel last_link_velocity(const LongLinks& L, int ia, int io) {
  LinkVel v{L.at(io, 0), 0.0f, 0.0f};
  float pth = L.at(ia, 0), pom = v.w;
#pragma unroll 4
  for (int i = 1; i < L.k; ++i) {
    const float th = L.at(ia, i), om = L.at(io, i);
    float s, c;
    joint_sincos(sub(th, pth), &s, &c);
    outward_link(s, c, sub(om, pom), v);
    pth = th;
    pom = om;
  }
  return v;
}

// One RK4 stage: accelerations of the stage whose angles and rates are arrays (ia, io) and
// whose last link's velocity is tip, applied at once as stage `stage`. Returns the last link's
// velocity of the state written (the next stage's, or with stage 3 the next step's), whose sum
// of cos theta_j over the links, from the special function unit, goes to height.
RLENV_D LinkVel aba_stage(const LongLinks& L, int ia, int io, float torque, int stage, LinkVel tip,
                          float& height) {
  const int k = L.k;
  Carry C{0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
  {
    LinkVel v = tip;
    float th = L.at(ia, k - 1), om = L.at(io, k - 1);
#pragma unroll 2
    for (int i = k - 1; i >= 1; --i) {
      const float pth = L.at(ia, i - 1), pom = L.at(io, i - 1);
      inward_link(th, om, pth, pom, v, C, L.at(kGu, i), L.at(kU1, i));
      th = pth;
      om = pom;
    }
  }
  LinkAcc a;
  const float th0 = L.at(ia, 0), om0 = L.at(io, 0);
  float run = root_accel(th0, torque, C, a);
  float nth, nom;
  stage_update(stage, L.at(kTh, 0), L.at(kOm, 0), om0, run, L.at(kDth, 0), L.at(kDom, 0), nth, nom);
  if (stage < 3) {
    L.at(kTs, 0) = nth;
    L.at(kOs, 0) = nom;
  } else {
    L.at(kTh, 0) = nth;
    L.at(kOm, 0) = nom;
  }
  LinkVel next{nom, 0.0f, 0.0f};  // the written state's link velocities, forward
  float hq = stage == 3 ? __cosf(nth) : 0.0f;
  float pth = th0, pom = om0, pnth = nth, pnom = nom;
  LinkVel v{om0, 0.0f, 0.0f};  // this stage's link velocities, forward again
#pragma unroll 4
  for (int i = 1; i < k; ++i) {
    const float th = L.at(ia, i), om = L.at(io, i);  // read before this link's update rewrites them
    const float q2 = last_link(th, om, pth, pom, L.at(kGu, i), L.at(kU1, i), v, a);
    run = add(run, q2);
    stage_update(stage, L.at(kTh, i), L.at(kOm, i), om, run, L.at(kDth, i), L.at(kDom, i), nth, nom);
    if (stage < 3) {
      L.at(kTs, i) = nth;
      L.at(kOs, i) = nom;
    } else {
      L.at(kTh, i) = nth;
      L.at(kOm, i) = nom;
    }
    float sn, cn;
    joint_sincos(sub(nth, pnth), &sn, &cn);
    outward_link(sn, cn, sub(nom, pnom), next);
    if (stage == 3) hq = add(hq, __cosf(nth));
    pth = th;
    pom = om;
    pnth = nth;
    pnom = nom;
  }
  height = hq;
  return next;
}

// T steps of environment e; step t reads actions[t * n + e], draws its resets from seed0 + t and
// writes reward_seq / done_seq row t when those are not null.
RLENV_D void run_shared(const LongLinks& L, const LongArgs& g, int64_t e) {
  const int k = g.k;
  const int64_t n = g.n;
  for (int j = 0; j < k; ++j) {
    L.at(kTh, j) = __ldg(g.state + j * n + e);
    L.at(kOm, j) = __ldg(g.state + (k + j) * n + e);
  }
  int act = g.T > 0 ? action_at(g.actions, g.dtype, e) : 0;
  const float half = float(k) * 0.5f, band = height_band(k);
  LinkVel tip = last_link_velocity(L, kTh, kOm);
  for (int64_t t = 0; t < g.T; ++t) {
    check_flag(act < 0 || act > 2, kCheckActionRange);
    const float torque = float(act - 1) * pd::TORQUE;
    if (t + 1 < g.T) act = action_at(g.actions, g.dtype, (t + 1) * n + e);
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
      const uint32_t hs = env_hash(g.seed0 + uint32_t(t), g.off + e);
      for (int j = 0; j < k; ++j) {
        L.at(kTh, j) = uniform_pm(pcg_hash(hs + uint32_t(j) * kRowStride), pd::RESET_BOUND);
        L.at(kOm, j) = uniform_pm(pcg_hash(hs + uint32_t(k + j) * kRowStride), pd::RESET_BOUND);
      }
      tip = last_link_velocity(L, kTh, kOm);
    }
    if (g.reward_seq) g.reward_seq[t * n + e] = d ? 0.0f : -1.0f;
    if (g.done_seq) g.done_seq[t * n + e] = d;
  }
  for (int j = 0; j < k; ++j) {
    check_flag(!(isfinite(L.at(kTh, j)) && isfinite(L.at(kOm, j))), kCheckNonFinite);
    g.next[j * n + e] = L.at(kTh, j);
    g.next[(k + j) * n + e] = L.at(kOm, j);
  }
}

// ============================== tensor-memory warps ==============================
// Every tcgen05 instruction below is warp-wide (.sync.aligned): all 32 lanes of a tensor-memory
// warp run the whole routine, lanes past the batch on zero state with nothing loaded from or
// stored to global memory, and a __syncwarp follows each stretch of code where lanes may take
// different branches (the wrap's exact division, resets, the height check, the check build's
// flags, the batch's tail) before the next tcgen05 instruction. Loads complete at
// tcgen05.wait::ld, which takes the loaded registers as operands so that no use of them is
// scheduled before it; stores complete at tcgen05.wait::st, which each pass issues before the
// next pass reads what it stored.

struct Pair {
  float a, b;
};
struct Record {
  float f[8];
};

RLENV_D Pair tm_ld2(uint32_t addr) {
  uint32_t r0, r1;
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x2.b32 {%0, %1}, [%2];"
               : "=r"(r0), "=r"(r1)
               : "r"(addr)
               : "memory");
  return Pair{__uint_as_float(r0), __uint_as_float(r1)};
}
RLENV_D void tm_wait(Pair& p) {
  asm volatile("tcgen05.wait::ld.sync.aligned;" : "+f"(p.a), "+f"(p.b)::"memory");
}
RLENV_D Record tm_ld8(uint32_t addr) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
                 "=r"(r[7])
               : "r"(addr)
               : "memory");
  Record out;
#pragma unroll
  for (int i = 0; i < 8; ++i) out.f[i] = __uint_as_float(r[i]);
  return out;
}
RLENV_D void tm_wait(Record& x) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+f"(x.f[0]), "+f"(x.f[1]), "+f"(x.f[2]), "+f"(x.f[3]), "+f"(x.f[4]), "+f"(x.f[5]),
                 "+f"(x.f[6]), "+f"(x.f[7])::"memory");
}
RLENV_D void tm_st2(uint32_t addr, float a, float b) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x2.b32 [%0], {%1, %2};" ::"r"(addr),
               "r"(__float_as_uint(a)), "r"(__float_as_uint(b))
               : "memory");
}
RLENV_D void tm_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

RLENV_D uint32_t tm_link(uint32_t lane_base, int i) { return lane_base + uint32_t(8 * i); }

// The last link's velocity for the angle and rate pair at field `in` of every record.
RLENV_D LinkVel tm_last_link_velocity(uint32_t tb, int k, int in) {
  Pair cur = tm_ld2(tm_link(tb, 0) + in);
  tm_wait(cur);
  LinkVel v{cur.b, 0.0f, 0.0f};
  Pair nxt = tm_ld2(tm_link(tb, 1) + in);
  for (int i = 1; i < k; ++i) {
    tm_wait(nxt);
    const Pair p = nxt;
    if (i + 1 < k) nxt = tm_ld2(tm_link(tb, i + 1) + in);
    float s, c;
    joint_sincos(sub(p.a, cur.a), &s, &c);
    outward_link(s, c, sub(p.b, cur.b), v);
    cur = p;
  }
  return v;
}

// aba_stage for a tensor-memory warp: the same arithmetic in the same order, each link's record
// loaded one link ahead of its use.
RLENV_D LinkVel tm_stage(uint32_t tb, int k, float torque, int stage, LinkVel tip, float& height) {
  const int in = stage == 0 ? tTh : tTs;  // field of the stage's angle and rate
  Carry C{0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
  {
    LinkVel v = tip;
    Pair cur = tm_ld2(tm_link(tb, k - 1) + in);
    tm_wait(cur);
    Pair nxt = tm_ld2(tm_link(tb, k - 2) + in);
#pragma unroll 2
    for (int i = k - 1; i >= 1; --i) {
      tm_wait(nxt);
      const Pair prev = nxt;
      if (i >= 2) nxt = tm_ld2(tm_link(tb, i - 2) + in);
      float g, u1;
      inward_link(cur.a, cur.b, prev.a, prev.b, v, C, g, u1);
      tm_st2(tm_link(tb, i) + tGu, g, u1);
      cur = prev;
    }
  }
  tm_wait_st();
  Record r = tm_ld8(tm_link(tb, 0));
  tm_wait(r);
  LinkAcc a;
  const float th0 = r.f[in], om0 = r.f[in + 1];
  float run = root_accel(th0, torque, C, a);
  float nth, nom, dth = r.f[tDth], dom = r.f[tDom];
  stage_update(stage, r.f[tTh], r.f[tOm], om0, run, dth, dom, nth, nom);
  if (stage < 3) {
    tm_st2(tm_link(tb, 0) + tTs, nth, nom);
    tm_st2(tm_link(tb, 0) + tDth, dth, dom);
  } else {
    __syncwarp();  // after the wrap
    tm_st2(tm_link(tb, 0) + tTh, nth, nom);
  }
  LinkVel next{nom, 0.0f, 0.0f};
  float hq = stage == 3 ? __cosf(nth) : 0.0f;
  float pth = th0, pom = om0, pnth = nth, pnom = nom;
  LinkVel v{om0, 0.0f, 0.0f};
  Record nx = tm_ld8(tm_link(tb, 1));
#pragma unroll 4  // as the shared-memory passes: +4% for the mixed kernel at K = 32 .. 64
  for (int i = 1; i < k; ++i) {
    tm_wait(nx);
    const Record cur = nx;
    if (i + 1 < k) nx = tm_ld8(tm_link(tb, i + 1));
    const float th = cur.f[in], om = cur.f[in + 1];
    const float q2 = last_link(th, om, pth, pom, cur.f[tGu], cur.f[tU1], v, a);
    run = add(run, q2);
    dth = cur.f[tDth];
    dom = cur.f[tDom];
    stage_update(stage, cur.f[tTh], cur.f[tOm], om, run, dth, dom, nth, nom);
    if (stage < 3) {
      tm_st2(tm_link(tb, i) + tTs, nth, nom);
      tm_st2(tm_link(tb, i) + tDth, dth, dom);
    } else {
      __syncwarp();  // after the wrap
      tm_st2(tm_link(tb, i) + tTh, nth, nom);
    }
    float sn, cn;
    joint_sincos(sub(nth, pnth), &sn, &cn);
    outward_link(sn, cn, sub(nom, pnom), next);
    if (stage == 3) hq = add(hq, __cosf(nth));
    pth = th;
    pom = om;
    pnth = nth;
    pnom = nom;
  }
  tm_wait_st();
  height = hq;
  return next;
}

// run_shared for a tensor-memory warp whose lane base address is tb; valid is false for lanes
// past the batch.
RLENV_D void run_tensor(uint32_t tb, const LongArgs& g, int64_t e, bool valid) {
  const int k = g.k;
  const int64_t n = g.n;
  for (int j = 0; j < k; ++j) {
    const float th = valid ? __ldg(g.state + j * n + e) : 0.0f;
    const float om = valid ? __ldg(g.state + (k + j) * n + e) : 0.0f;
    __syncwarp();
    tm_st2(tm_link(tb, j) + tTh, th, om);
  }
  tm_wait_st();
  int act = (g.T > 0 && valid) ? action_at(g.actions, g.dtype, e) : 1;
  const float half = float(k) * 0.5f, band = height_band(k);
  LinkVel tip = tm_last_link_velocity(tb, k, tTh);
  for (int64_t t = 0; t < g.T; ++t) {
    check_flag(act < 0 || act > 2, kCheckActionRange);
    const float torque = float(act - 1) * pd::TORQUE;
    if (t + 1 < g.T && valid) act = action_at(g.actions, g.dtype, (t + 1) * n + e);
    __syncwarp();
    float hq;
    tip = tm_stage(tb, k, torque, 0, tip, hq);
    tip = tm_stage(tb, k, torque, 1, tip, hq);
    tip = tm_stage(tb, k, torque, 2, tip, hq);
    tip = tm_stage(tb, k, torque, 3, tip, hq);
    const bool near = fabsf(-hq - half) <= band;
    bool d = -hq > half;
    if (__any_sync(0xffffffffu, near)) {
      float h = 0.0f;
      for (int j = 0; j < k; ++j) {
        __syncwarp();
        Pair p = tm_ld2(tm_link(tb, j) + tTh);
        tm_wait(p);
        h += cos_fast(p.a);
      }
      if (near) d = -h > half;
    }
    d = d && valid;
    if (__any_sync(0xffffffffu, d)) {
      const uint32_t hs = env_hash(g.seed0 + uint32_t(t), g.off + e);
      for (int j = 0; j < k; ++j) {
        Pair p = tm_ld2(tm_link(tb, j) + tTh);
        tm_wait(p);
        const float th = d ? uniform_pm(pcg_hash(hs + uint32_t(j) * kRowStride), pd::RESET_BOUND) : p.a;
        const float om = d ? uniform_pm(pcg_hash(hs + uint32_t(k + j) * kRowStride), pd::RESET_BOUND) : p.b;
        __syncwarp();
        tm_st2(tm_link(tb, j) + tTh, th, om);
      }
      tm_wait_st();
      const LinkVel fresh = tm_last_link_velocity(tb, k, tTh);
      if (d) tip = fresh;
    }
    if (valid) {
      if (g.reward_seq) g.reward_seq[t * n + e] = d ? 0.0f : -1.0f;
      if (g.done_seq) g.done_seq[t * n + e] = d;
    }
  }
  for (int j = 0; j < k; ++j) {
    __syncwarp();
    Pair p = tm_ld2(tm_link(tb, j) + tTh);
    tm_wait(p);
    if (valid) {
      check_flag(!(isfinite(p.a) && isfinite(p.b)), kCheckNonFinite);
      g.next[j * n + e] = p.a;
      g.next[(k + j) * n + e] = p.b;
    }
  }
}

// ============================== kernels ==============================

// Shared memory only (K > 64): one warp per block, as many blocks per SM as shared memory holds.
__global__ void __launch_bounds__(kLongBlock) pendulum_aba_long_kernel(LongArgs g) {
  extern __shared__ float links[];
  const int64_t e = int64_t(blockIdx.x) * kLongBlock + threadIdx.x;
  if (e >= g.n) return;
  run_shared(LongLinks{links + threadIdx.x, g.k}, g, e);
}

// K <= 64: warps 0-3 keep their environments in tensor memory (warp w reaches lanes 32 w ..
// 32 w + 31 of the block's 512 columns), warps 4 .. 4 + shared_warps - 1 in shared memory. The
// block is alone on its SM (at least kOneBlockPerSmSmem of dynamic shared memory), so warp 0's
// allocation of every column succeeds at once; every warp reaches the closing barrier, after
// which warp 0 frees the columns.
// (at least one block per SM: without the bound the compiler chose 48 registers and spilled)
__global__ void __launch_bounds__(kMixedMaxThreads, 1) pendulum_aba_mixed_kernel(LongArgs g, int shared_warps) {
  extern __shared__ float links[];
  __shared__ uint32_t tmem_base;
  const int warp = int(threadIdx.x) >> 5, lane = int(threadIdx.x) & 31;
  const int64_t e = int64_t(blockIdx.x) * (32 * (kTensorWarps + shared_warps)) + threadIdx.x;
  if (warp == 0) {
    const uint32_t slot = static_cast<uint32_t>(__cvta_generic_to_shared(&tmem_base));
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot),
                 "r"(kTensorColumns)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tb = tmem_base;
  if (warp < kTensorWarps) {
    run_tensor(tb + (uint32_t(32 * warp) << 16), g, e, e < g.n);
  } else if (e < g.n) {
    float* region = links + size_t(warp - kTensorWarps) * kLongArrays * g.k * kLongBlock;
    run_shared(LongLinks{region + lane, g.k}, g, e);
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (warp == 0) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tb), "r"(kTensorColumns)
                 : "memory");
  }
}

// Which kernel steps a batch of n, and with how many shared-memory warps beside the four
// tensor-memory ones (-1: the shared-memory kernel). Measured on a B200 (M env-steps/s, shared
// memory kernel against the best mixed block):
//   K = 64: N = 16,384  346 / 555 (0 shared warps), 65,536  535 / 836 (3), 262,144  514 / 771 (3)
//   K = 48: N = 65,536  889 / 1,127 (4), 262,144  899 / 1,161 (4)
//   K = 32: N = 65,536  1,574 / 1,696 (4), 262,144  1,707 / 1,765 (4)
//   K = 24: N = 65,536  2,542 / 2,259 (4), 262,144  2,730 / 2,646 (8)
//   K = 17: N = 262,144  4,428 / 3,764 (12); N = 4,096 or 16,384: the shared kernel at every K
// A tensor-memory warp alone runs about 15% slower than a shared-memory warp alone, so the mixed
// kernel pays where it needs fewer waves of blocks: from K = 32, where shared memory alone fits
// at most six warps per SM. More than four shared-memory warps put three warps on a
// sub-partition and lose; a count that is not a multiple of four leaves the block waiting on its
// busiest sub-partition. So at most four, the fewest that reach the fewest waves, and the mixed
// kernel only when that is fewer waves than the shared-memory kernel needs.
int mixed_shared_warps(int k, int64_t n, int sms) {
  if (k < 32 || k > kTensorMaxLinks) return -1;
  const int64_t per_warp = int64_t(kLongArrays) * k * kLongBlock * int64_t(sizeof(float));
  // one-warp blocks of the shared-memory kernel per SM (228 KB per SM, 1 KB reserved per block)
  const int64_t cap = std::min<int64_t>(32, (228 * 1024) / (per_warp + 1024));
  const int64_t warps = (n + 31) / 32;
  const int64_t shared_waves = (warps + sms * cap - 1) / (sms * cap);
  const int fit = int(std::min<int64_t>(kMaxSharedWarps, (kMaxDynamicSmem - 64) / per_warp));
  int best = -1;
  int64_t best_waves = shared_waves;
  for (int sw = 0; sw <= fit; ++sw) {
    const int64_t per_block = int64_t(32) * (kTensorWarps + sw);
    const int64_t waves = ((n + per_block - 1) / per_block + sms - 1) / sms;
    if (waves < best_waves) {
      best_waves = waves;
      best = sw;
    }
  }
  return best;
}

int launch_aba_long(int k, const float* state, const void* actions, int dtype, uint32_t seed0,
                    int64_t T, int64_t n, int64_t off, float* next, float* reward_seq,
                    uint8_t* done_seq, void* stream) {
  if (k < 2 || k > kMaxLongLinks) return RLENV_EUNSUPPORTED;
  if (n == 0) return RLENV_OK;
  const LongArgs g{k, state, actions, dtype, seed0, T, n, off, next, reward_seq, done_seq};
  int sw = -1;
  if (k <= kTensorMaxLinks) {
    int dev = 0, sms = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return int(e);
    sw = mixed_shared_warps(k, n, sms);
  }
  if (sw >= 0) {
    const size_t smem = std::max<size_t>(size_t(sw) * long_smem_bytes(k), size_t(kOneBlockPerSmSmem));
    cudaError_t e = cudaFuncSetAttribute(pendulum_aba_mixed_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(pendulum_aba_mixed_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                               int(cudaSharedmemCarveoutMaxShared));
    if (e != cudaSuccess) return int(e);
    const int64_t per_block = int64_t(32) * (kTensorWarps + sw);
    const int64_t blocks = (n + per_block - 1) / per_block;
    if (blocks > int64_t(0x7fffffff)) return RLENV_EINVAL;
    pendulum_aba_mixed_kernel<<<int(blocks), int(per_block), smem, as_stream(stream)>>>(g, sw);
    return launch_status();
  }
  const size_t smem = long_smem_bytes(k);
  cudaError_t e = cudaFuncSetAttribute(pendulum_aba_long_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(pendulum_aba_long_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                             int(cudaSharedmemCarveoutMaxShared));
  if (e != cudaSuccess) return int(e);
  const int64_t blocks = (n + kLongBlock - 1) / kLongBlock;
  if (blocks > int64_t(0x7fffffff)) return RLENV_EINVAL;
  pendulum_aba_long_kernel<<<int(blocks), kLongBlock, smem, as_stream(stream)>>>(g);
  return launch_status();
}

}  // namespace pend
}  // namespace rlenv
