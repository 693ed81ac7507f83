// Shared device helpers for every kernel of librlenv: the reset hash, the
// action loader, the Philox noise generator and the launch/status plumbing.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "rlenv.h"

#define RLENV_HD __host__ __device__ __forceinline__
#define RLENV_D __device__ __forceinline__

namespace rlenv {

constexpr int kThreads = 256;  // block size of the streaming step kernels

// ---------------------------------------------------------------------------
// Reset stream. The PCG hash of Jarzynski & Olano, "Hash Functions for GPU
// Rendering" (JCGT 9(3), 2020), applied to seed ^ (i * 0x9E3779B9) plus a
// per-row offset: the reference's in-kernel reset generator
// (cartpole_metal.py:40-51, 89-93; pendulum_metal.py:86-90). Keeping the same
// constants keeps the reset values of every environment equal to the
// reference kernel's.
RLENV_HD uint32_t pcg_hash(uint32_t v) {
  uint32_t s = v * 747796405u + 2891336453u;
  uint32_t w = ((s >> ((s >> 28u) + 4u)) ^ s) * 277803737u;
  return (w >> 22u) ^ w;
}

// The top 24 bits of a hash as a float in [-bound, bound). Every step before
// the final product is exact; the product is one correctly rounded multiply
// (__fmul_rn is never fused into a neighbouring add).
RLENV_D float uniform_pm(uint32_t h, float bound) {
  float t = float(h >> 8) * (1.0f / 16777216.0f) * 2.0f - 1.0f;
  return __fmul_rn(t, bound);
}

RLENV_D uint32_t env_hash(uint32_t seed, int64_t global_index) {
  return seed ^ (uint32_t(global_index) * 0x9E3779B9u);
}

constexpr uint32_t kRowStride = 0x85EBCA6Bu;  // per-row offset for the K-link, hopper and legged resets
// CartPole and Acrobot use four explicit offsets (cartpole_metal.py:90-93).
RLENV_D uint32_t classic_row_offset(int r) {
  return r == 0 ? 0u : r == 1 ? 0x85EBCA6Bu : r == 2 ? 0xC2B2AE35u : 0x27D4EB2Fu;
}

// ---------------------------------------------------------------------------
// Actions arrive as int32 (MLX randint), int64 (numpy, torch) or uint8.
template <typename A>
RLENV_D int load_action(const A* __restrict__ a, int64_t i) {
  return int(__ldg(a + i));
}
template <>
RLENV_D int load_action<int64_t>(const int64_t* __restrict__ a, int64_t i) {
  return int(__ldg(reinterpret_cast<const long long*>(a) + i));
}

// ---------------------------------------------------------------------------
// Philox-4x32-10 (Salmon, Moraes, Dror & Shaw, "Parallel random numbers: as
// easy as 1, 2, 3", SC 2011), written from the paper: ten rounds of two
// 32x32->64 multiplies with the published multipliers and Weyl key increments.
struct U4 {
  uint32_t x, y, z, w;
};

RLENV_HD U4 philox4x32_10(U4 c, uint32_t k0, uint32_t k1) {
  const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u;
  const uint32_t W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    uint64_t p0 = uint64_t(M0) * c.x;
    uint64_t p1 = uint64_t(M1) * c.z;
    U4 n;
    n.x = uint32_t(p1 >> 32) ^ c.y ^ k0;
    n.y = uint32_t(p1);
    n.z = uint32_t(p0 >> 32) ^ c.w ^ k1;
    n.w = uint32_t(p0);
    c = n;
    k0 += W0;
    k1 += W1;
  }
  return c;
}

// Four standard normals for block `blk` (parameters 4*blk .. 4*blk+3) of
// antithetic pair `pair` in generation `gen`: two Box-Muller transforms
// (Box & Muller 1958) of the four Philox words. u1 is in (0, 1], so the
// logarithm is finite.
RLENV_D void normal4(uint64_t seed, uint64_t gen, int64_t pair, int64_t blk, float out[4]) {
  U4 c{uint32_t(blk), uint32_t(pair), uint32_t(gen), uint32_t(gen >> 32)};
  U4 r = philox4x32_10(c, uint32_t(seed), uint32_t(seed >> 32) ^ uint32_t(uint64_t(pair) >> 32));
  const float inv24 = 1.0f / 16777216.0f;
  float u1a = float((r.x >> 8) + 1u) * inv24;  // (0, 1]
  float u2a = float(r.y >> 8) * inv24;          // [0, 1)
  float u1b = float((r.z >> 8) + 1u) * inv24;
  float u2b = float(r.w >> 8) * inv24;
  float ra = sqrtf(-2.0f * logf(u1a));
  float rb = sqrtf(-2.0f * logf(u1b));
  float sa, ca, sb, cb;
  sincospif(2.0f * u2a, &sa, &ca);
  sincospif(2.0f * u2b, &sb, &cb);
  out[0] = ra * ca;
  out[1] = ra * sa;
  out[2] = rb * cb;
  out[3] = rb * sb;
}

RLENV_D float noise_at(uint64_t seed, uint64_t gen, int64_t pair, int64_t j) {
  float v[4];
  normal4(seed, gen, pair, j >> 2, v);
  return v[j & 3];
}

// An unsigned key whose order is numpy's sort order of float32: every number
// by value (-0 and +0 equal), then NaN, every NaN equal. Negative numbers have
// their bits inverted, the rest get the sign bit set (the usual order-preserving
// map of IEEE floats to unsigned integers).
RLENV_D uint32_t rank_order_key(float f) {
  if (f != f) return 0xFFFFFFFFu;
  const uint32_t b = __float_as_uint(f == 0.0f ? 0.0f : f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// Centred rank of sorted position r among p members (es.py:214-215).
RLENV_D float centered_rank(int64_t r, int64_t p) { return float(r) / float(p - 1) - 0.5f; }

// x - 2 pi floor((x + pi) / 2 pi): an angle to [-pi, pi), bit for bit as that
// float32 expression (acrobot_np.py:87-89, pendulum_np.py:110-111). The quotient is
// formed by a multiply; it can fall on the other side of an integer than the
// division only within a few ulp of one, and there (or far outside the angles a
// step produces) the division decides. The floor of the quotient is the nearest
// integer to q - 1/2, formed by adding and subtracting 1.5 * 2^23 (two additions on the
// FMA pipe instead of a rounding instruction on the special function unit's pipe, which
// the Acrobot step keeps busy with its sines, cosines and reciprocals: 1% faster). It is
// floor(q) unless q is within rounding of an integer, and there the fraction r falls
// outside [2e-6, 1 - 2e-6] and the division decides as before; every float32 x with
// |x| <= 1e6 gives the same bits as with floorf (checked exhaustively on the host), and
// larger |x| takes the division.
RLENV_D float wrap_to_pi(float x) {
  constexpr float kPi = 3.141592653589793f, kTwoPi = 6.283185307179586f;
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
  const float y = x + kPi;
  const float q = y * (1.0f / kTwoPi);
  float f = __fsub_rn(__fadd_rn(__fsub_rn(q, 0.5f), kRound), kRound);
  const float r = q - f;
  if (r < 2e-6f || r > 1.0f - 2e-6f || fabsf(q) > 8.0f) f = floorf(y / kTwoPi);
  return x - kTwoPi * f;
}

// ---------------------------------------------------------------------------
// Sine and cosine of one angle, for the physics kernels (every angle a step
// forms is within a few tens of radians of zero).
// - Reduction by pi/2 after Cody & Waite (1980): k = rint(2x/pi) by the 1.5 * 2^23
//   rounding constant, whose low mantissa bits are then k mod 4; r = x - k pi/2 with
//   pi/2 in three float32 parts. With fused multiply-adds the first part's step is
//   exact, so r carries at most half an ulp of rounding.
// - sin r = r + r^3 P(r^2) and cos r = 1 + r^2 (-1/2 + r^2 Q(r^2)), P and Q quadratics
//   fitted for least maximum relative error on |r| <= 1.02 pi/4 (trig_coeffs.py
//   derives every constant below; a test checks they match).
// - Both results are within 1.6 ulp of the exact values for |x| <= 1024 (float32
//   numpy's own sin and cos are within 1.5). Beyond that, and for NaN and infinities,
//   sincosf answers.
namespace trig {
constexpr float kTwoOverPi = 6.3661975e-01f;
constexpr float kPio2Hi = 1.5707964e+00f;
constexpr float kPio2Mid = -4.371139e-08f;
constexpr float kPio2Lo = -1.7151245e-15f;
constexpr float kSin1 = -1.6666654e-01f;
constexpr float kSin2 = 8.332063e-03f;
constexpr float kSin3 = -1.9502117e-04f;
constexpr float kCos1 = 4.166664e-02f;
constexpr float kCos2 = -1.3887185e-03f;
constexpr float kCos3 = 2.441811e-05f;
constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
constexpr float kFastLimit = 1024.0f;
}  // namespace trig

// Where the rare branch finds sincosf. kShared: one out-of-line copy per kernel,
// the smaller code (on a B200 the Acrobot T-step kernel runs 5% faster with it).
// kInline: a copy at every call site, for kernels at a register limit (the call's
// preserved registers take the legged C = 4 kernel from 128 to 133 registers, and
// from four resident blocks per SM to three).
enum class TrigFar { kShared, kInline };

static __device__ __noinline__ float2 sincos_far(float x) {
  float2 sc;
  sincosf(x, &sc.x, &sc.y);
  return sc;
}

template <TrigFar kFar = TrigFar::kShared>
RLENV_D void sincos_fast(float x, float* s, float* c) {
  if (!(fabsf(x) <= trig::kFastLimit)) {
    if constexpr (kFar == TrigFar::kShared) {
      const float2 sc = sincos_far(x);
      *s = sc.x;
      *c = sc.y;
    } else {
      sincosf(x, s, c);
    }
    return;
  }
  const float j = fmaf(x, trig::kTwoOverPi, trig::kRound);
  const float k = j - trig::kRound;
  const uint32_t quadrant = __float_as_uint(j);
  float r = fmaf(-k, trig::kPio2Hi, x);
  r = fmaf(-k, trig::kPio2Mid, r);
  r = fmaf(-k, trig::kPio2Lo, r);
  const float r2 = r * r;
  const float ps = fmaf(fmaf(r2, trig::kSin3, trig::kSin2), r2, trig::kSin1);
  const float sr = fmaf(r * r2, ps, r);
  const float pc = fmaf(fmaf(r2, trig::kCos3, trig::kCos2), r2, trig::kCos1);
  const float cr = fmaf(r2, fmaf(r2, pc, -0.5f), 1.0f);
  const bool odd = quadrant & 1u;
  const float a = odd ? cr : sr, b = odd ? sr : cr;
  *s = __uint_as_float(__float_as_uint(a) ^ ((quadrant & 2u) << 30));
  *c = __uint_as_float(__float_as_uint(b) ^ (((quadrant + 1u) & 2u) << 30));
}

// Sine and cosine from the special function unit (__sinf, __cosf), after a reduction
// to [-pi, pi] by 2 pi in two float32 parts (k = rint(x / 2 pi) by the same rounding
// constant). CUDA documents both within 2^-21.41 absolute on [-pi, pi]; with the
// reduction, the worst measured on a B200 over |x| <= 1024 is 5.9e-7. About 8
// instructions against sincos_fast's 29, for intermediate values whose error the caller
// bounds: the Acrobot's RK4 stage derivatives. |x| < 2^22 keeps the reduction exact to
// 2^-48 relative; larger arguments give bounded but inaccurate results.
namespace trig {
constexpr float kInvTwoPi = 1.5915494e-01f;
constexpr float kTwoPiHi = 6.2831855e+00f;
constexpr float kTwoPiLo = -1.7484555e-07f;
}  // namespace trig

RLENV_D void sincos_sfu(float x, float* s, float* c) {
  const float k = fmaf(x, trig::kInvTwoPi, trig::kRound) - trig::kRound;
  float r = fmaf(-k, trig::kTwoPiHi, x);
  r = fmaf(-k, trig::kTwoPiLo, r);
  *s = __sinf(r);
  *c = __cosf(r);
}

// Sine and cosine from the special function unit on the argument as given, with no
// reduction. Beyond pi the unit reduces the argument itself after scaling it to revolutions,
// and its error grows with |x|: measured on a B200 over every float32 with |x| <= pi, 4, 8, 10
// and 16, at most 4.1e-7, 6.5e-7, 1.21e-6, 1.27e-6 and 2.27e-6 (sincos_sfu: 4.9e-7 over
// |x| <= 16).
RLENV_D void sincos_sfu_near(float x, float* s, float* c) {
  *s = __sinf(x);
  *c = __cosf(x);
}

RLENV_D float cos_fast(float x) {
  float s, c;
  sincos_fast(x, &s, &c);
  return c;
}

// Index of element (i, j), j <= i, of a lower triangle stored row by row.
RLENV_HD constexpr int tri(int i, int j) { return i * (i + 1) / 2 + j; }

// ---------------------------------------------------------------------------
inline int grid_for(int64_t threads, int block = kThreads) {
  int64_t g = (threads + block - 1) / block;
  return int(g < 1 ? 1 : g);
}

inline int launch_status() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? RLENV_OK : int(e);
}

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool valid_dtype(int dt) { return dt == RLENV_I32 || dt == RLENV_I64 || dt == RLENV_U8; }

// Call f with the action pointer typed by dtype; f receives a typed null
// pointer whose type selects the template instance.
template <typename F>
int with_action_type(int dtype, F&& f) {
  switch (dtype) {
    case RLENV_I32: return f(static_cast<const int32_t*>(nullptr));
    case RLENV_I64: return f(static_cast<const int64_t*>(nullptr));
    case RLENV_U8: return f(static_cast<const uint8_t*>(nullptr));
    default: return RLENV_EINVAL;
  }
}

}  // namespace rlenv

// ---- the check build -----------------------------------------------------------
// Compiled with -DRLENV_CHECKS (rlenv_build.build(checks=True), librlenv_checks.so), the
// kernels record what they find wrong in a device word instead of trapping: an action
// outside its body's range, a non-finite value in an output. Each translation unit has its
// own word and registers a host reader for it when the library loads; rlenv_checks_status
// (checks.cu) reads and clears all of them. In the normal build check_flag is empty.
namespace rlenv {
enum CheckBit : unsigned { kCheckActionRange = 1u, kCheckNonFinite = 2u };
}  // namespace rlenv
#ifdef RLENV_CHECKS
namespace rlenv {
static __device__ unsigned int g_check_word;
void register_check_reader(int (*reader)(unsigned int*, bool));
namespace {
int read_check_word(unsigned int* out, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(out, g_check_word, sizeof(unsigned int));
  if (e == cudaSuccess && clear && *out) {
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbol(g_check_word, &zero, sizeof(unsigned int));
  }
  return e == cudaSuccess ? RLENV_OK : int(e);
}
struct CheckReaderRegistration {
  CheckReaderRegistration() { register_check_reader(&read_check_word); }
};
CheckReaderRegistration g_check_reader_registration;
}  // namespace
RLENV_D void check_flag(bool bad, unsigned int bit) {
  if (bad) atomicOr(&g_check_word, bit);
}
}  // namespace rlenv
#else
namespace rlenv {
RLENV_D void check_flag(bool, unsigned int) {}
}  // namespace rlenv
#endif
