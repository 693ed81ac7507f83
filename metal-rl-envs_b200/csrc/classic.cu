// CartPole and Acrobot: the single-step kernels that replace the reference's
// `cartpole_step` / `acrobot_step` Metal kernels, and T-step kernels that keep
// the state in registers across steps.
//
// Per environment-step the single-step kernels read 16 B of state and one
// action and write 16 B of state, a 4 B reward and a 1 B done flag; the T-step
// kernels move the state once per launch and per step only the action, reward
// and flag. CartPole threads own 4 consecutive environments (16-byte vector
// accesses) when N is a multiple of 4 and every buffer is 16-byte aligned;
// Acrobot, whose RK4 step is bound by instruction issue, owns one per thread.
#include <type_traits>

#include "classic.cuh"

namespace rlenv {
namespace {

// Each environment advances one state in place by one step: physics,
// termination, the masked reset from the hash stream, the reward. `Aux` is
// whatever the next step can reuse from this one (Acrobot: the sines and
// cosines of the stepped state, which its termination test computes and its
// next first RK4 stage needs). kVec is the number of consecutive environments
// a thread owns: 4 (16-byte accesses) where the step is light enough to be
// bound by memory, 1 where it is bound by instruction issue and the
// occupancy of one environment per thread hides latency better. kBlock is the
// block size and kMinBlocks the launch bound on resident blocks per SM.
struct CartPoleEnv {
  using S = CartPole;
  struct Aux {};
  static constexpr int kActions = 2;
  static constexpr int kVec = 4;
  // 128 threads: 131,072 environments make 1,024 blocks, 6.9 per SM, against 3.5 (so
  // 4 on some SMs, 3 on others) with 256 threads: 145 against 133 B env-steps/s on a B200
  static constexpr int kBlock = 128;
  static constexpr int kMinBlocks = 1;
  RLENV_D static S from(const float (&r)[4]) { return S{r[0], r[1], r[2], r[3]}; }
  RLENV_D static void to(const S& s, float (&r)[4]) {
    r[0] = s.x; r[1] = s.xd; r[2] = s.th; r[3] = s.thd;
  }
  RLENV_D static Aux aux(const S&) { return Aux{}; }
  RLENV_D static bool step(S& s, Aux&, int a, uint32_t h, float& reward) {
    const S nx = cartpole_physics(s, cartpole_force(a));
    const bool d = cartpole_terminated(nx);
    s.x = d ? uniform_pm(pcg_hash(h + classic_row_offset(0)), cp::RESET_BOUND) : nx.x;
    s.xd = d ? uniform_pm(pcg_hash(h + classic_row_offset(1)), cp::RESET_BOUND) : nx.xd;
    s.th = d ? uniform_pm(pcg_hash(h + classic_row_offset(2)), cp::RESET_BOUND) : nx.th;
    s.thd = d ? uniform_pm(pcg_hash(h + classic_row_offset(3)), cp::RESET_BOUND) : nx.thd;
    reward = 1.0f;
    return d;
  }
};

struct AcrobotEnv {
  using S = Acrobot;
  using Aux = AcrobotTrig;
  static constexpr int kActions = 3;
  static constexpr int kVec = 1;
  // 8 resident blocks of 256 threads (at most 32 registers): the whole batch of a
  // 262,144-environment launch is resident at once instead of 1.15 waves
  static constexpr int kBlock = 256;
  static constexpr int kMinBlocks = 8;
  RLENV_D static S from(const float (&r)[4]) { return S{r[0], r[1], r[2], r[3]}; }
  RLENV_D static void to(const S& s, float (&r)[4]) {
    r[0] = s.th1; r[1] = s.th2; r[2] = s.dth1; r[3] = s.dth2;
  }
  RLENV_D static Aux aux(const S& s) { return acrobot_stage_trig(s); }
  RLENV_D static bool step(S& s, Aux& t, int a, uint32_t h, float& reward) {
    const S nx = acrobot_physics(s, t, float(a - 1));
    Aux tn;
    const bool d = acrobot_trig_terminated(nx, tn);
    if (d) {  // rare under random actions: the fresh state's trig only on this branch
      s = S{uniform_pm(pcg_hash(h + classic_row_offset(0)), ac::RESET_BOUND),
            uniform_pm(pcg_hash(h + classic_row_offset(1)), ac::RESET_BOUND),
            uniform_pm(pcg_hash(h + classic_row_offset(2)), ac::RESET_BOUND),
            uniform_pm(pcg_hash(h + classic_row_offset(3)), ac::RESET_BOUND)};
      t = acrobot_stage_trig(s);
    } else {
      s = nx;
      t = tn;
    }
    reward = d ? 0.0f : -1.0f;
    return d;
  }
};

// RLENV_U2: actions packed along time, four steps to a byte: byte (r, i) of the (ceil(T / 4), n)
// array holds environment i's actions of steps 4r .. 4r + 3, step 4r + u in bits 2u. Packed2 is
// its element type in the kernels. A thread reads one byte (four for four environments) per four
// steps and shifts two bits out per step.
struct Packed2 {
  uint8_t bits;
};
template <typename A>
constexpr bool kPacked = std::is_same_v<A, Packed2>;

// The packed bytes of V consecutive environments from byte offset `at` (four bytes in one
// 32-bit load for V = 4, whose offset is a multiple of four).
template <int V>
RLENV_D uint32_t load_packed(const Packed2* __restrict__ a, int64_t at) {
  const uint8_t* p = reinterpret_cast<const uint8_t*>(a) + at;
  if constexpr (V == 4) return __ldg(reinterpret_cast<const unsigned int*>(p));
  else return __ldg(p);
}

// Load V consecutive actions starting at element `i` (i is a multiple of V).
template <typename A, int V>
RLENV_D void load_actions(const A* __restrict__ a, int64_t i, int (&out)[V]) {
#pragma unroll
  for (int u = 0; u < V; ++u) out[u] = load_action(a, i + u);
}
template <>
RLENV_D void load_actions<uint8_t, 4>(const uint8_t* __restrict__ a, int64_t i, int (&out)[4]) {
  uchar4 v = __ldg(reinterpret_cast<const uchar4*>(a + i));
  out[0] = v.x; out[1] = v.y; out[2] = v.z; out[3] = v.w;
}
template <>
RLENV_D void load_actions<int32_t, 4>(const int32_t* __restrict__ a, int64_t i, int (&out)[4]) {
  int4 v = __ldg(reinterpret_cast<const int4*>(a + i));
  out[0] = v.x; out[1] = v.y; out[2] = v.z; out[3] = v.w;
}

// State rows of V consecutive environments: st[r][u] is row r of env i + u.
template <int V>
RLENV_D void load_rows(const float* __restrict__ s, int64_t n, int64_t i, float (&st)[4][V]) {
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    if (V == 4) {
      float4 v = __ldg(reinterpret_cast<const float4*>(s + r * n + i));
      st[r][0] = v.x; st[r][1] = v.y; st[r][2] = v.z; st[r][V > 3 ? 3 : 0] = v.w;
    } else {
#pragma unroll
      for (int u = 0; u < V; ++u) st[r][u] = __ldg(s + r * n + i + u);
    }
  }
}

template <int V>
RLENV_D void store_rows(float* __restrict__ s, int64_t n, int64_t i, const float (&st)[4][V]) {
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    if (V == 4) {
      *reinterpret_cast<float4*>(s + r * n + i) =
          make_float4(st[r][0], st[r][1], st[r][2], st[r][V > 3 ? 3 : 0]);
    } else {
#pragma unroll
      for (int u = 0; u < V; ++u) s[r * n + i + u] = st[r][u];
    }
  }
}

template <int V>
RLENV_D void store_vec(float* __restrict__ p, int64_t i, const float (&x)[V]) {
  if (V == 4) *reinterpret_cast<float4*>(p + i) = make_float4(x[0], x[1], x[2], x[V > 3 ? 3 : 0]);
  else
#pragma unroll
    for (int u = 0; u < V; ++u) p[i + u] = x[u];
}

template <int V>
RLENV_D void store_flags(uint8_t* __restrict__ p, int64_t i, const bool (&d)[V]) {
  if (V == 4) *reinterpret_cast<uchar4*>(p + i) = make_uchar4(d[0], d[1], d[2], d[V > 3 ? 3 : 0]);
  else
#pragma unroll
    for (int u = 0; u < V; ++u) p[i + u] = d[u];
}

template <typename Env, int V>
RLENV_D void load_states(const float* __restrict__ s, int64_t n, int64_t i, typename Env::S (&st)[V]) {
  float rows[4][V];
  load_rows<V>(s, n, i, rows);
#pragma unroll
  for (int u = 0; u < V; ++u) {
    const float r[4] = {rows[0][u], rows[1][u], rows[2][u], rows[3][u]};
    st[u] = Env::from(r);
  }
}

template <typename Env, int V>
RLENV_D void store_states(float* __restrict__ s, int64_t n, int64_t i, const typename Env::S (&st)[V]) {
  float rows[4][V];
#pragma unroll
  for (int u = 0; u < V; ++u) {
    float r[4];
    Env::to(st[u], r);
#pragma unroll
    for (int k = 0; k < 4; ++k) rows[k][u] = r[k];
  }
  store_rows<V>(s, n, i, rows);
}

// SUMS selects the instance that also accumulates per-environment reward sums
// and termination counts; the plain chain keeps those registers free. SEQ says which
// per-step sequences are written: kSeqBoth (the loop then has no per-step test of their
// pointers: 3.5% of the Acrobot kernel's time on a B200), kSeqNone (no per-step row offset
// either: the sums-only Acrobot instance then fits 32 registers without spilling), or
// kSeqEither (either pointer may be null, tested per step).
constexpr int kSeqEither = 0, kSeqBoth = 1, kSeqNone = 2;
template <typename Env, typename A, int V, bool SUMS, int SEQ>
__global__ void __launch_bounds__(Env::kBlock, Env::kMinBlocks)
step_many_kernel(const float* __restrict__ state_in, const A* __restrict__ actions, uint32_t seed0,
                 int64_t T, int64_t n, int64_t off, float* __restrict__ state_out,
                 float* __restrict__ reward_seq, uint8_t* __restrict__ done_seq,
                 float* __restrict__ reward_sum, float* __restrict__ done_count) {
  const int64_t i = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) * V;
  if (i >= n) return;
  typename Env::S st[V];
  typename Env::Aux aux[V];
  load_states<Env, V>(state_in, n, i, st);
  float rsum[V], dcnt[V];
#pragma unroll
  for (int u = 0; u < V; ++u) {
    aux[u] = Env::aux(st[u]);
    rsum[u] = dcnt[u] = 0.0f;
  }
  // the next step's actions are loaded one step ahead, so their latency hides behind a step
  int act[V];
  // packed actions: the bytes of the current block of four steps (two bits shifted out per
  // step) and of the next block, loaded four steps ahead; pat is the offset of the block after
  [[maybe_unused]] uint32_t pcur = 0, pnxt = 0;
  [[maybe_unused]] int64_t pat = 0;
  if constexpr (kPacked<A>) {
    if (T > 0) pcur = load_packed<V>(actions, i);
    if (T > 4) pnxt = load_packed<V>(actions, n + i);
    pat = 2 * n + i;
  } else {
    if (T > 0) load_actions<A, V>(actions, i, act);
  }
  int64_t row = i;  // t * n + i, advanced by n per step
  for (int64_t t = 0; t < T; ++t, row += n) {
    int nxt[V] = {};
    if constexpr (kPacked<A>) {
#pragma unroll
      for (int u = 0; u < V; ++u) act[u] = int((pcur >> (8 * u)) & 3u);
      pcur = V == 1 ? pcur >> 2 : (pcur >> 2) & 0x3F3F3F3Fu;
      if ((t & 3) == 3) {
        pcur = pnxt;
        if (t + 5 < T) pnxt = load_packed<V>(actions, pat);
        pat += n;
      }
    } else {
      if (t + 1 < T) load_actions<A, V>(actions, row + n, nxt);
    }
    bool d[V];
    float rw[V];
#pragma unroll
    for (int u = 0; u < V; ++u) check_flag(act[u] < 0 || act[u] >= Env::kActions, kCheckActionRange);
#pragma unroll
    for (int u = 0; u < V; ++u)
      d[u] = Env::step(st[u], aux[u], act[u], env_hash(seed0 + uint32_t(t), off + i + u), rw[u]);
    if constexpr (!kPacked<A>) {
#pragma unroll
      for (int u = 0; u < V; ++u) act[u] = nxt[u];
    }
    if constexpr (SEQ == kSeqBoth) {
      store_vec<V>(reward_seq, row, rw);
      store_flags<V>(done_seq, row, d);
    } else if constexpr (SEQ == kSeqEither) {
      if (reward_seq) store_vec<V>(reward_seq, row, rw);
      if (done_seq) store_flags<V>(done_seq, row, d);
    }
    if constexpr (SUMS) {
#pragma unroll
      for (int u = 0; u < V; ++u) {
        rsum[u] += rw[u];
        dcnt[u] += d[u] ? 1.0f : 0.0f;
      }
    }
  }
#pragma unroll
  for (int u = 0; u < V; ++u) {
    float r[4];
    Env::to(st[u], r);
    check_flag(!(isfinite(r[0]) && isfinite(r[1]) && isfinite(r[2]) && isfinite(r[3])), kCheckNonFinite);
  }
  store_states<Env, V>(state_out, n, i, st);
  if constexpr (SUMS) {
    if (reward_sum) store_vec<V>(reward_sum, i, rsum);
    if (done_count) store_vec<V>(done_count, i, dcnt);
  }
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Four environments per thread (16-byte state accesses, one load of four actions) pay off
// only when the batch still fills the GPU at a quarter of the threads: from about 32
// resident warps per SM on the 148 SMs of a B200. Below that one environment per thread
// is faster (measured with T = 1,000 on a B200: at N = 131,072, 145 against 80 B
// env-steps/s; at N = 1,048,576, 188 against 201 B).
constexpr int64_t kVecMinEnvs = int64_t(4) * 32 * 32 * 148;

template <typename Env>
int launch_step_many(const float* state_in, const void* actions, int dtype, uint32_t seed0,
                     int64_t T, int64_t n, int64_t off, float* state_out, float* reward_seq,
                     uint8_t* done_seq, float* reward_sum, float* done_count, void* stream) {
  if (n < 0 || T < 0 || !(valid_dtype(dtype) || dtype == RLENV_U2)) return RLENV_EINVAL;
  if (n == 0) return RLENV_OK;
  if (!state_in || !state_out || (T > 0 && !actions)) return RLENV_EINVAL;
  const int esz = dtype == RLENV_I64 ? 8 : dtype == RLENV_I32 ? 4 : 1;
  const bool vec = Env::kVec == 4 && n >= kVecMinEnvs && (n % 4 == 0) && aligned16(state_in) &&
                   aligned16(state_out) &&
                   (!reward_seq || aligned16(reward_seq)) &&
                   (!done_seq || (reinterpret_cast<uintptr_t>(done_seq) & 3u) == 0) &&
                   (!reward_sum || aligned16(reward_sum)) && (!done_count || aligned16(done_count)) &&
                   (dtype == RLENV_I64 || (reinterpret_cast<uintptr_t>(actions) % (4 * esz)) == 0);
  cudaStream_t s = as_stream(stream);
  auto typed = [&](auto&& f) {
    return dtype == RLENV_U2 ? f(static_cast<const Packed2*>(nullptr)) : with_action_type(dtype, f);
  };
  return typed([&](auto tag) {
    using A = std::remove_const_t<std::remove_pointer_t<decltype(tag)>>;
    const A* a = static_cast<const A*>(actions);
    auto go = [&](auto sums, auto seq) {
      constexpr bool S = decltype(sums)::value;
      constexpr int Q = decltype(seq)::value;
      constexpr int B = Env::kBlock;
      if constexpr (Env::kVec == 4) {
        if (vec) {
          step_many_kernel<Env, A, 4, S, Q><<<grid_for(n / 4, B), B, 0, s>>>(
              state_in, a, seed0, T, n, off, state_out, reward_seq, done_seq, reward_sum, done_count);
          return launch_status();
        }
      }
      step_many_kernel<Env, A, 1, S, Q><<<grid_for(n, B), B, 0, s>>>(
          state_in, a, seed0, T, n, off, state_out, reward_seq, done_seq, reward_sum, done_count);
      return launch_status();
    };
    using Both = std::integral_constant<int, kSeqBoth>;
    using None = std::integral_constant<int, kSeqNone>;
    using Either = std::integral_constant<int, kSeqEither>;
    const bool sums = reward_sum || done_count;
    const int seq = reward_seq && done_seq ? kSeqBoth : !reward_seq && !done_seq ? kSeqNone : kSeqEither;
    auto with_seq = [&](auto s) {
      return seq == kSeqBoth ? go(s, Both{}) : seq == kSeqNone ? go(s, None{}) : go(s, Either{});
    };
    return sums ? with_seq(std::true_type{}) : with_seq(std::false_type{});
  });
}

// One step is the T-step kernel with T = 1, writing the step's reward and done
// flag as its one-row sequences: a chain of single-step calls and one T-step
// call then run the same machine code and agree bit for bit.
template <typename Env>
int launch_step(const float* state, const void* action, int dtype, uint32_t seed, int64_t n,
                int64_t off, float* next, float* reward, uint8_t* done, void* stream) {
  if (n > 0 && (!state || !action || !next || !reward || !done)) return RLENV_EINVAL;
  return launch_step_many<Env>(state, action, dtype, seed, 1, n, off, next, reward, done, nullptr,
                               nullptr, stream);
}

}  // namespace
}  // namespace rlenv

extern "C" {

int rlenv_cartpole_step(const float* state, const void* action, int action_dtype, uint32_t seed,
                        int64_t n, int64_t index_offset, float* next_state, float* reward,
                        uint8_t* done, void* stream) {
  return rlenv::launch_step<rlenv::CartPoleEnv>(state, action, action_dtype, seed, n, index_offset,
                                                next_state, reward, done, stream);
}

int rlenv_cartpole_step_many(const float* state_in, const void* actions, int action_dtype,
                             uint32_t seed0, int64_t steps, int64_t n, int64_t index_offset,
                             float* state_out, float* reward_seq, uint8_t* done_seq,
                             float* reward_sum, float* done_count, void* stream) {
  return rlenv::launch_step_many<rlenv::CartPoleEnv>(state_in, actions, action_dtype, seed0, steps,
                                                     n, index_offset, state_out, reward_seq,
                                                     done_seq, reward_sum, done_count, stream);
}

int rlenv_acrobot_step(const float* state, const void* action, int action_dtype, uint32_t seed,
                       int64_t n, int64_t index_offset, float* next_state, float* reward,
                       uint8_t* done, void* stream) {
  return rlenv::launch_step<rlenv::AcrobotEnv>(state, action, action_dtype, seed, n, index_offset,
                                               next_state, reward, done, stream);
}

int rlenv_acrobot_step_many(const float* state_in, const void* actions, int action_dtype,
                            uint32_t seed0, int64_t steps, int64_t n, int64_t index_offset,
                            float* state_out, float* reward_seq, uint8_t* done_seq,
                            float* reward_sum, float* done_count, void* stream) {
  return rlenv::launch_step_many<rlenv::AcrobotEnv>(state_in, actions, action_dtype, seed0, steps,
                                                    n, index_offset, state_out, reward_seq,
                                                    done_seq, reward_sum, done_count, stream);
}

}  // extern "C"
