// rlscan.cu -- C ABI entry points of librlscan.so (declared in include/rlscan.h).
//
// Host side: argument checks, kernel configuration and template dispatch.
// Nothing here allocates memory: outputs and the workspace are owned by the
// caller (the Python shim allocates them with torch, like the reference).
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "rlscan.h"
#include "scan_kernel.cuh"

using namespace rls;

namespace {

constexpr int kWarps = 4;
constexpr int64_t kMinTileElems = kWarps * 1 * 32 * 4;  // smallest tile of any launch

inline bool aligned16(const void* p) { return p == nullptr || ((uintptr_t)p & 15u) == 0; }

int env_rounds() {
  static int v = [] {
    const char* s = std::getenv("RLS_ROUNDS");
    if (!s) return 0;
    int r = std::atoi(s);
    return (r == 1 || r == 2 || r == 4) ? r : 0;
  }();
  return v;
}

// Rounds per warp: larger tiles for large inputs (fewer look-back hops, more
// bytes in flight per thread); small inputs keep enough CTAs to fill 148 SMs.
int pick_rounds(int64_t M, int vec, int max_rounds) {
  int r = env_rounds();
  if (!r) {
    const int64_t per_round_tile = (int64_t)kWarps * 32 * vec;
    const int64_t tiles_r2 = (M + 2 * per_round_tile - 1) / (2 * per_round_tile);
    const int64_t tiles_r4 = (M + 4 * per_round_tile - 1) / (4 * per_round_tile);
    if (tiles_r4 >= 8 * 148) r = 4;
    else if (tiles_r2 >= 2 * 148) r = 2;
    else r = 1;
  }
  if (r > max_rounds) r = max_rounds;
  return r;
}

template <class Alg, int R>
int launch_r(const typename Alg::Params& p, Geom g, void* ws, size_t ws_bytes, cudaStream_t s) {
  constexpr int64_t tile = (int64_t)kWarps * R * 32 * Alg::kVec;
  g.num_tiles = (g.M + tile - 1) / tile;
  if (g.num_tiles == 0) return RLS_OK;
  if (!ws || ws_bytes < ws_bytes_for_tiles(g.num_tiles)) return RLS_EWORKSPACE;
  if (g.num_tiles > 0x3fffffffLL) return RLS_EINVAL;
  const size_t smem = (size_t)g.smem_per_warp * kWarps;
  auto kern = scan_kernel<Alg, kWarps, R>;
  if (smem > 0) {
    // Opt in to more than the default 48 KB (dynamic + static) once per
    // instantiation and thread.
    static thread_local int configured = 0;
    if (!configured) {
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024) != cudaSuccess)
        return RLS_ECUDA;
      configured = 1;
    }
  }
  kern<<<(unsigned)g.num_tiles, kWarps * 32, smem, s>>>(p, g, ws);
  return cudaPeekAtLastError() == cudaSuccess ? RLS_OK : RLS_ECUDA;
}

template <class Alg, int MAXR = 4>
int launch(const typename Alg::Params& p, Geom g, void* ws, size_t ws_bytes, cudaStream_t s) {
  if (g.M == 0) return RLS_OK;
  const int r = pick_rounds(g.M, Alg::kVec, MAXR);
  if (r >= 4 && MAXR >= 4) return launch_r<Alg, (MAXR >= 4 ? 4 : 1)>(p, g, ws, ws_bytes, s);
  if (r >= 2 && MAXR >= 2) return launch_r<Alg, (MAXR >= 2 ? 2 : 1)>(p, g, ws, ws_bytes, s);
  return launch_r<Alg, 1>(p, g, ws, ws_bytes, s);
}

int make_geom(int64_t N, int64_t T, const rls_segment_t* seg, bool backward, Geom& g) {
  if (N < 0 || T < 0) return RLS_EINVAL;
  if (T > 0 && N > INT64_MAX / T) return RLS_EINVAL;
  g.M = N * T;
  g.S = T;
  g.N = N;
  g.num_tiles = 0;
  g.seg = 0;
  g.edge_global = 1;
  g.smem_per_warp = 0;
  g.tma = 0;
  if (seg) {
    if (seg->t0 < 0 || seg->total_len < seg->t0 + T) return RLS_EINVAL;
    g.seg = 1;
    g.edge_global = backward ? (seg->t0 + T == seg->total_len) : (seg->t0 == 0);
  }
  return RLS_OK;
}

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

bool valid_dtype(int d) { return d == RLS_F32 || d == RLS_BF16; }

}  // namespace

extern "C" {

size_t rls_workspace_bytes(int64_t num_elements) {
  if (num_elements <= 0) return 64;
  const int64_t tiles = (num_elements + kMinTileElems - 1) / kMinTileElems;
  return ws_bytes_for_tiles(tiles);
}

int rls_workspace_error(void* ws, void* stream) {
  if (!ws) return 0;
  unsigned h = 0;
  cudaStream_t s = as_stream(stream);
  if (cudaMemcpyAsync(&h, (char*)ws + offsetof(WsHeader, error), 4, cudaMemcpyDeviceToHost, s) != cudaSuccess)
    return -1;
  if (cudaStreamSynchronize(s) != cudaSuccess) return -1;
  if (h) {
    const unsigned z = 0;
    cudaMemcpyAsync((char*)ws + offsetof(WsHeader, error), &z, 4, cudaMemcpyHostToDevice, s);
    cudaStreamSynchronize(s);
  }
  return (int)h;
}

const char* rls_status_string(int status) {
  switch (status) {
    case RLS_OK: return "ok";
    case RLS_EINVAL: return "invalid argument";
    case RLS_EALIGN: return "pointer not 16-byte aligned";
    case RLS_EWORKSPACE: return "workspace missing or too small";
    case RLS_ECUDA: {
      static thread_local char buf[256];
      cudaError_t e = cudaGetLastError();
      std::snprintf(buf, sizeof(buf), "CUDA error: %s", cudaGetErrorString(e));
      return buf;
    }
    case RLS_EUNSUPPORTED: return "unsupported argument combination";
    default: return "unknown status";
  }
}

const char* rls_build_info(void) {
  return "librlscan: sm_100a affine scans (single-pass decoupled look-back, 4 warps/CTA, "
         "rounds 1/2/4, fp32 + bf16 inputs)";
}

// ---------------------------------------------------------------------------
int rls_gae(const void* rewards, const void* values, const void* terminateds, const void* truncateds,
            const void* bootstrap, int boot_kind, float* advantages, int64_t num_envs, int64_t seq_len,
            float gamma, float lambda_, int in_dtype, const rls_segment_t* seg, void* ws, size_t ws_bytes,
            void* stream) {
  if (num_envs == 0 || seq_len == 0) return (num_envs < 0 || seq_len < 0) ? RLS_EINVAL : RLS_OK;
  if (!rewards || !values || !terminateds || !advantages || !valid_dtype(in_dtype)) return RLS_EINVAL;
  if (boot_kind < RLS_BOOT_NONE || boot_kind > RLS_BOOT_FULL_SEL) return RLS_EINVAL;
  if ((boot_kind == RLS_BOOT_ROW || boot_kind == RLS_BOOT_LASTCOL) && !bootstrap) return RLS_EINVAL;
  if (seg && !seg->halo && seg->t0 + seq_len < seg->total_len) return RLS_EINVAL;
  if (!aligned16(rewards) || !aligned16(values) || !aligned16(terminateds) || !aligned16(truncateds) ||
      !aligned16(advantages) || (boot_kind >= RLS_BOOT_LASTCOL && !aligned16(bootstrap)))
    return RLS_EALIGN;
  Geom g;
  int st = make_geom(num_envs, seq_len, seg, true, g);
  if (st) return st;
  cudaStream_t s = as_stream(stream);
  const float gl = gamma * lambda_;
#define GAE_PARAMS(T)                                                                                     \
  typename GaeAlg<T>::Params p;                                                                           \
  p.r = (const T*)rewards; p.v = (const T*)values; p.term = (const T*)terminateds;                         \
  p.trunc = (const T*)truncateds;                                                                          \
  p.boot = boot_kind >= RLS_BOOT_LASTCOL ? (const T*)bootstrap : nullptr;                                  \
  p.boot_row = boot_kind == RLS_BOOT_ROW ? (const float*)bootstrap : nullptr;                              \
  p.halo = seg ? seg->halo : nullptr;                                                                      \
  p.out0 = advantages; p.out1 = nullptr; p.boot_kind = boot_kind; p.gamma = gamma; p.gl = gl;
  if (in_dtype == RLS_F32) {
    GAE_PARAMS(float)
    return launch<GaeAlg<float>>(p, g, ws, ws_bytes, s);
  } else {
    GAE_PARAMS(__nv_bfloat16)
    return launch<GaeAlg<__nv_bfloat16>, 2>(p, g, ws, ws_bytes, s);
  }
#undef GAE_PARAMS
}

int rls_vtrace(const void* log_pi_target, const void* log_pi_behavior, const void* values, const void* rewards,
               const void* terminateds, const void* truncateds, const void* bootstrap, int boot_kind,
               float* targets, float* advantages, int64_t num_envs, int64_t seq_len, float gamma, float rho_bar,
               float c_bar, int in_dtype, void* ws, size_t ws_bytes, void* stream) {
  if (num_envs == 0 || seq_len == 0) return (num_envs < 0 || seq_len < 0) ? RLS_EINVAL : RLS_OK;
  if (!log_pi_target || !log_pi_behavior || !values || !rewards || !terminateds || !targets || !advantages ||
      !valid_dtype(in_dtype))
    return RLS_EINVAL;
  if (boot_kind < RLS_BOOT_NONE || boot_kind > RLS_BOOT_FULL_ADD) return RLS_EINVAL;
  if ((boot_kind == RLS_BOOT_ROW || boot_kind == RLS_BOOT_LASTCOL) && !bootstrap) return RLS_EINVAL;
  if (!aligned16(log_pi_target) || !aligned16(log_pi_behavior) || !aligned16(values) || !aligned16(rewards) ||
      !aligned16(terminateds) || !aligned16(truncateds) || !aligned16(targets) || !aligned16(advantages) ||
      (boot_kind >= RLS_BOOT_LASTCOL && !aligned16(bootstrap)))
    return RLS_EALIGN;
  Geom g;
  int st = make_geom(num_envs, seq_len, nullptr, true, g);
  if (st) return st;
  cudaStream_t s = as_stream(stream);
#define VT_PARAMS(T)                                                                                      \
  typename VtraceAlg<T>::Params p;                                                                        \
  p.lpt = (const T*)log_pi_target; p.lpb = (const T*)log_pi_behavior; p.v = (const T*)values;              \
  p.r = (const T*)rewards; p.term = (const T*)terminateds; p.trunc = (const T*)truncateds;                 \
  p.boot = boot_kind >= RLS_BOOT_LASTCOL ? (const T*)bootstrap : nullptr;                                  \
  p.boot_row = boot_kind == RLS_BOOT_ROW ? (const float*)bootstrap : nullptr;                              \
  p.halo = nullptr; p.out0 = targets; p.out1 = advantages; p.boot_kind = boot_kind;                        \
  p.gamma = gamma; p.rho_bar = rho_bar; p.c_bar = c_bar;
  if (in_dtype == RLS_F32) {
    VT_PARAMS(float)
    return launch<VtraceAlg<float>, 2>(p, g, ws, ws_bytes, s);
  } else {
    VT_PARAMS(__nv_bfloat16)
    return launch<VtraceAlg<__nv_bfloat16>, 2>(p, g, ws, ws_bytes, s);
  }
#undef VT_PARAMS
}

int rls_retrace(const float* action_probs_target, const float* action_probs_behavior, const float* q_values,
                const float* next_q_values_all, const int64_t* actions, const float* rewards,
                const float* terminateds, const float* truncateds, float* targets, float* advantages,
                int64_t num_envs, int64_t seq_len, int64_t num_actions, float gamma, float lambda_, float c_bar,
                float rho_bar, void* ws, size_t ws_bytes, void* stream) {
  if (num_envs == 0 || seq_len == 0) return (num_envs < 0 || seq_len < 0) ? RLS_EINVAL : RLS_OK;
  if (!action_probs_target || !action_probs_behavior || !q_values || !next_q_values_all || !actions ||
      !rewards || !terminateds || !truncateds || !targets || !advantages || num_actions <= 0)
    return RLS_EINVAL;
  if (!aligned16(action_probs_target) || !aligned16(action_probs_behavior) || !aligned16(q_values) ||
      !aligned16(next_q_values_all) || !aligned16(actions) || !aligned16(rewards) || !aligned16(terminateds) ||
      !aligned16(truncateds) || !aligned16(targets) || !aligned16(advantages))
    return RLS_EALIGN;
  Geom g;
  int st = make_geom(num_envs, seq_len, nullptr, true, g);
  if (st) return st;
  cudaStream_t s = as_stream(stream);
  RetraceAlg::Params p;
  p.pi = action_probs_target; p.mu = action_probs_behavior; p.q = q_values; p.nq = next_q_values_all;
  p.act = actions; p.r = rewards; p.term = terminateds; p.trunc = truncateds;
  p.out0 = targets; p.out1 = advantages; p.A = num_actions;
  p.gamma = gamma; p.lam = lambda_; p.c_bar = c_bar; p.rho_bar = rho_bar;
  if (g.M == 0) return RLS_OK;
  // Staging: one warp span of pi and Qn rows plus actions, E and pi_a.
  int rounds = pick_rounds(g.M, 4, 2);
  auto per_warp = [&](int r) {
    const int64_t we = (int64_t)r * 128;
    int64_t b = we * (2 * num_actions + 2) * 4 + we * 8;
    return (b + 127) & ~(int64_t)127;
  };
  int64_t pw = per_warp(rounds);
  if (pw * kWarps > 160 * 1024 && rounds > 1) { rounds = 1; pw = per_warp(1); }
  const bool staged = num_actions <= 64 && pw * kWarps <= 160 * 1024;
  g.smem_per_warp = staged ? (int)pw : 0;
  g.tma = 1;
  p.warp_elems = rounds * 128;
  if (rounds == 2) return launch_r<RetraceAlg, 2>(p, g, ws, ws_bytes, s);
  return launch_r<RetraceAlg, 1>(p, g, ws, ws_bytes, s);
}

int rls_lambda_returns(const void* rewards, const void* next_values, const void* terminateds,
                       const void* truncateds, const void* bootstrap, int boot_kind, float* out, int64_t num_envs,
                       int64_t seq_len, float gamma, float lambda_, int in_dtype, const rls_segment_t* seg,
                       void* ws, size_t ws_bytes, void* stream) {
  if (num_envs == 0 || seq_len == 0) return (num_envs < 0 || seq_len < 0) ? RLS_EINVAL : RLS_OK;
  if (!rewards || !next_values || !terminateds || !out || !valid_dtype(in_dtype)) return RLS_EINVAL;
  if (!(boot_kind == RLS_BOOT_NONE || boot_kind == RLS_BOOT_LASTCOL || boot_kind == RLS_BOOT_FULL_ADD))
    return RLS_EINVAL;
  if ((boot_kind == RLS_BOOT_ROW || boot_kind == RLS_BOOT_LASTCOL) && !bootstrap) return RLS_EINVAL;
  if (!aligned16(rewards) || !aligned16(next_values) || !aligned16(terminateds) || !aligned16(truncateds) ||
      !aligned16(bootstrap) || !aligned16(out))
    return RLS_EALIGN;
  Geom g;
  int st = make_geom(num_envs, seq_len, seg, true, g);
  if (st) return st;
  cudaStream_t s = as_stream(stream);
#define LAM_PARAMS(T)                                                                                     \
  typename LambdaAlg<T>::Params p;                                                                        \
  p.r = (const T*)rewards; p.nv = (const T*)next_values; p.term = (const T*)terminateds;                   \
  p.trunc = (const T*)truncateds; p.boot = (const T*)bootstrap; p.out0 = out; p.out1 = nullptr;            \
  p.boot_kind = boot_kind; p.gamma = gamma; p.g1l = gamma * (1.0f - lambda_); p.gl = gamma * lambda_;
  if (in_dtype == RLS_F32) {
    LAM_PARAMS(float)
    return launch<LambdaAlg<float>>(p, g, ws, ws_bytes, s);
  } else {
    LAM_PARAMS(__nv_bfloat16)
    return launch<LambdaAlg<__nv_bfloat16>, 2>(p, g, ws, ws_bytes, s);
  }
#undef LAM_PARAMS
}

int rls_discounted_returns(const void* rewards, const void* terminateds, const void* truncateds,
                           const void* bootstrap, int boot_kind, float* out, int64_t num_envs, int64_t seq_len,
                           float gamma, int in_dtype, const rls_segment_t* seg, void* ws, size_t ws_bytes,
                           void* stream) {
  if (num_envs == 0 || seq_len == 0) return (num_envs < 0 || seq_len < 0) ? RLS_EINVAL : RLS_OK;
  if (!rewards || !terminateds || !out || !valid_dtype(in_dtype)) return RLS_EINVAL;
  if (!(boot_kind == RLS_BOOT_NONE || boot_kind == RLS_BOOT_LASTCOL || boot_kind == RLS_BOOT_FULL_ADD))
    return RLS_EINVAL;
  if ((boot_kind == RLS_BOOT_ROW || boot_kind == RLS_BOOT_LASTCOL) && !bootstrap) return RLS_EINVAL;
  if (!aligned16(rewards) || !aligned16(terminateds) || !aligned16(truncateds) || !aligned16(bootstrap) ||
      !aligned16(out))
    return RLS_EALIGN;
  Geom g;
  int st = make_geom(num_envs, seq_len, seg, true, g);
  if (st) return st;
  cudaStream_t s = as_stream(stream);
#define DISC_PARAMS(T)                                                                                    \
  typename DiscountedAlg<T>::Params p;                                                                    \
  p.r = (const T*)rewards; p.term = (const T*)terminateds; p.trunc = (const T*)truncateds;                 \
  p.boot = (const T*)bootstrap; p.out0 = out; p.out1 = nullptr; p.boot_kind = boot_kind; p.gamma = gamma;
  if (in_dtype == RLS_F32) {
    DISC_PARAMS(float)
    return launch<DiscountedAlg<float>>(p, g, ws, ws_bytes, s);
  } else {
    DISC_PARAMS(__nv_bfloat16)
    return launch<DiscountedAlg<__nv_bfloat16>, 2>(p, g, ws, ws_bytes, s);
  }
#undef DISC_PARAMS
}

static int forward_common(const void* x, const void* dones, const float* seed, float* out, int64_t num_envs,
                          int64_t seq_len, float k, int prev, int in_dtype, const rls_segment_t* seg, void* ws,
                          size_t ws_bytes, void* stream) {
  if (num_envs == 0 || seq_len == 0) return (num_envs < 0 || seq_len < 0) ? RLS_EINVAL : RLS_OK;
  if (!x || !dones || !out || !valid_dtype(in_dtype)) return RLS_EINVAL;
  if (seg && prev && seg->t0 > 0 && !seg->halo) return RLS_EINVAL;
  if (!aligned16(x) || !aligned16(dones) || !aligned16(out)) return RLS_EALIGN;
  Geom g;
  int st = make_geom(num_envs, seq_len, seg, false, g);
  if (st) return st;
  cudaStream_t s = as_stream(stream);
#define FWD_PARAMS(T)                                                                                     \
  typename ForwardAlg<T>::Params p;                                                                       \
  p.x = (const T*)x; p.done = (const T*)dones; p.seed = seed; p.halo = seg ? seg->halo : nullptr;          \
  p.out0 = out; p.out1 = nullptr; p.k = k; p.prev = prev;
  if (in_dtype == RLS_F32) {
    FWD_PARAMS(float)
    return launch<ForwardAlg<float>>(p, g, ws, ws_bytes, s);
  } else {
    FWD_PARAMS(__nv_bfloat16)
    return launch<ForwardAlg<__nv_bfloat16>, 2>(p, g, ws, ws_bytes, s);
  }
#undef FWD_PARAMS
}

int rls_eligibility_traces(const void* gradients, const void* dones, const float* seed_values, float* out,
                           int64_t num_envs, int64_t seq_len, float gamma, float lambda_, int in_dtype,
                           const rls_segment_t* seg, void* ws, size_t ws_bytes, void* stream) {
  return forward_common(gradients, dones, seed_values, out, num_envs, seq_len, gamma * lambda_, 1, in_dtype, seg,
                        ws, ws_bytes, stream);
}

int rls_prefix_sum(const void* inputs, const void* dones, const float* seed_values, int boundary_ends_at,
                   float* out, int64_t num_envs, int64_t seq_len, int in_dtype, const rls_segment_t* seg, void* ws,
                   size_t ws_bytes, void* stream) {
  return forward_common(inputs, dones, seed_values, out, num_envs, seq_len, 1.0f, boundary_ends_at ? 1 : 0,
                        in_dtype, seg, ws, ws_bytes, stream);
}

int rls_affine_scan(const float* u, const float* v, const float* carry, int direction, float* out,
                    int64_t num_envs, int64_t seq_len, const rls_segment_t* seg, void* ws, size_t ws_bytes,
                    void* stream) {
  if (num_envs == 0 || seq_len == 0) return (num_envs < 0 || seq_len < 0) ? RLS_EINVAL : RLS_OK;
  if (!u || !v || !out || (direction != 0 && direction != 1)) return RLS_EINVAL;
  if (!aligned16(u) || !aligned16(v) || !aligned16(out)) return RLS_EALIGN;
  Geom g;
  int st = make_geom(num_envs, seq_len, seg, direction == 0, g);
  if (st) return st;
  cudaStream_t s = as_stream(stream);
  if (direction == 0) {
    AffineAlg<true>::Params p{u, v, carry, out, nullptr};
    return launch<AffineAlg<true>>(p, g, ws, ws_bytes, s);
  }
  AffineAlg<false>::Params p{u, v, carry, out, nullptr};
  return launch<AffineAlg<false>>(p, g, ws, ws_bytes, s);
}

}  // extern "C"
