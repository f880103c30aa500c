// ppo.cu -- fused epilogues of GAE for a PPO update (no kernel counterpart in
// the reference; src/rl_triton ROADMAP.md v0.2 lists "fused GAE + advantage
// normalisation" as future work).
//
// rls_gae_normalized: advantages normalised over the whole batch,
//   A = GAE, mean = sum(A)/M, std = sqrt(sum((A - mean)^2)/(M - 1)),
//   norm = (A - mean) / (std + eps)   (torch: (A - A.mean()) / (A.std() + eps)),
// plus, optionally, the value targets A + V and the raw advantages.
//
// Two passes, both launched with programmatic dependent launch so they overlap
// their neighbours' launch and tail: pass 1 is GAE (the row kernels' chunk
// walk) writing the advantages with ordinary stores -- at RL batch sizes they
// stay in the 126 MB L2 -- and one fp64 (sum, sum of squares) per CTA; pass 2
// reduces the CTA partials in a fixed order (every CTA gets the same mean and
// std) and writes the normalised advantages and the returns.  Rows that do not
// start 16-byte aligned take GAE, a statistics pass and a normalise pass.  All
// deterministic (no floating-point atomics).
#include <cmath>
#include <cstdint>
#include <mutex>

#include "rlscan.h"
#include "scan_kernel.cuh"
#include "tile_policies.cuh"
#include "rows2_kernel.cuh"
#include "host_shared.h"

using namespace rls;

namespace {

constexpr int kNormWarps = 8;
constexpr int kStatThreads = 256;

struct NormArgs {
  float* norm;          // [N, S] normalised advantages
  float* rets;          // [N, S] A + V, or null
  float* raw;           // [N, S] A, or null
  float* stats;         // fp32[2] (mean, std), or null
  const void* values;   // V, for the returns
  int bf16;
  double2* partials;    // per CTA (sum, sum of squares)
  unsigned* counter;    // CTAs done with pass 1 (the last one resets it)
  float* mean_den;      // pass 1's last CTA: {mean, std + eps}
  float eps;
};

__device__ __forceinline__ float load_value(const void* p, int bf16, int64_t i) {
  if (bf16) return bf16_bits_to_float(reinterpret_cast<const unsigned short*>(p)[i]);
  return reinterpret_cast<const float*>(p)[i];
}

// Walk one row from the window end (backward), chunk by chunk with the next
// chunk's loads in flight, handing each emitted vector to `sink(col, v)`.
// SINGLE: the row is one chunk (seq_len <= 32 x VEC): one buffer, no loop.
template <class P, bool SINGLE, class Sink>
__device__ __forceinline__ void walk_row(const typename P::Params& p, const Geom& g, int64_t row, int lane,
                                         Sink&& sink) {
  constexpr int VEC = Rows2Chunk<P, 1>::VEC;
  constexpr int64_t CH = 32 * VEC;
  const int64_t S = g.S, rbase = row * S;
  const int64_t nch = (S + CH - 1) / CH;
  auto cb_of = [&](int64_t k) { return (nch - 1 - k) * CH; };
  // Two named chunk buffers (an array indexed by k & 1 would live in local memory).
  Rows2Chunk<P, 1> a;
  typename P::Nbr edge_nbr{};
  float carry = 0.f;
  auto chunk = [&](int64_t k, const Rows2Chunk<P, 1>& ch) {
    ChunkScan<P, 1> cs;
    cs.col0[0] = cb_of(k) + lane * VEC;
    cs.row[0] = row;
    cs.i0[0] = rbase + cs.col0[0];
    cs.valid[0] = cs.col0[0] < S;
    cs.edge_v[0] = cs.valid[0] && (cs.col0[0] + VEC == S);
    edge_nbr = cs.pass1(p, g, lane, ch, edge_nbr);
    const int64_t col0 = cs.col0[0];
    carry = cs.pass2(p, g, ch, carry, [&](int, int q, float4 v0, float4) { sink(col0 + q, v0); });
  };
  rows2_load<P, 1>(p, rbase, S, cb_of(0), lane, a);
  if constexpr (SINGLE) {
    chunk(0, a);
  } else {
    Rows2Chunk<P, 1> b;
    for (int64_t k = 0; k < nch; k += 2) {
      if (k + 1 < nch) rows2_load<P, 1>(p, rbase, S, cb_of(k + 1), lane, b);
      chunk(k, a);
      if (k + 1 >= nch) break;
      if (k + 2 < nch) rows2_load<P, 1>(p, rbase, S, cb_of(k + 2), lane, a);
      chunk(k + 1, b);
    }
  }
}

// Block-wide fp64 sum of (a, b); every thread gets the result.  Fixed order.
template <int NT>
__device__ double2 block_sum2(double a, double b) {
  __shared__ double2 red[NT / 32];
#pragma unroll
  for (int d = 16; d >= 1; d >>= 1) {
    a += __shfl_xor_sync(0xffffffffu, a, d);
    b += __shfl_xor_sync(0xffffffffu, b, d);
  }
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = make_double2(a, b);
  __syncthreads();
  double2 t = make_double2(0.0, 0.0);
  for (int w = 0; w < NT / 32; ++w) {
    t.x += red[w].x;
    t.y += red[w].y;
  }
  return t;
}

// mean / (std + eps) from the partials, in a fixed order.
template <int NT>
__device__ void finish_stats(const double2* partials, int n, int64_t count, float eps, float* mean_f, float* den_f,
                             float* std_f) {
  double a = 0.0, b = 0.0;
  for (int i = threadIdx.x; i < n; i += NT) {
    const double2 v = __ldcg(partials + i);  // written by other CTAs: bypass L1
    a += v.x;
    b += v.y;
  }
  const double2 t = block_sum2<NT>(a, b);
  const double mean = t.x / (double)count;
  double var = count > 1 ? (t.y - t.x * mean) / (double)(count - 1) : 0.0;
  if (var < 0.0) var = 0.0;
  *mean_f = (float)mean;
  *std_f = (float)sqrt(var);
  *den_f = *std_f + eps;
}

// Pass 1 (one warp per row, rows strided over the grid): GAE into `tmp` with
// ordinary stores (at RL batch sizes the advantages stay in L2 for pass 2) and
// the per-CTA fp64 (sum, sum of squares).  Launched with programmatic stream
// serialization: it triggers its dependents at once and waits for its
// predecessor before its first store (and before its first load when an input
// may be the predecessor's output, Geom::pdl == 1).
template <class P, bool SINGLE>
__global__ void __launch_bounds__(kNormWarps * 32) gae_stats_kernel(const typename P::Params p, const Geom g,
                                                                     float* tmp, NormArgs na) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t S = g.S;
  const int64_t W = (int64_t)gridDim.x * kNormWarps;
  pdl_trigger();
  if (g.pdl == 1) pdl_wait();
  bool waited = g.pdl == 1;
  double s1 = 0.0, s2 = 0.0;
  for (int64_t row = (int64_t)blockIdx.x * kNormWarps + warp; row < g.N; row += W) {
    walk_row<P, SINGLE>(p, g, row, lane, [&](int64_t col, float4 v) {
      if (!waited) {
        pdl_wait();
        waited = true;
      }
      *reinterpret_cast<float4*>(tmp + row * S + col) = v;
      s1 += (double)v.x + (double)v.y + (double)v.z + (double)v.w;
      s2 += (double)v.x * v.x + (double)v.y * v.y + (double)v.z * v.z + (double)v.w * v.w;
    });
  }
  const double2 part = block_sum2<kNormWarps * 32>(s1, s2);
  pdl_wait();  // also in CTAs that stored nothing: the partials follow the predecessor
  // The last CTA to finish reduces the partials (fixed order) once for pass 2.
  __shared__ int s_last;
  if (threadIdx.x == 0) {
    na.partials[blockIdx.x] = part;
    __threadfence();
    s_last = atomicAdd(na.counter, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (s_last) {
    __threadfence();
    float m, d, sd;
    finish_stats<kNormWarps * 32>(na.partials, gridDim.x, g.M, na.eps, &m, &d, &sd);
    if (threadIdx.x == 0) {
      na.mean_den[0] = m;
      na.mean_den[1] = d;
      if (na.stats) {
        na.stats[0] = m;
        na.stats[1] = sd;
      }
      *na.counter = 0u;
    }
  }
}

// Pass 2: the normalised advantages and the returns, one float4 group per
// thread per step, from the mean and std pass 1's last CTA left.  `tmp` may be
// `norm` itself.  Waits for pass 1, then lets its own dependents start.
__global__ void __launch_bounds__(kStatThreads) norm_finish_kernel(const float* tmp, int64_t M, NormArgs na) {
  pdl_wait();
  pdl_trigger();
  const float mean = __ldcg(na.mean_den), den = __ldcg(na.mean_den + 1);
  const int64_t M4 = M / 4;  // rows are a multiple of 4 steps on this path
  const int64_t stride = (int64_t)gridDim.x * kStatThreads;
  for (int64_t gi = (int64_t)blockIdx.x * kStatThreads + threadIdx.x; gi < M4; gi += stride) {
    const int64_t i = gi * 4;
    const float4 a = __ldcs(reinterpret_cast<const float4*>(tmp + i));
    if (na.rets) {
      float4 v;
      if (na.bf16) {
        const uint2 u = __ldcs(reinterpret_cast<const uint2*>(reinterpret_cast<const unsigned short*>(na.values) + i));
        v = make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u), __uint_as_float(u.y << 16),
                        __uint_as_float(u.y & 0xffff0000u));
      } else {
        v = __ldcs(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(na.values) + i));
      }
      st_stream_f4(na.rets + i, make_float4(a.x + v.x, a.y + v.y, a.z + v.z, a.w + v.w));
    }
    st_stream_f4(na.norm + i, make_float4((a.x - mean) / den, (a.y - mean) / den, (a.z - mean) / den,
                                          (a.w - mean) / den));
  }
}

// ---- large batches: statistics, then normalise ---------------------------------
// Grid-stride over float4 groups, UNR groups per thread in flight per step so
// the whole GPU keeps enough bytes in flight; M % 4 == 0 for the vector part,
// the tail (< 4 elements) is handled by the first threads.
constexpr int kStatUnroll = 4;
__global__ void __launch_bounds__(kStatThreads) norm_stats_kernel(const float* adv, int64_t M, double2* partials) {
  double a = 0.0, b = 0.0;
  const int64_t M4 = M / 4;
  const float4* a4 = reinterpret_cast<const float4*>(adv);
  const int64_t stride = (int64_t)gridDim.x * kStatThreads;
  for (int64_t g0 = (int64_t)blockIdx.x * kStatThreads + threadIdx.x; g0 < M4; g0 += stride * kStatUnroll) {
    float4 v[kStatUnroll];
#pragma unroll
    for (int u = 0; u < kStatUnroll; ++u) {
      const int64_t gi = g0 + u * stride;
      v[u] = gi < M4 ? __ldcg(a4 + gi) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < kStatUnroll; ++u) {
      a += (double)v[u].x + (double)v[u].y + (double)v[u].z + (double)v[u].w;
      b += (double)v[u].x * v[u].x + (double)v[u].y * v[u].y + (double)v[u].z * v[u].z + (double)v[u].w * v[u].w;
    }
  }
  if (blockIdx.x == 0 && threadIdx.x < (unsigned)(M - M4 * 4)) {
    const float v = adv[M4 * 4 + threadIdx.x];
    a += v;
    b += (double)v * v;
  }
  const double2 t = block_sum2<kStatThreads>(a, b);
  if (threadIdx.x == 0) partials[blockIdx.x] = t;
}

__global__ void __launch_bounds__(kStatThreads) norm_apply_kernel(const float* adv, int64_t M, const double2* partials,
                                                                  int nparts, NormArgs na) {
  __shared__ float s_mean, s_den;
  {
    float m, d, sd;
    finish_stats<kStatThreads>(partials, nparts, M, na.eps, &m, &d, &sd);
    if (threadIdx.x == 0) {
      s_mean = m;
      s_den = d;
      if (blockIdx.x == 0 && na.stats) {
        na.stats[0] = m;
        na.stats[1] = sd;
      }
    }
  }
  __syncthreads();
  const float mean = s_mean, den = s_den;
  const int64_t M4 = M / 4;
  const float4* a4 = reinterpret_cast<const float4*>(adv);
  const int64_t stride = (int64_t)gridDim.x * kStatThreads;
  for (int64_t g0 = (int64_t)blockIdx.x * kStatThreads + threadIdx.x; g0 < M4; g0 += stride * kStatUnroll) {
    float4 v[kStatUnroll];
#pragma unroll
    for (int u = 0; u < kStatUnroll; ++u) {
      const int64_t gi = g0 + u * stride;
      v[u] = gi < M4 ? __ldcs(a4 + gi) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < kStatUnroll; ++u) {
      const int64_t gi = g0 + u * stride;
      if (gi >= M4) break;
      const int64_t i = gi * 4;
      if (na.rets)
        st_stream_f4(na.rets + i, make_float4(v[u].x + load_value(na.values, na.bf16, i),
                                              v[u].y + load_value(na.values, na.bf16, i + 1),
                                              v[u].z + load_value(na.values, na.bf16, i + 2),
                                              v[u].w + load_value(na.values, na.bf16, i + 3)));
      st_stream_f4(na.norm + i, make_float4((v[u].x - mean) / den, (v[u].y - mean) / den, (v[u].z - mean) / den,
                                            (v[u].w - mean) / den));
    }
  }
  if (blockIdx.x == 0 && threadIdx.x < (unsigned)(M - M4 * 4)) {
    const int64_t i = M4 * 4 + threadIdx.x;
    const float a = adv[i];
    if (na.rets) na.rets[i] = a + load_value(na.values, na.bf16, i);
    na.norm[i] = (a - mean) / den;
  }
}

// ---- GAE + value loss ------------------------------------------------------------
// One pass: A = GAE, returns = A + V, and for the value head's predictions
// V' the loss mean(l(V' - returns)) with l = d^2 (MSE) or Huber(delta), plus
// its gradient dl/dV' / M, written per element for the backward pass.
struct ValueArgs {
  float* adv;            // A, or null
  float* rets;           // A + V, or null
  float* grad;           // d loss / d V'
  const float* new_v;    // V' (fp32)
  const void* values;    // V
  int bf16;
  double* partials;      // per CTA loss sums
  unsigned* counter;     // CTAs done (the last one resets it)
  float* loss;           // written by the last CTA
  int huber;
  float delta;
  float inv_count;
};

template <class P, bool SINGLE>
__global__ void __launch_bounds__(kNormWarps * 32) gae_value_kernel(const typename P::Params p, const Geom g,
                                                                     const ValueArgs va) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t S = g.S;
  const int64_t W = (int64_t)gridDim.x * kNormWarps;
  pdl_trigger();
  if (g.pdl == 1) pdl_wait();
  bool waited = g.pdl == 1;
  double acc = 0.0;
  for (int64_t row = (int64_t)blockIdx.x * kNormWarps + warp; row < g.N; row += W) {
    walk_row<P, SINGLE>(p, g, row, lane, [&](int64_t col, float4 a) {
      if (!waited) {
        pdl_wait();
        waited = true;
      }
      const int64_t i = row * S + col;
      const float av[4] = {a.x, a.y, a.z, a.w};
      const float4 nv4 = __ldcs(reinterpret_cast<const float4*>(va.new_v + i));
      const float nv[4] = {nv4.x, nv4.y, nv4.z, nv4.w};
      float rt[4], gr[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        rt[k] = av[k] + load_value(va.values, va.bf16, i + k);
        const float d = nv[k] - rt[k];
        float l, gd;
        if (va.huber) {
          const float ad = fabsf(d);
          l = ad < va.delta ? 0.5f * d * d : va.delta * (ad - 0.5f * va.delta);
          gd = ad < va.delta ? d : copysignf(va.delta, d);
        } else {
          l = d * d;
          gd = 2.f * d;
        }
        acc += (double)l;
        gr[k] = gd * va.inv_count;
      }
      if (va.adv) st_stream_f4(va.adv + i, a);
      if (va.rets) st_stream_f4(va.rets + i, make_float4(rt[0], rt[1], rt[2], rt[3]));
      st_stream_f4(va.grad + i, make_float4(gr[0], gr[1], gr[2], gr[3]));
    });
  }
  const double2 t = block_sum2<kNormWarps * 32>(acc, 0.0);
  pdl_wait();  // also in CTAs that stored nothing
  // The last CTA to finish sums the partials in a fixed order into the loss.
  __shared__ int s_last;
  if (threadIdx.x == 0) {
    va.partials[blockIdx.x] = t.x;
    __threadfence();
    s_last = atomicAdd(va.counter, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (s_last) {
    __threadfence();
    double a = 0.0;
    for (int i = threadIdx.x; i < (int)gridDim.x; i += kNormWarps * 32) a += __ldcg(va.partials + i);
    const double2 tot = block_sum2<kNormWarps * 32>(a, 0.0);
    if (threadIdx.x == 0) {
      *va.loss = (float)(tot.x * (double)va.inv_count);
      *va.counter = 0u;
    }
  }
}

// Rows that do not start 16-byte aligned: GAE first, then this elementwise pass.
__global__ void __launch_bounds__(kStatThreads) value_loss_elementwise(const float* adv, int64_t M, ValueArgs va) {
  double acc = 0.0;
  for (int64_t i = (int64_t)blockIdx.x * kStatThreads + threadIdx.x; i < M; i += (int64_t)gridDim.x * kStatThreads) {
    const float a = adv[i];
    const float rt = a + load_value(va.values, va.bf16, i);
    const float d = va.new_v[i] - rt;
    float l, gd;
    if (va.huber) {
      const float ad = fabsf(d);
      l = ad < va.delta ? 0.5f * d * d : va.delta * (ad - 0.5f * va.delta);
      gd = ad < va.delta ? d : copysignf(va.delta, d);
    } else {
      l = d * d;
      gd = 2.f * d;
    }
    acc += (double)l;
    if (va.rets) va.rets[i] = rt;
    va.grad[i] = gd * va.inv_count;
  }
  const double2 t = block_sum2<kStatThreads>(acc, 0.0);
  if (threadIdx.x == 0) va.partials[blockIdx.x] = t.x;
}

__global__ void __launch_bounds__(kStatThreads) value_loss_finish(const double* partials, int n, float inv_count,
                                                                  float* loss) {
  pdl_wait();  // then trigger: a dependent starts after the loss pass has completed
  pdl_trigger();
  double a = 0.0;
  for (int i = threadIdx.x; i < n; i += kStatThreads) a += __ldcg(partials + i);
  const double2 t = block_sum2<kStatThreads>(a, 0.0);
  if (threadIdx.x == 0) *loss = (float)(t.x * (double)inv_count);
}

int num_sms_of(int dev) {
  static int cache[64] = {0};
  if (dev < 0 || dev >= 64) return 148;
  if (!cache[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

// The two passes; RLS_EUNSUPPORTED for rows that do not start 16-byte aligned.
template <class P>
int launch_gae_norm(const typename P::Params& p, Geom g, NormArgs na, size_t ws_bytes, cudaStream_t s) {
  constexpr int VEC = Rows2Chunk<P, 1>::VEC;
  if (g.S % VEC != 0) return RLS_EUNSUPPORTED;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return RLS_ECUDA;
  const int sms = num_sms_of(dev);
  // One warp per row: too few rows to fill the GPU take the GAE kernel choice
  // (virtual rows, look-back) and the separate statistics passes instead.
  if (g.N < 8LL * sms) return RLS_EUNSUPPORTED;
  int64_t blocks = (g.N + kNormWarps - 1) / kNormWarps;
  if (blocks > 8LL * sms) blocks = 8LL * sms;
  if ((size_t)64 + (size_t)blocks * sizeof(double2) > ws_bytes) return RLS_EWORKSPACE;
  float* tmp = na.raw ? na.raw : na.norm;
  const size_t mb = (size_t)g.M * (na.bf16 ? 2 : 4);
  g.pdl = pdl_mode(s, {{p.r, mb}, {p.v, mb}, {p.term, mb}, {p.trunc, mb}, {p.boot, mb},
                       {p.boot_row, (size_t)g.N * 4}});
  constexpr int64_t CH = 32 * VEC;
  int st = g.S <= CH
               ? launch_rowk(gae_stats_kernel<P, true>, blocks, kNormWarps * 32, s, g.pdl, g.M, tmp, nullptr, p, g,
                             tmp, na)
               : launch_rowk(gae_stats_kernel<P, false>, blocks, kNormWarps * 32, s, g.pdl, g.M, tmp, nullptr, p, g,
                             tmp, na);
  if (st) return st;
  const int64_t groups = g.M / 4;
  int64_t fb = (groups + kStatThreads - 1) / kStatThreads;
  if (fb > 8LL * sms) fb = 8LL * sms;
  if (fb < 1) fb = 1;
  return launch_rowk(norm_finish_kernel, fb, kStatThreads, s, 1, g.M, na.norm, na.rets, (const float*)tmp, g.M, na);
}

template <class T>
int gae_norm_dispatch(const typename GaeAlg<T>::Params& p, const Geom& g, const NormArgs& na, size_t wsb,
                      cudaStream_t s) {
  const bool tr = p.trunc != nullptr;
  const int pb = p.boot_kind == RLS_BOOT_FULL_ADD ? 1 : ((p.boot_kind == RLS_BOOT_FULL_SEL && tr) ? 2 : 0);
  if (!tr && pb == 0) return launch_gae_norm<GaeT<T, false, 0>>(p, g, na, wsb, s);
  if (tr && pb == 0) return launch_gae_norm<GaeT<T, true, 0>>(p, g, na, wsb, s);
  if (tr && pb == 2) return launch_gae_norm<GaeT<T, true, 2>>(p, g, na, wsb, s);
  if (!tr && pb == 1) return launch_gae_norm<GaeT<T, false, 1>>(p, g, na, wsb, s);
  return launch_gae_norm<GaeT<T, true, 1>>(p, g, na, wsb, s);
}

}  // namespace

extern "C" int rls_gae_normalized(const void* rewards, const void* values, const void* terminateds,
                                  const void* truncateds, const void* bootstrap, int boot_kind, float* normalized,
                                  float* returns, float* advantages, float* stats, int64_t num_envs, int64_t seq_len,
                                  float gamma, float lambda_, float eps, int in_dtype, void* ws, size_t ws_bytes,
                                  void* stream) {
  if (num_envs < 0 || seq_len < 0) return RLS_EINVAL;
  if (num_envs == 0 || seq_len == 0) return RLS_OK;
  if (!rewards || !values || !terminateds || !normalized || !ws) return RLS_EINVAL;
  if (in_dtype != RLS_F32 && in_dtype != RLS_BF16) return RLS_EINVAL;
  if (boot_kind < RLS_BOOT_NONE || boot_kind > RLS_BOOT_FULL_SEL) return RLS_EINVAL;
  if ((boot_kind == RLS_BOOT_ROW || boot_kind == RLS_BOOT_LASTCOL) && !bootstrap) return RLS_EINVAL;
  if (num_envs > INT64_MAX / seq_len) return RLS_EINVAL;
  auto al = [](const void* q) { return q == nullptr || ((uintptr_t)q & 15u) == 0; };
  if (!al(rewards) || !al(values) || !al(terminateds) || !al(truncateds) || !al(normalized) || !al(returns) ||
      !al(advantages) || (boot_kind >= RLS_BOOT_LASTCOL && !al(bootstrap)) || !al(ws))
    return RLS_EALIGN;
  DeviceGuard guard{rewards, values, terminateds, truncateds, bootstrap, normalized, returns, advantages, stats, ws};
  if (guard.status()) return guard.status();
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int64_t M = num_envs * seq_len;
  std::lock_guard<std::recursive_mutex> launch_lock(launch_mutex());

  Geom g{};
  g.M = M;
  g.S = seq_len;
  g.N = num_envs;
  g.edge_global = 1;
  NormArgs na{};
  na.norm = normalized;
  na.rets = returns;
  na.raw = advantages;
  na.stats = stats;
  na.values = values;
  na.bf16 = in_dtype == RLS_BF16;
  na.partials = reinterpret_cast<double2*>(static_cast<char*>(ws) + 64);
  na.counter = &reinterpret_cast<WsHeader*>(ws)->pad[0];
  na.mean_den = reinterpret_cast<float*>(&reinterpret_cast<WsHeader*>(ws)->pad[2]);
  na.eps = eps;

#define NORM_PARAMS(T)                                                                                    \
  typename GaeAlg<T>::Params p{};                                                                         \
  p.r = (const T*)rewards; p.v = (const T*)values; p.term = (const T*)terminateds;                         \
  p.trunc = (const T*)truncateds;                                                                          \
  p.boot = boot_kind >= RLS_BOOT_LASTCOL ? (const T*)bootstrap : nullptr;                                  \
  p.boot_row = boot_kind == RLS_BOOT_ROW ? (const float*)bootstrap : nullptr;                              \
  p.halo = nullptr; p.out0 = nullptr; p.out1 = nullptr; p.boot_kind = boot_kind; p.gamma = gamma;          \
  p.gl = gamma * lambda_;
  int st = prepare_layout(ws, ws_bytes, kLayoutScratch, s);
  if (st) return st;
  if (in_dtype == RLS_F32) {
    NORM_PARAMS(float)
    st = gae_norm_dispatch<float>(p, g, na, ws_bytes, s);
  } else {
    NORM_PARAMS(__nv_bfloat16)
    st = gae_norm_dispatch<__nv_bfloat16>(p, g, na, ws_bytes, s);
  }
#undef NORM_PARAMS
  if (st != RLS_EUNSUPPORTED) return st;

  // Rows that do not start 16-byte aligned, or too few rows for one warp per
  // row: GAE into the advantages (or the output as scratch), then a statistics
  // pass and a normalise pass.
  float* adv = advantages ? advantages : normalized;
  int cur = 0;
  if (cudaGetDevice(&cur) != cudaSuccess) return RLS_ECUDA;
  const int nparts = 8 * num_sms_of(cur);
  if ((size_t)64 + (size_t)nparts * sizeof(double2) > ws_bytes) return RLS_EWORKSPACE;
  st = rls_gae(rewards, values, terminateds, truncateds, bootstrap, boot_kind, adv, num_envs, seq_len, gamma,
               lambda_, in_dtype, nullptr, ws, ws_bytes, stream);
  if (st) return st;
  // rls_gae may have used the workspace's records; the partials take their place.
  st = prepare_layout(ws, ws_bytes, kLayoutScratch, s);
  if (st) return st;
  norm_stats_kernel<<<nparts, kStatThreads, 0, s>>>(adv, M, na.partials);
  norm_apply_kernel<<<nparts, kStatThreads, 0, s>>>(adv, M, na.partials, nparts, na);
  return cudaPeekAtLastError() == cudaSuccess ? RLS_OK : RLS_ECUDA;
}

namespace {
template <class P>
int launch_gae_value(const typename P::Params& p, const Geom& g, ValueArgs va, float* loss, size_t ws_bytes,
                     cudaStream_t s) {
  constexpr int VEC = Rows2Chunk<P, 1>::VEC;
  if (g.S % VEC != 0) return RLS_EUNSUPPORTED;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return RLS_ECUDA;
  if (g.N < 8LL * num_sms_of(dev)) return RLS_EUNSUPPORTED;  // few rows: GAE's own kernel choice, then the loss pass
  int64_t blocks = (g.N + kNormWarps - 1) / kNormWarps;
  const int64_t cap = (int64_t)8 * num_sms_of(dev);
  if (blocks > cap) blocks = cap;
  if ((size_t)64 + (size_t)blocks * sizeof(double) > ws_bytes) return RLS_EWORKSPACE;
  const size_t mb = (size_t)g.M * (va.bf16 ? 2 : 4);
  Geom g2 = g;
  g2.pdl = pdl_mode(s, {{p.r, mb}, {p.v, mb}, {p.term, mb}, {p.trunc, mb}, {p.boot, mb},
                        {p.boot_row, (size_t)g.N * 4}, {va.new_v, (size_t)g.M * 4}});
  va.loss = loss;
  constexpr int64_t CH = 32 * VEC;
  int st = g.S <= CH ? launch_rowk(gae_value_kernel<P, true>, blocks, kNormWarps * 32, s, g2.pdl, g.M, va.grad,
                                   va.rets, p, g2, va)
                     : launch_rowk(gae_value_kernel<P, false>, blocks, kNormWarps * 32, s, g2.pdl, g.M, va.grad,
                                   va.rets, p, g2, va);
  if (st) return st;
  // It triggers its dependents at once: all four outputs are the stream's record.
  const size_t ob = (size_t)g.M * 4;
  pdl_record(s, {{va.grad, ob}, {va.rets, ob}, {va.adv, ob}, {loss, 4}});
  return RLS_OK;
}

template <class T>
int gae_value_dispatch(const typename GaeAlg<T>::Params& p, const Geom& g, const ValueArgs& va, float* loss,
                       size_t wsb, cudaStream_t s) {
  const bool tr = p.trunc != nullptr;
  const int pb = p.boot_kind == RLS_BOOT_FULL_ADD ? 1 : ((p.boot_kind == RLS_BOOT_FULL_SEL && tr) ? 2 : 0);
  if (!tr && pb == 0) return launch_gae_value<GaeT<T, false, 0>>(p, g, va, loss, wsb, s);
  if (tr && pb == 0) return launch_gae_value<GaeT<T, true, 0>>(p, g, va, loss, wsb, s);
  if (tr && pb == 2) return launch_gae_value<GaeT<T, true, 2>>(p, g, va, loss, wsb, s);
  if (!tr && pb == 1) return launch_gae_value<GaeT<T, false, 1>>(p, g, va, loss, wsb, s);
  return launch_gae_value<GaeT<T, true, 1>>(p, g, va, loss, wsb, s);
}
}  // namespace

extern "C" int rls_gae_value_loss(const void* rewards, const void* values, const void* terminateds,
                                  const void* truncateds, const void* bootstrap, int boot_kind,
                                  const float* new_values, float* advantages, float* returns, float* grad,
                                  float* loss, int64_t num_envs, int64_t seq_len, float gamma, float lambda_,
                                  int loss_kind, float delta, int in_dtype, void* ws, size_t ws_bytes,
                                  void* stream) {
  if (num_envs < 0 || seq_len < 0) return RLS_EINVAL;
  if (!loss) return RLS_EINVAL;
  if (num_envs == 0 || seq_len == 0) return RLS_OK;
  if (!rewards || !values || !terminateds || !new_values || !grad || !ws) return RLS_EINVAL;
  if (in_dtype != RLS_F32 && in_dtype != RLS_BF16) return RLS_EINVAL;
  if (loss_kind != RLS_LOSS_MSE && loss_kind != RLS_LOSS_HUBER) return RLS_EINVAL;
  if (boot_kind < RLS_BOOT_NONE || boot_kind > RLS_BOOT_FULL_SEL) return RLS_EINVAL;
  if ((boot_kind == RLS_BOOT_ROW || boot_kind == RLS_BOOT_LASTCOL) && !bootstrap) return RLS_EINVAL;
  if (num_envs > INT64_MAX / seq_len) return RLS_EINVAL;
  auto al = [](const void* q) { return q == nullptr || ((uintptr_t)q & 15u) == 0; };
  if (!al(rewards) || !al(values) || !al(terminateds) || !al(truncateds) || !al(new_values) || !al(advantages) ||
      !al(returns) || !al(grad) || (boot_kind >= RLS_BOOT_LASTCOL && !al(bootstrap)) || !al(ws))
    return RLS_EALIGN;
  DeviceGuard guard{rewards, values, terminateds, truncateds, bootstrap, new_values, advantages, returns, grad, loss,
                    ws};
  if (guard.status()) return guard.status();
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  std::lock_guard<std::recursive_mutex> launch_lock(launch_mutex());
  int st = prepare_layout(ws, ws_bytes, kLayoutScratch, s);
  if (st) return st;
  Geom g{};
  g.M = num_envs * seq_len;
  g.S = seq_len;
  g.N = num_envs;
  g.edge_global = 1;
  ValueArgs va{};
  va.adv = advantages;
  va.rets = returns;
  va.grad = grad;
  va.new_v = new_values;
  va.values = values;
  va.bf16 = in_dtype == RLS_BF16;
  va.partials = reinterpret_cast<double*>(static_cast<char*>(ws) + 64);
  va.counter = &reinterpret_cast<WsHeader*>(ws)->pad[0];
  va.loss = loss;
  va.huber = loss_kind == RLS_LOSS_HUBER;
  va.delta = delta;
  va.inv_count = (float)(1.0 / (double)g.M);
#define VAL_PARAMS(T)                                                                                     \
  typename GaeAlg<T>::Params p{};                                                                         \
  p.r = (const T*)rewards; p.v = (const T*)values; p.term = (const T*)terminateds;                         \
  p.trunc = (const T*)truncateds;                                                                          \
  p.boot = boot_kind >= RLS_BOOT_LASTCOL ? (const T*)bootstrap : nullptr;                                  \
  p.boot_row = boot_kind == RLS_BOOT_ROW ? (const float*)bootstrap : nullptr;                              \
  p.halo = nullptr; p.out0 = nullptr; p.out1 = nullptr; p.boot_kind = boot_kind; p.gamma = gamma;          \
  p.gl = gamma * lambda_;
  if (in_dtype == RLS_F32) {
    VAL_PARAMS(float)
    st = gae_value_dispatch<float>(p, g, va, loss, ws_bytes, s);
  } else {
    VAL_PARAMS(__nv_bfloat16)
    st = gae_value_dispatch<__nv_bfloat16>(p, g, va, loss, ws_bytes, s);
  }
#undef VAL_PARAMS
  if (st != RLS_EUNSUPPORTED) return st;
  // Unaligned rows, or too few rows for one warp per row: GAE into the
  // advantages (the gradient buffer as scratch), then the elementwise loss pass.
  float* adv = advantages ? advantages : grad;
  st = rls_gae(rewards, values, terminateds, truncateds, bootstrap, boot_kind, adv, num_envs, seq_len, gamma,
               lambda_, in_dtype, nullptr, ws, ws_bytes, stream);
  if (st) return st;
  st = prepare_layout(ws, ws_bytes, kLayoutScratch, s);
  if (st) return st;
  int cur = 0;
  if (cudaGetDevice(&cur) != cudaSuccess) return RLS_ECUDA;
  const int nparts = 8 * num_sms_of(cur);
  if ((size_t)64 + (size_t)nparts * sizeof(double) > ws_bytes) return RLS_EWORKSPACE;
  value_loss_elementwise<<<nparts, kStatThreads, 0, s>>>(adv, g.M, va);
  if (cudaPeekAtLastError() != cudaSuccess) return RLS_ECUDA;
  // value_loss_finish triggers its dependents: launched through launch_rowk so
  // the stream's record names its output.
  return launch_rowk(value_loss_finish, 1, kStatThreads, s, 1, 1, loss, nullptr, (const double*)va.partials, nparts,
                     va.inv_count, loss);
}

// ---- GAE with observation-skip masking ---------------------------------------------
// Multi-turn / tool-use rollouts interleave generated tokens (mask 1) with
// observation tokens (mask 0).  Observation tokens pass the recurrence through
// unchanged, so credit flows across them:
//   NV[t] = value of the next generated token after t (0 past the window end),
//   A[t]  = m[t] ? r[t] + gamma*NV[t] - V[t] + gamma*lambda*A[t+1] : A[t+1],
//   A[T]  = 0,  returns = A + V.
// Two chained backward affine scans per chunk, in one warp per row:
//   NV: x[t] = m[t+1]*V[t+1] + (1 - m[t+1]) * x[t+1]   (x[T-1] = 0),
//   A:  x[t] = m[t]*delta[t] + (m[t]*gamma*lambda + 1 - m[t]) * x[t+1].
namespace {
constexpr int kSkipWarps = 8;

template <class InT>
__device__ __forceinline__ void load_vec(const InT* p, int64_t i, bool vec_ok, int64_t left, float (&o)[16 / sizeof(InT)]) {
  constexpr int V = 16 / sizeof(InT);
  if (vec_ok && left >= V) {
    const uint4 u = __ldcs(reinterpret_cast<const uint4*>(p + i));
    const unsigned w[4] = {u.x, u.y, u.z, u.w};
    if constexpr (sizeof(InT) == 4) {
#pragma unroll
      for (int k = 0; k < 4; ++k) o[k] = __uint_as_float(w[k]);
    } else {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        o[2 * k] = __uint_as_float(w[k] << 16);
        o[2 * k + 1] = __uint_as_float(w[k] & 0xffff0000u);
      }
    }
  } else {
#pragma unroll
    for (int k = 0; k < V; ++k) {
      if (k < left) {
        if constexpr (sizeof(InT) == 4) o[k] = p[i + k];
        else o[k] = bf16_bits_to_float(reinterpret_cast<const unsigned short*>(p)[i + k]);
      } else {
        o[k] = 0.f;
      }
    }
  }
}

// Backward warp scan of per-lane maps: returns (exclusive map of the lanes
// after this one, total map of the chunk).
__device__ __forceinline__ void warp_suffix_scan(Pair m, int lane, Pair& excl, Pair& tot) {
  Pair incl = m;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const Pair o = shfl_pair_down(incl, d);
    if (lane + d < 32) incl = compose(incl, o);
  }
  const Pair x = shfl_pair_down(incl, 1);
  excl = (lane == 31) ? pair_identity() : x;
  tot = shfl_pair_idx(incl, 0);
}

template <class InT>
__global__ void __launch_bounds__(kSkipWarps * 32) gae_obs_skip_kernel(const InT* r, const InT* v, const InT* mask,
                                                                        float* adv, float* rets, int64_t N, int64_t S,
                                                                        float gamma, float gl, int pdl) {
  constexpr int VEC = 16 / sizeof(InT);
  constexpr int64_t CH = 32 * VEC;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kSkipWarps + (threadIdx.x >> 5);
  if (row >= N) return;
  const bool vec_ok = (S % VEC) == 0;
  const int64_t rbase = row * S;
  const int64_t nch = (S + CH - 1) / CH;
  pdl_trigger();
  if (pdl == 1) pdl_wait();
  bool waited = pdl == 1;
  float carry_nv = 0.f, carry_a = 0.f;
  float next_m = 0.f, next_v = 0.f;  // m, V of the element after the current chunk
  for (int64_t k = 0; k < nch; ++k) {
    const int64_t cb = (nch - 1 - k) * CH;
    const int64_t col0 = cb + lane * VEC;
    const int64_t left = S - col0;  // elements of this lane's run inside the row
    float rr[VEC], vv[VEC], mm[VEC];
    load_vec<InT>(r, rbase + col0, vec_ok, left, rr);
    load_vec<InT>(v, rbase + col0, vec_ok, left, vv);
    load_vec<InT>(mask, rbase + col0, vec_ok, left, mm);
    // neighbour (m, V) after this lane's last element
    float nm = __shfl_down_sync(0xffffffffu, mm[0], 1), nvv = __shfl_down_sync(0xffffffffu, vv[0], 1);
    if (lane == 31) { nm = next_m; nvv = next_v; }
    const float chunk_m0 = __shfl_sync(0xffffffffu, mm[0], 0), chunk_v0 = __shfl_sync(0xffffffffu, vv[0], 0);
    // scan 1: next generated value
    float a1[VEC], b1[VEC];
#pragma unroll
    for (int e = VEC - 1; e >= 0; --e) {
      const float m1 = e + 1 < VEC ? mm[e + 1] : nm;
      const float v1 = e + 1 < VEC ? vv[e + 1] : nvv;
      const int64_t col = col0 + e;
      if (col >= S) { a1[e] = 0.f; b1[e] = 1.f; continue; }
      if (col == S - 1) { a1[e] = 0.f; b1[e] = 0.f; continue; }
      a1[e] = m1 * v1;
      b1[e] = 1.f - m1;
    }
    Pair m = pair_identity();
#pragma unroll
    for (int e = VEC - 1; e >= 0; --e) m = compose(Pair{a1[e], b1[e]}, m);
    Pair ex, tot;
    warp_suffix_scan(m, lane, ex, tot);
    float x = apply(ex, carry_nv);
    float nvs[VEC];
#pragma unroll
    for (int e = VEC - 1; e >= 0; --e) {
      x = fmaf(b1[e], x, a1[e]);
      nvs[e] = x;
    }
    carry_nv = apply(tot, carry_nv);
    // scan 2: advantages
    float a2[VEC], b2[VEC];
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      if (col0 + e >= S) { a2[e] = 0.f; b2[e] = 1.f; continue; }
      const float delta = rr[e] + gamma * nvs[e] - vv[e];
      a2[e] = mm[e] * delta;
      b2[e] = mm[e] * gl + (1.f - mm[e]);
    }
    m = pair_identity();
#pragma unroll
    for (int e = VEC - 1; e >= 0; --e) m = compose(Pair{a2[e], b2[e]}, m);
    warp_suffix_scan(m, lane, ex, tot);
    x = apply(ex, carry_a);
    float out[VEC];
#pragma unroll
    for (int e = VEC - 1; e >= 0; --e) {
      x = fmaf(b2[e], x, a2[e]);
      out[e] = x;
    }
    carry_a = apply(tot, carry_a);
    next_m = chunk_m0;
    next_v = chunk_v0;
    if (!waited) {  // the first chunk is loaded and scanned; nothing is stored before the predecessor ends
      pdl_wait();
      waited = true;
    }
    const int64_t i = rbase + col0;
    if (vec_ok && left >= VEC) {
#pragma unroll
      for (int q = 0; q < VEC; q += 4) {
        st_stream_f4(adv + i + q, make_float4(out[q], out[q + 1], out[q + 2], out[q + 3]));
        if (rets) st_stream_f4(rets + i + q, make_float4(out[q] + vv[q], out[q + 1] + vv[q + 1], out[q + 2] + vv[q + 2],
                                                         out[q + 3] + vv[q + 3]));
      }
    } else {
#pragma unroll
      for (int e = 0; e < VEC; ++e)
        if (e < left) {
          adv[i + e] = out[e];
          if (rets) rets[i + e] = out[e] + vv[e];
        }
    }
  }
}
}  // namespace

extern "C" int rls_gae_obs_skip(const void* rewards, const void* values, const void* mask, float* advantages,
                                float* returns, int64_t num_envs, int64_t seq_len, float gamma, float lambda_,
                                int in_dtype, void* stream) {
  if (num_envs < 0 || seq_len < 0) return RLS_EINVAL;
  if (num_envs == 0 || seq_len == 0) return RLS_OK;
  if (!rewards || !values || !mask || !advantages) return RLS_EINVAL;
  if (in_dtype != RLS_F32 && in_dtype != RLS_BF16) return RLS_EINVAL;
  if (num_envs > INT64_MAX / seq_len) return RLS_EINVAL;
  auto al = [](const void* q) { return q == nullptr || ((uintptr_t)q & 15u) == 0; };
  if (!al(rewards) || !al(values) || !al(mask) || !al(advantages) || !al(returns)) return RLS_EALIGN;
  DeviceGuard guard{rewards, values, mask, advantages, returns};
  if (guard.status()) return guard.status();
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  std::lock_guard<std::recursive_mutex> launch_lock(launch_mutex());
  const int64_t blocks = (num_envs + kSkipWarps - 1) / kSkipWarps;
  if (blocks > 0x7fffffffLL) return RLS_EINVAL;
  const float gl = gamma * lambda_;
  const size_t mb = (size_t)num_envs * seq_len * (in_dtype == RLS_BF16 ? 2 : 4);
  const int pdl = pdl_mode(s, {{rewards, mb}, {values, mb}, {mask, mb}});
  const int64_t M = num_envs * seq_len;
  if (in_dtype == RLS_F32)
    return launch_rowk(gae_obs_skip_kernel<float>, blocks, kSkipWarps * 32, s, pdl, M, advantages, returns,
                       (const float*)rewards, (const float*)values, (const float*)mask, advantages, returns, num_envs,
                       seq_len, gamma, gl, pdl);
  return launch_rowk(gae_obs_skip_kernel<__nv_bfloat16>, blocks, kSkipWarps * 32, s, pdl, M, advantages, returns,
                     (const __nv_bfloat16*)rewards, (const __nv_bfloat16*)values, (const __nv_bfloat16*)mask,
                     advantages, returns, num_envs, seq_len, gamma, gl, pdl);
}
