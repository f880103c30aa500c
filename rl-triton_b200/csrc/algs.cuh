// algs.cuh -- per-estimator element rules for the generic affine scan kernel.
//
// Each policy turns the inputs of one element into its affine coefficients
// (a, b) -- x[t] = a + b * x[t(+/-)1] -- and turns the solved state back into
// the estimator's outputs.  The formulas follow the reference's fused Triton
// kernels (file:line cited per policy); the float operation order mirrors
// theirs so the results agree to a few ulp.
//
// Edge handling (shared by every policy).  The kernel scans ONE flat array of
// num_envs*seq_len elements; a row edge is folded into the coefficients:
//   * at the window end of a backward row (t = T-1) the carry coming from the
//     next row is cut (b = 0) and the row's own boundary carry C is folded in
//     as a += b_orig * C;
//   * at the start of a forward row (t = 0) the seed is folded in the same way;
//   * at a time-split cut (a local segment edge that is not the global edge)
//     b = 0 as well, and the neighbour values across the cut come from the
//     per-row halo array; the true carry is applied later by the segment fix-up.
#pragma once
#include "common.cuh"

namespace rls {

// Boot kinds (mirror include/rlscan.h).
constexpr int kBootNone = 0, kBootRow = 1, kBootLastCol = 2, kBootFullAdd = 3, kBootFullSel = 4;

struct EdgeCtx {
  int64_t i;    // flat element index
  int64_t row;
  bool edge;    // backward: local col == S-1; forward: local col == 0
  bool global;  // the edge is the real window end (backward) / start (forward)
};

struct Geom {
  int64_t M;          // elements in the flat buffer = N * S
  int64_t S;          // local row length
  int64_t N;          // rows
  int64_t num_tiles;  // tiles of the launch
  int64_t ws_cap;     // tiles the workspace can describe (its layout key)
  int edge_global;    // 1: local row edges are global row edges (no time split)
  int seg;            // 1: time-split launch (halo neighbours at cuts)
  int smem_per_warp;  // dynamic shared memory per warp (Retrace staging)
  int tma;            // 1: staging uses cp.async.bulk
  int l2_prefetch;    // flat3: bulk L2 prefetch of each super-tile before its first walk
  int pdl;            // row kernels launched with programmatic stream serialization:
                      // 0 none; 1 wait for the preceding kernel before the first load;
                      // 2 issue the first chunk's loads, then wait (inputs are not
                      //   outputs of the preceding library launch on this stream)
};

// Struct-generic warp shuffles for neighbour records (all 32-bit members).
template <class T>
__device__ __forceinline__ T shfl_down_any(const T& v, int d) {
  static_assert(sizeof(T) % 4 == 0, "32-bit members");
  T r;
  const unsigned* s = reinterpret_cast<const unsigned*>(&v);
  unsigned* o = reinterpret_cast<unsigned*>(&r);
#pragma unroll
  for (int k = 0; k < (int)(sizeof(T) / 4); ++k) o[k] = __shfl_down_sync(0xffffffffu, s[k], d);
  return r;
}
template <class T>
__device__ __forceinline__ T shfl_up_any(const T& v, int d) {
  T r;
  const unsigned* s = reinterpret_cast<const unsigned*>(&v);
  unsigned* o = reinterpret_cast<unsigned*>(&r);
#pragma unroll
  for (int k = 0; k < (int)(sizeof(T) / 4); ++k) o[k] = __shfl_up_sync(0xffffffffu, s[k], d);
  return r;
}
template <class T>
__device__ __forceinline__ T shfl_idx_any(const T& v, int src) {
  T r;
  const unsigned* s = reinterpret_cast<const unsigned*>(&v);
  unsigned* o = reinterpret_cast<unsigned*>(&r);
#pragma unroll
  for (int k = 0; k < (int)(sizeof(T) / 4); ++k) o[k] = __shfl_sync(0xffffffffu, s[k], src);
  return r;
}

struct NoStage {
  template <class P>
  __device__ __forceinline__ static void stage(const P&, const Geom&, int64_t, int, int, unsigned char*,
                                               uint64_t*, WsHeader*) {}
};

// =========================================================================
// GAE -- src/rl_triton/kernels/gae.py:62-180 (flat), src/rl_triton/ops/gae.py:192-215
// (chunked).  delta = r + gamma*(1-term)*v_next - v ; b = gamma*lambda*(1-done);
// the additive carry at the window end is always 0 (kernels/gae.py:86-96).
// =========================================================================
template <class InT>
struct GaeAlg : NoStage {
  static constexpr bool kBackward = true;
  static constexpr bool kNeedsNbr = true;
  static constexpr int kVec = InTraits<InT>::kVec;
  static constexpr int kOuts = 1;
  struct Params {
    const InT *r, *v, *term, *trunc, *boot;
    const float* boot_row;
    const float* halo;
    float* out0;
    float* out1;
    int boot_kind;
    float gamma, gl;
  };
  struct Run {
    float r[kVec], v[kVec], term[kVec], trunc[kVec], boot[kVec];
  };
  using Nbr = float;  // V of the neighbouring element
  __device__ __forceinline__ static void load(const Params& p, int64_t i, int64_t M, bool full, Run& x,
                                              const unsigned char*, int) {
    load_run<InT, kVec>(p.r, i, M, full, 0.f, x.r);
    load_run<InT, kVec>(p.v, i, M, full, 0.f, x.v);
    load_run<InT, kVec>(p.term, i, M, full, 1.f, x.term);
    if (p.trunc) load_run<InT, kVec>(p.trunc, i, M, full, 0.f, x.trunc);
    else {
#pragma unroll
      for (int k = 0; k < kVec; ++k) x.trunc[k] = 0.f;
    }
    if (p.boot && p.boot_kind >= kBootFullAdd) load_run<InT, kVec>(p.boot, i, M, full, 0.f, x.boot);
    else {
#pragma unroll
      for (int k = 0; k < kVec; ++k) x.boot[k] = 0.f;
    }
  }
  __device__ __forceinline__ static Nbr nbr_at(const Run& x, int j) { return x.v[j]; }
  __device__ __forceinline__ static Nbr nbr_global(const Params& p, int64_t i) {
    return InTraits<InT>::scalar(p.v, i);
  }
  __device__ __forceinline__ static Nbr nbr_halo(const Params& p, int64_t row) { return p.halo[row]; }

  // Next-state value at the window end.
  __device__ __forceinline__ static float window_value(const Params& p, const Run& x, int j, const EdgeCtx& e) {
    if (p.boot_kind == kBootNone) return 0.f;
    if (p.boot_kind == kBootRow) return p.boot_row[e.row];
    if (p.boot_kind == kBootLastCol) return InTraits<InT>::scalar(p.boot, e.i);  // column T-1 only
    return x.boot[j];
  }
  __device__ __forceinline__ static void coeff(const Params& p, Run& x, int j, Nbr vnext, const EdgeCtx& e,
                                               float& a, float& b) {
    const float term = x.term[j];
    const float trunc = x.trunc[j];
    const float done = p.trunc ? fminf(term + trunc, 1.f) : term;
    float vn;
    if (e.edge && e.global) {
      vn = window_value(p, x, j, e);
    } else if (p.boot_kind == kBootFullSel) {
      // flat path with truncations: kernels/gae.py:153-154
      vn = (trunc == 1.f) ? x.boot[j] : vnext;
    } else {
      // masked + additive form: ops/gae.py:200-205
      vn = p.trunc ? ((trunc == 0.f) ? vnext : 0.f) : vnext;
      if (p.boot_kind == kBootFullAdd) vn = vn + x.boot[j];
    }
    const float nt = 1.f - term;
    a = x.r[j] + p.gamma * vn * nt - x.v[j];
    b = e.edge ? 0.f : p.gl * (1.f - done);
  }
  __device__ __forceinline__ static void emit(const Params&, const Run&, int, float xs, float, Nbr,
                                              const EdgeCtx&, float& o0, float&) {
    o0 = xs;
  }
};

// =========================================================================
// V-trace -- src/rl_triton/kernels/vtrace_fused.py:98-196 (flat) and
// src/rl_triton/ops/vtrace.py:161-201 (chunked).
//   rho = min(rho_bar, e^{lpt-lpb}), c = min(c_bar, .)
//   a = rho*(r + gamma*v_next*(1-term) - v),  b = gamma*c*(1-done)
//   targets = Delta + v;  adv = rho*(r + gamma*vs_next*(1-term) - v)
// vs_next = vs[t+1] = Delta[t+1] + v[t+1]; the solved Delta[t+1] is exactly the
// carry that enters element t, so no store/reload round trip is needed.
// =========================================================================
template <class InT>
struct VtraceAlg : NoStage {
  static constexpr bool kBackward = true;
  static constexpr bool kNeedsNbr = true;
  static constexpr int kVec = InTraits<InT>::kVec;
  static constexpr int kOuts = 2;
  struct Params {
    const InT *lpt, *lpb, *v, *r, *term, *trunc, *boot;
    const float* boot_row;
    const float* halo;
    float* out0;  // targets
    float* out1;  // advantages
    int boot_kind;
    float gamma, rho_bar, c_bar;
  };
  struct Run {
    float lpt[kVec], lpb[kVec], v[kVec], r[kVec], term[kVec], trunc[kVec], boot[kVec];
  };
  using Nbr = float;
  __device__ __forceinline__ static void load(const Params& p, int64_t i, int64_t M, bool full, Run& x,
                                              const unsigned char*, int) {
    load_run<InT, kVec>(p.lpt, i, M, full, 0.f, x.lpt);
    load_run<InT, kVec>(p.lpb, i, M, full, 0.f, x.lpb);
    load_run<InT, kVec>(p.v, i, M, full, 0.f, x.v);
    load_run<InT, kVec>(p.r, i, M, full, 0.f, x.r);
    load_run<InT, kVec>(p.term, i, M, full, 1.f, x.term);
    if (p.trunc) load_run<InT, kVec>(p.trunc, i, M, full, 0.f, x.trunc);
    else {
#pragma unroll
      for (int k = 0; k < kVec; ++k) x.trunc[k] = 0.f;
    }
    if (p.boot && p.boot_kind >= kBootFullAdd) load_run<InT, kVec>(p.boot, i, M, full, 0.f, x.boot);
    else {
#pragma unroll
      for (int k = 0; k < kVec; ++k) x.boot[k] = 0.f;
    }
  }
  __device__ __forceinline__ static Nbr nbr_at(const Run& x, int j) { return x.v[j]; }
  __device__ __forceinline__ static Nbr nbr_global(const Params& p, int64_t i) {
    return InTraits<InT>::scalar(p.v, i);
  }
  __device__ __forceinline__ static Nbr nbr_halo(const Params& p, int64_t row) { return p.halo[row]; }
  __device__ __forceinline__ static float window_value(const Params& p, const Run& x, int j, const EdgeCtx& e) {
    if (p.boot_kind == kBootNone) return 0.f;
    if (p.boot_kind == kBootRow) return p.boot_row[e.row];
    if (p.boot_kind == kBootLastCol) return InTraits<InT>::scalar(p.boot, e.i);  // column T-1 only
    return x.boot[j];
  }
  __device__ __forceinline__ static void coeff(const Params& p, Run& x, int j, Nbr vnext, const EdgeCtx& e,
                                               float& a, float& b) {
    const float ratio = expf(x.lpt[j] - x.lpb[j]);
    const float rho = fminf(ratio, p.rho_bar);
    const float c = fminf(ratio, p.c_bar);
    x.lpt[j] = rho;  // keep rho for the advantage
    const float term = x.term[j];
    const float trunc = x.trunc[j];
    const float done = p.trunc ? fminf(term + trunc, 1.f) : term;
    float vn;
    if (e.edge && e.global) {
      vn = window_value(p, x, j, e);
    } else {
      // kernels/vtrace_fused.py:120-122 (masked + additive bootstrap)
      vn = p.trunc ? ((trunc == 0.f) ? vnext : 0.f) : vnext;
      if (p.boot_kind == kBootFullAdd) vn = vn + x.boot[j];
    }
    const float nt = 1.f - term;
    a = rho * (x.r[j] + p.gamma * vn * nt - x.v[j]);
    b = e.edge ? 0.f : p.gamma * c * (1.f - done);
  }
  __device__ __forceinline__ static void emit(const Params& p, const Run& x, int j, float xs, float xnext,
                                              Nbr vnext, const EdgeCtx& e, float& o0, float& o1) {
    const float rho = x.lpt[j];
    const float term = x.term[j];
    float vsn;
    if (e.edge && e.global) {
      vsn = window_value(p, x, j, e);
    } else {
      // kernels/vtrace_fused.py:179-181
      vsn = p.trunc ? ((x.trunc[j] == 0.f) ? (xnext + vnext) : 0.f) : (xnext + vnext);
      if (p.boot_kind == kBootFullAdd) vsn = vsn + x.boot[j];
    }
    o0 = xs + x.v[j];
    o1 = rho * (x.r[j] + p.gamma * vsn * (1.f - term) - x.v[j]);
  }
};

// =========================================================================
// Retrace(lambda) -- src/rl_triton/kernels/retrace_fused.py:112-201 and
// src/rl_triton/ops/retrace.py:177-196.
//   E = sum_a pi[t,a]*Qn[t,a];  pi_a = pi[t, a_t];  a = r + gamma*E*(1-term) - Q
//   b = gamma * lambda*min(c_bar, pi_a[t+1]/mu[t+1]) * (1-done),  c[T] := 0
//   targets = Delta + Q;  adv = min(rho_bar, pi_a/mu) * (r + gamma*Q_ret[t+1]*(1-term) - Q)
// with Q_ret[T] := 0 and no truncation masking of Q_ret[t+1] (the reference's
// own convention, kernels/retrace_fused.py:197-201).
// The [N,T,A] tensors are staged per warp into shared memory with one bulk
// copy each (cp.async.bulk, no multicast), and E / pi_a are reduced there.
// =========================================================================
struct RetraceAlg {
  static constexpr bool kBackward = true;
  static constexpr bool kNeedsNbr = true;
  static constexpr int kVec = 4;
  static constexpr int kOuts = 2;
  struct Params {
    const float *pi, *mu, *q, *nq, *r, *term, *trunc;
    const int64_t* act;
    float* out0;
    float* out1;
    int64_t A;
    float gamma, lam, c_bar, rho_bar;
    int warp_elems;  // elements per warp span (staging layout)
  };
  struct Run {
    float e[kVec], pa[kVec], mu[kVec], q[kVec], r[kVec], term[kVec], trunc[kVec];
  };
  struct Nbr {
    float pa, mu, q;
  };

  __device__ __forceinline__ static float pi_at(const float* pi_row, int64_t a, int64_t A) {
    return (a >= 0 && a < A) ? pi_row[a] : 0.f;
  }

  // Stage the warp's [warp_elems, A] spans of pi and Qn and its actions into
  // shared memory, then reduce E and pi_a per element (striped over lanes).
  __device__ static void stage(const Params& p, const Geom& g, int64_t wbase, int warp_elems, int lane,
                               unsigned char* smem, uint64_t* mbar, WsHeader* hdr) {
    if (g.smem_per_warp == 0) return;  // direct (unstaged) mode for large A
    const int64_t A = p.A;
    float* pi_s = reinterpret_cast<float*>(smem);
    float* nq_s = pi_s + (int64_t)warp_elems * A;
    float* e_s = nq_s + (int64_t)warp_elems * A;
    float* pa_s = e_s + warp_elems;
    int64_t* act_s = reinterpret_cast<int64_t*>(pa_s + warp_elems);
    const bool full = wbase + warp_elems <= g.M;
    if (full && g.tma) {
      const unsigned mb = (unsigned)__cvta_generic_to_shared(mbar);
      if (lane == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(mb) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
      }
      __syncwarp();
      if (lane == 0) {
        const unsigned span = (unsigned)(warp_elems * A * 4);
        const unsigned abytes = (unsigned)(warp_elems * 8);
        const unsigned total = 2u * span + abytes;
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(mb), "r"(total) : "memory");
        const unsigned d0 = (unsigned)__cvta_generic_to_shared(pi_s);
        const unsigned d1 = (unsigned)__cvta_generic_to_shared(nq_s);
        const unsigned d2 = (unsigned)__cvta_generic_to_shared(act_s);
        asm volatile(
            "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(d0),
            "l"(p.pi + wbase * A), "r"(span), "r"(mb)
            : "memory");
        asm volatile(
            "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(d1),
            "l"(p.nq + wbase * A), "r"(span), "r"(mb)
            : "memory");
        asm volatile(
            "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(d2),
            "l"(p.act + wbase), "r"(abytes), "r"(mb)
            : "memory");
      }
      // Bounded wait for phase 0 of the barrier.
      unsigned done = 0;
      for (unsigned it = 0; it < kSpinLimit; ++it) {
        asm volatile(
            "{\n\t.reg .pred P;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 P, [%1], 0;\n\t"
            "selp.u32 %0, 1, 0, P;\n\t}"
            : "=r"(done)
            : "r"(mb)
            : "memory");
        if (done) break;
      }
      if (!done) {
        if (lane == 0) atomicOr(&hdr->error, 2u);
        // Fill with zeros so the rest of the kernel stays well defined.
        for (int idx = lane; idx < warp_elems; idx += 32) { e_s[idx] = 0.f; pa_s[idx] = 0.f; }
        __syncwarp();
        return;
      }
    } else {
      for (int idx = lane; idx < warp_elems; idx += 32) {
        const int64_t i = wbase + idx;
        if (i < g.M) {
          for (int64_t k = 0; k < A; ++k) {
            pi_s[idx * A + k] = __ldg(p.pi + i * A + k);
            nq_s[idx * A + k] = __ldg(p.nq + i * A + k);
          }
          act_s[idx] = __ldg(p.act + i);
        } else {
          for (int64_t k = 0; k < A; ++k) { pi_s[idx * A + k] = 0.f; nq_s[idx * A + k] = 0.f; }
          act_s[idx] = 0;
        }
      }
      __syncwarp();
    }
    if (A == 4) {
      const float4* pi4 = reinterpret_cast<const float4*>(pi_s);
      const float4* nq4 = reinterpret_cast<const float4*>(nq_s);
      for (int idx = lane; idx < warp_elems; idx += 32) {
        const float4 pv = pi4[idx];
        const float4 qv = nq4[idx];
        float e = pv.x * qv.x;
        e = fmaf(pv.y, qv.y, e);
        e = fmaf(pv.z, qv.z, e);
        e = fmaf(pv.w, qv.w, e);
        const int64_t a = act_s[idx];
        const float pw[4] = {pv.x, pv.y, pv.z, pv.w};
        float pa = 0.f;
#pragma unroll
        for (int k = 0; k < 4; ++k) pa = (a == k) ? pw[k] : pa;
        e_s[idx] = e;
        pa_s[idx] = pa;
      }
    } else {
      for (int idx = lane; idx < warp_elems; idx += 32) {
        const float* prow = pi_s + idx * A;
        const float* qrow = nq_s + idx * A;
        float e = 0.f;
        for (int64_t k = 0; k < A; ++k) e = fmaf(prow[k], qrow[k], e);
        e_s[idx] = e;
        pa_s[idx] = pi_at(prow, act_s[idx], A);
      }
    }
    __syncwarp();
  }

  __device__ __forceinline__ static void load(const Params& p, int64_t i, int64_t M, bool full, Run& x,
                                              const unsigned char* smem, int local) {
    if (smem) {
      const float* e_s = reinterpret_cast<const float*>(smem) + (int64_t)p.warp_elems * 2 * p.A;
      const float* pa_s = e_s + p.warp_elems;
      const float4 ev = *reinterpret_cast<const float4*>(e_s + local);
      const float4 pv = *reinterpret_cast<const float4*>(pa_s + local);
      x.e[0] = ev.x; x.e[1] = ev.y; x.e[2] = ev.z; x.e[3] = ev.w;
      x.pa[0] = pv.x; x.pa[1] = pv.y; x.pa[2] = pv.z; x.pa[3] = pv.w;
    } else if (p.A == 4 && full) {
      // Row-kernel path, A = 4: one 16-byte vector per element of pi and Qn,
      // the four int64 actions as two 16-byte vectors.
      const longlong2 a01 = __ldcs(reinterpret_cast<const longlong2*>(p.act + i));
      const longlong2 a23 = __ldcs(reinterpret_cast<const longlong2*>(p.act + i + 2));
      const int64_t acts[4] = {a01.x, a01.y, a23.x, a23.y};
#pragma unroll
      for (int k = 0; k < kVec; ++k) {
        const float4 pv = __ldcs(reinterpret_cast<const float4*>(p.pi + (i + k) * 4));
        const float4 qv = __ldcs(reinterpret_cast<const float4*>(p.nq + (i + k) * 4));
        float e = pv.x * qv.x;
        e = fmaf(pv.y, qv.y, e);
        e = fmaf(pv.z, qv.z, e);
        e = fmaf(pv.w, qv.w, e);
        const int64_t a = acts[k];
        float pa = 0.f;
        pa = (a == 0) ? pv.x : pa;
        pa = (a == 1) ? pv.y : pa;
        pa = (a == 2) ? pv.z : pa;
        pa = (a == 3) ? pv.w : pa;
        x.e[k] = e;
        x.pa[k] = pa;
      }
    } else {
#pragma unroll
      for (int k = 0; k < kVec; ++k) {
        const int64_t ii = i + k;
        float e = 0.f, pa = 0.f;
        if (ii < M) {
          const float* prow = p.pi + ii * p.A;
          const float* qrow = p.nq + ii * p.A;
          for (int64_t c = 0; c < p.A; ++c) e = fmaf(__ldg(prow + c), __ldg(qrow + c), e);
          const int64_t a = __ldg(p.act + ii);
          pa = (a >= 0 && a < p.A) ? __ldg(prow + a) : 0.f;
        }
        x.e[k] = e;
        x.pa[k] = pa;
      }
    }
    load_run<float, kVec>(p.mu, i, M, full, 1.f, x.mu);
    load_run<float, kVec>(p.q, i, M, full, 0.f, x.q);
    load_run<float, kVec>(p.r, i, M, full, 0.f, x.r);
    load_run<float, kVec>(p.term, i, M, full, 1.f, x.term);
    load_run<float, kVec>(p.trunc, i, M, full, 0.f, x.trunc);
  }
  __device__ __forceinline__ static Nbr nbr_at(const Run& x, int j) { return Nbr{x.pa[j], x.mu[j], x.q[j]}; }
  __device__ __forceinline__ static Nbr nbr_global(const Params& p, int64_t i) {
    const int64_t a = __ldg(p.act + i);
    const float pa = (a >= 0 && a < p.A) ? __ldg(p.pi + i * p.A + a) : 0.f;
    return Nbr{pa, __ldg(p.mu + i), __ldg(p.q + i)};
  }
  __device__ __forceinline__ static Nbr nbr_halo(const Params&, int64_t) { return Nbr{0.f, 1.f, 0.f}; }
  __device__ __forceinline__ static void coeff(const Params& p, Run& x, int j, Nbr nx, const EdgeCtx& e,
                                               float& a, float& b) {
    const float term = x.term[j];
    const float done = fminf(term + x.trunc[j], 1.f);
    a = x.r[j] + p.gamma * x.e[j] * (1.f - term) - x.q[j];
    if (e.edge) {
      b = 0.f;
    } else {
      const float c_next = p.lam * fminf(nx.pa / nx.mu, p.c_bar);
      b = p.gamma * c_next * (1.f - done);
    }
  }
  __device__ __forceinline__ static void emit(const Params& p, const Run& x, int j, float xs, float xnext,
                                              Nbr nx, const EdgeCtx& e, float& o0, float& o1) {
    const float qn = e.edge ? 0.f : (xnext + nx.q);
    const float rho = fminf(x.pa[j] / x.mu[j], p.rho_bar);
    o0 = xs + x.q[j];
    o1 = rho * (x.r[j] + p.gamma * qn * (1.f - x.term[j]) - x.q[j]);
  }
};

// =========================================================================
// TD(lambda) returns -- src/rl_triton/kernels/lambda_returns_fused.py:62-89.
//   a = r + gamma*(1-lambda)*(1-done)*nv [+ gamma*trunc*boot],  b = gamma*lambda*(1-done)
// carry at the window end = bootstrap[:, -1] (or 0).
// =========================================================================
template <class InT>
struct LambdaAlg : NoStage {
  static constexpr bool kBackward = true;
  static constexpr bool kNeedsNbr = false;
  static constexpr int kVec = InTraits<InT>::kVec;
  static constexpr int kOuts = 1;
  struct Params {
    const InT *r, *nv, *term, *trunc, *boot;
    float* out0;
    float* out1;
    int boot_kind;
    float gamma, g1l, gl;  // gamma, gamma*(1-lambda), gamma*lambda
  };
  struct Run {
    float r[kVec], nv[kVec], term[kVec], trunc[kVec], boot[kVec];
  };
  using Nbr = float;
  __device__ __forceinline__ static void load(const Params& p, int64_t i, int64_t M, bool full, Run& x,
                                              const unsigned char*, int) {
    load_run<InT, kVec>(p.r, i, M, full, 0.f, x.r);
    load_run<InT, kVec>(p.nv, i, M, full, 0.f, x.nv);
    load_run<InT, kVec>(p.term, i, M, full, 1.f, x.term);
    if (p.trunc) load_run<InT, kVec>(p.trunc, i, M, full, 0.f, x.trunc);
    else {
#pragma unroll
      for (int k = 0; k < kVec; ++k) x.trunc[k] = 0.f;
    }
    if (p.boot && p.boot_kind >= kBootFullAdd) load_run<InT, kVec>(p.boot, i, M, full, 0.f, x.boot);
    else {
#pragma unroll
      for (int k = 0; k < kVec; ++k) x.boot[k] = 0.f;
    }
  }
  __device__ __forceinline__ static Nbr nbr_at(const Run&, int) { return 0.f; }
  __device__ __forceinline__ static Nbr nbr_global(const Params&, int64_t) { return 0.f; }
  __device__ __forceinline__ static Nbr nbr_halo(const Params&, int64_t) { return 0.f; }
  __device__ __forceinline__ static void coeff(const Params& p, Run& x, int j, Nbr, const EdgeCtx& e, float& a,
                                               float& b) {
    const float trunc = x.trunc[j];
    const float done = p.trunc ? fminf(x.term[j] + trunc, 1.f) : x.term[j];
    const float nd = 1.f - done;
    a = x.r[j] + p.g1l * nd * x.nv[j];
    if (p.boot_kind == kBootFullAdd) a = a + p.gamma * trunc * x.boot[j];
    b = p.gl * nd;
    if (e.edge) {
      if (e.global) {
        if (p.boot_kind == kBootFullAdd && p.boot) a = fmaf(b, x.boot[j], a);
        else if (p.boot_kind == kBootLastCol) a = fmaf(b, InTraits<InT>::scalar(p.boot, e.i), a);
      }
      b = 0.f;
    }
  }
  __device__ __forceinline__ static void emit(const Params&, const Run&, int, float xs, float, Nbr,
                                              const EdgeCtx&, float& o0, float&) {
    o0 = xs;
  }
};

// =========================================================================
// Discounted returns -- src/rl_triton/kernels/discounted_returns_fused.py:56-82.
//   a = r [+ gamma*trunc*boot],  b = gamma*(1-done);  carry = bootstrap[:, -1] (or 0)
// =========================================================================
template <class InT>
struct DiscountedAlg : NoStage {
  static constexpr bool kBackward = true;
  static constexpr bool kNeedsNbr = false;
  static constexpr int kVec = InTraits<InT>::kVec;
  static constexpr int kOuts = 1;
  struct Params {
    const InT *r, *term, *trunc, *boot;
    float* out0;
    float* out1;
    int boot_kind;
    float gamma;
  };
  struct Run {
    float r[kVec], term[kVec], trunc[kVec], boot[kVec];
  };
  using Nbr = float;
  __device__ __forceinline__ static void load(const Params& p, int64_t i, int64_t M, bool full, Run& x,
                                              const unsigned char*, int) {
    load_run<InT, kVec>(p.r, i, M, full, 0.f, x.r);
    load_run<InT, kVec>(p.term, i, M, full, 1.f, x.term);
    if (p.trunc) load_run<InT, kVec>(p.trunc, i, M, full, 0.f, x.trunc);
    else {
#pragma unroll
      for (int k = 0; k < kVec; ++k) x.trunc[k] = 0.f;
    }
    if (p.boot && p.boot_kind >= kBootFullAdd) load_run<InT, kVec>(p.boot, i, M, full, 0.f, x.boot);
    else {
#pragma unroll
      for (int k = 0; k < kVec; ++k) x.boot[k] = 0.f;
    }
  }
  __device__ __forceinline__ static Nbr nbr_at(const Run&, int) { return 0.f; }
  __device__ __forceinline__ static Nbr nbr_global(const Params&, int64_t) { return 0.f; }
  __device__ __forceinline__ static Nbr nbr_halo(const Params&, int64_t) { return 0.f; }
  __device__ __forceinline__ static void coeff(const Params& p, Run& x, int j, Nbr, const EdgeCtx& e, float& a,
                                               float& b) {
    const float trunc = x.trunc[j];
    const float done = p.trunc ? fminf(x.term[j] + trunc, 1.f) : x.term[j];
    a = x.r[j];
    if (p.boot_kind == kBootFullAdd) a = a + p.gamma * trunc * x.boot[j];
    b = p.gamma * (1.f - done);
    if (e.edge) {
      if (e.global) {
        if (p.boot_kind == kBootFullAdd && p.boot) a = fmaf(b, x.boot[j], a);
        else if (p.boot_kind == kBootLastCol) a = fmaf(b, InTraits<InT>::scalar(p.boot, e.i), a);
      }
      b = 0.f;
    }
  }
  __device__ __forceinline__ static void emit(const Params&, const Run&, int, float xs, float, Nbr,
                                              const EdgeCtx&, float& o0, float&) {
    o0 = xs;
  }
};

// =========================================================================
// Forward scans.
// Eligibility traces -- src/rl_triton/kernels/eligibility_traces_fused.py:66-84:
//   z[t] = g[t] + gamma*lambda*(1-done[t-1]) z[t-1], done[-1] := 0, z[-1] = seed
// Episodic prefix sum -- src/rl_triton/kernels/prefix_sum_fused.py:62-84:
//   C[t] = x[t] + (1-done[t-1]) C[t-1]  ("ends_at")  or  (1-done[t]) ("starts_at")
// Both have the form a = x[t], b = k*(1 - flag), handled by one policy.
// =========================================================================
template <class InT>
struct ForwardAlg : NoStage {
  static constexpr bool kBackward = false;
  static constexpr bool kNeedsNbr = true;
  static constexpr int kVec = InTraits<InT>::kVec;
  static constexpr int kOuts = 1;
  struct Params {
    const InT *x, *done;
    const float* seed;
    const float* halo;  // done[t0-1] per row at a time-split cut
    float* out0;
    float* out1;
    float k;            // gamma*lambda for traces, 1 for the prefix sum
    int prev;           // 1: gate on done[t-1] ("ends_at" / traces), 0: on done[t]
  };
  struct Run {
    float x[kVec], done[kVec];
  };
  using Nbr = float;  // done of the previous element
  __device__ __forceinline__ static void load(const Params& p, int64_t i, int64_t M, bool full, Run& r,
                                              const unsigned char*, int) {
    load_run<InT, kVec>(p.x, i, M, full, 0.f, r.x);
    load_run<InT, kVec>(p.done, i, M, full, 0.f, r.done);
  }
  __device__ __forceinline__ static Nbr nbr_at(const Run& r, int j) { return r.done[j]; }
  __device__ __forceinline__ static Nbr nbr_global(const Params& p, int64_t i) {
    return InTraits<InT>::scalar(p.done, i);
  }
  __device__ __forceinline__ static Nbr nbr_halo(const Params& p, int64_t row) { return p.halo[row]; }
  __device__ __forceinline__ static void coeff(const Params& p, Run& r, int j, Nbr dprev, const EdgeCtx& e,
                                               float& a, float& b) {
    float flag;
    if (p.prev) flag = (e.edge && e.global) ? 0.f : dprev;
    else flag = r.done[j];
    a = r.x[j];
    b = p.k * (1.f - flag);
    if (e.edge) {
      if (e.global && p.seed) a = fmaf(b, p.seed[e.row], a);
      b = 0.f;
    }
  }
  __device__ __forceinline__ static void emit(const Params&, const Run&, int, float xs, float, Nbr,
                                              const EdgeCtx&, float& o0, float&) {
    o0 = xs;
  }
};

// =========================================================================
// Generic affine scan on materialised coefficients (fp32) --
// src/rl_triton/kernels/scan.py:39-138 and kernels/scan_chunked.py:7-85.
// =========================================================================
template <bool BWD>
struct AffineAlg : NoStage {
  static constexpr bool kBackward = BWD;
  static constexpr bool kNeedsNbr = false;
  static constexpr int kVec = 4;
  static constexpr int kOuts = 1;
  struct Params {
    const float *u, *v;
    const float* carry;
    float* out0;
    float* out1;
  };
  struct Run {
    float u[kVec], v[kVec];
  };
  using Nbr = float;
  __device__ __forceinline__ static void load(const Params& p, int64_t i, int64_t M, bool full, Run& r,
                                              const unsigned char*, int) {
    load_run<float, kVec>(p.u, i, M, full, 0.f, r.u);
    load_run<float, kVec>(p.v, i, M, full, 1.f, r.v);
  }
  __device__ __forceinline__ static Nbr nbr_at(const Run&, int) { return 0.f; }
  __device__ __forceinline__ static Nbr nbr_global(const Params&, int64_t) { return 0.f; }
  __device__ __forceinline__ static Nbr nbr_halo(const Params&, int64_t) { return 0.f; }
  __device__ __forceinline__ static void coeff(const Params& p, Run& r, int j, Nbr, const EdgeCtx& e, float& a,
                                               float& b) {
    a = r.u[j];
    b = r.v[j];
    if (e.edge) {
      if (e.global && p.carry) a = fmaf(b, p.carry[e.row], a);
      b = 0.f;
    }
  }
  __device__ __forceinline__ static void emit(const Params&, const Run&, int, float xs, float, Nbr,
                                              const EdgeCtx&, float& o0, float&) {
    o0 = xs;
  }
};

}  // namespace rls
