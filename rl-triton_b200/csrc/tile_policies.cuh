// tile_policies.cuh -- per-estimator element rules for the TMA-staged tile kernel.
//
// A policy names the input streams staged per tile (`sptr`, `esz`), turns one
// element into its affine map (`coeff`: x = a + b * x_carry) and turns the
// solved state back into outputs (`emit`).  The formulas and their float
// operation order are those of the reference's fused Triton kernels (file:line
// per policy), so results agree with its sequential references to a few ulp.
//
// Variants.  Whatever touches every element is a template parameter -- TR:
// truncations present; PB: per-step bootstrap values (1 additive, 2 selected
// at truncations); PREV: the forward decay is gated by done[t-1] -- so the hot
// loop has no runtime branches.  What only touches row edges (window values
// from last_value / the last bootstrap column, seeds, time-split halos) is
// read at run time inside the out-of-line edge helpers.
//
// Edge rule shared by all policies: at a backward row's last column (forward:
// first column) b = 0 and the row's boundary value is folded into a; at a
// time-split cut (edge, not global) the neighbour comes from the per-row halo
// and the true carry is applied later by the segment fix-up.
//
// The Params structs are shared with the register kernels (algs.cuh).
#pragma once
#include "tile_kernel.cuh"

namespace rls {

template <class InT>
__host__ __device__ constexpr int vec_of() { return 16 / (int)sizeof(InT); }

// Common part of the policies whose staged streams are all [N, T] of one type.
template <class InT_, int NSTREAMS>
struct HomogeneousStreams {
  using InT = InT_;
  static constexpr int kNS = NSTREAMS;
  static constexpr int kNI = NSTREAMS;
  static constexpr bool kElemLoad = false;
  // Decays that are only ever 0 or 1 (running sums): the flat2 look-back may
  // stop at any published inclusive value.
  template <class Params>
  __device__ __forceinline__ static bool unit_decay(const Params&) { return false; }
  template <int K>
  __host__ __device__ static constexpr int vec() { return (K % vec_of<InT>() == 0) ? vec_of<InT>() : 1; }
  template <class Params>
  __host__ __device__ static int esz(const Params&, int) { return (int)sizeof(InT); }
  template <int VEC, class Params>
  __device__ __forceinline__ static void load(const Params&, const SView& s, int idx0, int64_t,
                                              float (&in)[NSTREAMS][VEC]) {
    load_streams<InT, NSTREAMS, VEC>(s, idx0, in);
  }
};

// ===========================================================================
// GAE -- src/rl_triton/kernels/gae.py:62-180, src/rl_triton/ops/gae.py:192-215.
//   delta = r + gamma*(1-term)*v_next - v,  b = gamma*lambda*(1-done)
// Streams: r, v, term, [trunc], [boot].
// ===========================================================================
template <class InT, bool TR, int PB>
struct GaeT : HomogeneousStreams<InT, 3 + (TR ? 1 : 0) + (PB ? 1 : 0)> {
  using Base = HomogeneousStreams<InT, 3 + (TR ? 1 : 0) + (PB ? 1 : 0)>;
  using Params = typename GaeAlg<InT>::Params;
  using Nbr = float;
  static constexpr bool kBackward = true, kNeedsNbr = true, kNextInEmit = false, kEmitReads = false;
  static constexpr int kOuts = 1, kOutSlots = 1, kScratch = 0;
  static constexpr int iR = 0, iV = 1, iTerm = 2, iTrunc = 3, iBoot = TR ? 4 : 3;
  __host__ __device__ static const void* sptr(const Params& p, int k) {
    if (k == iR) return p.r;
    if (k == iV) return p.v;
    if (k == iTerm) return p.term;
    if (TR && k == iTrunc) return p.trunc;
    return p.boot;
  }
  template <int VEC>
  __device__ __forceinline__ static Nbr nbr_of(const float (&in)[Base::kNI][VEC], int e) { return in[iV][e]; }
  __device__ __forceinline__ static Nbr nbr_smem(const Params&, const SView& s, int idx, int64_t) {
    return s.f<InT>(iV, idx);
  }
  __device__ __forceinline__ static Nbr nbr_global(const Params& p, int64_t i) { return gload(p.v, i); }

  __device__ __forceinline__ static float vnext_rule(float vnext, float trunc, float boot) {
    if constexpr (PB == 2) {
      return (trunc == 1.f) ? boot : vnext;  // kernels/gae.py:153-154
    } else {
      float vn = TR ? ((trunc == 0.f) ? vnext : 0.f) : vnext;  // ops/gae.py:200-205
      if constexpr (PB == 1) vn = vn + boot;
      return vn;
    }
  }
  // Next-state value at a row edge: the window value (kernels/gae.py:86-96,
  // 153-177) or, at a time-split cut, the next segment's first value.
  __device__ __noinline__ static float edge_vn(const float* boot_row, const InT* boot, int kind, const float* halo,
                                               EdgeLoc L, int j, float trunc, float boot_e) {
    if (L.glob) {
      if (PB) return boot_e;
      if (kind == kBootRow) return boot_row[L.row(j)];
      if (kind >= kBootLastCol) return gload(boot, L.gi(j));
      return 0.f;
    }
    return vnext_rule(halo[L.row(j)], trunc, boot_e);
  }
  template <int VEC>
  __device__ __forceinline__ static void coeff(const Params& p, const float (&in)[Base::kNI][VEC], int e,
                                               Nbr vnext, bool edge, const EdgeLoc& L, int j, float*, float& a,
                                               float& b) {
    const float term = in[iTerm][e];
    const float trunc = TR ? in[iTrunc][e] : 0.f;
    const float boot = PB ? in[iBoot][e] : 0.f;
    const float done = TR ? fminf(term + trunc, 1.f) : term;
    float vn = vnext_rule(vnext, trunc, boot);
    if (edge) vn = edge_vn(p.boot_row, p.boot, p.boot_kind, p.halo, L, j, trunc, boot);
    const float nt = 1.f - term;
    a = in[iR][e] + p.gamma * vn * nt - in[iV][e];
    b = edge ? 0.f : p.gl * (1.f - done);
  }
  template <int VEC>
  __device__ __forceinline__ static void emit(const Params&, const float (&)[Base::kNI][VEC], int, float x, float,
                                              Nbr, bool, const EdgeLoc&, int, const float*, float& o0, float&) {
    o0 = x;
  }
};

// ===========================================================================
// V-trace -- src/rl_triton/kernels/vtrace_fused.py:98-196, ops/vtrace.py:161-201.
//   rho = min(rho_bar, e^{lpt-lpb}), c = min(c_bar, .)
//   a = rho*(r + gamma*v_next*(1-term) - v),  b = gamma*c*(1-done)
//   targets = Delta + v;  adv = rho*(r + gamma*vs_next*(1-term) - v)
// vs_next = Delta[t+1] + v[t+1]: Delta[t+1] is exactly the state the walk held
// before element t, so no store / barrier / reload round trip is needed.
// Streams: lpt, lpb, v, r, term, [trunc], [boot].  rho waits in scratch.
// ===========================================================================
template <class InT, bool TR, bool PB>
struct VtraceT : HomogeneousStreams<InT, 5 + (TR ? 1 : 0) + (PB ? 1 : 0)> {
  using Base = HomogeneousStreams<InT, 5 + (TR ? 1 : 0) + (PB ? 1 : 0)>;
  using Params = typename VtraceAlg<InT>::Params;
  using Nbr = float;
  static constexpr bool kBackward = true, kNeedsNbr = true, kNextInEmit = false, kEmitReads = true;
  static constexpr int kOuts = 2, kOutSlots = 2, kScratch = 1;
  static constexpr int iLpt = 0, iLpb = 1, iV = 2, iR = 3, iTerm = 4, iTrunc = 5, iBoot = TR ? 6 : 5;
  // Streams the advantage reads again in pass 2 (all but the log-probs).
  static constexpr unsigned kEmitMask = ~((1u << iLpt) | (1u << iLpb));
  __host__ __device__ static const void* sptr(const Params& p, int k) {
    switch (k) {
      case iLpt: return p.lpt;
      case iLpb: return p.lpb;
      case iV: return p.v;
      case iR: return p.r;
      case iTerm: return p.term;
      default: return (TR && k == iTrunc) ? (const void*)p.trunc : (const void*)p.boot;
    }
  }
  template <int VEC>
  __device__ __forceinline__ static Nbr nbr_of(const float (&in)[Base::kNI][VEC], int e) { return in[iV][e]; }
  __device__ __forceinline__ static Nbr nbr_smem(const Params&, const SView& s, int idx, int64_t) {
    return s.f<InT>(iV, idx);
  }
  __device__ __forceinline__ static Nbr nbr_global(const Params& p, int64_t i) { return gload(p.v, i); }
  __device__ __forceinline__ static float next_rule(float vnext, float trunc, float boot) {
    float vn = TR ? ((trunc == 0.f) ? vnext : 0.f) : vnext;  // kernels/vtrace_fused.py:120-122, 179-181
    if constexpr (PB) vn = vn + boot;
    return vn;
  }
  // Window value at the row end (V-trace has no time split: edges are global).
  __device__ __noinline__ static float edge_wv(const float* boot_row, const InT* boot, int kind, EdgeLoc L, int j,
                                               float boot_e) {
    if (PB) return boot_e;
    if (kind == kBootRow) return boot_row[L.row(j)];
    if (kind >= kBootLastCol) return gload(boot, L.gi(j));
    return 0.f;
  }
  template <int VEC>
  __device__ __forceinline__ static void coeff(const Params& p, const float (&in)[Base::kNI][VEC], int e,
                                               Nbr vnext, bool edge, const EdgeLoc& L, int j, float* scratch,
                                               float& a, float& b) {
    const float ratio = expf(in[iLpt][e] - in[iLpb][e]);
    const float rho = fminf(ratio, p.rho_bar);
    const float c = fminf(ratio, p.c_bar);
    *scratch = rho;
    const float term = in[iTerm][e];
    const float trunc = TR ? in[iTrunc][e] : 0.f;
    const float boot = PB ? in[iBoot][e] : 0.f;
    const float done = TR ? fminf(term + trunc, 1.f) : term;
    float vn = next_rule(vnext, trunc, boot);
    if (edge) vn = edge_wv(p.boot_row, p.boot, p.boot_kind, L, j, boot);
    const float nt = 1.f - term;
    a = rho * (in[iR][e] + p.gamma * vn * nt - in[iV][e]);
    b = edge ? 0.f : p.gamma * c * (1.f - done);
  }
  template <int VEC>
  __device__ __forceinline__ static void emit(const Params& p, const float (&in)[Base::kNI][VEC], int e, float x,
                                              float xnext, Nbr vnext, bool edge, const EdgeLoc& L, int j,
                                              const float* scratch, float& o0, float& o1) {
    const float rho = *scratch;
    const float v = in[iV][e];
    const float trunc = TR ? in[iTrunc][e] : 0.f;
    const float boot = PB ? in[iBoot][e] : 0.f;
    float vsn = next_rule(xnext + vnext, trunc, boot);
    if (edge) vsn = edge_wv(p.boot_row, p.boot, p.boot_kind, L, j, boot);
    o0 = x + v;
    o1 = rho * (in[iR][e] + p.gamma * vsn * (1.f - in[iTerm][e]) - v);
  }
};

// ===========================================================================
// Retrace(lambda) -- src/rl_triton/kernels/retrace_fused.py:112-201,
// src/rl_triton/ops/retrace.py:177-196.
//   E = sum_a pi[t,a]*Qn[t,a];  a = r + gamma*E*(1-term) - Q
//   b = gamma * lambda*min(c_bar, pi_a[t+1]/mu[t+1]) * (1-done)
//   targets = Delta + Q;  adv = min(rho_bar, pi_a/mu) * (r + gamma*Q_ret[t+1]*(1-term) - Q)
// with Q_ret[T] := 0 and no truncation masking of Q_ret[t+1].
// Staged streams: [pi, Qn] (A floats per step, while STAGED), actions (int64),
// mu, q, r, term, trunc.  Per-element values: E, pi_a, mu, q, r, term, trunc.
// ===========================================================================
template <bool STAGED>
struct RetraceT {
  using Params = RetraceAlg::Params;
  using Nbr = RetraceAlg::Nbr;
  using InT = float;
  static constexpr bool kBackward = true, kNeedsNbr = true, kEmitReads = true, kElemLoad = true;
  // Q_ret[t+1] enters the advantage even at a truncated step (b == 0 there),
  // so only a row edge makes the incoming carry irrelevant.
  static constexpr bool kNextInEmit = true;
  static constexpr int kOuts = 2, kOutSlots = 2, kScratch = 1;
  static constexpr int kNS = STAGED ? 8 : 6;
  static constexpr int kNI = 7;
  static constexpr int sPi = 0, sNq = 1, sAct = STAGED ? 2 : 0, sMu = sAct + 1, sQ = sAct + 2, sR = sAct + 3,
                       sTerm = sAct + 4, sTrunc = sAct + 5;
  static constexpr int iE = 0, iPa = 1, iMu = 2, iQ = 3, iR = 4, iTerm = 5, iTrunc = 6;
  template <int K>
  __host__ __device__ static constexpr int vec() { return 1; }
  __host__ __device__ static const void* sptr(const Params& p, int k) {
    if (STAGED && k == sPi) return p.pi;
    if (STAGED && k == sNq) return p.nq;
    if (k == sAct) return p.act;
    if (k == sMu) return p.mu;
    if (k == sQ) return p.q;
    if (k == sR) return p.r;
    if (k == sTerm) return p.term;
    return p.trunc;
  }
  __host__ __device__ static int esz(const Params& p, int k) {
    if (STAGED && k <= sNq) return (int)(p.A * 4);
    return k == sAct ? 8 : 4;
  }
  __device__ __forceinline__ static float pi_at(const Params& p, const SView& s, int idx, int64_t gi, int64_t a) {
    if (a < 0 || a >= p.A) return 0.f;
    if (STAGED) return s.ld<float>(sPi, (int)(idx * p.A + a));
    return __ldg(p.pi + gi * p.A + a);
  }
  template <int VEC>
  __device__ __forceinline__ static void load(const Params& p, const SView& s, int idx, int64_t gi,
                                              float (&in)[kNI][VEC]) {
    static_assert(VEC == 1, "Retrace reads one step at a time");
    float E;
    if (STAGED && p.A == 4) {
      const float4 pv = s.ld<float4>(sPi, idx);
      const float4 qv = s.ld<float4>(sNq, idx);
      E = pv.x * qv.x;
      E = fmaf(pv.y, qv.y, E);
      E = fmaf(pv.z, qv.z, E);
      E = fmaf(pv.w, qv.w, E);
    } else if (STAGED) {
      const float* prow = reinterpret_cast<const float*>(s.st + s.off[sPi]) + (int64_t)idx * p.A;
      const float* qrow = reinterpret_cast<const float*>(s.st + s.off[sNq]) + (int64_t)idx * p.A;
      E = prow[0] * qrow[0];
      for (int64_t c = 1; c < p.A; ++c) E = fmaf(prow[c], qrow[c], E);
    } else {
      const float* prow = p.pi + gi * p.A;
      const float* qrow = p.nq + gi * p.A;
      E = __ldg(prow) * __ldg(qrow);
      for (int64_t c = 1; c < p.A; ++c) E = fmaf(__ldg(prow + c), __ldg(qrow + c), E);
    }
    in[iE][0] = E;
    in[iPa][0] = pi_at(p, s, idx, gi, s.ld<int64_t>(sAct, idx));
    in[iMu][0] = s.ld<float>(sMu, idx);
    in[iQ][0] = s.ld<float>(sQ, idx);
    in[iR][0] = s.ld<float>(sR, idx);
    in[iTerm][0] = s.ld<float>(sTerm, idx);
    in[iTrunc][0] = s.ld<float>(sTrunc, idx);
  }
  template <int VEC>
  __device__ __forceinline__ static Nbr nbr_of(const float (&in)[kNI][VEC], int e) {
    return Nbr{in[iPa][e], in[iMu][e], in[iQ][e]};
  }
  __device__ __forceinline__ static Nbr nbr_smem(const Params& p, const SView& s, int idx, int64_t gi) {
    return Nbr{pi_at(p, s, idx, gi, s.ld<int64_t>(sAct, idx)), s.ld<float>(sMu, idx), s.ld<float>(sQ, idx)};
  }
  __device__ __forceinline__ static Nbr nbr_global(const Params& p, int64_t i) {
    const int64_t a = __ldg(p.act + i);
    const float pa = (a >= 0 && a < p.A) ? __ldg(p.pi + i * p.A + a) : 0.f;
    return Nbr{pa, __ldg(p.mu + i), __ldg(p.q + i)};
  }
  template <int VEC>
  __device__ __forceinline__ static void coeff(const Params& p, const float (&in)[kNI][VEC], int e, Nbr nx,
                                               bool edge, const EdgeLoc&, int, float* scratch, float& a,
                                               float& b) {
    const float term = in[iTerm][e];
    const float done = fminf(term + in[iTrunc][e], 1.f);
    *scratch = fminf(in[iPa][e] / in[iMu][e], p.rho_bar);
    a = in[iR][e] + p.gamma * in[iE][e] * (1.f - term) - in[iQ][e];
    if (edge) {
      b = 0.f;
    } else {
      const float c_next = p.lam * fminf(nx.pa / nx.mu, p.c_bar);
      b = p.gamma * c_next * (1.f - done);
    }
  }
  template <int VEC>
  __device__ __forceinline__ static void emit(const Params& p, const float (&in)[kNI][VEC], int e, float x,
                                              float xnext, Nbr nx, bool edge, const EdgeLoc&, int,
                                              const float* scratch, float& o0, float& o1) {
    const float qn = edge ? 0.f : (xnext + nx.q);
    const float q = in[iQ][e];
    o0 = x + q;
    o1 = *scratch * (in[iR][e] + p.gamma * qn * (1.f - in[iTerm][e]) - q);
  }
};

// Window value folded in at a backward row end by the returns estimators
// (only the last-column bootstrap kind reads memory there).
template <class InT>
__device__ __noinline__ float returns_window(const InT* boot, EdgeLoc L, int j) {
  return gload(boot, L.gi(j));
}

// ===========================================================================
// TD(lambda) returns -- src/rl_triton/kernels/lambda_returns_fused.py:62-89.
//   a = r + gamma*(1-lambda)*(1-done)*nv [+ gamma*trunc*boot],  b = gamma*lambda*(1-done)
// carry at the window end = bootstrap[:, -1] (or 0).
// Streams: r, next_values, term, [trunc], [boot].
// ===========================================================================
template <class InT, bool TR, bool PB>
struct LambdaT : HomogeneousStreams<InT, 3 + (TR ? 1 : 0) + (PB ? 1 : 0)> {
  using Base = HomogeneousStreams<InT, 3 + (TR ? 1 : 0) + (PB ? 1 : 0)>;
  using Params = typename LambdaAlg<InT>::Params;
  using Nbr = float;
  static constexpr bool kBackward = true, kNeedsNbr = false, kNextInEmit = false, kEmitReads = false;
  static constexpr int kOuts = 1, kOutSlots = 1, kScratch = 0;
  static constexpr int iR = 0, iNv = 1, iTerm = 2, iTrunc = 3, iBoot = TR ? 4 : 3;
  __host__ __device__ static const void* sptr(const Params& p, int k) {
    if (k == iR) return p.r;
    if (k == iNv) return p.nv;
    if (k == iTerm) return p.term;
    if (TR && k == iTrunc) return p.trunc;
    return p.boot;
  }
  template <int VEC>
  __device__ __forceinline__ static Nbr nbr_of(const float (&)[Base::kNI][VEC], int) { return 0.f; }
  __device__ __forceinline__ static Nbr nbr_smem(const Params&, const SView&, int, int64_t) { return 0.f; }
  __device__ __forceinline__ static Nbr nbr_global(const Params&, int64_t) { return 0.f; }
  template <int VEC>
  __device__ __forceinline__ static void coeff(const Params& p, const float (&in)[Base::kNI][VEC], int e, Nbr,
                                               bool edge, const EdgeLoc& L, int j, float*, float& a, float& b) {
    const float trunc = TR ? in[iTrunc][e] : 0.f;
    const float term = in[iTerm][e];
    const float done = TR ? fminf(term + trunc, 1.f) : term;
    const float nd = 1.f - done;
    a = in[iR][e] + p.g1l * nd * in[iNv][e];
    if constexpr (PB) a = a + p.gamma * trunc * in[iBoot][e];
    b = p.gl * nd;
    if (edge) {
      if constexpr (PB) {
        if (L.glob) a = fmaf(b, in[iBoot][e], a);
      } else {
        if (L.glob && p.boot_kind == kBootLastCol) a = fmaf(b, returns_window(p.boot, L, j), a);
      }
      b = 0.f;
    }
  }
  template <int VEC>
  __device__ __forceinline__ static void emit(const Params&, const float (&)[Base::kNI][VEC], int, float x, float,
                                              Nbr, bool, const EdgeLoc&, int, const float*, float& o0, float&) {
    o0 = x;
  }
};

// ===========================================================================
// Discounted returns -- src/rl_triton/kernels/discounted_returns_fused.py:56-82.
//   a = r [+ gamma*trunc*boot],  b = gamma*(1-done);  carry = bootstrap[:, -1] (or 0)
// Streams: r, term, [trunc], [boot].
// ===========================================================================
template <class InT, bool TR, bool PB>
struct DiscountedT : HomogeneousStreams<InT, 2 + (TR ? 1 : 0) + (PB ? 1 : 0)> {
  using Base = HomogeneousStreams<InT, 2 + (TR ? 1 : 0) + (PB ? 1 : 0)>;
  using Params = typename DiscountedAlg<InT>::Params;
  using Nbr = float;
  static constexpr bool kBackward = true, kNeedsNbr = false, kNextInEmit = false, kEmitReads = false;
  static constexpr int kOuts = 1, kOutSlots = 1, kScratch = 0;
  static constexpr int iR = 0, iTerm = 1, iTrunc = 2, iBoot = TR ? 3 : 2;
  __host__ __device__ static const void* sptr(const Params& p, int k) {
    if (k == iR) return p.r;
    if (k == iTerm) return p.term;
    if (TR && k == iTrunc) return p.trunc;
    return p.boot;
  }
  template <int VEC>
  __device__ __forceinline__ static Nbr nbr_of(const float (&)[Base::kNI][VEC], int) { return 0.f; }
  __device__ __forceinline__ static Nbr nbr_smem(const Params&, const SView&, int, int64_t) { return 0.f; }
  __device__ __forceinline__ static Nbr nbr_global(const Params&, int64_t) { return 0.f; }
  template <int VEC>
  __device__ __forceinline__ static void coeff(const Params& p, const float (&in)[Base::kNI][VEC], int e, Nbr,
                                               bool edge, const EdgeLoc& L, int j, float*, float& a, float& b) {
    const float trunc = TR ? in[iTrunc][e] : 0.f;
    const float term = in[iTerm][e];
    const float done = TR ? fminf(term + trunc, 1.f) : term;
    a = in[iR][e];
    if constexpr (PB) a = a + p.gamma * trunc * in[iBoot][e];
    b = p.gamma * (1.f - done);
    if (edge) {
      if constexpr (PB) {
        if (L.glob) a = fmaf(b, in[iBoot][e], a);
      } else {
        if (L.glob && p.boot_kind == kBootLastCol) a = fmaf(b, returns_window(p.boot, L, j), a);
      }
      b = 0.f;
    }
  }
  template <int VEC>
  __device__ __forceinline__ static void emit(const Params&, const float (&)[Base::kNI][VEC], int, float x, float,
                                              Nbr, bool, const EdgeLoc&, int, const float*, float& o0, float&) {
    o0 = x;
  }
};

// Per-row value (seed, carry) read at a forward row start / affine row edge.
__device__ __noinline__ inline float row_value(const float* arr, EdgeLoc L, int j) { return arr[L.row(j)]; }

// ===========================================================================
// Forward scans: eligibility traces (kernels/eligibility_traces_fused.py:66-84)
// and the episodic prefix sum (kernels/prefix_sum_fused.py:62-84).
//   x[t] = in[t] + k*(1 - flag) * x[t-1],  flag = done[t-1] (PREV) or done[t]
// Streams: inputs, dones.
// ===========================================================================
template <class InT, bool PREV>
struct ForwardT : HomogeneousStreams<InT, 2> {
  using Params = typename ForwardAlg<InT>::Params;
  using Nbr = float;
  static constexpr bool kBackward = false, kNeedsNbr = PREV, kNextInEmit = false, kEmitReads = false;
  __device__ __forceinline__ static bool unit_decay(const Params& p) { return p.k == 1.f; }
  static constexpr int kOuts = 1, kOutSlots = 1, kScratch = 0;
  __host__ __device__ static const void* sptr(const Params& p, int k) { return k == 0 ? (const void*)p.x : p.done; }
  template <int VEC>
  __device__ __forceinline__ static Nbr nbr_of(const float (&in)[2][VEC], int e) { return in[1][e]; }
  __device__ __forceinline__ static Nbr nbr_smem(const Params&, const SView& s, int idx, int64_t) {
    return s.f<InT>(1, idx);
  }
  __device__ __forceinline__ static Nbr nbr_global(const Params& p, int64_t i) { return gload(p.done, i); }
  template <int VEC>
  __device__ __forceinline__ static void coeff(const Params& p, const float (&in)[2][VEC], int e, Nbr dprev,
                                               bool edge, const EdgeLoc& L, int j, float*, float& a, float& b) {
    a = in[0][e];
    if (edge) {
      // At the window start the gate reads done[-1] := 0 (PREV) or done[0].
      const float bo = p.k * (1.f - (PREV ? 0.f : in[1][e]));
      if (L.glob && p.seed) a = fmaf(bo, row_value(p.seed, L, j), a);
      b = 0.f;
    } else {
      b = p.k * (1.f - (PREV ? dprev : in[1][e]));
    }
  }
  template <int VEC>
  __device__ __forceinline__ static void emit(const Params&, const float (&)[2][VEC], int, float x, float, Nbr,
                                              bool, const EdgeLoc&, int, const float*, float& o0, float&) {
    o0 = x;
  }
};

// ===========================================================================
// Generic affine scan on materialised coefficients (fp32) --
// src/rl_triton/kernels/scan.py:39-138, kernels/scan_chunked.py:7-85.
// Streams: u, v.
// ===========================================================================
template <bool BWD>
struct AffineT : HomogeneousStreams<float, 2> {
  using Params = typename AffineAlg<BWD>::Params;
  using Nbr = float;
  static constexpr bool kBackward = BWD, kNeedsNbr = false, kNextInEmit = false, kEmitReads = false;
  __device__ __forceinline__ static bool unit_decay(const Params&) { return true; }
  static constexpr int kOuts = 1, kOutSlots = 1, kScratch = 0;
  __host__ __device__ static const void* sptr(const Params& p, int k) { return k == 0 ? p.u : p.v; }
  template <int VEC>
  __device__ __forceinline__ static Nbr nbr_of(const float (&)[2][VEC], int) { return 0.f; }
  __device__ __forceinline__ static Nbr nbr_smem(const Params&, const SView&, int, int64_t) { return 0.f; }
  __device__ __forceinline__ static Nbr nbr_global(const Params&, int64_t) { return 0.f; }
  template <int VEC>
  __device__ __forceinline__ static void coeff(const Params& p, const float (&in)[2][VEC], int e, Nbr, bool edge,
                                               const EdgeLoc& L, int j, float*, float& a, float& b) {
    a = in[0][e];
    b = in[1][e];
    if (edge) {
      if (L.glob && p.carry) a = fmaf(b, row_value(p.carry, L, j), a);
      b = 0.f;
    }
  }
  template <int VEC>
  __device__ __forceinline__ static void emit(const Params&, const float (&)[2][VEC], int, float x, float, Nbr,
                                              bool, const EdgeLoc&, int, const float*, float& o0, float&) {
    o0 = x;
  }
};

}  // namespace rls
