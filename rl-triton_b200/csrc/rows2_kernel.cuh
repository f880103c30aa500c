// rows2_kernel.cuh -- lean row-parallel scan: one warp per row, compile-time policies.
//
// Same schedule as rows_kernel.cuh (a warp walks its row in chunks from the
// edge where the carry enters, carrying the state between chunks in a
// register: no workspace, no shared memory, no barrier), but with the
// per-element rules of the tile policies (tile_policies.cuh), whose variants
// are template parameters, and with the next chunk's loads issued before the
// current chunk is scanned:
//  * a lane owns VEC consecutive elements per round (one 16-byte vector per
//    input stream: 4 fp32 or 8 bf16), R rounds per chunk; the vectors stay raw
//    in registers and are converted on use;
//  * chunk c+1's vectors are requested while chunk c is scanned (two register
//    buffers), so a warp keeps up to 2 * R * streams * 16 B per lane in flight;
//  * seq_len % VEC == 0, so a vector lies in one row and can only hold the
//    row's edge at its last (backward) / first (forward) element.
#pragma once
#include "tile_policies.cuh"

namespace rls {

template <class P, int R>
struct Rows2Chunk {
  static constexpr int VEC = 16 / (int)sizeof(typename P::InT);
  uint4 v[R][P::kNS];
};

template <class P, int R>
__device__ __forceinline__ void rows2_load(const typename P::Params& p, int64_t rbase, int64_t S, int64_t cbase,
                                           int lane, Rows2Chunk<P, R>& ch) {
  constexpr int VEC = Rows2Chunk<P, R>::VEC;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int64_t col0 = cbase + (int64_t)r * 32 * VEC + lane * VEC;
#pragma unroll
    for (int k = 0; k < P::kNS; ++k) {
      const typename P::InT* src = reinterpret_cast<const typename P::InT*>(P::sptr(p, k));
      ch.v[r][k] = (col0 < S) ? __ldcs(reinterpret_cast<const uint4*>(src + rbase + col0)) : make_uint4(0, 0, 0, 0);
    }
  }
}

template <class P, int R>
__device__ __forceinline__ void rows2_unpack(const Rows2Chunk<P, R>& ch, int r,
                                             float (&in)[P::kNI][Rows2Chunk<P, R>::VEC], unsigned mask = ~0u) {
#pragma unroll
  for (int k = 0; k < P::kNS; ++k) {
    if (!((mask >> k) & 1u)) continue;
    const uint4 v = ch.v[r][k];
    if constexpr (sizeof(typename P::InT) == 4) {
      in[k][0] = __uint_as_float(v.x); in[k][1] = __uint_as_float(v.y);
      in[k][2] = __uint_as_float(v.z); in[k][3] = __uint_as_float(v.w);
    } else {
      const unsigned w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        in[k][2 * h] = __uint_as_float(w[h] << 16);
        in[k][2 * h + 1] = __uint_as_float(w[h] & 0xffff0000u);
      }
    }
  }
}

// Scan one chunk with the carry entering it; returns the carry leaving it.
template <class P, int R>
__device__ __forceinline__ float rows2_chunk(const typename P::Params& p, const Geom& g, int64_t row,
                                             int64_t rbase, int64_t cbase, int lane, const Rows2Chunk<P, R>& ch,
                                             float carry, typename P::Nbr& edge_nbr) {
  using Nbr = typename P::Nbr;
  constexpr int VEC = Rows2Chunk<P, R>::VEC;
  constexpr int NI = P::kNI;
  constexpr bool BWD = P::kBackward;
  constexpr int JE = BWD ? VEC - 1 : 0;
  const int64_t S = g.S;
  const int glob = g.edge_global;

  int64_t col0[R];
  bool valid[R], edge_v[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    col0[r] = cbase + (int64_t)r * 32 * VEC + lane * VEC;
    valid[r] = col0[r] < S;
    edge_v[r] = valid[r] && (BWD ? (col0[r] + VEC == S) : (col0[r] == 0));
  }

  // Neighbour entering each lane's vector (backward: the element after it).
  Nbr nbe[R];
  if constexpr (P::kNeedsNbr) {
    Nbr own[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      float in[NI][VEC];
      rows2_unpack<P, R>(ch, r, in);
      own[r] = P::template nbr_of<VEC>(in, BWD ? 0 : VEC - 1);
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
      if constexpr (BWD) {
        Nbr h = shfl_down_any(own[r], 1);
        const Nbr w = (r + 1 < R) ? shfl_idx_any(own[(r + 1) % R], 0) : edge_nbr;
        if (lane == 31) h = w;
        nbe[r] = h;
      } else {
        Nbr h = shfl_up_any(own[r], 1);
        const Nbr w = (r > 0) ? shfl_idx_any(own[(r + R - 1) % R], 31) : edge_nbr;
        if (lane == 0) h = w;
        nbe[r] = h;
      }
    }
    edge_nbr = BWD ? shfl_idx_any(own[0], 0) : shfl_idx_any(own[R - 1], 31);
  }

  // Pass 1: coefficients, lane maps, shuffle scan per round.
  float ca[R][VEC], cb[R][VEC], scr[R][VEC];
  Pair excl[R], tot[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    float in[NI][VEC];
    rows2_unpack<P, R>(ch, r, in);
    const EdgeLoc L{rbase + col0[r], row, col0[r], S, glob};
    Nbr nb{};
    if constexpr (P::kNeedsNbr) nb = nbe[r];
#pragma unroll
    for (int q = 0; q < VEC; ++q) {
      const int e = BWD ? (VEC - 1 - q) : q;
      P::template coeff<VEC>(p, in, e, nb, (e == JE) && edge_v[r], L, e, &scr[r][e], ca[r][e], cb[r][e]);
      if constexpr (P::kNeedsNbr) nb = P::template nbr_of<VEC>(in, e);
    }
    if (!valid[r]) {
#pragma unroll
      for (int e = 0; e < VEC; ++e) { ca[r][e] = 0.f; cb[r][e] = 1.f; }
    }
    Pair m = pair_identity();
#pragma unroll
    for (int q = 0; q < VEC; ++q) {
      const int e = BWD ? (VEC - 1 - q) : q;
      m = compose(Pair{ca[r][e], cb[r][e]}, m);
    }
    Pair incl = m;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      if constexpr (BWD) {
        const Pair o = shfl_pair_down(incl, d);
        if (lane + d < 32) incl = compose(incl, o);
      } else {
        const Pair o = shfl_pair_up(incl, d);
        if (lane >= d) incl = compose(incl, o);
      }
    }
    if constexpr (BWD) {
      const Pair x = shfl_pair_down(incl, 1);
      excl[r] = (lane == 31) ? pair_identity() : x;
      tot[r] = shfl_pair_idx(incl, 0);
    } else {
      const Pair x = shfl_pair_up(incl, 1);
      excl[r] = (lane == 0) ? pair_identity() : x;
      tot[r] = shfl_pair_idx(incl, 31);
    }
  }

  // Round carries from the chunk's carry-entry edge inward.
  float cr[R];
  float c = carry;
  if constexpr (BWD) {
#pragma unroll
    for (int r = R - 1; r >= 0; --r) { cr[r] = c; c = apply(tot[r], c); }
  } else {
#pragma unroll
    for (int r = 0; r < R; ++r) { cr[r] = c; c = apply(tot[r], c); }
  }

  // Pass 2: emit and store.
#pragma unroll
  for (int r = 0; r < R; ++r) {
    float in[NI][VEC];
    if constexpr (P::kEmitReads) rows2_unpack<P, R>(ch, r, in, P::kEmitMask);
    const EdgeLoc L{rbase + col0[r], row, col0[r], S, glob};
    float x = apply(excl[r], cr[r]);
    float o0[VEC], o1[VEC];
    Nbr nb{};
    if constexpr (P::kNeedsNbr) nb = nbe[r];
#pragma unroll
    for (int q = 0; q < VEC; ++q) {
      const int e = BWD ? (VEC - 1 - q) : q;
      const float xo = x;
      x = fmaf(cb[r][e], x, ca[r][e]);
      P::template emit<VEC>(p, in, e, x, xo, nb, (e == JE) && edge_v[r], L, e, &scr[r][e], o0[e], o1[e]);
      if constexpr (P::kNeedsNbr && P::kEmitReads) nb = P::template nbr_of<VEC>(in, e);
    }
    if (valid[r]) {
      const int64_t i0 = rbase + col0[r];
#pragma unroll
      for (int q = 0; q < VEC; q += 4) {
        st_stream_f4(p.out0 + i0 + q, make_float4(o0[q], o0[q + 1], o0[q + 2], o0[q + 3]));
        if constexpr (P::kOuts > 1)
          st_stream_f4(p.out1 + i0 + q, make_float4(o1[q], o1[q + 1], o1[q + 2], o1[q + 3]));
      }
    }
  }
  return c;
}

template <class P, int WPB, int R>
__global__ void __launch_bounds__(WPB * 32) rows2_kernel(const typename P::Params p, const Geom g) {
  constexpr int VEC = Rows2Chunk<P, R>::VEC;
  constexpr int64_t CH = (int64_t)R * 32 * VEC;
  constexpr bool BWD = P::kBackward;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * WPB + (threadIdx.x >> 5);
  if (row >= g.N) return;  // whole warp exits together
  const int64_t S = g.S;
  const int64_t rbase = row * S;
  const int64_t nch = (S + CH - 1) / CH;
  auto cb_of = [&](int64_t k) { return (BWD ? (nch - 1 - k) : k) * CH; };

  Rows2Chunk<P, R> a, b;
  typename P::Nbr edge_nbr{};
  float carry = 0.f;
  rows2_load<P, R>(p, rbase, S, cb_of(0), lane, a);
  for (int64_t k = 0; k < nch; k += 2) {
    if (k + 1 < nch) rows2_load<P, R>(p, rbase, S, cb_of(k + 1), lane, b);
    carry = rows2_chunk<P, R>(p, g, row, rbase, cb_of(k), lane, a, carry, edge_nbr);
    if (k + 1 >= nch) break;
    if (k + 2 < nch) rows2_load<P, R>(p, rbase, S, cb_of(k + 2), lane, a);
    carry = rows2_chunk<P, R>(p, g, row, rbase, cb_of(k + 1), lane, b, carry, edge_nbr);
  }
}

}  // namespace rls
