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

// G: 16-byte vectors per lane and round, contiguous in memory (a lane owns
// VEC = G * 16 / sizeof(InT) consecutive steps); stream k's vector g is v[r][k * G + g].
template <class P, int R, int G = 1>
struct Rows2Chunk {
  static constexpr int V0 = 16 / (int)sizeof(typename P::InT);
  static constexpr int VEC = V0 * G;
  uint4 v[R][P::kNS * G];
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

template <class P, int R, int G = 1>
__device__ __forceinline__ void rows2_unpack(const Rows2Chunk<P, R, G>& ch, int r,
                                             float (&in)[P::kNI][Rows2Chunk<P, R, G>::VEC], unsigned mask = ~0u) {
  constexpr int V0 = Rows2Chunk<P, R, G>::V0;
#pragma unroll
  for (int k = 0; k < P::kNS; ++k) {
    if (!((mask >> k) & 1u)) continue;
#pragma unroll
    for (int gg = 0; gg < G; ++gg) {
      const uint4 v = ch.v[r][k * G + gg];
      if constexpr (sizeof(typename P::InT) == 4) {
        in[k][gg * V0 + 0] = __uint_as_float(v.x); in[k][gg * V0 + 1] = __uint_as_float(v.y);
        in[k][gg * V0 + 2] = __uint_as_float(v.z); in[k][gg * V0 + 3] = __uint_as_float(v.w);
      } else {
        const unsigned w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          in[k][gg * V0 + 2 * h] = __uint_as_float(w[h] << 16);
          in[k][gg * V0 + 2 * h + 1] = __uint_as_float(w[h] & 0xffff0000u);
        }
      }
    }
  }
}

// One chunk (R rounds x 32 lanes x VEC elements) in registers: pass 1 builds
// the element maps and the shuffle scans, pass 2 emits from the carry.  Lane
// l's vector of round r starts at flat index i0[r] = (row, col0[r]).
template <class P, int R, int G = 1>
struct ChunkScan {
  using Nbr = typename P::Nbr;
  using Chunk = Rows2Chunk<P, R, G>;
  static constexpr int VEC = Chunk::VEC;
  static constexpr int NI = P::kNI;
  static constexpr bool BWD = P::kBackward;
  static constexpr int JE = BWD ? VEC - 1 : 0;
  int64_t i0[R], row[R], col0[R];
  bool valid[R], edge_v[R];
  Nbr nbe[R];
  float ca[R][VEC], cb[R][VEC], scr[R][VEC];
  Pair excl[R], tot[R];

  // edge_nbr: the neighbour across the chunk's carry-entry edge (element after
  // the chunk backward, before it forward); returns the one the next chunk in
  // walk order needs from this chunk.
  // AGG_ONLY: only the chunk's total map is wanted (tot[]; excl[] is left
  // unset) -- one butterfly reduction instead of the scan.
  template <bool AGG_ONLY = false>
  __device__ __forceinline__ Nbr pass1(const typename P::Params& p, const Geom& g, int lane,
                                       const Chunk& ch, Nbr edge_nbr) {
    const int glob = g.edge_global;
    if constexpr (P::kNeedsNbr) {
      Nbr own[R];
#pragma unroll
      for (int r = 0; r < R; ++r) {
        float in[NI][VEC];
        rows2_unpack<P, R, G>(ch, r, in);
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
#pragma unroll
    for (int r = 0; r < R; ++r) {
      float in[NI][VEC];
      rows2_unpack<P, R, G>(ch, r, in);
      const EdgeLoc L{i0[r], row[r], col0[r], g.S, glob};
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
      if constexpr (AGG_ONLY) {
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
          const Pair o{__shfl_xor_sync(0xffffffffu, m.a, d), __shfl_xor_sync(0xffffffffu, m.b, d)};
          // the lane half that comes later in walk order composes on the outside
          const bool later = BWD ? !(lane & d) : (lane & d);
          m = later ? compose(m, o) : compose(o, m);
        }
        tot[r] = m;
        continue;
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
    return edge_nbr;
  }

  // The chunk's composed map (carry entering -> state leaving).
  __device__ __forceinline__ Pair aggregate() const {
    Pair agg = pair_identity();
    if constexpr (BWD) {
#pragma unroll
      for (int r = R - 1; r >= 0; --r) agg = compose(tot[r], agg);
    } else {
#pragma unroll
      for (int r = 0; r < R; ++r) agg = compose(tot[r], agg);
    }
    return agg;
  }

  // Emit and store with the carry entering the chunk; returns the carry leaving it.
  // `sink(r, q, v0, v1)` takes the outputs of elements q..q+3 of round r
  // (flat index i0[r] + q); the default streams them to out0 / out1.
  __device__ __forceinline__ float pass2(const typename P::Params& p, const Geom& g, const Chunk& ch,
                                         float carry) {
    return pass2(p, g, ch, carry, [&](int r, int q, float4 v0, float4 v1) {
      st_stream_f4(p.out0 + i0[r] + q, v0);
      if constexpr (P::kOuts > 1) st_stream_f4(p.out1 + i0[r] + q, v1);
    });
  }
  template <class Sink>
  __device__ __forceinline__ float pass2(const typename P::Params& p, const Geom& g, const Chunk& ch,
                                         float carry, Sink&& sink) {
    const int glob = g.edge_global;
    float cr[R];
    float c = carry;
    if constexpr (BWD) {
#pragma unroll
      for (int r = R - 1; r >= 0; --r) { cr[r] = c; c = apply(tot[r], c); }
    } else {
#pragma unroll
      for (int r = 0; r < R; ++r) { cr[r] = c; c = apply(tot[r], c); }
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
      float in[NI][VEC];
      if constexpr (P::kEmitReads) rows2_unpack<P, R, G>(ch, r, in, P::kEmitMask);
      const EdgeLoc L{i0[r], row[r], col0[r], g.S, glob};
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
#pragma unroll
        for (int q = 0; q < VEC; q += 4) {
          float4 v1 = make_float4(0.f, 0.f, 0.f, 0.f);
          if constexpr (P::kOuts > 1) v1 = make_float4(o1[q], o1[q + 1], o1[q + 2], o1[q + 3]);
          sink(r, q, make_float4(o0[q], o0[q + 1], o0[q + 2], o0[q + 3]), v1);
        }
      }
    }
    return c;
  }
};

// Scan one chunk of one row with the carry entering it; returns the carry leaving it.
// wait_before_emit: the first chunk of a kernel launched with programmatic
// stream serialization whose loads could start early (Geom::pdl == 2) waits
// for the preceding grid only between its scan and its first store.
template <class P, int R>
__device__ __forceinline__ float rows2_chunk(const typename P::Params& p, const Geom& g, int64_t row,
                                             int64_t rbase, int64_t cbase, int lane, const Rows2Chunk<P, R>& ch,
                                             float carry, typename P::Nbr& edge_nbr, bool wait_before_emit = false) {
  constexpr int VEC = Rows2Chunk<P, R>::VEC;
  constexpr bool BWD = P::kBackward;
  ChunkScan<P, R> cs;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    cs.col0[r] = cbase + (int64_t)r * 32 * VEC + lane * VEC;
    cs.row[r] = row;
    cs.i0[r] = rbase + cs.col0[r];
    cs.valid[r] = cs.col0[r] < g.S;
    cs.edge_v[r] = cs.valid[r] && (BWD ? (cs.col0[r] + VEC == g.S) : (cs.col0[r] == 0));
  }
  edge_nbr = cs.pass1(p, g, lane, ch, edge_nbr);
  if (wait_before_emit) pdl_wait();
  return cs.pass2(p, g, ch, carry);
}

// PDL: launched with programmatic stream serialization (Geom::pdl says when the
// first loads may precede the wait).  A separate instantiation keeps the wait
// out of the plain kernel's code, whose register allocation it would change.
template <class P, int WPB, int R, bool PDL = false>
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
  if constexpr (PDL) {
    pdl_trigger();
    if (g.pdl == 1) pdl_wait();
  }
  rows2_load<P, R>(p, rbase, S, cb_of(0), lane, a);
  if constexpr (PDL) {
    if (g.pdl == 2) pdl_wait();  // the first chunk's loads are in flight; nothing is stored before this
  }
  for (int64_t k = 0; k < nch; k += 2) {
    if (k + 1 < nch) rows2_load<P, R>(p, rbase, S, cb_of(k + 1), lane, b);
    carry = rows2_chunk<P, R>(p, g, row, rbase, cb_of(k), lane, a, carry, edge_nbr);
    if (k + 1 >= nch) break;
    if (k + 2 < nch) rows2_load<P, R>(p, rbase, S, cb_of(k + 2), lane, a);
    carry = rows2_chunk<P, R>(p, g, row, rbase, cb_of(k + 1), lane, b, carry, edge_nbr);
  }
}

// Rows of at most one chunk (seq_len <= 32 lanes x VEC, e.g. 4096 x 128 fp32):
// one warp per row, WPB rows per CTA, no loop.  Launched with programmatic
// stream serialization, such a kernel is short enough that the time between
// two launches matters: it loads and scans its row before griddepcontrol.wait
// (when its inputs are not the preceding launch's outputs, Geom::pdl == 2) and
// only emits and stores after it.
template <class P, int WPB>
__global__ void __launch_bounds__(WPB * 32) rows1_kernel(const typename P::Params p, const Geom g) {
  constexpr int VEC = Rows2Chunk<P, 1>::VEC;
  constexpr bool BWD = P::kBackward;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * WPB + (threadIdx.x >> 5);
  if (row >= g.N) return;  // whole warp exits together
  const int64_t S = g.S;
  pdl_trigger();
  if (g.pdl == 1) pdl_wait();
  Rows2Chunk<P, 1> ch;
  rows2_load<P, 1>(p, row * S, S, 0, lane, ch);
  typename P::Nbr edge_nbr{};
  rows2_chunk<P, 1>(p, g, row, row * S, 0, lane, ch, 0.f, edge_nbr, g.pdl == 2);
  (void)VEC;
  (void)BWD;
}

}  // namespace rls

namespace rls {

// ===========================================================================
// flat2: one warp per 512-element tile of the flat [N*S] array, for few long
// rows.  Each warp loads its tile straight into registers (the ChunkScan of the
// row kernel), publishes the tile's map, takes its carry from a decoupled
// look-back over the preceding tiles, and emits (every wait is bounded and
// latches an error bit instead of hanging).  A launch uses the
// workspace's current epoch, like the other look-back kernels, and a one-thread
// kernel launched right after it advances the epoch, so blocks need no exit
// counter.
// ===========================================================================

static __global__ void advance_epoch(void* ws_base) {
  WsHeader* h = reinterpret_cast<WsHeader*>(ws_base);
  h->epoch = (h->epoch + 1u) & kEpochMask;
}

constexpr int kLookWindows = 4;

// flat2's status words: per tile three 64-bit words, each carrying an fp32 value
// in its low half and (epoch << 2 | kind) in its high half -- inc (the inclusive
// value: kFlagIncl or kFlagSelf), aga / agb (the map's a and b: kFlagAgg).
// A value and its tag travel in one aligned 64-bit store, so readers need no
// fence and one round trip.  Layout: [64-byte header | inc | aga | agb].
struct PackedWs {
  WsHeader* hdr;
  unsigned long long *inc, *aga, *agb;
};
__host__ __device__ inline int64_t packed_capacity(size_t bytes) {
  return bytes < 64 ? 0 : (int64_t)((bytes - 64) / 24);
}
__device__ __forceinline__ PackedWs packed_carve(void* base, int64_t cap) {
  PackedWs w;
  w.hdr = reinterpret_cast<WsHeader*>(base);
  w.inc = reinterpret_cast<unsigned long long*>(reinterpret_cast<char*>(base) + 64);
  w.aga = w.inc + cap;
  w.agb = w.aga + cap;
  return w;
}
__device__ __forceinline__ unsigned long long pack_word(float v, unsigned tk) {
  return ((unsigned long long)tk << 32) | __float_as_uint(v);
}
__device__ __forceinline__ void st_word(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_word(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned word_tag(unsigned long long w) { return (unsigned)(w >> 32); }
__device__ __forceinline__ float word_val(unsigned long long w) { return __uint_as_float((unsigned)w); }

// Carry entering tile `ticket` (the state after tile ticket-1), read from the
// tiles published before it, 32 at a time (lane l reads tile ticket-1-32w-l).
// The carry is the serial fold c <- a_m + b_m * c from a stop point that
// depends only on the data, so the outputs are bit-identical from run to run:
//  * decaying recurrences: the nearest kFlagSelf tile, or the nearest tile where
//    the running product of b's (taken from ticket-1 backwards) is exactly 0 --
//    the fold starts from 0 there; for gamma*lambda decays this comes within a
//    few tiles;
//  * running sums (b only 0 or 1, `unit`): the nearest tile with any inclusive
//    value -- each is the same serial fold, so whichever is found first gives
//    the same result.
// Without a stop within kLookWindows windows, the predecessor's own inclusive
// value (computed by the same rule) is awaited instead.
__device__ __forceinline__ float flat2_look_back(const PackedWs& ws, int64_t ticket, unsigned tag, int lane,
                                                 bool unit, unsigned& err) {
  constexpr unsigned FULL = 0xffffffffu;
  float As[kLookWindows], Bs[kLookWindows];
  float cum = 1.f;
  float c = 0.f;
  bool found = false;
#pragma unroll
  for (int w = 0; w < kLookWindows; ++w) {
    if (found) break;
    const int64_t pj = ticket - 1 - 32 * w - lane;
    unsigned kind = kFlagSelf;
    float a = 0.f, b = 0.f, inc = 0.f;
    if (pj >= 0) {
      unsigned it = 0;
      while (true) {
        const unsigned long long wi = ld_word(ws.inc + pj);
        const unsigned ti = word_tag(wi);
        if (ti == (tag | kFlagSelf)) { kind = kFlagSelf; inc = a = word_val(wi); break; }
        const unsigned long long wa = ld_word(ws.aga + pj), wb = ld_word(ws.agb + pj);
        if (word_tag(wa) == (tag | kFlagAgg) && word_tag(wb) == (tag | kFlagAgg)) {
          a = word_val(wa);
          b = word_val(wb);
          kind = (ti == (tag | kFlagIncl)) ? kFlagIncl : kFlagAgg;
          inc = word_val(wi);
          break;
        }
        if (++it > kSpinLimit) { err |= 1u; kind = kFlagSelf; a = inc = 0.f; break; }
        if (it > 8) __nanosleep(32);
      }
    }
    float pr = b;  // running product of b, nearest tile first
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const float o = __shfl_up_sync(FULL, pr, d);
      if (lane >= d) pr *= o;
    }
    pr *= cum;
    const bool stop = (kind == kFlagSelf) || (unit ? (kind == kFlagIncl) : (pr == 0.f));
    const unsigned m = __ballot_sync(FULL, stop);
    if (m) {
      const int st = __ffs(m) - 1;
      const unsigned ks = __shfl_sync(FULL, kind, st);
      int l0;
      if (ks == kFlagSelf || (unit && ks == kFlagIncl)) {
        c = __shfl_sync(FULL, inc, st);
        l0 = st - 1;
      } else {
        c = 0.f;
        l0 = st;
      }
      for (int l = l0; l >= 0; --l) c = fmaf(__shfl_sync(FULL, b, l), c, __shfl_sync(FULL, a, l));
#pragma unroll
      for (int u = w - 1; u >= 0; --u)
        for (int l = 31; l >= 0; --l) c = fmaf(__shfl_sync(FULL, Bs[u], l), c, __shfl_sync(FULL, As[u], l));
      found = true;
    } else {
      As[w] = a;
      Bs[w] = b;
      cum = __shfl_sync(FULL, pr, 31);
    }
  }
  if (!found) {
    float v = 0.f;
    if (lane == 0) {
      unsigned it = 0;
      while (true) {
        const unsigned long long wi = ld_word(ws.inc + ticket - 1);
        const unsigned ti = word_tag(wi);
        if (ti == (tag | kFlagIncl) || ti == (tag | kFlagSelf)) { v = word_val(wi); break; }
        if (++it > kSpinLimit) { err |= 1u; break; }
        __nanosleep(64);
      }
    }
    c = __shfl_sync(FULL, v, 0);
  }
  return c;
}

// Scan, publish, look back and emit one loaded tile.
template <class P, int R>
__device__ __forceinline__ void flat2_tile(const typename P::Params& p, const Geom& g, const PackedWs& ws,
                                           int64_t ticket, int lane, unsigned tag, const Rows2Chunk<P, R>& ch,
                                           unsigned& err) {
  using CS = ChunkScan<P, R>;
  constexpr int VEC = CS::VEC;
  constexpr int64_t CH = (int64_t)R * 32 * VEC;
  constexpr bool BWD = P::kBackward;
  constexpr unsigned FULL = 0xffffffffu;
  const int64_t tile = BWD ? (g.num_tiles - 1 - ticket) : ticket;
  const int64_t base = tile * CH;
  CS cs;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    cs.i0[r] = base + (int64_t)r * 32 * VEC + lane * VEC;
    cs.valid[r] = cs.i0[r] < g.M;
    row_col(cs.i0[r], g.S, cs.row[r], cs.col0[r]);
    cs.edge_v[r] = cs.valid[r] && (BWD ? (cs.col0[r] + VEC == g.S) : (cs.col0[r] == 0));
  }
  typename P::Nbr nb{};
  if constexpr (P::kNeedsNbr) {
    const int64_t gn = BWD ? base + CH : base - 1;
    if (BWD ? (gn < g.M) : (gn >= 0)) nb = P::nbr_global(p, gn);
  }
  cs.pass1(p, g, lane, ch, nb);
  const Pair agg = cs.aggregate();
  if (lane == 0) {
    if (agg.b == 0.f || ticket == 0) {
      st_word(ws.inc + ticket, pack_word(agg.a, tag | kFlagSelf));
    } else {
      st_word(ws.aga + ticket, pack_word(agg.a, tag | kFlagAgg));
      st_word(ws.agb + ticket, pack_word(agg.b, tag | kFlagAgg));
    }
  }
  // The tile's entry element: backward the last lane's last element of the last round.
  const int rent = BWD ? R - 1 : 0;
  const bool keep = P::kNextInEmit ? !cs.edge_v[rent] : (cs.cb[rent][CS::JE] != 0.f);
  const bool need = ticket > 0 && __shfl_sync(FULL, keep ? 1 : 0, BWD ? 31 : 0);
  float carry = 0.f;
  if (need) {
    carry = flat2_look_back(ws, ticket, tag, lane, P::unit_decay(p), err);
    if (lane == 0 && agg.b != 0.f) st_word(ws.inc + ticket, pack_word(apply(agg, carry), tag | kFlagIncl));
  }
  cs.pass2(p, g, ch, carry);
}

template <class P, int R>
__device__ __forceinline__ int64_t flat2_base(const Geom& g, int64_t ticket) {
  constexpr int64_t CH = (int64_t)R * 32 * Rows2Chunk<P, R>::VEC;
  return (P::kBackward ? (g.num_tiles - 1 - ticket) : ticket) * CH;
}

// One tile per warp: tile t is scanned by warp t % 4 of block t / 4.  Blocks
// start in index order, so a tile's predecessors are running or done (the waits
// are bounded regardless); dynamic block scheduling keeps slow warps from
// holding up a fixed chain of successors.
template <class P, int R>
__global__ void __launch_bounds__(128) flat2_kernel(const typename P::Params p, const Geom g, void* ws_base) {
  __shared__ unsigned s_epoch;
  const PackedWs ws = packed_carve(ws_base, g.ws_cap);
  if (threadIdx.x == 0) s_epoch = ld_relaxed_u32(&ws.hdr->epoch);
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
  if (t >= g.num_tiles) return;
  unsigned err = 0;
  Rows2Chunk<P, R> ch;
  rows2_load<P, R>(p, 0, g.M, flat2_base<P, R>(g, t), lane, ch);
  flat2_tile<P, R>(p, g, ws, t, lane, s_epoch << 2, ch, err);
  if (err && lane == 0) atomicOr(&ws.hdr->error, err);
}

// ===========================================================================
// flat3: one warp per super-tile of NCH chunks of R vectors per lane, walked twice.
// Walk A streams the chunks from the carry-entry end (the next chunk's vectors
// requested before the current one is scanned) and only composes the
// super-tile's map; the map is published and the carry taken from the same
// look-back as flat2; walk B re-reads the chunks -- from L2, where walk A left
// them: the resident super-tiles hold ~50 MB -- and emits.  The look-back thus
// sits between two long stretches of independent loads instead of inside every
// small tile.
// ===========================================================================
template <class P, int R, bool LAST_USE>
__device__ __forceinline__ void flat_load(const typename P::Params& p, int64_t M, int64_t cbase, int lane,
                                          Rows2Chunk<P, R>& ch) {
  constexpr int VEC = Rows2Chunk<P, R>::VEC;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int64_t i = cbase + (int64_t)r * 32 * VEC + lane * VEC;
#pragma unroll
    for (int k = 0; k < P::kNS; ++k) {
      const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const typename P::InT*>(P::sptr(p, k)) + i);
      ch.v[r][k] = (i < M) ? (LAST_USE ? __ldcs(src) : __ldg(src)) : make_uint4(0, 0, 0, 0);
    }
  }
}

// Row and column of a lane's vector.  Within one walk the chunks are CH steps
// apart, so for rows of at least CH steps the position advances with one
// compare (at most one row boundary is crossed) instead of a division per chunk.
struct RowCursor {
  int64_t row, col;
};

template <class P, int R, int G = 1>
__device__ __forceinline__ void flat_chunk_setup(const Geom& g, int64_t cbase, int lane, bool first, RowCursor& c,
                                                 ChunkScan<P, R, G>& cs) {
  constexpr int VEC = ChunkScan<P, R, G>::VEC;
  constexpr int64_t CH = 32 * VEC * R;
  if constexpr (R == 1) {
    cs.i0[0] = cbase + lane * VEC;
    if (first || g.S < CH) {
      row_col(cs.i0[0], g.S, c.row, c.col);
    } else if (P::kBackward) {
      c.col -= CH;
      if (c.col < 0) { c.col += g.S; --c.row; }
    } else {
      c.col += CH;
      if (c.col >= g.S) { c.col -= g.S; ++c.row; }
    }
    cs.row[0] = c.row;
    cs.col0[0] = c.col;
    cs.valid[0] = cs.i0[0] < g.M;
    cs.edge_v[0] = cs.valid[0] && (P::kBackward ? (c.col + VEC == g.S) : (c.col == 0));
  } else {
#pragma unroll
    for (int r = 0; r < R; ++r) {
      cs.i0[r] = cbase + (int64_t)r * 32 * VEC + lane * VEC;
      cs.valid[r] = cs.i0[r] < g.M;
      row_col(cs.i0[r], g.S, cs.row[r], cs.col0[r]);
      cs.edge_v[r] = cs.valid[r] && (P::kBackward ? (cs.col0[r] + VEC == g.S) : (cs.col0[r] == 0));
    }
  }
}

template <class P, int NCH, int R, int MINB = 1>
__global__ void __launch_bounds__(128, MINB) flat3_kernel(const typename P::Params p, const Geom g, void* ws_base) {
  using CS = ChunkScan<P, R>;
  constexpr int RE = P::kBackward ? R - 1 : 0;  // round holding the entry element
  constexpr int VEC = CS::VEC;
  constexpr int64_t CH = 32 * VEC * R;
  constexpr int64_t ST = CH * NCH;
  constexpr bool BWD = P::kBackward;
  constexpr unsigned FULL = 0xffffffffu;
  __shared__ unsigned s_epoch;
  const PackedWs ws = packed_carve(ws_base, g.ws_cap);
  if (threadIdx.x == 0) s_epoch = ld_relaxed_u32(&ws.hdr->epoch);
  __syncthreads();
  const unsigned tag = s_epoch << 2;
  const int lane = threadIdx.x & 31;
  const int64_t ticket = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
  if (ticket >= g.num_tiles) return;
  const int64_t base = (BWD ? (g.num_tiles - 1 - ticket) : ticket) * ST;
  auto cbase = [&](int k) { return base + (BWD ? (NCH - 1 - k) : k) * CH; };
  unsigned err = 0;
  using Nbr = typename P::Nbr;
  Nbr nb0{};
  if constexpr (P::kNeedsNbr) {
    const int64_t gn = BWD ? base + ST : base - 1;
    if (BWD ? (gn < g.M) : (gn >= 0)) nb0 = P::nbr_global(p, gn);
  }

  // One bulk L2 prefetch per input stream for the whole super-tile: walk A's
  // loads then find their lines on the way, without registers held for them.
  if (g.l2_prefetch) {
    if (lane < P::kNS) {
      const int64_t n = (g.M - base < ST ? g.M - base : ST);
      const char* src = reinterpret_cast<const char*>(reinterpret_cast<const typename P::InT*>(P::sptr(p, lane)) + base);
      const unsigned bytes = (unsigned)(n * (int64_t)sizeof(typename P::InT));
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
    }
  }
  // ---- walk A: the super-tile's map --------------------------------------------
  Rows2Chunk<P, R> a, b;
  RowCursor cur;
  Pair M = pair_identity();
  bool keep = false;  // the entry element does not cut the carry
  {
    Nbr nb = nb0;
    flat_load<P, R, false>(p, g.M, cbase(0), lane, a);
#pragma unroll 1
    for (int k = 0; k < NCH; k += 2) {
      if (k + 1 < NCH) flat_load<P, R, false>(p, g.M, cbase(k + 1), lane, b);
      {
        CS cs;
        flat_chunk_setup<P, R>(g, cbase(k), lane, k == 0, cur, cs);
        nb = cs.template pass1<true>(p, g, lane, a, nb);
        M = compose(cs.aggregate(), M);
        if (k == 0) keep = P::kNextInEmit ? !cs.edge_v[RE] : (cs.cb[RE][CS::JE] != 0.f);
      }
      if (k + 1 >= NCH) break;
      if (k + 2 < NCH) flat_load<P, R, false>(p, g.M, cbase(k + 2), lane, a);
      {
        CS cs;
        flat_chunk_setup<P, R>(g, cbase(k + 1), lane, false, cur, cs);
        nb = cs.template pass1<true>(p, g, lane, b, nb);
        M = compose(cs.aggregate(), M);
      }
    }
  }
  if (lane == 0) {
    if (M.b == 0.f || ticket == 0) {
      st_word(ws.inc + ticket, pack_word(M.a, tag | kFlagSelf));
    } else {
      st_word(ws.aga + ticket, pack_word(M.a, tag | kFlagAgg));
      st_word(ws.agb + ticket, pack_word(M.b, tag | kFlagAgg));
    }
  }
  const bool need = ticket > 0 && __shfl_sync(FULL, keep ? 1 : 0, BWD ? 31 : 0);
  float carry = 0.f;
  if (need) {
    carry = flat2_look_back(ws, ticket, tag, lane, P::unit_decay(p), err);
    if (lane == 0 && M.b != 0.f) st_word(ws.inc + ticket, pack_word(apply(M, carry), tag | kFlagIncl));
  }

  // ---- walk B: re-read (from L2) and emit ---------------------------------------
  {
    Nbr nb = nb0;
    flat_load<P, R, true>(p, g.M, cbase(0), lane, a);
#pragma unroll 1
    for (int k = 0; k < NCH; k += 2) {
      if (k + 1 < NCH) flat_load<P, R, true>(p, g.M, cbase(k + 1), lane, b);
      {
        CS cs;
        flat_chunk_setup<P, R>(g, cbase(k), lane, k == 0, cur, cs);
        nb = cs.pass1(p, g, lane, a, nb);
        carry = cs.pass2(p, g, a, carry);
      }
      if (k + 1 >= NCH) break;
      if (k + 2 < NCH) flat_load<P, R, true>(p, g.M, cbase(k + 2), lane, a);
      {
        CS cs;
        flat_chunk_setup<P, R>(g, cbase(k + 1), lane, false, cur, cs);
        nb = cs.pass1(p, g, lane, b, nb);
        carry = cs.pass2(p, g, b, carry);
      }
    }
  }
  if (err && lane == 0) atomicOr(&ws.hdr->error, err);
}

// ===========================================================================
// flat4: flat3's two walks fed through a per-lane ring of D chunk slots in
// shared memory, filled by 16-byte cp.async copies.  Each lane copies and later
// reads back only its own vector of each stream, so the ring needs no barrier
// and no cross-lane fence: cp.async.wait_group on the lane's own copies is the
// whole protocol.  D-1 chunks per warp are in flight at all times, held in
// shared memory rather than registers, and the loads of walk B's first chunks
// are issued before the look-back, so they overlap it.
// Ring layout per warp: [slot][stream][lane] x 16 bytes (a warp touches 512
// contiguous bytes per stream: conflict-free).
// ===========================================================================
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, unsigned src_bytes) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// D == 0: the ring holds the whole super-tile (NCH slots); walk B then re-reads
// shared memory instead of L2.
template <class P, int D, int G, int NCH = 0>
constexpr int flat4_smem_per_warp() { return (D ? D : NCH) * P::kNS * 32 * G * 16; }

// cp.async.wait_group takes an immediate: dispatch a run-time count (< 16).
__device__ __forceinline__ void cp_async_wait_n(int n) {
  switch (n) {
    case 0: cp_async_wait<0>(); break;
    case 1: cp_async_wait<1>(); break;
    case 2: cp_async_wait<2>(); break;
    case 3: cp_async_wait<3>(); break;
    case 4: cp_async_wait<4>(); break;
    case 5: cp_async_wait<5>(); break;
    case 6: cp_async_wait<6>(); break;
    case 7: cp_async_wait<7>(); break;
    case 8: cp_async_wait<8>(); break;
    case 9: cp_async_wait<9>(); break;
    case 10: cp_async_wait<10>(); break;
    case 11: cp_async_wait<11>(); break;
    case 12: cp_async_wait<12>(); break;
    case 13: cp_async_wait<13>(); break;
    case 14: cp_async_wait<14>(); break;
    default: cp_async_wait<15>(); break;
  }
}

// Position of 16-byte vector v (0 .. 32G-1, in memory order) inside its slot.
// Copies are coalesced (lane l lands vectors g*32 + l), reads are per lane
// (lane l takes vectors l*G .. l*G+G-1); the XOR keeps both conflict-free: any
// 8 lanes of one phase hit 8 distinct 16-byte bank groups, for G = 2 and 4.
template <int G>
__device__ __forceinline__ int ring_pos(int v) {
  if constexpr (G == 1) return v;
  else return v ^ ((v >> (G == 2 ? 1 : 2)) & 7);
}

template <class P, int NCH, int D, int G, int WPB>
__global__ void __launch_bounds__(WPB * 32) flat4_kernel(const typename P::Params p, const Geom g, void* ws_base) {
  using CS = ChunkScan<P, 1, G>;
  constexpr int NS = P::kNS;
  constexpr int VEC = CS::VEC;
  constexpr int V0 = CS::Chunk::V0;
  static_assert(G == 1 || G == 2 || G == 4, "G");
  constexpr int64_t CH = 32 * VEC;
  constexpr int64_t ST = CH * NCH;
  constexpr bool BWD = P::kBackward;
  constexpr unsigned FULL = 0xffffffffu;
  constexpr bool RES = D == 0;  // resident super-tile
  constexpr int NSLOT = RES ? NCH : D;
  static_assert(RES || D >= 2, "ring of at least two slots");
  static_assert(!RES || NCH <= 16, "wait counts up to 15");
  extern __shared__ uint4 flat4_ring[];
  __shared__ unsigned s_epoch;
  const PackedWs ws = packed_carve(ws_base, g.ws_cap);
  if (threadIdx.x == 0) s_epoch = ld_relaxed_u32(&ws.hdr->epoch);
  __syncthreads();
  const unsigned tag = s_epoch << 2;
  const int lane = threadIdx.x & 31;
  const int64_t ticket = (int64_t)blockIdx.x * WPB + (threadIdx.x >> 5);
  if (ticket >= g.num_tiles) return;
  uint4* ring = flat4_ring + (threadIdx.x >> 5) * (NSLOT * NS * 32 * G);
  const int64_t base = (BWD ? (g.num_tiles - 1 - ticket) : ticket) * ST;
  auto cbase = [&](int k) { return base + (BWD ? (NCH - 1 - k) : k) * CH; };

  // Load j of the 2*NCH in walk order (walk A's chunks, then walk B's again)
  // into slot j % D; one commit group per load, empty past the end, so that
  // after load j + D - 1 is issued, wait_group<D-1> means "load j has landed".
  auto issue = [&](int j) {
    if (j < (RES ? NCH : 2 * NCH)) {
      const int64_t cb = cbase(j < NCH ? j : j - NCH);
      uint4* slot = ring + (j % NSLOT) * NS * 32 * G;
#pragma unroll
      for (int gg = 0; gg < G; ++gg) {
        const int v = gg * 32 + lane;
        const int64_t i = cb + (int64_t)v * V0;
        const bool ok = i < g.M;
        const int pos = ring_pos<G>(v);
#pragma unroll
        for (int k = 0; k < NS; ++k) {
          const typename P::InT* src = reinterpret_cast<const typename P::InT*>(P::sptr(p, k));
          cp_async16(slot + k * 32 * G + pos, ok ? src + i : src, ok ? 16u : 0u);
        }
      }
    }
    cp_async_commit();
  };
  auto take = [&](int j, typename CS::Chunk& ch) {
    if constexpr (RES) {
      if (j < NCH) cp_async_wait_n(NCH - 1 - j);
    } else {
      cp_async_wait<D - 1>();
    }
    const uint4* slot = ring + (j % NSLOT) * NS * 32 * G;
#pragma unroll
    for (int gg = 0; gg < G; ++gg) {
      const int pos = ring_pos<G>(lane * G + gg);
#pragma unroll
      for (int k = 0; k < NS; ++k) ch.v[0][k * G + gg] = slot[k * 32 * G + pos];
    }
  };

#pragma unroll
  for (int j = 0; j < (RES ? NCH : D - 1); ++j) issue(j);

  unsigned err = 0;
  using Nbr = typename P::Nbr;
  Nbr nb0{};
  if constexpr (P::kNeedsNbr) {
    const int64_t gn = BWD ? base + ST : base - 1;
    if (BWD ? (gn < g.M) : (gn >= 0)) nb0 = P::nbr_global(p, gn);
  }

  // ---- walk A: the super-tile's map --------------------------------------------
  typename CS::Chunk ch;
  RowCursor cur;
  Pair M = pair_identity();
  bool keep = false;
  {
    Nbr nb = nb0;
#pragma unroll 1
    for (int k = 0; k < NCH; ++k) {
      // slot (k + D - 1) % D was read into registers by the previous step
      if constexpr (!RES) issue(k + D - 1);
      take(k, ch);
      CS cs;
      flat_chunk_setup<P, 1, G>(g, cbase(k), lane, k == 0, cur, cs);
      nb = cs.template pass1<true>(p, g, lane, ch, nb);
      M = compose(cs.aggregate(), M);
      if (k == 0) keep = P::kNextInEmit ? !cs.edge_v[0] : (cs.cb[0][CS::JE] != 0.f);
    }
  }
  if (lane == 0) {
    if (M.b == 0.f || ticket == 0) {
      st_word(ws.inc + ticket, pack_word(M.a, tag | kFlagSelf));
    } else {
      st_word(ws.aga + ticket, pack_word(M.a, tag | kFlagAgg));
      st_word(ws.agb + ticket, pack_word(M.b, tag | kFlagAgg));
    }
  }
  const bool need = ticket > 0 && __shfl_sync(FULL, keep ? 1 : 0, BWD ? 31 : 0);
  float carry = 0.f;
  if (need) {
    carry = flat2_look_back(ws, ticket, tag, lane, P::unit_decay(p), err);
    if (lane == 0 && M.b != 0.f) st_word(ws.inc + ticket, pack_word(apply(M, carry), tag | kFlagIncl));
  }

  // ---- walk B: the same chunks again (L2) and emit ----------------------------------
  {
    Nbr nb = nb0;
#pragma unroll 1
    for (int k = 0; k < NCH; ++k) {
      if constexpr (!RES) issue(NCH + k + D - 1);
      take(NCH + k, ch);
      CS cs;
      flat_chunk_setup<P, 1, G>(g, cbase(k), lane, k == 0, cur, cs);
      nb = cs.pass1(p, g, lane, ch, nb);
      carry = cs.pass2(p, g, ch, carry);
    }
  }
  cp_async_wait<0>();
  if (err && lane == 0) atomicOr(&ws.hdr->error, err);
}

// ===========================================================================
// vseg: virtual rows.  The flat buffer is cut into nseg segments of L steps
// (L a multiple of the chunk), each scanned by one warp in one walk -- the
// lean row kernel's loop over a flat range -- with carry 0 at its entry.  Real
// row edges inside a segment are handled as everywhere else (b = 0), and the
// neighbour across the entry cut is read from memory, so only the carry is
// missing; each segment leaves its map (A = state at the far end, B = product
// of b) for the carry composition and the bounded fix-up in segment.cu, and a
// fix-up code.  With binary flags every b is 0 or the constant bcoef (gamma,
// gamma*lambda, or 1 for the prefix sum), so the decay product k steps in is
// bcoef^(k+1) up to the first b = 0: the code is that element's offset from
// the segment start (-1 if the segment has none) and the fix-up needs no flag
// reads.  Any other b gives -2 (the fix-up walks the decay product).
// ===========================================================================
template <class P>
__global__ void __launch_bounds__(128) vseg_kernel(const typename P::Params p, const Geom g, int64_t L, int64_t nseg,
                                                   float bcoef, float* seg_a, float* seg_b, int* seg_code) {
  using CS = ChunkScan<P, 1>;
  constexpr int VEC = CS::VEC;
  constexpr int64_t CH = 32 * VEC;
  constexpr bool BWD = P::kBackward;
  constexpr unsigned FULL = 0xffffffffu;
  const int lane = threadIdx.x & 31;
  // The carry composition (a programmatic dependent) may launch once every
  // block of this one-wave grid is running; it waits for the grid to finish.
  pdl_trigger();
  const int64_t sidx = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
  if (sidx >= nseg) return;
  const int64_t s0 = sidx * L;
  const int64_t len = (g.M - s0 < L) ? g.M - s0 : L;
  const int64_t nch = (len + CH - 1) / CH;
  auto cbase = [&](int64_t k) { return s0 + (BWD ? (nch - 1 - k) : k) * CH; };
  using Nbr = typename P::Nbr;
  Nbr nb{};
  if constexpr (P::kNeedsNbr) {
    const int64_t gn = BWD ? s0 + len : s0 - 1;
    if (BWD ? (gn < g.M) : (gn >= 0)) nb = P::nbr_global(p, gn);
  }
  int code = -1;
  bool binary = true;  // every b seen so far is 0 or bcoef
  // First b = 0 of the chunk in walk order (called until one is found).
  auto first_zero = [&](const CS& cs, int64_t cb) {
    int q0 = VEC;
#pragma unroll
    for (int q = 0; q < VEC; ++q) {
      const int e = BWD ? VEC - 1 - q : q;
      const float c = cs.cb[0][e];
      binary = binary && (c == 0.f || c == bcoef);
      if (c == 0.f && q0 == VEC) q0 = q;
    }
    const unsigned m = __ballot_sync(FULL, q0 < VEC);
    if (m) {
      const int wl = BWD ? 31 - __clz(m) : __ffs(m) - 1;
      const int qq = __shfl_sync(FULL, q0, wl);
      code = (int)(cb + wl * VEC + (BWD ? VEC - 1 - qq : qq) - s0);
    }
  };
  RowCursor cur;
  Pair M = pair_identity();
  float carry = 0.f;
  // A ring of D chunks: the loads of the next D-1 chunks are in flight while
  // one is scanned (three for policies of up to three input streams, whose
  // chunks are small; two otherwise).
  constexpr int D = P::kNS <= 3 ? 3 : 2;
  Rows2Chunk<P, 1> buf[D];
#pragma unroll
  for (int u = 0; u < D - 1; ++u)
    if (u < nch) flat_load<P, 1, true>(p, g.M, cbase(u), lane, buf[u]);
#pragma unroll 1
  for (int64_t k = 0; k < nch; k += D) {
#pragma unroll
    for (int u = 0; u < D; ++u) {
      const int64_t kk = k + u;
      if (kk >= nch) break;
      if (kk + D - 1 < nch) flat_load<P, 1, true>(p, g.M, cbase(kk + D - 1), lane, buf[(u + D - 1) % D]);
      CS cs;
      flat_chunk_setup<P, 1>(g, cbase(kk), lane, kk == 0, cur, cs);
      nb = cs.pass1(p, g, lane, buf[u], nb);
      if (code == -1) first_zero(cs, cbase(kk));
      M = compose(cs.aggregate(), M);
      carry = cs.pass2(p, g, buf[u], carry);
    }
  }
  if (!__all_sync(FULL, binary)) code = -2;
  if (lane == 0) {
    seg_a[sidx] = carry;
    seg_b[sidx] = M.b;
    seg_code[sidx] = code;
  }
}

}  // namespace rls
