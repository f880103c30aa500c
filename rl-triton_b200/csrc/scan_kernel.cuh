// scan_kernel.cuh -- single-pass affine scan over a flat [rows*S] buffer.
//
// Layout.  A tile is WARPS warps x ROUNDS rounds x 32 lanes x VEC elements of
// consecutive memory.  In one round a lane owns VEC consecutive elements
// (one 16-byte vector per input stream), so every warp-wide load of a round is
// a fully coalesced 512-byte access.  All rounds' loads are issued before any
// arithmetic so each thread keeps ROUNDS x streams x 16 B in flight.
//
// Scan.  (1) each lane composes its VEC element maps serially; (2) a
// Kogge-Stone shuffle scan composes lanes per round; (3) rounds and warps are
// composed through registers / shared memory into the tile aggregate; (4) the
// tile carry comes from a decoupled look-back over the tiles already scheduled
// (Merrill & Garland 2016, "Single-pass Parallel Prefix Scan with Decoupled
// Look-back"), ordered by a dynamic ticket so every awaited tile is resident;
// (5) each lane re-walks its elements serially from its exact carry and emits.
// Row edges are folded into the coefficients (b = 0), so a tile whose
// aggregate has b == 0 publishes its inclusive value at once and every
// look-back stops at the first tile containing an episode reset / row edge
// (or where the decay product underflowed to 0).
#pragma once
#include "algs.cuh"

namespace rls {

__device__ __forceinline__ void row_col(int64_t i, int64_t S, int64_t& row, int64_t& col) {
  if (S == 1) {
    row = i;
    col = 0;
    return;
  }
  if (i < 0x7fffffffLL && S < 0x7fffffffLL) {
    const unsigned ui = (unsigned)i, us = (unsigned)S;
    row = ui / us;
    col = ui - (unsigned)row * us;
  } else {
    row = i / S;
    col = i - row * S;
  }
}

template <class Alg, int WARPS, int ROUNDS>
__global__ void __launch_bounds__(WARPS * 32)
scan_kernel(const typename Alg::Params p, const Geom g, void* ws_base) {
  constexpr int VEC = Alg::kVec;
  constexpr int RUN = 32 * VEC;
  constexpr int WARP_ELEMS = ROUNDS * RUN;
  constexpr int TILE = WARPS * WARP_ELEMS;
  constexpr bool BWD = Alg::kBackward;
  using Run = typename Alg::Run;
  using Nbr = typename Alg::Nbr;

  __shared__ unsigned s_ticket, s_epoch;
  __shared__ Pair s_warp[WARPS];
  __shared__ float s_carry;
  __shared__ uint64_t s_mbar[WARPS];
  extern __shared__ __align__(128) unsigned char s_dyn[];

  const Workspace ws = ws_carve(ws_base, g.ws_cap);
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;

  if (threadIdx.x == 0) {
    s_epoch = ld_relaxed_u32(&ws.hdr->epoch);
    s_ticket = atomicAdd(&ws.hdr->ticket, 1u);
  }
  __syncthreads();
  const unsigned ticket = s_ticket;
  const unsigned epoch = s_epoch;
  const int64_t tile = BWD ? (g.num_tiles - 1 - (int64_t)ticket) : (int64_t)ticket;
  const int64_t wbase = tile * TILE + (int64_t)warp * WARP_ELEMS;

  unsigned char* stage = g.smem_per_warp ? (s_dyn + (size_t)warp * g.smem_per_warp) : nullptr;
  Alg::stage(p, g, wbase, WARP_ELEMS, lane, stage, &s_mbar[warp], ws.hdr);

  // ---- loads: every round's vectors in flight at once --------------------
  Run run[ROUNDS];
#pragma unroll
  for (int r = 0; r < ROUNDS; ++r) {
    const int64_t i = wbase + r * RUN + lane * VEC;
    // Two call sites (not one with a runtime flag) keep `run` in registers.
    if (i + VEC <= g.M) Alg::load(p, i, g.M, true, run[r], stage, r * RUN + lane * VEC);
    else Alg::load(p, i, g.M, false, run[r], stage, r * RUN + lane * VEC);
  }

  // ---- neighbour across each lane's run edge ----------------------------
  Nbr halo[ROUNDS];
  if constexpr (Alg::kNeedsNbr) {
#pragma unroll
    for (int r = 0; r < ROUNDS; ++r) {
      if constexpr (BWD) {
        Nbr h = shfl_down_any(Alg::nbr_at(run[r], 0), 1);
        if (r + 1 < ROUNDS) {
          const Nbr w = shfl_idx_any(Alg::nbr_at(run[(r + 1) % ROUNDS], 0), 0);
          if (lane == 31) h = w;
        } else if (lane == 31) {
          const int64_t ii = wbase + WARP_ELEMS;
          if (ii < g.M) h = Alg::nbr_global(p, ii);
        }
        halo[r] = h;
      } else {
        Nbr h = shfl_up_any(Alg::nbr_at(run[r], VEC - 1), 1);
        if (r > 0) {
          const Nbr w = shfl_idx_any(Alg::nbr_at(run[(r + ROUNDS - 1) % ROUNDS], VEC - 1), 31);
          if (lane == 0) h = w;
        } else if (lane == 0) {
          const int64_t ii = wbase - 1;
          if (ii >= 0) h = Alg::nbr_global(p, ii);
        }
        halo[r] = h;
      }
    }
  }

  // ---- coefficients and per-lane maps ------------------------------------
  float ca[ROUNDS][VEC], cb[ROUNDS][VEC];
  Pair excl[ROUNDS];   // composition of the lanes after (bwd) / before (fwd) this lane
  Pair total[ROUNDS];  // composition of the whole round
#pragma unroll
  for (int r = 0; r < ROUNDS; ++r) {
    const int64_t i0 = wbase + r * RUN + lane * VEC;
    int64_t row, col;
    row_col(i0, g.S, row, col);
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
      if (i0 + j < g.M) {
        EdgeCtx e;
        e.i = i0 + j;
        e.row = row;
        e.edge = BWD ? (col == g.S - 1) : (col == 0);
        e.global = g.edge_global != 0;
        Nbr nb;
        if constexpr (Alg::kNeedsNbr) {
          if constexpr (BWD) nb = (j + 1 < VEC) ? Alg::nbr_at(run[r], (j + 1) % VEC) : halo[r];
          else nb = (j > 0) ? Alg::nbr_at(run[r], (j + VEC - 1) % VEC) : halo[r];
          if (g.seg && e.edge && !e.global) nb = Alg::nbr_halo(p, row);
        } else {
          nb = Nbr{};
        }
        Alg::coeff(p, run[r], j, nb, e, ca[r][j], cb[r][j]);
      } else {
        ca[r][j] = 0.f;
        cb[r][j] = 1.f;
      }
      if (++col == g.S) {
        col = 0;
        ++row;
      }
    }
    Pair m = pair_identity();
    if constexpr (BWD) {
#pragma unroll
      for (int j = VEC - 1; j >= 0; --j) m = compose(Pair{ca[r][j], cb[r][j]}, m);
    } else {
#pragma unroll
      for (int j = 0; j < VEC; ++j) m = compose(Pair{ca[r][j], cb[r][j]}, m);
    }
    // Kogge-Stone over lanes, in scan direction.
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
      Pair x = shfl_pair_down(incl, 1);
      excl[r] = (lane == 31) ? pair_identity() : x;
      total[r] = shfl_pair_idx(incl, 0);
    } else {
      Pair x = shfl_pair_up(incl, 1);
      excl[r] = (lane == 0) ? pair_identity() : x;
      total[r] = shfl_pair_idx(incl, 31);
    }
  }

  // ---- warp aggregate -> CTA aggregate ------------------------------------
  Pair wagg = pair_identity();
  if constexpr (BWD) {
#pragma unroll
    for (int r = ROUNDS - 1; r >= 0; --r) wagg = compose(total[r], wagg);
  } else {
#pragma unroll
    for (int r = 0; r < ROUNDS; ++r) wagg = compose(total[r], wagg);
  }
  if (lane == 0) s_warp[warp] = wagg;
  __syncthreads();

  if (threadIdx.x == 0) {
    // Exclusive warp maps (towards the tile's carry entry) and tile aggregate.
    Pair acc = pair_identity();
    if constexpr (BWD) {
      for (int w = WARPS - 1; w >= 0; --w) {
        const Pair t = s_warp[w];
        s_warp[w] = acc;
        acc = compose(t, acc);
      }
    } else {
      for (int w = 0; w < WARPS; ++w) {
        const Pair t = s_warp[w];
        s_warp[w] = acc;
        acc = compose(t, acc);
      }
    }
    const Pair agg = acc;
    const unsigned tag = epoch << 2;
    bool published = false;
    if (agg.b == 0.f || ticket == 0) {
      // The aggregate does not depend on the incoming carry (a reset / row
      // edge inside the tile, or the first tile whose entry is a row edge).
      __stcg(&ws.incl[ticket], make_float2(agg.a, 0.f));
      st_release_u32(&ws.flags[ticket], tag | kFlagIncl);
      published = true;
    } else {
      __stcg(&ws.agg[ticket], make_float2(agg.a, agg.b));
      st_release_u32(&ws.flags[ticket], tag | kFlagAgg);
    }
    // Deterministic decoupled look-back.  Phase 1 walks back to the nearest
    // tile whose inclusive value is published; phase 2 folds the aggregates
    // of the tiles in between in scan order.  Every inclusive value is thus
    // the same serial fold  c <- a_m + b_m * c  over tile aggregates, whatever
    // the scheduling, so repeated runs are bit-identical.
    float carry = 0.f;
    if (ticket > 0) {
      int64_t j = (int64_t)ticket - 1;
      float base = 0.f;
      bool ok = true;
      while (true) {
        unsigned f = 0, it = 0;
        while (true) {
          f = ld_acquire_u32(&ws.flags[j]);
          if ((f & ~3u) == tag && (f & 3u)) break;
          if (++it > kSpinLimit) {
            ok = false;
            break;
          }
          if (it > 32) __nanosleep(64);
          // Another tile already gave up: do not wait out a second limit.
          if ((it & 1023u) == 0 && ld_relaxed_u32(&ws.hdr->error) != 0u) {
            ok = false;
            break;
          }
        }
        if (!ok) break;
        if ((f & 3u) == kFlagIncl) {
          base = __ldcg(&ws.incl[j]).x;
          break;
        }
        if (j == 0) {  // cannot happen: the first tile always publishes inclusive
          ok = false;
          break;
        }
        --j;
      }
      if (ok) {
        carry = base;
        for (int64_t m = j + 1; m < (int64_t)ticket; ++m) {
          const float2 v = __ldcg(&ws.agg[m]);
          carry = fmaf(v.y, carry, v.x);
        }
      } else {
        atomicOr(&ws.hdr->error, 1u);
        carry = 0.f;
      }
    }
    if (!published) {
      __stcg(&ws.incl[ticket], make_float2(apply(agg, carry), 0.f));
      st_release_u32(&ws.flags[ticket], tag | kFlagIncl);
    }
    s_carry = carry;
    // Last CTA to finish re-arms the workspace for the next launch.
    __threadfence();
    const unsigned n = atomicAdd(&ws.hdr->finished, 1u);
    if (n == (unsigned)(g.num_tiles - 1)) {
      ws.hdr->ticket = 0u;
      ws.hdr->finished = 0u;
      ws.hdr->epoch = (epoch + 1u) & kEpochMask;
      __threadfence();
    }
  }
  __syncthreads();

  // ---- distribute carries and emit ----------------------------------------
  float c_round = apply(s_warp[warp], s_carry);
  float c_r[ROUNDS];
  if constexpr (BWD) {
#pragma unroll
    for (int r = ROUNDS - 1; r >= 0; --r) {
      c_r[r] = c_round;
      c_round = apply(total[r], c_round);
    }
  } else {
#pragma unroll
    for (int r = 0; r < ROUNDS; ++r) {
      c_r[r] = c_round;
      c_round = apply(total[r], c_round);
    }
  }

#pragma unroll
  for (int r = 0; r < ROUNDS; ++r) {
    const int64_t i0 = wbase + r * RUN + lane * VEC;
    float x = apply(excl[r], c_r[r]);
    float o0[VEC], o1[VEC];
    int64_t row, col;
    row_col(i0, g.S, row, col);
    if constexpr (BWD) {
      // Edge flags in memory order first, then the backward walk.
      bool edge[VEC];
      int64_t rows[VEC];
#pragma unroll
      for (int j = 0; j < VEC; ++j) {
        edge[j] = (col == g.S - 1);
        rows[j] = row;
        if (++col == g.S) {
          col = 0;
          ++row;
        }
      }
#pragma unroll
      for (int j = VEC - 1; j >= 0; --j) {
        const float xn = x;
        x = fmaf(cb[r][j], x, ca[r][j]);
        EdgeCtx e;
        e.i = i0 + j;
        e.row = rows[j];
        e.edge = edge[j];
        e.global = g.edge_global != 0;
        Nbr nb;
        if constexpr (Alg::kNeedsNbr) {
          nb = (j + 1 < VEC) ? Alg::nbr_at(run[r], (j + 1) % VEC) : halo[r];
          if (g.seg && e.edge && !e.global) nb = Alg::nbr_halo(p, rows[j]);
        } else {
          nb = Nbr{};
        }
        if (i0 + j < g.M) Alg::emit(p, run[r], j, x, xn, nb, e, o0[j], o1[j]);
        else { o0[j] = 0.f; o1[j] = 0.f; }
      }
    } else {
#pragma unroll
      for (int j = 0; j < VEC; ++j) {
        const float xp = x;
        x = fmaf(cb[r][j], x, ca[r][j]);
        EdgeCtx e;
        e.i = i0 + j;
        e.row = row;
        e.edge = (col == 0);
        e.global = g.edge_global != 0;
        Nbr nb = Nbr{};
        if (i0 + j < g.M) Alg::emit(p, run[r], j, x, xp, nb, e, o0[j], o1[j]);
        else { o0[j] = 0.f; o1[j] = 0.f; }
        if (++col == g.S) {
          col = 0;
          ++row;
        }
      }
    }
    const bool full = i0 + VEC <= g.M;
    if (i0 < g.M) {
      store_run<VEC>(p.out0, i0, g.M, full, o0);
      if constexpr (Alg::kOuts > 1) store_run<VEC>(p.out1, i0, g.M, full, o1);
    }
  }
}

}  // namespace rls
