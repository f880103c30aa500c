// rows_kernel.cuh -- row-parallel affine scan: one warp owns one row.
//
// When there are enough rows to fill the GPU (the common RL batch shape,
// e.g. 4096 x 128 or 131072 x 1024), time-parallelism across CTAs buys
// nothing: every row is independent.  This kernel gives each row to one warp,
// which walks the row in chunks of ROUNDS x 32 lanes x VEC elements, starting
// at the edge where the carry enters (the window end for backward scans, the
// window start for forward scans).  The carry between chunks stays in a
// register, so the kernel needs no workspace, no shared memory, no block
// barrier and no atomics -- the only cross-lane traffic is the warp-shuffle
// composition inside a round.
//
// Per chunk: every round's 16-byte vectors of every input stream are loaded
// before any arithmetic (ROUNDS x streams x 16 B in flight per lane); each
// lane composes its VEC element maps serially; a Kogge-Stone shuffle scan
// composes lanes; the carry is applied and outputs are emitted with 16-byte
// streaming stores.  The element rules (coefficients, edges, emitted outputs)
// are the same policies the flat look-back kernel uses (algs.cuh).
//
// Rows whose length is a multiple of VEC start on a 16-byte boundary and use
// 16-byte vector accesses; other lengths take per-element accesses (the rows
// then start anywhere), with the same per-element row-end handling.
#pragma once
#include "algs.cuh"

namespace rls {

template <class Alg, int WPB, int ROUNDS>
__global__ void __launch_bounds__(WPB * 32)
rows_kernel(const typename Alg::Params p, const Geom g) {
  constexpr int VEC = Alg::kVec;
  constexpr int RUN = 32 * VEC;
  constexpr int CH = ROUNDS * RUN;
  constexpr bool BWD = Alg::kBackward;
  using Run = typename Alg::Run;
  using Nbr = typename Alg::Nbr;

  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * WPB + (threadIdx.x >> 5);
  if (row >= g.N) return;  // whole warp exits together
  const int64_t S = g.S;
  const int64_t rbase = row * S;
  const int64_t rend = rbase + S;
  const int64_t nch = (S + CH - 1) / CH;
  const bool glob = g.edge_global != 0;
  // Rows of a length that is not a multiple of VEC do not start 16-byte
  // aligned: every access is then per element (coalesced across the warp).
  const bool vec_ok = (S % VEC) == 0;

  float carry = 0.f;  // state entering the chunk (edges fold the boundary in)
  Nbr edge_nbr{};     // neighbour across the chunk edge, from the previous chunk
  pdl_trigger();
  if (g.pdl == 1) pdl_wait();

  for (int64_t k = 0; k < nch; ++k) {
    const int64_t c = BWD ? (nch - 1 - k) : k;
    const int64_t cbase = c * CH;

    Run run[ROUNDS];
#pragma unroll
    for (int r = 0; r < ROUNDS; ++r) {
      const int64_t col = cbase + r * RUN + lane * VEC;
      const int64_t i = rbase + col;
      if (vec_ok && col + VEC <= S) Alg::load(p, i, rend, true, run[r], nullptr, 0);
      else Alg::load(p, i, rend, false, run[r], nullptr, 0);
    }
    if (g.pdl == 2 && k == 0) pdl_wait();  // the first loads are in flight; no store before this

    Nbr halo[ROUNDS];
    if constexpr (Alg::kNeedsNbr) {
#pragma unroll
      for (int r = 0; r < ROUNDS; ++r) {
        if constexpr (BWD) {
          Nbr h = shfl_down_any(Alg::nbr_at(run[r], 0), 1);
          const Nbr w = (r + 1 < ROUNDS) ? shfl_idx_any(Alg::nbr_at(run[(r + 1) % ROUNDS], 0), 0) : edge_nbr;
          if (lane == 31) h = w;
          halo[r] = h;
        } else {
          Nbr h = shfl_up_any(Alg::nbr_at(run[r], VEC - 1), 1);
          const Nbr w = (r > 0) ? shfl_idx_any(Alg::nbr_at(run[(r + ROUNDS - 1) % ROUNDS], VEC - 1), 31)
                                : edge_nbr;
          if (lane == 0) h = w;
          halo[r] = h;
        }
      }
      // The neighbour the next chunk (in walk order) needs from this one.
      if constexpr (BWD) edge_nbr = shfl_idx_any(Alg::nbr_at(run[0], 0), 0);
      else edge_nbr = shfl_idx_any(Alg::nbr_at(run[ROUNDS - 1], VEC - 1), 31);
    }

    float ca[ROUNDS][VEC], cb[ROUNDS][VEC];
    Pair excl[ROUNDS], total[ROUNDS];
#pragma unroll
    for (int r = 0; r < ROUNDS; ++r) {
      const int64_t col0 = cbase + r * RUN + lane * VEC;
#pragma unroll
      for (int j = 0; j < VEC; ++j) {
        const int64_t col = col0 + j;
        if (col < S) {
          EdgeCtx e;
          e.i = rbase + col;
          e.row = row;
          e.edge = BWD ? (col == S - 1) : (col == 0);
          e.global = glob;
          Nbr nb;
          if constexpr (Alg::kNeedsNbr) {
            if constexpr (BWD) nb = (j + 1 < VEC) ? Alg::nbr_at(run[r], (j + 1) % VEC) : halo[r];
            else nb = (j > 0) ? Alg::nbr_at(run[r], (j + VEC - 1) % VEC) : halo[r];
            if (g.seg && e.edge && !glob) nb = Alg::nbr_halo(p, row);
          } else {
            nb = Nbr{};
          }
          Alg::coeff(p, run[r], j, nb, e, ca[r][j], cb[r][j]);
        } else {
          ca[r][j] = 0.f;
          cb[r][j] = 1.f;
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
        total[r] = shfl_pair_idx(incl, 0);
      } else {
        const Pair x = shfl_pair_up(incl, 1);
        excl[r] = (lane == 0) ? pair_identity() : x;
        total[r] = shfl_pair_idx(incl, 31);
      }
    }

    // Carries of the rounds, from the chunk's carry-entry edge inward.
    float c_r[ROUNDS];
    float c_round = carry;
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
    carry = c_round;

#pragma unroll
    for (int r = 0; r < ROUNDS; ++r) {
      const int64_t col0 = cbase + r * RUN + lane * VEC;
      float x = apply(excl[r], c_r[r]);
      float o0[VEC], o1[VEC];
      if constexpr (BWD) {
#pragma unroll
        for (int j = VEC - 1; j >= 0; --j) {
          const float xn = x;
          x = fmaf(cb[r][j], x, ca[r][j]);
          const int64_t col = col0 + j;
          EdgeCtx e;
          e.i = rbase + col;
          e.row = row;
          e.edge = (col == S - 1);
          e.global = glob;
          Nbr nb;
          if constexpr (Alg::kNeedsNbr) {
            nb = (j + 1 < VEC) ? Alg::nbr_at(run[r], (j + 1) % VEC) : halo[r];
            if (g.seg && e.edge && !glob) nb = Alg::nbr_halo(p, row);
          } else {
            nb = Nbr{};
          }
          if (col < S) Alg::emit(p, run[r], j, x, xn, nb, e, o0[j], o1[j]);
          else { o0[j] = 0.f; o1[j] = 0.f; }
        }
      } else {
#pragma unroll
        for (int j = 0; j < VEC; ++j) {
          const float xp = x;
          x = fmaf(cb[r][j], x, ca[r][j]);
          const int64_t col = col0 + j;
          EdgeCtx e;
          e.i = rbase + col;
          e.row = row;
          e.edge = (col == 0);
          e.global = glob;
          Nbr nb = Nbr{};
          if (col < S) Alg::emit(p, run[r], j, x, xp, nb, e, o0[j], o1[j]);
          else { o0[j] = 0.f; o1[j] = 0.f; }
        }
      }
      if (col0 < S) {
        const bool full = vec_ok && col0 + VEC <= S;
        store_run<VEC>(p.out0, rbase + col0, rend, full, o0);
        if constexpr (Alg::kOuts > 1) store_run<VEC>(p.out1, rbase + col0, rend, full, o1);
      }
    }
  }
}

}  // namespace rls
