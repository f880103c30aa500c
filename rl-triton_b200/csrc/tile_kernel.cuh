// tile_kernel.cuh -- persistent, TMA-staged single-pass affine scan.
//
// The [num_envs, seq_len] inputs are scanned as ONE flat array of M = N*S
// elements; row edges are folded into the coefficients (b = 0 at an edge, the
// row's boundary value folded into a), so the same kernel serves 4096 short
// rows, 131072 medium rows and a single 2^28-step row.
//
// Data movement.  The flat array is cut into tiles of THREADS*K elements.  A
// persistent CTA (a few per SM) keeps NS tiles in flight in a shared-memory
// ring: for every input stream ONE bulk copy (cp.async.bulk global->shared, no
// multicast) moves the tile's bytes and completes on the stage's mbarrier.
// Outputs are written to a shared-memory slot and leave with one bulk copy
// shared->global per output.  HBM sees only full-line streaming traffic and
// no thread ever waits on a global load.
//
// Scan.  Thread `th` owns the K consecutive elements [th*K, th*K+K) of a tile
// and reads them from the stage as 16-byte vectors.  Pass 1 turns every
// element into its affine map (a, b) (kept in registers) and composes them
// serially; a shuffle scan composes the threads of a warp and thread 0 the
// warps, giving the tile aggregate.  The tile's carry comes from a decoupled
// look-back over the preceding tiles (Merrill & Garland 2016, "Single-pass
// Parallel Prefix Scan with Decoupled Look-back"), skipped when the tile's
// entry element cuts the carry.  Pass 2 re-walks each thread's elements from
// its exact carry and emits.
//
// Per-element cost.  Everything that varies per element is a compile-time
// property of the policy (truncations present, per-step bootstrap values,
// forward boundary mode); row edges are found from a per-thread bit mask and
// their boundary values are fetched in a rarely-taken, out-of-line branch.
//
// Schedule and liveness.  Each CTA takes ONE ticket when it starts and then
// owns tiles ticket, ticket + G, ticket + 2G, ... (G = grid size): in every
// round the G CTAs hold G consecutive tiles, so a tile's predecessor is always
// in progress in the same (or the previous) round and never queued behind
// other tiles.  The launch is cooperative, so all G CTAs are co-resident;
// every wait is nonetheless bounded (kSpinLimit) and latches an error bit in
// the workspace instead of hanging.
#pragma once
#include "algs.cuh"

namespace rls {

constexpr int kTileThreads = 128;
constexpr int kMaxStreams = 8;
constexpr int kMaxStages = 4;

// Launch geometry of the tile kernel (by value, lives in the param space).
struct TileGeom {
  int64_t M, S, N;
  int64_t num_tiles;
  int64_t ws_cap;   // tiles the workspace can describe (its layout key)
  int edge_global;  // 1: local row edges are global window edges
  int seg;          // 1: time-split launch (halo values at cuts)
  int stages;       // NS
  int stage_bytes;  // bytes of one ring stage
  int off[kMaxStreams];  // byte offset of each staged stream in a stage
};

// Where an edge element sits, for the out-of-line edge handlers.
struct EdgeLoc {
  int64_t i0;    // flat index of the thread's first element
  int64_t row0;  // its row
  int64_t col0;  // its column
  int64_t S;
  int glob;      // edges are real window edges (not time-split cuts)
  __device__ __forceinline__ int64_t gi(int j) const { return i0 + j; }
  __device__ __forceinline__ int64_t row(int j) const { return row0 + (col0 + j) / S; }
};

// Staged-tile view: element idx of stream k.
struct SView {
  const unsigned char* st;
  const int* off;
  template <class T>
  __device__ __forceinline__ T ld(int k, int idx) const {
    return *reinterpret_cast<const T*>(st + off[k] + (size_t)idx * sizeof(T));
  }
  template <class InT>
  __device__ __forceinline__ float f(int k, int idx) const;
};
template <>
__device__ __forceinline__ float SView::f<float>(int k, int idx) const { return ld<float>(k, idx); }
template <>
__device__ __forceinline__ float SView::f<__nv_bfloat16>(int k, int idx) const {
  return bf16_bits_to_float(ld<unsigned short>(k, idx));
}

template <class InT>
__device__ __forceinline__ float gload(const InT* p, int64_t i) {
  return InTraits<InT>::scalar(p, i);
}

// VEC consecutive elements (idx0 a multiple of VEC) of the first NS streams.
template <class InT, int NS, int VEC>
__device__ __forceinline__ void load_streams(const SView& s, int idx0, float (&in)[NS][VEC]) {
#pragma unroll
  for (int k = 0; k < NS; ++k) {
    if constexpr (VEC == 1) {
      in[k][0] = s.f<InT>(k, idx0);
    } else if constexpr (sizeof(InT) == 4) {
#pragma unroll
      for (int q = 0; q < VEC; q += 4) {
        const float4 v = s.ld<float4>(k, (idx0 + q) >> 2);
        in[k][q] = v.x; in[k][q + 1] = v.y; in[k][q + 2] = v.z; in[k][q + 3] = v.w;
      }
    } else {
#pragma unroll
      for (int q = 0; q < VEC; q += 8) {
        const uint4 v = s.ld<uint4>(k, (idx0 + q) >> 3);
        const unsigned w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          in[k][q + 2 * h] = __uint_as_float(w[h] << 16);
          in[k][q + 2 * h + 1] = __uint_as_float(w[h] & 0xffff0000u);
        }
      }
    }
  }
}

// ---- PTX wrappers ------------------------------------------------------------
__device__ __forceinline__ unsigned smem_u32(const void* p) { return (unsigned)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* b, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* b, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* b, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, P;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, unsigned bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void bulk_s2g(void* dst, const void* src, unsigned bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(smem_u32(src)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Issue the bulk copies of one tile into a ring stage (one thread).
template <class P, int K>
__device__ void issue_tile_loads(const typename P::Params& p, const TileGeom& g, int64_t tile,
                                 unsigned char* stage, uint64_t* bar) {
  constexpr int TILE = kTileThreads * K;
  const int64_t start = tile * TILE;
  const int64_t n = (g.M - start < TILE) ? (g.M - start) : TILE;
  unsigned total = 0;
  // Tail bytes (below a 16-byte multiple) first, with plain loads; the arrive
  // below releases them to the waiting threads together with the bulk bytes.
#pragma unroll
  for (int k = 0; k < P::kNS; ++k) {
    const int es = P::esz(p, k);
    const unsigned bytes = (unsigned)(n * es);
    const unsigned bulk = bytes & ~15u;
    if (bulk != bytes) {
      const unsigned char* src = reinterpret_cast<const unsigned char*>(P::sptr(p, k)) + start * es;
      for (unsigned b = bulk; b < bytes; ++b) stage[g.off[k] + b] = src[b];
    }
    total += bulk;
  }
  mbar_arrive_expect_tx(bar, total);
#pragma unroll
  for (int k = 0; k < P::kNS; ++k) {
    const int es = P::esz(p, k);
    const unsigned bulk = (unsigned)(n * es) & ~15u;
    if (bulk) {
      const unsigned char* src = reinterpret_cast<const unsigned char*>(P::sptr(p, k)) + start * es;
      bulk_g2s(stage + g.off[k], src, bulk, bar);
    }
  }
}

template <class P, int K>
__global__ void __launch_bounds__(kTileThreads)
tile_kernel(const typename P::Params p, const TileGeom g, void* ws_base) {
  constexpr int TH = kTileThreads;
  constexpr int TILE = TH * K;
  constexpr bool BWD = P::kBackward;
  constexpr int NW = TH / 32;
  constexpr int NI = P::kNI;
  constexpr int VEC = P::template vec<K>();
  constexpr int NV = K / VEC;
  static_assert(K % VEC == 0, "a run is a whole number of vectors");
  static_assert(K <= 64, "edge mask is 64 bits");
  using Nbr = typename P::Nbr;

  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ uint64_t s_full[kMaxStages];
  __shared__ Pair s_warp[NW];
  __shared__ float s_carry;
  __shared__ int s_need;
  __shared__ unsigned s_first, s_epoch;

  const Workspace ws = ws_carve(ws_base, g.ws_cap);
  const int th = threadIdx.x;
  const int lane = th & 31;
  const int warp = th >> 5;
  const int NS = g.stages;
  const int64_t G = gridDim.x;
  unsigned char* out_slot = smem + (size_t)NS * g.stage_bytes;
  float* out0_s = reinterpret_cast<float*>(out_slot);
  float* out1_s = out0_s + TILE;
  float* scratch = out0_s + (size_t)TILE * P::kOutSlots;

  if (th == 0) {
    s_epoch = ld_relaxed_u32(&ws.hdr->epoch);
    s_first = atomicAdd(&ws.hdr->ticket, 1u);
    for (int s = 0; s < NS; ++s) mbar_init(&s_full[s], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    for (int s = 0; s < NS; ++s) {
      const int64_t t = (int64_t)s_first + s * G;
      if (t < g.num_tiles) {
        const int64_t tile = BWD ? (g.num_tiles - 1 - t) : t;
        issue_tile_loads<P, K>(p, g, tile, smem + (size_t)s * g.stage_bytes, &s_full[s]);
      }
    }
  }
  __syncthreads();
  const unsigned epoch = s_epoch;
  const unsigned tag = epoch << 2;
  const int glob = g.edge_global;
  const int64_t first = s_first;

  for (int it = 0;; ++it) {
    const int s = it % NS;
    const unsigned parity = (unsigned)((it / NS) & 1);
    const int64_t ticket = first + (int64_t)it * G;
    if (ticket >= g.num_tiles) break;
    const int64_t tile = BWD ? (g.num_tiles - 1 - ticket) : ticket;
    const int64_t start = tile * TILE;
    const int nvalid = (int)((g.M - start < TILE) ? (g.M - start) : TILE);
    unsigned char* stw = smem + (size_t)s * g.stage_bytes;
    const SView sv{stw, g.off};

    // Wait for the stage (bounded).
    {
      bool ok = false;
      for (unsigned i = 0; i < kSpinLimit; ++i) {
        if (mbar_try_wait(&s_full[s], parity)) { ok = true; break; }
      }
      if (!ok && lane == 0) atomicOr(&ws.hdr->error, 2u);
    }
    // Partial tile: zero the staged bytes past the valid elements so the scan
    // over the padding stays finite (nothing past nvalid is stored).
    if (nvalid < TILE) {
#pragma unroll
      for (int k = 0; k < P::kNS; ++k) {
        const int es = P::esz(p, k);
        for (int b = nvalid * es + th; b < TILE * es; b += TH) stw[g.off[k] + b] = 0;
      }
      __syncthreads();
    }

    // Row geometry of this thread's run; bit j of emask <=> element j is a row edge.
    const int64_t i0 = start + (int64_t)th * K;
    int64_t row0, col0;
    row_col(i0, g.S, row0, col0);
    uint64_t emask = 0;
    {
      const int64_t firste = BWD ? (g.S - 1 - col0) : ((col0 == 0) ? 0 : g.S - col0);
      for (int64_t e = firste; e < K; e += g.S) emask |= 1ull << e;
      const int nm = nvalid - th * K;
      if (nm < K) emask &= (nm <= 0) ? 0ull : ((1ull << nm) - 1ull);
    }
    const EdgeLoc L{i0, row0, col0, g.S, glob};

    // Neighbour entering the run (backward: element th*K+K, forward: th*K-1).
    Nbr nb0{};
    if constexpr (P::kNeedsNbr) {
      const int idxn = BWD ? (th + 1) * K : th * K - 1;
      const int64_t gn = i0 + (BWD ? K : -1);
      if (BWD ? (idxn < nvalid) : (idxn >= 0)) nb0 = P::nbr_smem(p, sv, idxn, gn);
      else if (BWD ? (gn < g.M) : (gn >= 0)) nb0 = P::nbr_global(p, gn);
    }

    // ---- pass 1: coefficients and the thread's composed map -----------------
    float ca[K], cb[K];
    {
      Nbr nb = nb0;
#pragma unroll
      for (int vq = 0; vq < NV; ++vq) {
        const int v = BWD ? (NV - 1 - vq) : vq;
        float in[NI][VEC];
        // (global reads of element-wise policies stay inside the array)
        const int64_t gv = i0 + v * VEC;
        P::template load<VEC>(p, sv, th * K + v * VEC, gv < g.M ? gv : g.M - 1, in);
#pragma unroll
        for (int eq = 0; eq < VEC; ++eq) {
          const int e = BWD ? (VEC - 1 - eq) : eq;
          const int j = v * VEC + e;
          const bool edge = (emask >> j) & 1ull;
          P::template coeff<VEC>(p, in, e, nb, edge, L, j, scratch + th * K + j, ca[j], cb[j]);
          if constexpr (P::kNeedsNbr) nb = P::template nbr_of<VEC>(in, e);
        }
      }
    }
    // Padding past the end of the array is the identity map exactly.
    if (nvalid < TILE) {
#pragma unroll
      for (int j = 0; j < K; ++j)
        if (th * K + j >= nvalid) { ca[j] = 0.f; cb[j] = 1.f; }
    }
    Pair m = pair_identity();
#pragma unroll
    for (int q = 0; q < K; ++q) {
      const int j = BWD ? (K - 1 - q) : q;
      m = compose(Pair{ca[j], cb[j]}, m);
    }

    // ---- warp scan (towards the carry entry) ---------------------------------
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
    Pair excl;
    if constexpr (BWD) {
      const Pair x = shfl_pair_down(incl, 1);
      excl = (lane == 31) ? pair_identity() : x;
      if (lane == 0) s_warp[warp] = incl;
    } else {
      const Pair x = shfl_pair_up(incl, 1);
      excl = (lane == 0) ? pair_identity() : x;
      if (lane == 31) s_warp[warp] = incl;
    }
    // The carry matters unless the tile's entry element cuts it.
    if (BWD ? (th == TH - 1) : (th == 0)) {
      const int je = BWD ? K - 1 : 0;
      s_need = P::kNextInEmit ? !((emask >> je) & 1ull) : (cb[je] != 0.f);
    }
    __syncthreads();

    if (th == 0) {
      Pair acc = pair_identity();
      if constexpr (BWD) {
        for (int w = NW - 1; w >= 0; --w) {
          const Pair t = s_warp[w];
          s_warp[w] = acc;
          acc = compose(t, acc);
        }
      } else {
        for (int w = 0; w < NW; ++w) {
          const Pair t = s_warp[w];
          s_warp[w] = acc;
          acc = compose(t, acc);
        }
      }
      const Pair agg = acc;
      bool published = false;
      if (agg.b == 0.f || ticket == 0) {
        __stcg(&ws.incl[ticket], make_float2(agg.a, 0.f));
        st_release_u32(&ws.flags[ticket], tag | kFlagIncl);
        published = true;
      } else {
        __stcg(&ws.agg[ticket], make_float2(agg.a, agg.b));
        st_release_u32(&ws.flags[ticket], tag | kFlagAgg);
      }
      float carry = 0.f;
      if (ticket > 0 && (s_need || !published)) {
        int64_t j = ticket - 1;
        float base = 0.f;
        bool ok = true;
        while (true) {
          unsigned f = 0, itn = 0;
          while (true) {
            f = ld_acquire_u32(&ws.flags[j]);
            if ((f & ~3u) == tag && (f & 3u)) break;
            if (++itn > kSpinLimit) { ok = false; break; }
            if (itn > 32) __nanosleep(32);
            if ((itn & 1023u) == 0 && ld_relaxed_u32(&ws.hdr->error) != 0u) { ok = false; break; }
          }
          if (!ok) break;
          if ((f & 3u) == kFlagIncl) {
            base = __ldcg(&ws.incl[j]).x;
            break;
          }
          if (j == 0) { ok = false; break; }
          --j;
        }
        if (ok) {
          carry = base;
          for (int64_t q = j + 1; q < ticket; ++q) {
            const float2 v = __ldcg(&ws.agg[q]);
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
      // The output slot is rewritten below: the previous tile's bulk stores
      // must have finished reading it.
      bulk_wait_read0();
    }
    __syncthreads();

    // ---- pass 2: emit ---------------------------------------------------------
    {
      float x = apply(excl, apply(s_warp[warp], s_carry));
      Nbr nb = nb0;
#pragma unroll
      for (int vq = 0; vq < NV; ++vq) {
        const int v = BWD ? (NV - 1 - vq) : vq;
        float in[NI][VEC];
        const int64_t gv = i0 + v * VEC;
        if constexpr (P::kEmitReads) P::template load<VEC>(p, sv, th * K + v * VEC, gv < g.M ? gv : g.M - 1, in);
        float o0[VEC], o1[VEC];
#pragma unroll
        for (int eq = 0; eq < VEC; ++eq) {
          const int e = BWD ? (VEC - 1 - eq) : eq;
          const int j = v * VEC + e;
          const bool edge = (emask >> j) & 1ull;
          const float xo = x;
          x = fmaf(cb[j], x, ca[j]);
          P::template emit<VEC>(p, in, e, x, xo, nb, edge, L, j, scratch + th * K + j, o0[e], o1[e]);
          if constexpr (P::kNeedsNbr && P::kEmitReads) nb = P::template nbr_of<VEC>(in, e);
        }
        const int o = th * K + v * VEC;
        if constexpr (VEC % 4 == 0) {
#pragma unroll
          for (int q = 0; q < VEC; q += 4) {
            *reinterpret_cast<float4*>(out0_s + o + q) = make_float4(o0[q], o0[q + 1], o0[q + 2], o0[q + 3]);
            if constexpr (P::kOuts > 1)
              *reinterpret_cast<float4*>(out1_s + o + q) = make_float4(o1[q], o1[q + 1], o1[q + 2], o1[q + 3]);
          }
        } else {
#pragma unroll
          for (int q = 0; q < VEC; ++q) {
            out0_s[o + q] = o0[q];
            if constexpr (P::kOuts > 1) out1_s[o + q] = o1[q];
          }
        }
      }
    }
    fence_proxy_async();
    __syncthreads();

    if (th == 0) {
      // Outputs: 16-byte-multiple prefix by bulk copy, the rest by plain stores.
      const unsigned bytes = (unsigned)nvalid * 4u;
      const unsigned bulk = bytes & ~15u;
      if (bulk) {
        bulk_s2g(p.out0 + start, out0_s, bulk);
        if constexpr (P::kOuts > 1) bulk_s2g(p.out1 + start, out1_s, bulk);
        bulk_commit();
      }
      for (int q = (int)(bulk / 4); q < nvalid; ++q) {
        p.out0[start + q] = out0_s[q];
        if constexpr (P::kOuts > 1) p.out1[start + q] = out1_s[q];
      }
      // Refill this stage with this CTA's tile NS rounds ahead.
      const int64_t t = ticket + (int64_t)NS * G;
      if (t < g.num_tiles) {
        const int64_t nt = BWD ? (g.num_tiles - 1 - t) : t;
        issue_tile_loads<P, K>(p, g, nt, stw, &s_full[s]);
      }
    }
    __syncthreads();
  }

  if (th == 0) {
    bulk_wait0();
    __threadfence();
    // Last CTA out re-arms the workspace for the next launch on this stream.
    const unsigned n = atomicAdd(&ws.hdr->finished, 1u);
    if (n == gridDim.x - 1) {
      ws.hdr->ticket = 0u;
      ws.hdr->finished = 0u;
      ws.hdr->epoch = (epoch + 1u) & kEpochMask;
      __threadfence();
    }
  }
}

}  // namespace rls
