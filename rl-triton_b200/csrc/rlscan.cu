// rlscan.cu -- C ABI entry points of librlscan.so (declared in include/rlscan.h).
//
// Host side: argument checks, kernel configuration and template dispatch.
// Nothing here allocates memory: outputs and the workspace are owned by the
// caller (the Python shim allocates them with torch, like the reference).
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <algorithm>
#include <cmath>
#include <mutex>
#include <utility>

#include "rlscan.h"
#include "scan_kernel.cuh"
#include "rows_kernel.cuh"
#include "tile_policies.cuh"
#include "rows2_kernel.cuh"
#include "host_shared.h"

using namespace rls;

namespace rls {
std::recursive_mutex& launch_mutex() {
  static std::recursive_mutex mu;
  return mu;
}

// Record layouts share one workspace: the flags | aggregates | inclusive
// layout of the flat look-back and tile kernels (ws_carve), the packed 64-bit
// value|tag words of flat2/3/4 (packed_carve), and the fp64 partial sums of the
// normalising GAE (ppo.cu).  A stale float left by
// one layout could carry bits equal to a valid tag of the other, so the first
// launch of a layout on a workspace last used by the other one clears the
// records (the header, with the epoch, is kept).  Tracked per workspace
// pointer on the host, under the launch lock.
int prepare_layout(void* ws, size_t wsb, int layout, cudaStream_t s) {
  static void* last_ws[64] = {nullptr};
  static int last_layout[64] = {0};
  static int next_slot = 0;
  if (!ws || wsb <= 64) return RLS_OK;
  int slot = -1;
  for (int i = 0; i < 64; ++i)
    if (last_ws[i] == ws) { slot = i; break; }
  if (slot < 0) {  // first sight: a workspace starts zero-filled
    slot = next_slot;
    next_slot = (next_slot + 1) % 64;
    const bool evicted = last_ws[slot] != nullptr;
    last_ws[slot] = ws;
    last_layout[slot] = evicted ? kLayoutNone : layout;
    if (!evicted) return RLS_OK;
  }
  if (last_layout[slot] != layout) {
    if (cudaMemsetAsync(static_cast<char*>(ws) + 64, 0, wsb - 64, s) != cudaSuccess) return RLS_ECUDA;
    last_layout[slot] = layout;
  }
  return RLS_OK;
}

// ---- programmatic dependent launch of the row kernels ------------------------
// The row kernels (one warp per row, no workspace) are launched with
// programmatic stream serialization: the next one's launch and CTA ramp overlap
// the tail of the one before, which at 4096 x 128 is most of a launch.  A
// kernel waits (griddepcontrol.wait) for the preceding grid before its first
// store, and before its first load unless none of its inputs can be an output
// of the preceding library launch on the stream.  Only the row kernels trigger
// their dependents early across calls (the virtual-row scan and carry kernels
// trigger too, but their dependents are the next kernels of the same call,
// which wait before touching memory); any other preceding kernel (this
// library's or not) completes before a dependent starts, so the overlap check needs only the
// outputs of the last row-kernel launch per stream, kept here under the launch
// lock.
struct PdlRange {
  uintptr_t lo, hi;
};
struct PdlRecord {
  cudaStream_t s;
  PdlRange out[4];
  bool used;
};
static PdlRecord g_pdl[64];
static int g_pdl_next = 0;

static PdlRecord* pdl_find(cudaStream_t s) {
  for (auto& r : g_pdl)
    if (r.used && r.s == s) return &r;
  return nullptr;
}

// 2: the inputs are disjoint from the last row-kernel outputs on this stream
// (loads may start before the wait); 1: they may overlap (wait first).
int pdl_mode(cudaStream_t s, std::initializer_list<PdlIn> ins) {
  const PdlRecord* r = pdl_find(s);
  if (!r) return 2;
  for (const PdlIn& in : ins) {
    if (!in.p || !in.bytes) continue;
    const uintptr_t lo = (uintptr_t)in.p, hi = lo + in.bytes;
    for (const PdlRange& o : r->out)
      if (o.lo < hi && lo < o.hi) return 1;
  }
  return 2;
}

void pdl_record(cudaStream_t s, std::initializer_list<PdlIn> outs) {
  PdlRecord* r = pdl_find(s);
  if (!r) {
    r = &g_pdl[g_pdl_next];
    g_pdl_next = (g_pdl_next + 1) % 64;
    r->s = s;
    r->used = true;
  }
  int k = 0;
  for (const PdlIn& o : outs) {
    if (k == 4) break;
    r->out[k++] = PdlRange{(uintptr_t)o.p, o.p ? (uintptr_t)o.p + o.bytes : 0};
  }
  for (; k < 4; ++k) r->out[k] = PdlRange{0, 0};
}

void pdl_record(cudaStream_t s, const void* out0, const void* out1, size_t bytes) {
  pdl_record(s, {{out0, bytes}, {out1, bytes}});
}

}  // namespace rls

namespace {

constexpr int kWarps = 4;
constexpr int64_t kMinTileElems = 128;  // smallest tile of any launch (a one-round fp32 flat2 tile)

inline bool aligned16(const void* p) { return p == nullptr || ((uintptr_t)p & 15u) == 0; }

// Rounds per warp: larger tiles for large inputs (fewer look-back hops, more
// bytes in flight per thread); small inputs keep enough CTAs to fill 148 SMs.
int pick_rounds(int64_t M, int vec, int max_rounds) {
  int r = 0;
  {
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
  if (g.num_tiles > 0x3fffffffLL) return RLS_EINVAL;
  g.ws_cap = ws ? ws_capacity(ws_bytes) : 0;
  if (g.ws_cap < g.num_tiles) return RLS_EWORKSPACE;
  if (int st = prepare_layout(ws, ws_bytes, kLayoutFlags, s)) return st;
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

// ---- row-parallel path ------------------------------------------------
constexpr int kRowWarps = 4;  // rows (warps) per CTA of the row kernel


// The first row kernel takes any row length (per-element accesses when rows do
// not start 16-byte aligned).
template <class Alg>
bool use_rows(const Geom&) {
  return true;  // any length: unaligned rows take per-element accesses
}

template <class Alg, int R>
int launch_rows_r(const typename Alg::Params& p, const Geom& g, cudaStream_t s) {
  const int64_t blocks = (g.N + kRowWarps - 1) / kRowWarps;
  return launch_rowk(rows_kernel<Alg, kRowWarps, R>, blocks, kRowWarps * 32, s, g.pdl, g.M, p.out0, p.out1, p, g);
}

// Rounds per chunk: enough 16-byte vectors in flight per lane without
// padding short rows (a 128-step fp32 row is exactly one round).
template <class Alg, int MAXR>
int launch_rows(const typename Alg::Params& p, const Geom& g, cudaStream_t s) {
  const int64_t run = 32 * Alg::kVec;
  int r = (int)std::min<int64_t>((g.S + run - 1) / run, MAXR);
  if (r >= 4 && MAXR >= 4) return launch_rows_r<Alg, (MAXR >= 4 ? 4 : 1)>(p, g, s);
  if (r >= 2 && MAXR >= 2) return launch_rows_r<Alg, (MAXR >= 2 ? 2 : 1)>(p, g, s);
  return launch_rows_r<Alg, 1>(p, g, s);
}

// ---- kernel family ----------------------------------------------------------
// RLS_PATH=auto (default) | rows2 | vrows | flat4 | flat3 | flat2 | rows | flat |
// tile.  auto: the lean row kernel (rows2) when every row starts 16-byte
// aligned and there are enough rows to fill the GPU (one warp per row, no
// workspace, no barrier); else, for aligned rows, virtual rows (vrows: the
// flat buffer cut into ~32 segments per SM, one walk each with carry 0, then a
// carry composition and a bounded fix-up) for scans whose output is the state
// and whose segments reach 16K steps, and flat3 (one warp per 2048-step
// super-tile walked twice around one look-back) for the rest; unaligned rows
// take the TMA-staged tile kernel.  flat4 feeds flat3's walks through a
// cp.async ring; flat2 is their one-walk predecessor (one warp per 512-step
// tile).  The others force one family (the row kernels fall back to flat when
// rows are not aligned); rows is the first row kernel with generic policies,
// kept as a cross-check and for Retrace.
int path_mode() {
  const char* s = std::getenv("RLS_PATH");
  if (!s || !*s) return 0;
  if (!std::strcmp(s, "rows")) return 1;
  if (!std::strcmp(s, "flat")) return 2;
  if (!std::strcmp(s, "tile")) return 3;
  if (!std::strcmp(s, "rows2")) return 4;
  if (!std::strcmp(s, "flat2")) return 5;
  if (!std::strcmp(s, "flat3")) return 6;
  if (!std::strcmp(s, "flat4")) return 7;
  if (!std::strcmp(s, "vrows")) return 8;
  return 0;
}

constexpr int64_t kRowsMinEnvs = 8 * 148;  // rows that give every SM 8 warps


int num_sms(int dev) {
  static int cache[64] = {0};
  if (dev < 0 || dev >= 64) return 148;
  if (!cache[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

template <class P, int K>
int launch_tile_k(const typename P::Params& p, TileGeom tg, void* ws, size_t ws_bytes, cudaStream_t s) {
  constexpr int64_t TILE = (int64_t)kTileThreads * K;
  tg.num_tiles = (tg.M + TILE - 1) / TILE;
  if (tg.num_tiles == 0) return RLS_OK;
  if (tg.num_tiles > 0x3fffffffLL) return RLS_EINVAL;
  tg.ws_cap = ws ? ws_capacity(ws_bytes) : 0;
  if (tg.ws_cap < tg.num_tiles) return RLS_EWORKSPACE;
  if (int st = prepare_layout(ws, ws_bytes, kLayoutFlags, s)) return st;
  const size_t smem = (size_t)tg.stages * tg.stage_bytes + (size_t)TILE * 4 * (P::kOutSlots + P::kScratch);
  auto kern = tile_kernel<P, K>;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return RLS_ECUDA;
  // Per-device opt-in to large dynamic shared memory, and the resident CTAs
  // per SM for the smem size last used (occupancy is a host-side query).
  static unsigned long long configured = 0;
  static size_t occ_smem[64] = {0};
  static int occ_val[64] = {0};
  if (dev < 64 && !(configured & (1ull << dev))) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024) != cudaSuccess)
      return RLS_ECUDA;
    configured |= 1ull << dev;
  }
  int per_sm = 1;
  if (dev < 64 && occ_smem[dev] == smem && occ_val[dev] > 0) {
    per_sm = occ_val[dev];
  } else {
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kTileThreads, smem) != cudaSuccess ||
        per_sm <= 0)
      return RLS_ECUDA;
    if (dev < 64) { occ_smem[dev] = smem; occ_val[dev] = per_sm; }
  }
  int64_t grid = (int64_t)per_sm * num_sms(dev);
  if (grid > tg.num_tiles) grid = tg.num_tiles;
  // Cooperative launch: the round-robin tile order needs all CTAs resident.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kTileThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, p, tg, ws) != cudaSuccess) return RLS_ECUDA;
  return RLS_OK;
}

// Stage layout: every staged stream gets a 128-byte-aligned slot of TILE*esz
// bytes; returns the stage size.
template <class P>
int stage_layout(const typename P::Params& p, int K, int* off) {
  const int64_t tile = (int64_t)kTileThreads * K;
  int64_t cur = 0;
  for (int k = 0; k < kMaxStreams; ++k) off[k] = 0;
  for (int k = 0; k < P::kNS; ++k) {
    off[k] = (int)cur;
    cur += (tile * P::esz(p, k) + 127) & ~(int64_t)127;
  }
  return (int)cur;
}

// Ring depth: the deepest ring (4..2 stages) within the per-CTA budget, which
// by default leaves room for two CTAs per SM.
template <class P, int K>
int launch_tile(const typename P::Params& p, const Geom& g, void* ws, size_t ws_bytes, cudaStream_t s) {
  if (g.M == 0) return RLS_OK;
  TileGeom tg;
  tg.M = g.M; tg.S = g.S; tg.N = g.N; tg.num_tiles = 0; tg.ws_cap = 0;
  tg.edge_global = g.edge_global; tg.seg = g.seg;
  tg.stage_bytes = stage_layout<P>(p, K, tg.off);
  const int64_t outb = (int64_t)kTileThreads * K * 4 * (P::kOutSlots + P::kScratch);
  const int64_t budget = 112 * 1024;  // leaves room for two CTAs per SM
  int ns = 0;
  for (int c = kMaxStages; c >= 2 && !ns; --c)
    if (c * (int64_t)tg.stage_bytes + outb <= budget) ns = c;
  if (!ns) ns = 2;
  if (ns * (int64_t)tg.stage_bytes + outb > 220 * 1024) return RLS_EUNSUPPORTED;
  tg.stages = ns;
  return launch_tile_k<P, K>(p, tg, ws, ws_bytes, s);
}

constexpr int kTileK = 16;  // elements per thread: 4 float4 (fp32) or 2 x 8 bf16 per stream

// Launchers of the two kernels that take the compile-time policies.
template <class P>
struct TileL {
  static int run(const typename P::Params& p, const Geom& g, void* ws, size_t wsb, cudaStream_t s) {
    return launch_tile<P, kTileK>(p, g, ws, wsb, s);
  }
};
template <class P>
struct Rows2L {
  static int run(const typename P::Params& p, const Geom& g, void*, size_t, cudaStream_t s) {
    // Rows of one chunk: the loop-free kernel, 8 rows per CTA (4 for the
    // two-output policies, whose registers limit the resident CTAs); longer
    // rows: one round per chunk (the leanest registers measured fastest).
    constexpr int64_t kChunk = 32 * (16 / (int)sizeof(typename P::InT));
    if (g.S <= kChunk) {
      constexpr int W = P::kOuts > 1 ? 4 : 8;
      return launch_rowk(rows1_kernel<P, W>, (g.N + W - 1) / W, W * 32, s, g.pdl, g.M, p.out0, p.out1, p, g);
    }
    // Grids of many waves (e.g. 131072 x 1024) gain nothing from overlapping
    // launches, and dependents parked in griddepcontrol.wait would hold SM
    // slots during the tail: launch them plainly.
    const int64_t blocks = (g.N + 3) / 4;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return RLS_ECUDA;
    if (blocks > 16LL * num_sms(dev)) {
      Geom g2 = g;
      g2.pdl = 0;
      return launch_rowk(rows2_kernel<P, 4, 1, false>, blocks, 128, s, 0, g2.M, p.out0, p.out1, p, g2);
    }
    return launch_rowk(rows2_kernel<P, 4, 1, true>, blocks, 128, s, g.pdl, g.M, p.out0, p.out1, p, g);
  }
};

template <class P, int R>
int launch_flat2(const typename P::Params& p, const Geom& g0, void* ws, size_t wsb, cudaStream_t s) {
  constexpr int64_t CH = 32LL * R * (16 / (int)sizeof(typename P::InT));
  Geom g = g0;
  g.num_tiles = (g.M + CH - 1) / CH;
  if (g.num_tiles == 0) return RLS_OK;
  if (g.num_tiles > 0x3fffffffLL) return RLS_EINVAL;
  g.ws_cap = ws ? packed_capacity(wsb) : 0;
  // A workspace sized for fewer, larger tiles (e.g. the fixed scratch of
  // rls_gae_noalloc) may be too small for flat2's records: the tile kernel
  // then serves the call.
  if (g.ws_cap < g.num_tiles) return launch_tile<P, kTileK>(p, g0, ws, wsb, s);
  // Same convention as the other look-back kernels: a launch uses the current
  // epoch and leaves the next one for the following launch on this workspace.
  if (int st = prepare_layout(ws, wsb, kLayoutPacked, s)) return st;
  flat2_kernel<P, R><<<(unsigned)((g.num_tiles + 3) / 4), 128, 0, s>>>(p, g, ws);
  advance_epoch<<<1, 1, 0, s>>>(ws);
  return cudaPeekAtLastError() == cudaSuccess ? RLS_OK : RLS_ECUDA;
}

template <class P, int NCH, int R>
int launch_flat3(const typename P::Params& p, const Geom& g0, void* ws, size_t wsb, cudaStream_t s) {
  constexpr int64_t ST = 32LL * NCH * R * (16 / (int)sizeof(typename P::InT));
  Geom g = g0;
  g.num_tiles = (g.M + ST - 1) / ST;
  if (g.num_tiles == 0) return RLS_OK;
  if (g.num_tiles > 0x3fffffffLL) return RLS_EINVAL;
  g.ws_cap = ws ? packed_capacity(wsb) : 0;
  if (g.ws_cap < g.num_tiles) return launch_tile<P, kTileK>(p, g0, ws, wsb, s);
  if (int st = prepare_layout(ws, wsb, kLayoutPacked, s)) return st;
  g.l2_prefetch = 0;  // the bulk L2 prefetch measured within noise; kept off
  flat3_kernel<P, NCH, R><<<(unsigned)((g.num_tiles + 3) / 4), 128, 0, s>>>(p, g, ws);
  advance_epoch<<<1, 1, 0, s>>>(ws);
  return cudaPeekAtLastError() == cudaSuccess ? RLS_OK : RLS_ECUDA;
}

// Super-tiles of 2048 steps in chunks of one 16-byte vector per lane (sweeps of
// 1024-4096 steps and of two vectors per lane measured no better).
template <class P>
struct Flat3L {
  static int run(const typename P::Params& p, const Geom& g, void* ws, size_t wsb, cudaStream_t s) {
    constexpr int kChunk = 32 * (16 / (int)sizeof(typename P::InT));
    return launch_flat3<P, 2048 / kChunk, 1>(p, g, ws, wsb, s);
  }
};

template <class P, int NCH, int D, int G>
int launch_flat4(const typename P::Params& p, const Geom& g0, void* ws, size_t wsb, cudaStream_t s) {
  constexpr int64_t ST = 32LL * NCH * G * (16 / (int)sizeof(typename P::InT));
  constexpr int kWarp = flat4_smem_per_warp<P, D, G, NCH>();
  if constexpr (kWarp > 200 * 1024) {
    return launch_flat4<P, NCH, 4, G>(p, g0, ws, wsb, s);  // a resident super-tile this large does not fit
  } else {
  constexpr int WPB = 4 * kWarp <= 200 * 1024 ? 4 : (2 * kWarp <= 200 * 1024 ? 2 : 1);
  constexpr int kSmem = WPB * kWarp;
  static_assert(kSmem <= 200 * 1024, "ring too large");
  Geom g = g0;
  g.num_tiles = (g.M + ST - 1) / ST;
  if (g.num_tiles == 0) return RLS_OK;
  if (g.num_tiles > 0x3fffffffLL) return RLS_EINVAL;
  g.ws_cap = ws ? packed_capacity(wsb) : 0;
  if (g.ws_cap < g.num_tiles) return launch_tile<P, kTileK>(p, g0, ws, wsb, s);
  if (int st = prepare_layout(ws, wsb, kLayoutPacked, s)) return st;
  g.l2_prefetch = 0;
  static bool attr = false;  // per instantiation; racing first calls set the same value
  if (!attr) {
    if (cudaFuncSetAttribute(flat4_kernel<P, NCH, D, G, WPB>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem) !=
        cudaSuccess)
      return RLS_ECUDA;
    attr = true;
  }
  flat4_kernel<P, NCH, D, G, WPB><<<(unsigned)((g.num_tiles + WPB - 1) / WPB), WPB * 32, kSmem, s>>>(p, g, ws);
  advance_epoch<<<1, 1, 0, s>>>(ws);
  return cudaPeekAtLastError() == cudaSuccess ? RLS_OK : RLS_ECUDA;
  }
}

// flat4: 2048-step super-tiles, a 4-slot ring, one vector per lane and chunk (the
// kernel's other options -- resident super-tile, contiguous per-lane runs --
// measured no better and are not instantiated).
template <class P>
struct Flat4L {
  static int run(const typename P::Params& p, const Geom& g, void* ws, size_t wsb, cudaStream_t s) {
    constexpr int kChunk = 32 * (16 / (int)sizeof(typename P::InT));
    return launch_flat4<P, 2048 / kChunk, 4, 1>(p, g, ws, wsb, s);
  }
};

}  // namespace

namespace rls {
// segment.cu: carry composition and bounded fix-up of the virtual rows.
int vrows_finish(int alg, const void* f0, const void* f1, int bf16, float* out, int64_t M, int64_t S, float coef,
                 int ends_at, float* seg_a, float* seg_b, float* carry, int* seg_code, int64_t nseg, int64_t L,
                 cudaStream_t s);
int vrows_finish_vtrace(const void* lpt, const void* lpb, const void* term, const void* trunc, int bf16, float* out0,
                        float* out1, int64_t M, int64_t S, float gamma, float rho_bar, float c_bar, float* seg_a,
                        float* seg_b, float* carry, int* seg_code, int64_t nseg, int64_t L, cudaStream_t s);
}  // namespace rls

namespace {

// ---- virtual rows -------------------------------------------------------------
// Scans whose output is the state itself (GAE, lambda and discounted returns,
// eligibility traces, prefix sums) on few long rows: cut the flat buffer into
// one resident warp's worth of segments per SM slot, scan each with carry 0 in one walk (vseg_kernel: no
// second pass, no look-back), then compose the carries and apply the bounded
// fix-up out[t] += P[t] * carry (vrows_finish), which touches each segment
// only up to its first reset (or until P underflows).  Auto picks it when the
// segments reach 24K steps (unit decay) or 4K steps and three times the decay's
// underflow length (decays below one); shorter ones take flat4.
struct VrowsSpec {
  int alg;
  const void* f0;
  const void* f1;
  float coef;
  int ends_at;
};
template <class P>
struct VSpec {
  static constexpr bool ok = false;
  static VrowsSpec get(const typename P::Params&) { return {}; }
};
template <class T, bool TR, int PB>
struct VSpec<GaeT<T, TR, PB>> {
  static constexpr bool ok = true;
  static VrowsSpec get(const typename GaeT<T, TR, PB>::Params& p) { return {RLS_ALG_GAE, p.term, p.trunc, p.gl, 0}; }
};
template <class T, bool TR, bool PB>
struct VSpec<LambdaT<T, TR, PB>> {
  static constexpr bool ok = true;
  static VrowsSpec get(const typename LambdaT<T, TR, PB>::Params& p) {
    return {RLS_ALG_LAMBDA, p.term, p.trunc, p.gl, 0};
  }
};
template <class T, bool TR, bool PB>
struct VSpec<DiscountedT<T, TR, PB>> {
  static constexpr bool ok = true;
  static VrowsSpec get(const typename DiscountedT<T, TR, PB>::Params& p) {
    return {RLS_ALG_DISCOUNTED, p.term, p.trunc, p.gamma, 0};
  }
};
// V-trace: two outputs and a per-step decay gamma * min(c_bar, ratio); the
// fix-up (vrows_finish_vtrace) walks the decay product, bounded by gamma*c_bar.
template <class T, bool TR, bool PB>
struct VSpec<VtraceT<T, TR, PB>> {
  static constexpr bool ok = true;
  static VrowsSpec get(const typename VtraceT<T, TR, PB>::Params& p) {
    return {-1, p.term, p.trunc, p.gamma * p.c_bar, 0};
  }
};
template <class T>
struct IsVtrace {
  static constexpr bool value = false;
};
template <class T, bool TR, bool PB>
struct IsVtrace<VtraceT<T, TR, PB>> {
  static constexpr bool value = true;
};
template <class T, bool PREV>
struct VSpec<ForwardT<T, PREV>> {
  static constexpr bool ok = true;
  static VrowsSpec get(const typename ForwardT<T, PREV>::Params& p) {
    // traces gate on done[t-1] with k = gamma*lambda; the prefix sum has k = 1
    if (PREV && p.k != 1.f) return {RLS_ALG_ELIGIBILITY, p.done, nullptr, p.k, 1};
    return {RLS_ALG_PREFIX, p.done, nullptr, 1.f, PREV ? 1 : 0};
  }
};

constexpr int64_t kVrowsSegs = 32 * 148;  // segments if the occupancy query fails: 32 warps per SM
// auto: shortest segments worth their fix-up (measured against flat3 / flat4 on
// one row of 2^22 .. 2^27 steps at a 1e-4 reset rate).  A unit decay (prefix
// sums) adds the carry up to each segment's first reset; a decay below one
// also stops where the product underflows (kVrowsUnderflows x that length is
// the minimum); V-trace's per-step c < 1 usually ends its walk within a few
// hundred steps.
constexpr int64_t kVrowsMinLen = 4096;
constexpr int64_t kVrowsMinLenUnit = 24576;
constexpr double kVrowsUnderflows = 3.0;
constexpr int64_t kVrowsMinLenVtrace = 1024;

// forced (RLS_PATH=vrows): any length; auto: only when segments reach the
// minimum above, else flat4.  Policies without a virtual-row fix-up and decay
// coefficients outside (0, 1] take flat3.
template <class P>
int launch_vrows(const typename P::Params& p, const Geom& g, void* ws, size_t wsb, cudaStream_t s, bool forced) {
  constexpr int64_t CH = 32 * (16 / (int)sizeof(typename P::InT));
  if constexpr (!VSpec<P>::ok) {
    return Flat3L<P>::run(p, g, ws, wsb, s);
  } else {
    if (g.M == 0) return RLS_OK;
    // segments: one full wave of vseg_kernel (4 warps per block, resident blocks
    // per SM from its register count x the SMs), or as many as the workspace
    // holds (four words each).  A partial second wave would leave most SMs idle
    // at the end.
    const VrowsSpec v = VSpec<P>::get(p);
    // The bounded fix-up assumes the decay product stays within [0, 1] and
    // only shrinks: other coefficients take flat3.
    if (!(v.coef > 0.f && v.coef <= 1.f)) return Flat3L<P>::run(p, g, ws, wsb, s);
    // Per instantiation and device (devices may differ in SM count); racing
    // first calls compute the same value.
    static int64_t wave_of[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return RLS_ECUDA;
    int64_t wave = dev >= 0 && dev < 64 ? wave_of[dev] : 0;
    if (wave == 0) {
      int nb = 0;
      const int sms = num_sms(dev);
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, vseg_kernel<P>, 128, 0) != cudaSuccess || nb < 1)
        wave = kVrowsSegs;
      else
        wave = std::min<int64_t>((int64_t)nb * 4 * sms, 6144);  // vrows_carry stages <= 6144 maps
      if (dev >= 0 && dev < 64) wave_of[dev] = wave;
    }
    const int64_t room = ws && wsb > 64 ? (int64_t)((wsb - 64) / 16) : 0;
    const int64_t want = room < wave ? room : wave;
    if (want < 1) return Flat3L<P>::run(p, g, ws, wsb, s);
    int64_t L = (g.M + want - 1) / want;
    L = (L + CH - 1) / CH * CH;
    const int64_t nseg = (g.M + L - 1) / L;
    // auto: the fix-up reaches up to -110 / ln(coef) steps into a segment (the
    // decay product underflows there); keep that under a quarter of it.
    int64_t min_len = v.coef == 1.f ? kVrowsMinLenUnit : kVrowsMinLen;
    if (IsVtrace<P>::value) {
      // The fix-up walks to the first reset or until the product of the
      // per-step c < 1 underflows (a few hundred steps at c_bar = 1); even a
      // walk over a whole segment re-reads fewer bytes than the scan did.
      min_len = kVrowsMinLenVtrace;
    } else if (v.coef > 0.f && v.coef < 1.f) {
      min_len = std::max(min_len, (int64_t)(kVrowsUnderflows * -110.0 / std::log((double)v.coef)));
    }
    if (L > 0x7fffffffLL) return Flat3L<P>::run(p, g, ws, wsb, s);
    if (!forced && L < min_len) return Flat4L<P>::run(p, g, ws, wsb, s);
    // The segment words live in the stream's workspace across three launches,
    // enqueued under the caller's launch lock.
    float* seg_a = reinterpret_cast<float*>(static_cast<char*>(ws) + 64);
    float* seg_b = seg_a + nseg;
    float* carry = seg_b + nseg;
    int* code = reinterpret_cast<int*>(carry + nseg);
    vseg_kernel<P><<<(unsigned)((nseg + 3) / 4), 128, 0, s>>>(p, g, L, nseg, v.coef, seg_a, seg_b, code);
    if (cudaPeekAtLastError() != cudaSuccess) return RLS_ECUDA;
    if constexpr (IsVtrace<P>::value)
      return vrows_finish_vtrace(p.lpt, p.lpb, p.term, p.trunc, sizeof(typename P::InT) == 2, p.out0, p.out1, g.M,
                                 g.S, p.gamma, p.rho_bar, p.c_bar, seg_a, seg_b, carry, code, nseg, L, s);
    return vrows_finish(v.alg, v.f0, v.f1, sizeof(typename P::InT) == 2, p.out0, g.M, g.S, v.coef, v.ends_at, seg_a,
                        seg_b, carry, code, nseg, L, s);
  }
}
template <class P>
struct VrowsL {
  static int run(const typename P::Params& p, const Geom& g, void* ws, size_t wsb, cudaStream_t s) {
    return launch_vrows<P>(p, g, ws, wsb, s, path_mode() == 8);
  }
};

// flat2 tiles: 4 rounds of 32 lanes x one 16-byte vector (512 fp32 steps).
template <class P>
struct Flat2L {
  static int run(const typename P::Params& p, const Geom& g, void* ws, size_t wsb, cudaStream_t s) {
    return launch_flat2<P, 4>(p, g, ws, wsb, s);
  }
};

// Compile-time variant dispatch (truncations present, per-step bootstrap kind).
template <template <class> class L, class T>
int gae_v(const typename GaeAlg<T>::Params& p, const Geom& g, void* ws, size_t wsb, cudaStream_t s) {
  const bool tr = p.trunc != nullptr;
  const int pb = p.boot_kind == RLS_BOOT_FULL_ADD ? 1 : ((p.boot_kind == RLS_BOOT_FULL_SEL && tr) ? 2 : 0);
  if (!tr && pb == 0) return L<GaeT<T, false, 0>>::run(p, g, ws, wsb, s);
  if (tr && pb == 0) return L<GaeT<T, true, 0>>::run(p, g, ws, wsb, s);
  if (tr && pb == 2) return L<GaeT<T, true, 2>>::run(p, g, ws, wsb, s);
  if (!tr && pb == 1) return L<GaeT<T, false, 1>>::run(p, g, ws, wsb, s);
  return L<GaeT<T, true, 1>>::run(p, g, ws, wsb, s);
}
template <template <class> class L, class T>
int vtrace_v(const typename VtraceAlg<T>::Params& p, const Geom& g, void* ws, size_t wsb, cudaStream_t s) {
  const bool tr = p.trunc != nullptr, pb = p.boot_kind == RLS_BOOT_FULL_ADD;
  if (!tr && !pb) return L<VtraceT<T, false, false>>::run(p, g, ws, wsb, s);
  if (tr && !pb) return L<VtraceT<T, true, false>>::run(p, g, ws, wsb, s);
  if (!tr && pb) return L<VtraceT<T, false, true>>::run(p, g, ws, wsb, s);
  return L<VtraceT<T, true, true>>::run(p, g, ws, wsb, s);
}
template <template <class> class L, class T>
int lambda_v(const typename LambdaAlg<T>::Params& p, const Geom& g, void* ws, size_t wsb, cudaStream_t s) {
  const bool tr = p.trunc != nullptr, pb = p.boot_kind == RLS_BOOT_FULL_ADD && p.boot;
  if (!tr && !pb) return L<LambdaT<T, false, false>>::run(p, g, ws, wsb, s);
  if (tr && !pb) return L<LambdaT<T, true, false>>::run(p, g, ws, wsb, s);
  if (!tr && pb) return L<LambdaT<T, false, true>>::run(p, g, ws, wsb, s);
  return L<LambdaT<T, true, true>>::run(p, g, ws, wsb, s);
}
template <template <class> class L, class T>
int discounted_v(const typename DiscountedAlg<T>::Params& p, const Geom& g, void* ws, size_t wsb, cudaStream_t s) {
  const bool tr = p.trunc != nullptr, pb = p.boot_kind == RLS_BOOT_FULL_ADD && p.boot;
  if (!tr && !pb) return L<DiscountedT<T, false, false>>::run(p, g, ws, wsb, s);
  if (tr && !pb) return L<DiscountedT<T, true, false>>::run(p, g, ws, wsb, s);
  if (!tr && pb) return L<DiscountedT<T, false, true>>::run(p, g, ws, wsb, s);
  return L<DiscountedT<T, true, true>>::run(p, g, ws, wsb, s);
}
template <template <class> class L, class T>
int forward_v(const typename ForwardAlg<T>::Params& p, const Geom& g, void* ws, size_t wsb, cudaStream_t s) {
  if (p.prev) return L<ForwardT<T, true>>::run(p, g, ws, wsb, s);
  return L<ForwardT<T, false>>::run(p, g, ws, wsb, s);
}
template <template <class> class L, bool B>
int affine_v(const typename AffineAlg<B>::Params& p, const Geom& g, void* ws, size_t wsb, cudaStream_t s) {
  return L<AffineT<B>>::run(p, g, ws, wsb, s);
}

// Which family serves a call (see path_mode): 3 = tile, 4 = lean rows, else the
// register kernels behind launch().
template <class Alg>
int family(const Geom& g) {
  const int m = path_mode();
  const bool rows_ok = g.S % Alg::kVec == 0;
  if (m == 3) return 3;
  if (m == 4) return rows_ok ? 4 : 0;
  if (m == 5) return rows_ok ? 5 : 3;
  if (m == 6) return rows_ok ? 6 : 3;
  if (m == 7) return rows_ok ? 7 : 3;
  if (m == 8) return rows_ok ? 8 : 3;
  if (m != 0) return 0;
  if (rows_ok && g.N >= kRowsMinEnvs) return 4;
  if (g.N >= kRowsMinEnvs) return 0;  // many unaligned rows: the first row kernel, per-element accesses
  return rows_ok ? 8 : 3;  // virtual rows where the policy and the length allow, else flat3
}

template <class Alg, int MAXR = 4>
int launch(const typename Alg::Params& p, Geom g, void* ws, size_t ws_bytes, cudaStream_t s) {
  if (g.M == 0) return RLS_OK;
  const int pm = path_mode();
  if ((pm == 0 || pm == 1) && use_rows<Alg>(g)) return launch_rows<Alg, MAXR>(p, g, s);
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
  g.l2_prefetch = 0;
  g.pdl = 0;
  if (seg) {
    if (seg->t0 < 0 || seg->total_len < seg->t0 + T) return RLS_EINVAL;
    g.seg = 1;
    g.edge_global = backward ? (seg->t0 + T == seg->total_len) : (seg->t0 == 0);
  }
  return RLS_OK;
}

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Every call enqueues its launches under one process-wide lock.  A call may
// take several launches that share the stream's workspace (a look-back kernel
// and the epoch advance after it; the three virtual-row launches), and host
// threads that share a stream must not interleave those sequences.  Only the
// enqueue is serialised (microseconds), never the GPU work.


bool valid_dtype(int d) { return d == RLS_F32 || d == RLS_BF16; }

#define RLS_DEVICE_GUARD(...)              \
  DeviceGuard device_guard_{__VA_ARGS__};  \
  if (device_guard_.status()) return device_guard_.status();

}  // namespace

extern "C" {

size_t rls_workspace_bytes(int64_t num_elements) {
  if (num_elements <= 0) return 64;
  const int64_t tiles = (num_elements + kMinTileElems - 1) / kMinTileElems;
  const size_t packed = 64 + (size_t)tiles * 24;  // flat2's three 8-byte words per tile
  const size_t flags = ws_bytes_for_tiles(tiles);
  return packed > flags ? packed : flags;
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
    case RLS_ENOTDEVICE: return "an array argument is not device memory of one GPU (host pointer, or arrays on different GPUs)";
    case RLS_ETOOLARGE: return "num_envs * seq_len exceeds RLS_NOALLOC_MAX_ELEMENTS (the fixed scratch of rls_gae_noalloc)";
    default: return "unknown status";
  }
}

const char* rls_build_info(void) {
  return "librlscan: sm_100a affine scans (warp-per-row kernels with programmatic dependent launch, "
         "virtual rows and decoupled look-back for long rows, bulk-copy tiles for unaligned rows; "
         "fp32 + bf16 inputs, fp32 arithmetic)";
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
  RLS_DEVICE_GUARD(rewards, values, terminateds, truncateds, bootstrap, advantages, seg ? seg->halo : nullptr, ws)
  Geom g;
  int st = make_geom(num_envs, seq_len, seg, true, g);
  if (st) return st;
  cudaStream_t s = as_stream(stream);
  std::lock_guard<std::recursive_mutex> launch_lock(launch_mutex());
  const size_t esz = in_dtype == RLS_BF16 ? 2 : 4, mb = (size_t)g.M * esz, nb = (size_t)g.N * 4;
  g.pdl = pdl_mode(s, {{rewards, mb}, {values, mb}, {terminateds, mb}, {truncateds, mb},
                      {bootstrap, boot_kind == RLS_BOOT_ROW ? nb : mb}, {seg ? seg->halo : nullptr, nb}});
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
    {
      const int fam = family<GaeAlg<float>>(g);
      if (fam == 3) return gae_v<TileL, float>(p, g, ws, ws_bytes, s);
      if (fam == 4) return gae_v<Rows2L, float>(p, g, ws, ws_bytes, s);
      if (fam == 5) return gae_v<Flat2L, float>(p, g, ws, ws_bytes, s);
      if (fam == 6) return gae_v<Flat3L, float>(p, g, ws, ws_bytes, s);
      if (fam == 7) return gae_v<Flat4L, float>(p, g, ws, ws_bytes, s);
      if (fam == 8) return gae_v<VrowsL, float>(p, g, ws, ws_bytes, s);
    }
    return launch<GaeAlg<float>>(p, g, ws, ws_bytes, s);
  } else {
    GAE_PARAMS(__nv_bfloat16)
    {
      const int fam = family<GaeAlg<__nv_bfloat16>>(g);
      if (fam == 3) return gae_v<TileL, __nv_bfloat16>(p, g, ws, ws_bytes, s);
      if (fam == 4) return gae_v<Rows2L, __nv_bfloat16>(p, g, ws, ws_bytes, s);
      if (fam == 5) return gae_v<Flat2L, __nv_bfloat16>(p, g, ws, ws_bytes, s);
      if (fam == 6) return gae_v<Flat3L, __nv_bfloat16>(p, g, ws, ws_bytes, s);
      if (fam == 7) return gae_v<Flat4L, __nv_bfloat16>(p, g, ws, ws_bytes, s);
      if (fam == 8) return gae_v<VrowsL, __nv_bfloat16>(p, g, ws, ws_bytes, s);
    }
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
  RLS_DEVICE_GUARD(log_pi_target, log_pi_behavior, values, rewards, terminateds, truncateds, bootstrap, targets,
                   advantages, ws)
  Geom g;
  int st = make_geom(num_envs, seq_len, nullptr, true, g);
  if (st) return st;
  cudaStream_t s = as_stream(stream);
  std::lock_guard<std::recursive_mutex> launch_lock(launch_mutex());
  const size_t esz = in_dtype == RLS_BF16 ? 2 : 4, mb = (size_t)g.M * esz, nb = (size_t)g.N * 4;
  g.pdl = pdl_mode(s, {{log_pi_target, mb}, {log_pi_behavior, mb}, {values, mb}, {rewards, mb},
                      {terminateds, mb}, {truncateds, mb}, {bootstrap, boot_kind == RLS_BOOT_ROW ? nb : mb}});
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
    {
      const int fam = family<VtraceAlg<float>>(g);
      if (fam == 3) return vtrace_v<TileL, float>(p, g, ws, ws_bytes, s);
      if (fam == 4) return vtrace_v<Rows2L, float>(p, g, ws, ws_bytes, s);
      if (fam == 5) return vtrace_v<Flat2L, float>(p, g, ws, ws_bytes, s);
      if (fam == 6) return vtrace_v<Flat3L, float>(p, g, ws, ws_bytes, s);
      if (fam == 7) return vtrace_v<Flat4L, float>(p, g, ws, ws_bytes, s);
      if (fam == 8) return vtrace_v<VrowsL, float>(p, g, ws, ws_bytes, s);
    }
    return launch<VtraceAlg<float>, 2>(p, g, ws, ws_bytes, s);
  } else {
    VT_PARAMS(__nv_bfloat16)
    {
      const int fam = family<VtraceAlg<__nv_bfloat16>>(g);
      if (fam == 3) return vtrace_v<TileL, __nv_bfloat16>(p, g, ws, ws_bytes, s);
      if (fam == 4) return vtrace_v<Rows2L, __nv_bfloat16>(p, g, ws, ws_bytes, s);
      if (fam == 5) return vtrace_v<Flat2L, __nv_bfloat16>(p, g, ws, ws_bytes, s);
      if (fam == 6) return vtrace_v<Flat3L, __nv_bfloat16>(p, g, ws, ws_bytes, s);
      if (fam == 7) return vtrace_v<Flat4L, __nv_bfloat16>(p, g, ws, ws_bytes, s);
      if (fam == 8) return vtrace_v<VrowsL, __nv_bfloat16>(p, g, ws, ws_bytes, s);
    }
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
  RLS_DEVICE_GUARD(action_probs_target, action_probs_behavior, q_values, next_q_values_all, actions, rewards,
                   terminateds, truncateds, targets, advantages, ws)
  Geom g;
  int st = make_geom(num_envs, seq_len, nullptr, true, g);
  if (st) return st;
  cudaStream_t s = as_stream(stream);
  std::lock_guard<std::recursive_mutex> launch_lock(launch_mutex());
  {
    const size_t m4 = (size_t)g.M * 4, ma = m4 * (size_t)num_actions;
    g.pdl = pdl_mode(s, {{action_probs_target, ma}, {action_probs_behavior, m4}, {q_values, m4},
                         {next_q_values_all, ma}, {actions, 2 * m4}, {rewards, m4}, {terminateds, m4},
                         {truncateds, m4}});
  }
  RetraceAlg::Params p;
  p.pi = action_probs_target; p.mu = action_probs_behavior; p.q = q_values; p.nq = next_q_values_all;
  p.act = actions; p.r = rewards; p.term = terminateds; p.trunc = truncateds;
  p.out0 = targets; p.out1 = advantages; p.A = num_actions;
  p.gamma = gamma; p.lam = lambda_; p.c_bar = c_bar; p.rho_bar = rho_bar;
  if (g.M == 0) return RLS_OK;
  const int mode = path_mode();
  if (family<RetraceAlg>(g) >= 5 || family<RetraceAlg>(g) == 3) {
    // Stage pi / Qn in the tile ring while a two-stage ring of them fits.
    const int64_t per_step = 8 * num_actions + 28;
    const bool staged = num_actions <= 16 && 2 * per_step * kTileThreads * 9 + 12 * kTileThreads * 9 <= 220 * 1024;
    p.warp_elems = staged ? 1 : 0;
    if (staged) return launch_tile<RetraceT<true>, 9>(p, g, ws, ws_bytes, s);
    return launch_tile<RetraceT<false>, 9>(p, g, ws, ws_bytes, s);
  }
  if ((mode == 0 || mode == 1 || mode == 4) && use_rows<RetraceAlg>(g)) return launch_rows<RetraceAlg, 1>(p, g, s);
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
  RLS_DEVICE_GUARD(rewards, next_values, terminateds, truncateds, bootstrap, out, seg ? seg->halo : nullptr, ws)
  Geom g;
  int st = make_geom(num_envs, seq_len, seg, true, g);
  if (st) return st;
  cudaStream_t s = as_stream(stream);
  std::lock_guard<std::recursive_mutex> launch_lock(launch_mutex());
  const size_t esz = in_dtype == RLS_BF16 ? 2 : 4, mb = (size_t)g.M * esz, nb = (size_t)g.N * 4;
  g.pdl = pdl_mode(s, {{rewards, mb}, {next_values, mb}, {terminateds, mb}, {truncateds, mb},
                      {bootstrap, mb}, {seg ? seg->halo : nullptr, nb}});
#define LAM_PARAMS(T)                                                                                     \
  typename LambdaAlg<T>::Params p;                                                                        \
  p.r = (const T*)rewards; p.nv = (const T*)next_values; p.term = (const T*)terminateds;                   \
  p.trunc = (const T*)truncateds; p.boot = (const T*)bootstrap; p.out0 = out; p.out1 = nullptr;            \
  p.boot_kind = boot_kind; p.gamma = gamma; p.g1l = gamma * (1.0f - lambda_); p.gl = gamma * lambda_;
  if (in_dtype == RLS_F32) {
    LAM_PARAMS(float)
    {
      const int fam = family<LambdaAlg<float>>(g);
      if (fam == 3) return lambda_v<TileL, float>(p, g, ws, ws_bytes, s);
      if (fam == 4) return lambda_v<Rows2L, float>(p, g, ws, ws_bytes, s);
      if (fam == 5) return lambda_v<Flat2L, float>(p, g, ws, ws_bytes, s);
      if (fam == 6) return lambda_v<Flat3L, float>(p, g, ws, ws_bytes, s);
      if (fam == 7) return lambda_v<Flat4L, float>(p, g, ws, ws_bytes, s);
      if (fam == 8) return lambda_v<VrowsL, float>(p, g, ws, ws_bytes, s);
    }
    return launch<LambdaAlg<float>>(p, g, ws, ws_bytes, s);
  } else {
    LAM_PARAMS(__nv_bfloat16)
    {
      const int fam = family<LambdaAlg<__nv_bfloat16>>(g);
      if (fam == 3) return lambda_v<TileL, __nv_bfloat16>(p, g, ws, ws_bytes, s);
      if (fam == 4) return lambda_v<Rows2L, __nv_bfloat16>(p, g, ws, ws_bytes, s);
      if (fam == 5) return lambda_v<Flat2L, __nv_bfloat16>(p, g, ws, ws_bytes, s);
      if (fam == 6) return lambda_v<Flat3L, __nv_bfloat16>(p, g, ws, ws_bytes, s);
      if (fam == 7) return lambda_v<Flat4L, __nv_bfloat16>(p, g, ws, ws_bytes, s);
      if (fam == 8) return lambda_v<VrowsL, __nv_bfloat16>(p, g, ws, ws_bytes, s);
    }
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
  RLS_DEVICE_GUARD(rewards, terminateds, truncateds, bootstrap, out, seg ? seg->halo : nullptr, ws)
  Geom g;
  int st = make_geom(num_envs, seq_len, seg, true, g);
  if (st) return st;
  cudaStream_t s = as_stream(stream);
  std::lock_guard<std::recursive_mutex> launch_lock(launch_mutex());
  const size_t esz = in_dtype == RLS_BF16 ? 2 : 4, mb = (size_t)g.M * esz, nb = (size_t)g.N * 4;
  g.pdl = pdl_mode(s, {{rewards, mb}, {terminateds, mb}, {truncateds, mb}, {bootstrap, mb},
                      {seg ? seg->halo : nullptr, nb}});
#define DISC_PARAMS(T)                                                                                    \
  typename DiscountedAlg<T>::Params p;                                                                    \
  p.r = (const T*)rewards; p.term = (const T*)terminateds; p.trunc = (const T*)truncateds;                 \
  p.boot = (const T*)bootstrap; p.out0 = out; p.out1 = nullptr; p.boot_kind = boot_kind; p.gamma = gamma;
  if (in_dtype == RLS_F32) {
    DISC_PARAMS(float)
    {
      const int fam = family<DiscountedAlg<float>>(g);
      if (fam == 3) return discounted_v<TileL, float>(p, g, ws, ws_bytes, s);
      if (fam == 4) return discounted_v<Rows2L, float>(p, g, ws, ws_bytes, s);
      if (fam == 5) return discounted_v<Flat2L, float>(p, g, ws, ws_bytes, s);
      if (fam == 6) return discounted_v<Flat3L, float>(p, g, ws, ws_bytes, s);
      if (fam == 7) return discounted_v<Flat4L, float>(p, g, ws, ws_bytes, s);
      if (fam == 8) return discounted_v<VrowsL, float>(p, g, ws, ws_bytes, s);
    }
    return launch<DiscountedAlg<float>>(p, g, ws, ws_bytes, s);
  } else {
    DISC_PARAMS(__nv_bfloat16)
    {
      const int fam = family<DiscountedAlg<__nv_bfloat16>>(g);
      if (fam == 3) return discounted_v<TileL, __nv_bfloat16>(p, g, ws, ws_bytes, s);
      if (fam == 4) return discounted_v<Rows2L, __nv_bfloat16>(p, g, ws, ws_bytes, s);
      if (fam == 5) return discounted_v<Flat2L, __nv_bfloat16>(p, g, ws, ws_bytes, s);
      if (fam == 6) return discounted_v<Flat3L, __nv_bfloat16>(p, g, ws, ws_bytes, s);
      if (fam == 7) return discounted_v<Flat4L, __nv_bfloat16>(p, g, ws, ws_bytes, s);
      if (fam == 8) return discounted_v<VrowsL, __nv_bfloat16>(p, g, ws, ws_bytes, s);
    }
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
  RLS_DEVICE_GUARD(x, dones, seed, out, seg ? seg->halo : nullptr, ws)
  Geom g;
  int st = make_geom(num_envs, seq_len, seg, false, g);
  if (st) return st;
  cudaStream_t s = as_stream(stream);
  std::lock_guard<std::recursive_mutex> launch_lock(launch_mutex());
  const size_t esz = in_dtype == RLS_BF16 ? 2 : 4, mb = (size_t)g.M * esz, nb = (size_t)g.N * 4;
  g.pdl = pdl_mode(s, {{x, mb}, {dones, mb}, {seed, nb}, {seg ? seg->halo : nullptr, nb}});
#define FWD_PARAMS(T)                                                                                     \
  typename ForwardAlg<T>::Params p;                                                                       \
  p.x = (const T*)x; p.done = (const T*)dones; p.seed = seed; p.halo = seg ? seg->halo : nullptr;          \
  p.out0 = out; p.out1 = nullptr; p.k = k; p.prev = prev;
  if (in_dtype == RLS_F32) {
    FWD_PARAMS(float)
    {
      const int fam = family<ForwardAlg<float>>(g);
      if (fam == 3) return forward_v<TileL, float>(p, g, ws, ws_bytes, s);
      if (fam == 4) return forward_v<Rows2L, float>(p, g, ws, ws_bytes, s);
      if (fam == 5) return forward_v<Flat2L, float>(p, g, ws, ws_bytes, s);
      if (fam == 6) return forward_v<Flat3L, float>(p, g, ws, ws_bytes, s);
      if (fam == 7) return forward_v<Flat4L, float>(p, g, ws, ws_bytes, s);
      if (fam == 8) return forward_v<VrowsL, float>(p, g, ws, ws_bytes, s);
    }
    return launch<ForwardAlg<float>>(p, g, ws, ws_bytes, s);
  } else {
    FWD_PARAMS(__nv_bfloat16)
    {
      const int fam = family<ForwardAlg<__nv_bfloat16>>(g);
      if (fam == 3) return forward_v<TileL, __nv_bfloat16>(p, g, ws, ws_bytes, s);
      if (fam == 4) return forward_v<Rows2L, __nv_bfloat16>(p, g, ws, ws_bytes, s);
      if (fam == 5) return forward_v<Flat2L, __nv_bfloat16>(p, g, ws, ws_bytes, s);
      if (fam == 6) return forward_v<Flat3L, __nv_bfloat16>(p, g, ws, ws_bytes, s);
      if (fam == 7) return forward_v<Flat4L, __nv_bfloat16>(p, g, ws, ws_bytes, s);
      if (fam == 8) return forward_v<VrowsL, __nv_bfloat16>(p, g, ws, ws_bytes, s);
    }
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
  RLS_DEVICE_GUARD(u, v, carry, out, seg ? seg->halo : nullptr, ws)
  Geom g;
  int st = make_geom(num_envs, seq_len, seg, direction == 0, g);
  if (st) return st;
  cudaStream_t s = as_stream(stream);
  std::lock_guard<std::recursive_mutex> launch_lock(launch_mutex());
  g.pdl = pdl_mode(s, {{u, (size_t)g.M * 4}, {v, (size_t)g.M * 4}, {carry, (size_t)g.N * 4},
                      {seg ? seg->halo : nullptr, (size_t)g.N * 4}});
  if (direction == 0) {
    AffineAlg<true>::Params p{u, v, carry, out, nullptr};
    {
      const int fam = family<AffineAlg<true>>(g);
      if (fam == 3) return affine_v<TileL, true>(p, g, ws, ws_bytes, s);
      if (fam == 4) return affine_v<Rows2L, true>(p, g, ws, ws_bytes, s);
      if (fam == 5) return affine_v<Flat2L, true>(p, g, ws, ws_bytes, s);
      if (fam == 6) return affine_v<Flat3L, true>(p, g, ws, ws_bytes, s);
      if (fam == 7) return affine_v<Flat4L, true>(p, g, ws, ws_bytes, s);
      if (fam == 8) return affine_v<VrowsL, true>(p, g, ws, ws_bytes, s);
    }
    return launch<AffineAlg<true>>(p, g, ws, ws_bytes, s);
  }
  AffineAlg<false>::Params p{u, v, carry, out, nullptr};
  {
      const int fam = family<AffineAlg<false>>(g);
      if (fam == 3) return affine_v<TileL, false>(p, g, ws, ws_bytes, s);
      if (fam == 4) return affine_v<Rows2L, false>(p, g, ws, ws_bytes, s);
      if (fam == 5) return affine_v<Flat2L, false>(p, g, ws, ws_bytes, s);
      if (fam == 6) return affine_v<Flat3L, false>(p, g, ws, ws_bytes, s);
      if (fam == 7) return affine_v<Flat4L, false>(p, g, ws, ws_bytes, s);
      if (fam == 8) return affine_v<VrowsL, false>(p, g, ws, ws_bytes, s);
    }
  return launch<AffineAlg<false>>(p, g, ws, ws_bytes, s);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// rls_gae_noalloc: GAE whose look-back scratch is a fixed array in this file,
// for callers that cannot allocate device memory.  Every GAE launch family
// uses tiles of at least kNoAllocMinTile elements (the flat look-back kernel:
// 4 warps x 32 lanes x one fp32 vector; flat2: 32 lanes x 4 rounds x 4; the
// tile kernel, flat3 and the row kernels use larger tiles or none), so
// RLS_NOALLOC_MAX_ELEMENTS / kNoAllocMinTile tile records in the larger of the
// two record layouts (24 bytes per tile, flat2's packed words) cover every path
// up to the maximum size.  The array starts zero-filled, as the look-back
// protocol requires; the kernels keep it consistent from call to call
// (epoch-tagged flags), and each call clears the ticket and exit counters
// before launching.  The error latch is left alone: rls_gae_noalloc_error()
// reads and clears it.
namespace {
constexpr int64_t kNoAllocMinTile = 512;
static_assert((int64_t)kWarps * 32 * InTraits<float>::kVec >= kNoAllocMinTile,
              "flat look-back tiles are at least kNoAllocMinTile elements");
static_assert(32LL * 4 * (16 / (int)sizeof(float)) >= kNoAllocMinTile, "flat2 tiles are at least kNoAllocMinTile");
static_assert((int64_t)kTileThreads * kTileK >= kNoAllocMinTile, "tile-kernel tiles are at least kNoAllocMinTile");
constexpr int64_t kNoAllocTiles = RLS_NOALLOC_MAX_ELEMENTS / kNoAllocMinTile;
constexpr size_t kNoAllocBytes = 64 + (size_t)kNoAllocTiles * 24;
static_assert(kNoAllocBytes >= 64 + (size_t)kNoAllocTiles * 20 + 16, "room for the flags layout too");

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[64] = {nullptr};
}  // namespace

static __device__ __align__(256) unsigned char g_noalloc_ws[kNoAllocBytes];

// Device address of this GPU's copy of the scratch (looked up once per device,
// with that device current).
static void* noalloc_scratch(int* status) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) { *status = RLS_ECUDA; return nullptr; }
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    // The host-side name of the array is not a device address.
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_ws) != cudaSuccess || !p) { *status = RLS_ECUDA; return nullptr; }
    g_noalloc_ptr[dev] = p;
  }
  *status = RLS_OK;
  return g_noalloc_ptr[dev];
}

extern "C" int rls_gae_noalloc(const void* rewards, const void* values, const void* terminateds,
                               const void* truncateds, const void* bootstrap, int boot_kind, float* advantages,
                               int64_t num_envs, int64_t seq_len, float gamma, float lambda_, int in_dtype,
                               const rls_segment_t* seg, void* stream) {
  if (num_envs < 0 || seq_len < 0) return RLS_EINVAL;
  if (num_envs == 0 || seq_len == 0) return RLS_OK;
  if (num_envs > RLS_NOALLOC_MAX_ELEMENTS / seq_len) return RLS_ETOOLARGE;
  if (!rewards || !values || !terminateds || !advantages) return RLS_EINVAL;
  // The scratch used is the copy on the GPU that holds the arrays.
  RLS_DEVICE_GUARD(rewards, values, terminateds, truncateds, bootstrap, advantages, seg ? seg->halo : nullptr)
  int st = RLS_OK;
  void* ws = noalloc_scratch(&st);
  if (!ws) return st;
  cudaStream_t s = as_stream(stream);
  std::lock_guard<std::recursive_mutex> launch_lock(launch_mutex());
  // Ticket and exit counters (bytes 0-7); the epoch (8-11) must keep counting
  // up and the error latch (12-15) keeps its bits until it is read.
  if (cudaMemsetAsync(ws, 0, 8, s) != cudaSuccess) return RLS_ECUDA;
  return rls_gae(rewards, values, terminateds, truncateds, bootstrap, boot_kind, advantages, num_envs, seq_len,
                 gamma, lambda_, in_dtype, seg, ws, kNoAllocBytes, stream);
}

extern "C" int rls_gae_noalloc_error(void* stream) {
  int st = RLS_OK;
  void* ws = noalloc_scratch(&st);
  if (!ws) return -1;
  return rls_workspace_error(ws, stream);
}
