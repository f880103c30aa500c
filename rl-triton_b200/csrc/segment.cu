// segment.cu -- carry exchange helpers for sequences split along time.
//
// A rank holding columns [t0, t0+S) of every row first runs the ordinary scan
// with the segment edge treated as a cut (carry 0).  Each row's segment is then
// summarised as the affine map (A, B) from the carry entering at the near edge
// to the state at the far edge; the ranks exchange these tiny maps, compose the
// true carry, and apply it with a bounded fix-up:
//   out[t] += P[t] * carry,   P[t] = prod of b over the elements between t and
//   the edge where the carry enters.
// P becomes exactly 0 at the first episode reset (b = 0) and underflows to 0
// after a few thousand steps when b < 1, so both walks stop early; a segment
// without any reset is still handled, just by walking all of it.
//
// Many rows: one warp per row walks 32 elements per step from the edge inward
// with a shuffle product scan.  Few rows (a single long sequence split across
// GPUs): one 512-thread block per row walks 2048 elements per step with a
// block-wide product scan, so the walk to the first reset (~10^4 steps for a
// 1e-4 done rate) takes a handful of steps instead of hundreds of dependent
// loads.
#include "rlscan.h"
#include "common.cuh"

using namespace rls;

namespace {

struct SegArgs {
  int alg;
  const void* f0;
  const void* f1;
  int bf16;
  float* out;
  const float* carry;   // fix-up: carry per row
  float* seg_a;         // reduce outputs
  float* seg_b;
  int64_t N, S;
  float coef;
  int ends_at;
  const float* halo;
  int global_edge;      // the segment holds the global row edge where the carry would enter
  int backward;
  int exclusive;        // the entry element's own decay is left out of P (backward summaries)
  const void* values;   // summary (GAE): V at the segment's first column
  float gamma;          // summary (GAE): discount of the entry element's next value
  float* summary;       // summary: [5][N]
};

__device__ __forceinline__ float load_in(const void* p, int bf16, int64_t i) {
  if (bf16) return bf16_bits_to_float(__ldg(reinterpret_cast<const unsigned short*>(p) + i));
  return __ldg(reinterpret_cast<const float*>(p) + i);
}

// Decay b at local column `col` of row `row` (original value, no cut).
__device__ float decay_at(const SegArgs& a, int64_t row, int64_t col) {
  const int64_t i = row * a.S + col;
  switch (a.alg) {
    case RLS_ALG_GAE:
    case RLS_ALG_LAMBDA:
    case RLS_ALG_DISCOUNTED: {
      float done = load_in(a.f0, a.bf16, i);
      if (a.f1) done = fminf(done + load_in(a.f1, a.bf16, i), 1.f);
      return a.coef * (1.f - done);
    }
    case RLS_ALG_ELIGIBILITY:
    case RLS_ALG_PREFIX: {
      const bool prev = (a.alg == RLS_ALG_ELIGIBILITY) || a.ends_at;
      float flag;
      if (prev) flag = (col == 0) ? (a.halo ? a.halo[row] : 0.f) : load_in(a.f0, a.bf16, i - 1);
      else flag = load_in(a.f0, a.bf16, i);
      const float k = (a.alg == RLS_ALG_ELIGIBILITY) ? a.coef : 1.f;
      return k * (1.f - flag);
    }
    default:  // generic scans: v
      return __ldg(reinterpret_cast<const float*>(a.f0) + i);
  }
}

// Summary fields 2-4 of a row (fields 0-1, A and B, are the reduce's seg_a /
// seg_b, which point into the same [5][N] buffer):
//   backward: 2 = alpha, the weight of the next segment's first value V in the
//             entry element (GAE: gamma (1 - term) where not truncated, else 0),
//             3 = beta, the entry element's own decay b, 4 = V at column 0
//             (GAE; 0 otherwise);
//   forward:  2 = m, the factor the next segment's entry gate takes from this
//             segment's last flag (1 - done[last] when the gate reads done[t-1],
//             else 1); 3, 4 = 0.
__device__ void write_summary(const SegArgs& a, int64_t row) {
  const int64_t N = a.N, S = a.S;
  float f2 = 0.f, f3 = 0.f, f4 = 0.f;
  if (S > 0) {
    const int64_t last = row * S + S - 1;
    if (a.backward) {
      f3 = decay_at(a, row, S - 1);
      if (a.alg == RLS_ALG_GAE) {
        const float term = load_in(a.f0, a.bf16, last);
        const float trunc = a.f1 ? load_in(a.f1, a.bf16, last) : 0.f;
        f2 = trunc == 0.f ? a.gamma * (1.f - term) : 0.f;
        f4 = load_in(a.values, a.bf16, row * S);
      }
    } else {
      const bool prev = (a.alg == RLS_ALG_ELIGIBILITY) || (a.alg == RLS_ALG_PREFIX && a.ends_at);
      f2 = prev ? 1.f - load_in(a.f0, a.bf16, last) : 1.f;
    }
  }
  a.summary[2 * N + row] = f2;
  a.summary[3 * N + row] = f3;
  a.summary[4 * N + row] = f4;
}

// mode 0: reduce (seg_a, seg_b) [+ summary]; mode 1: fix-up with carry.
template <int MODE>
__global__ void __launch_bounds__(128) segment_walk(const SegArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
  if (row >= a.N) return;
  const int64_t S = a.S;
  float c = 0.f;
  if (MODE == 1) {
    c = a.carry[row];
    if (c == 0.f || a.global_edge) return;
  }
  float P = 1.f;  // product of b from the edge to the current position
  bool zero = (MODE == 0) && a.global_edge;
  for (int64_t k0 = 0; k0 < S && !zero; k0 += 32) {
    const int64_t k = k0 + lane;  // distance from the edge
    float b = 1.f;
    int64_t col = 0;
    if (k < S) {
      col = a.backward ? (S - 1 - k) : k;
      b = (a.exclusive && k == 0) ? 1.f : decay_at(a, row, col);
    }
    // inclusive product scan over lanes in walk order
    float incl = b;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const float o = __shfl_up_sync(0xffffffffu, incl, d);
      if (lane >= d) incl *= o;
    }
    const float Pk = P * incl;
    if (MODE == 1 && k < S && Pk != 0.f) {
      float* o = a.out + row * S + col;
      *o = fmaf(Pk, c, *o);
    }
    P = __shfl_sync(0xffffffffu, Pk, 31);
    if (P == 0.f) zero = true;
  }
  if (MODE == 0 && lane == 0) {
    const int64_t far = a.backward ? 0 : (S - 1);
    a.seg_a[row] = S > 0 ? a.out[row * S + far] : 0.f;
    a.seg_b[row] = zero ? 0.f : P;
    if (a.summary) write_summary(a, row);
  }
}

constexpr int kBlockWalk = 512;   // threads of the virtual-row fix-up block
constexpr int kBlockElems = 4;    // consecutive (walk-order) elements per thread there
// The time-split walks (one block per row): 8192 steps per pass, so the walk
// to the first reset of a 1e-4 done rate takes one or two passes.
constexpr int kSegWalk = 1024;
constexpr int kSegElems = 8;

// Block-per-row version of segment_walk (same results up to the rounding of
// the decay products).
template <int MODE>
__global__ void __launch_bounds__(kSegWalk) segment_walk_block(const SegArgs a) {
  constexpr int NW = kSegWalk / 32;
  constexpr int STEP = kSegWalk * kSegElems;
  __shared__ float s_w[NW];
  __shared__ float s_base;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t row = blockIdx.x;
  const int64_t S = a.S;
  float c = 0.f;
  if (MODE == 1) {
    c = a.carry[row];
    if (c == 0.f || a.global_edge) return;  // uniform across the block
  }
  float base = 1.f;  // product of b over all earlier steps
  bool zero = (MODE == 0) && a.global_edge;
  for (int64_t k0 = 0; k0 < S && !zero; k0 += STEP) {
    float b[kSegElems];
    int64_t col[kSegElems];
#pragma unroll
    for (int q = 0; q < kSegElems; ++q) {
      const int64_t k = k0 + (int64_t)threadIdx.x * kSegElems + q;
      col[q] = k < S ? (a.backward ? (S - 1 - k) : k) : -1;
      b[q] = col[q] >= 0 ? ((a.exclusive && k == 0) ? 1.f : decay_at(a, row, col[q])) : 1.f;
    }
    float mine = 1.f;
#pragma unroll
    for (int q = 0; q < kSegElems; ++q) mine *= b[q];
    float incl = mine;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const float o = __shfl_up_sync(0xffffffffu, incl, d);
      if (lane >= d) incl *= o;
    }
    if (lane == 31) s_w[warp] = incl;
    __syncthreads();
    float before = 1.f, total = 1.f;
    for (int w = 0; w < NW; ++w) {
      if (w == warp) before = total;
      total *= s_w[w];
    }
    const float excl = __shfl_up_sync(0xffffffffu, incl, 1);
    float P = base * before * (lane == 0 ? 1.f : excl);
    if (MODE == 1) {
#pragma unroll
      for (int q = 0; q < kSegElems; ++q) {
        P *= b[q];
        if (col[q] >= 0 && P != 0.f) {
          float* o = a.out + row * S + col[q];
          *o = fmaf(P, c, *o);
        }
      }
    }
    if (threadIdx.x == 0) s_base = base * total;
    __syncthreads();
    base = s_base;
    if (base == 0.f) zero = true;
    __syncthreads();  // s_w / s_base are rewritten next step
  }
  if (MODE == 0 && threadIdx.x == 0) {
    const int64_t far = a.backward ? 0 : (S - 1);
    a.seg_a[row] = S > 0 ? a.out[row * S + far] : 0.f;
    a.seg_b[row] = zero ? 0.f : base;
    if (a.summary) write_summary(a, row);
  }
}

// Few rows: a block per row; many rows: a warp per row.
template <int MODE>
int launch_walk(const SegArgs& a, void* stream) {
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (a.N <= 64) segment_walk_block<MODE><<<(unsigned)a.N, kSegWalk, 0, s>>>(a);
  else segment_walk<MODE><<<(unsigned)((a.N + 3) / 4), 128, 0, s>>>(a);
  return cudaPeekAtLastError() == cudaSuccess ? RLS_OK : RLS_ECUDA;
}

int fill_args(int alg, const void* flag0, const void* flag1, int in_dtype, int64_t N, int64_t S, float coef,
              int flags, const rls_segment_t* seg, SegArgs& a, bool null_halo_is_zero = false) {
  if (alg < RLS_ALG_GAE || alg > RLS_ALG_SCAN_FWD || !flag0 || !seg || N < 0 || S < 0) return RLS_EINVAL;
  if (in_dtype != RLS_F32 && in_dtype != RLS_BF16) return RLS_EINVAL;
  if ((alg == RLS_ALG_SCAN_BWD || alg == RLS_ALG_SCAN_FWD) && in_dtype != RLS_F32) return RLS_EINVAL;
  a.alg = alg;
  a.f0 = flag0;
  a.f1 = flag1;
  a.bf16 = in_dtype == RLS_BF16;
  a.N = N;
  a.S = S;
  a.coef = coef;
  a.ends_at = flags & 1;
  a.halo = seg->halo;
  a.backward = !(alg == RLS_ALG_ELIGIBILITY || alg == RLS_ALG_PREFIX || alg == RLS_ALG_SCAN_FWD);
  a.global_edge = a.backward ? (seg->t0 + S == seg->total_len) : (seg->t0 == 0);
  const bool needs_halo = (alg == RLS_ALG_ELIGIBILITY) || (alg == RLS_ALG_PREFIX && a.ends_at);
  if (needs_halo && !a.halo && !a.global_edge && !null_halo_is_zero) return RLS_EINVAL;
  a.exclusive = (flags & RLS_SEG_EXCLUSIVE) && a.backward;
  a.values = nullptr;
  a.gamma = 0.f;
  a.summary = nullptr;
  return RLS_OK;
}

// ---------------------------------------------------------------------------
// Virtual rows (one long buffer cut into nseg segments of L steps, scanned with
// carry 0 at each segment's entry by vseg_kernel): compose the carries in walk
// order, then add P[t] * carry from each segment's entry inward until P is 0.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void flat_row_col(int64_t i, int64_t S, int64_t& row, int64_t& col) {
  if (i < 0x7fffffffLL && S < 0x7fffffffLL) {
    const unsigned q = (unsigned)i / (unsigned)S;
    row = q;
    col = i - (int64_t)q * S;
  } else {
    row = i / S;
    col = i - row * S;
  }
}

// Decay of flat element i inside a virtual-row walk: 0 at the edge of a (local)
// row on the side the carry enters from, else the recurrence's b.
__device__ float vrow_decay(const SegArgs& a, int64_t i) {
  int64_t row, col;
  flat_row_col(i, a.S, row, col);
  if (a.backward ? (col == a.S - 1) : (col == 0)) return 0.f;
  return decay_at(a, row, col);
}

// One block: each thread composes a run of up to six consecutive segments (in
// walk order), the block scans the runs (warp shuffles, then the 32 warp
// totals), and each thread re-walks its run from its exclusive prefix, storing
// the carry entering every segment.  Launched as a programmatic dependent of
// vseg_kernel: it starts while the scan drains and waits for it in pdl_wait.
constexpr int kCarryThreads = 1024;
__global__ void __launch_bounds__(kCarryThreads) vrows_carry(const float* seg_a, const float* seg_b, float* carry,
                                                             int64_t nseg, int backward) {
  __shared__ Pair s_warp[kCarryThreads / 32];
  pdl_trigger();  // the fix-up may launch now; it waits for this grid in pdl_wait
  pdl_wait();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t run = (nseg + kCarryThreads - 1) / kCarryThreads;
  const int64_t w0 = threadIdx.x * run, w1 = (w0 + run < nseg) ? w0 + run : nseg;
  auto seg_of = [&](int64_t w) { return backward ? nseg - 1 - w : w; };
  Pair m = pair_identity();
  for (int64_t w = w0; w < w1; ++w) {
    const int64_t sg = seg_of(w);
    m = compose(Pair{seg_a[sg], seg_b[sg]}, m);
  }
  Pair incl = m;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const Pair o{__shfl_up_sync(0xffffffffu, incl.a, d), __shfl_up_sync(0xffffffffu, incl.b, d)};
    if (lane >= d) incl = compose(incl, o);
  }
  if (lane == 31) s_warp[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    Pair x = s_warp[lane];
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const Pair o{__shfl_up_sync(0xffffffffu, x.a, d), __shfl_up_sync(0xffffffffu, x.b, d)};
      if (lane >= d) x = compose(x, o);
    }
    s_warp[lane] = x;
  }
  __syncthreads();
  Pair ex{__shfl_up_sync(0xffffffffu, incl.a, 1), __shfl_up_sync(0xffffffffu, incl.b, 1)};
  if (lane == 0) ex = pair_identity();
  if (warp > 0) ex = compose(ex, s_warp[warp - 1]);
  float c = ex.a;  // the walk starts with carry 0
  for (int64_t w = w0; w < w1; ++w) {
    const int64_t sg = seg_of(w);
    const float next = fmaf(seg_b[sg], c, seg_a[sg]);
    carry[sg] = c;
    c = next;
  }
}

// Launch with programmatic stream serialization (the kernel calls pdl_wait()
// before touching memory the preceding kernel writes).
template <typename... KArgs, typename... Args>
int launch_dependent(void (*kern)(KArgs...), unsigned blocks, unsigned threads, size_t smem, cudaStream_t s,
                     Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(blocks);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...) == cudaSuccess ? RLS_OK : RLS_ECUDA;
}

// Block per segment.  Code >= -1 (binary flags: b is 0 or coef): the decay
// product k steps in from the entry is coef^(k+1) up to the first b = 0 and
// underflows to 0 within ~-104/ln(coef) steps, so the carry is applied over
// that range with no flag reads, eight loads in flight per thread before
// their stores.  Code -2: 2048 walk-order steps per pass with a block product
// scan until P is 0.  Either way the block clears the segment's four words.
constexpr int kFixBatch = 8;
__global__ void __launch_bounds__(kBlockWalk) vrows_fixup(const SegArgs a, int64_t L, float* seg_a, float* seg_b,
                                                          float* carry, int* seg_code) {
  constexpr int NW = kBlockWalk / 32;
  constexpr int STEP = kBlockWalk * kBlockElems;
  __shared__ float s_w[NW];
  __shared__ float s_base;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t sg = blockIdx.x;
  pdl_wait();
  const float c = carry[sg];
  const int code = seg_code[sg];
  __syncthreads();  // every thread has read its words before they are cleared
  if (threadIdx.x == 0) {
    seg_a[sg] = 0.f;
    seg_b[sg] = 0.f;
    carry[sg] = 0.f;
    seg_code[sg] = 0;
  }
  if (c == 0.f) return;  // uniform across the block
  const int64_t s0 = sg * L;
  const int64_t len = (a.N - s0 < L) ? a.N - s0 : L;  // a.N holds the flat length here
  if (code >= -1) {
    int64_t n = code >= 0 ? (a.backward ? len - 1 - code : code) : len;  // steps that take the carry
    const bool unit = a.coef == 1.f;
    if (!unit) {
      // |coef| < 1: the product underflows to 0 within -110 / ln|coef| steps;
      // otherwise it never does and every step up to the first reset takes it.
      const float ac = fabsf(a.coef);
      if (ac > 0.f && ac < 1.f) {
        const float lim = -110.f / logf(ac) + 64.f;
        if ((float)n > lim) n = (int64_t)lim;
      }
    }
    for (int64_t k0 = 0; k0 < n; k0 += (int64_t)kBlockWalk * kFixBatch) {
      float v[kFixBatch];
      int64_t idx[kFixBatch];
#pragma unroll
      for (int j = 0; j < kFixBatch; ++j) {
        const int64_t k = k0 + (int64_t)j * kBlockWalk + threadIdx.x;  // walk distance from the entry
        idx[j] = k < n ? (a.backward ? s0 + len - 1 - k : s0 + k) : -1;
        v[j] = idx[j] >= 0 ? a.out[idx[j]] : 0.f;
      }
#pragma unroll
      for (int j = 0; j < kFixBatch; ++j) {
        if (idx[j] < 0) continue;
        const int64_t k = k0 + (int64_t)j * kBlockWalk + threadIdx.x;
        const float P = unit ? 1.f : powf(a.coef, (float)(k + 1));
        a.out[idx[j]] = fmaf(P, c, v[j]);
      }
    }
    return;
  }
  float base = 1.f;
  for (int64_t k0 = 0; k0 < len; k0 += STEP) {
    float b[kBlockElems];
    int64_t idx[kBlockElems];
#pragma unroll
    for (int q = 0; q < kBlockElems; ++q) {
      const int64_t k = k0 + (int64_t)threadIdx.x * kBlockElems + q;
      idx[q] = k < len ? (a.backward ? s0 + len - 1 - k : s0 + k) : -1;
      b[q] = idx[q] >= 0 ? vrow_decay(a, idx[q]) : 1.f;
    }
    float mine = 1.f;
#pragma unroll
    for (int q = 0; q < kBlockElems; ++q) mine *= b[q];
    float incl = mine;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const float o = __shfl_up_sync(0xffffffffu, incl, d);
      if (lane >= d) incl *= o;
    }
    if (lane == 31) s_w[warp] = incl;
    __syncthreads();
    float before = 1.f, total = 1.f;
    for (int w = 0; w < NW; ++w) {
      if (w == warp) before = total;
      total *= s_w[w];
    }
    const float excl = __shfl_up_sync(0xffffffffu, incl, 1);
    float P = base * before * (lane == 0 ? 1.f : excl);
#pragma unroll
    for (int q = 0; q < kBlockElems; ++q) {
      P *= b[q];
      if (idx[q] >= 0 && P != 0.f) a.out[idx[q]] = fmaf(P, c, a.out[idx[q]]);
    }
    if (threadIdx.x == 0) s_base = base * total;
    __syncthreads();
    base = s_base;
    __syncthreads();  // s_w / s_base are rewritten next pass
    if (base == 0.f) break;  // uniform
  }
}

// V-trace virtual rows (kernels/vtrace_fused.py:98-196): each segment was
// scanned with Delta = 0 entering at its far edge, so the true result adds
// P[t] * c to the targets (P[t] = prod of b over t..far edge, b = gamma *
// min(c_bar, ratio) * (1 - done), 0 at a row's last column) and
// rho[t] * gamma * (1 - term[t]) * P[t+1] * c to the advantages where
// vs_next is vs[t+1] (not truncated, not a row's last column).  One warp per
// segment, 128 walk-order steps per pass (four per lane), until the product is
// 0: the first reset, or underflow after a few hundred steps of c < 1.  Reads
// lpt, lpb, term[, trunc] and both outputs only over that range.
struct VtraceFixArgs {
  const void *lpt, *lpb, *term, *trunc;
  float *out0, *out1;
  int bf16;
  float gamma, rho_bar, c_bar;
  int64_t M, S, L, nseg;
};
constexpr int kVfixElems = 8;
// One pass of the walk for one lane: input loads and the per-step decay b and
// advantage weight w of its kVfixElems steps.
struct VfixPass {
  float b[kVfixElems], w[kVfixElems];
  int64_t idx[kVfixElems];
  float mine;  // product of this lane's b
};
__device__ __forceinline__ void vfix_pass(const VtraceFixArgs& a, int64_t e, int64_t len, int64_t k0, int lane,
                                          VfixPass& f) {
  float lt[kVfixElems], lb[kVfixElems], tm[kVfixElems], tr[kVfixElems];
#pragma unroll
  for (int q = 0; q < kVfixElems; ++q) {
    const int64_t k = k0 + (int64_t)lane * kVfixElems + q;
    f.idx[q] = k < len ? e - 1 - k : -1;
    const int64_t i = f.idx[q] >= 0 ? f.idx[q] : e - 1;
    lt[q] = load_in(a.lpt, a.bf16, i);
    lb[q] = load_in(a.lpb, a.bf16, i);
    tm[q] = load_in(a.term, a.bf16, i);
    tr[q] = a.trunc ? load_in(a.trunc, a.bf16, i) : 0.f;
  }
  f.mine = 1.f;
#pragma unroll
  for (int q = 0; q < kVfixElems; ++q) {
    const bool row_end = f.idx[q] >= 0 && (f.idx[q] % a.S) == a.S - 1;
    const float ratio = expf(lt[q] - lb[q]);
    const float done = a.trunc ? fminf(tm[q] + tr[q], 1.f) : tm[q];
    f.b[q] = f.idx[q] < 0 ? 1.f : (row_end ? 0.f : a.gamma * fminf(ratio, a.c_bar) * (1.f - done));
    // weight of vs[t+1]'s correction in the advantage at t
    f.w[q] = (f.idx[q] < 0 || row_end || tr[q] != 0.f) ? 0.f : fminf(ratio, a.rho_bar) * a.gamma * (1.f - tm[q]);
    f.mine *= f.b[q];
  }
}

// Launched as a programmatic dependent of vrows_carry (which triggers as soon
// as it runs): the first pass's inputs -- which none of this call's kernels
// write -- are loaded and turned into decays before pdl_wait, while the scan
// and the carry composition finish; only the carry and the outputs are read
// after it.
__global__ void __launch_bounds__(128) vrows_fixup_vtrace(const VtraceFixArgs a, float* seg_a, float* seg_b,
                                                          float* carry, int* seg_code) {
  const int lane = threadIdx.x & 31;
  const int64_t sg = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
  const bool live = sg < a.nseg;
  const int64_t s0 = live ? sg * a.L : 0;
  const int64_t len = !live ? 0 : ((a.M - s0 < a.L) ? a.M - s0 : a.L);
  const int64_t e = s0 + len;  // the carry enters here (walk runs e-1, e-2, ...)
  VfixPass f;
  if (live) vfix_pass(a, e, len, 0, lane, f);
  pdl_wait();
  if (!live) return;
  // The carry and the first pass's outputs are loaded together (one round trip).
  const float c = carry[sg];
  float o0[kVfixElems], o1[kVfixElems];
  auto load_outs = [&]() {
#pragma unroll
    for (int q = 0; q < kVfixElems; ++q) {
      const int64_t i = f.idx[q] >= 0 ? f.idx[q] : e - 1;
      o0[q] = a.out0[i];
      o1[q] = a.out1[i];
    }
  };
  load_outs();
  __syncwarp();  // every lane has read the carry before it is cleared
  if (lane == 0) {
    seg_a[sg] = 0.f;
    seg_b[sg] = 0.f;
    carry[sg] = 0.f;
    seg_code[sg] = 0;
  }
  if (c == 0.f) return;  // uniform across the warp
  float base = 1.f;      // product of b over all earlier walk steps
  for (int64_t k0 = 0; k0 < len; k0 += 32 * kVfixElems) {
    if (k0 > 0) {
      vfix_pass(a, e, len, k0, lane, f);
      load_outs();
    }
    float incl = f.mine;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const float o = __shfl_up_sync(0xffffffffu, incl, d);
      if (lane >= d) incl *= o;
    }
    const float excl = __shfl_up_sync(0xffffffffu, incl, 1);
    float P = base * (lane == 0 ? 1.f : excl);  // product over the walk steps before this lane's first
#pragma unroll
    for (int q = 0; q < kVfixElems; ++q) {
      if (f.idx[q] < 0 || P == 0.f) break;
      const int64_t i = f.idx[q];
      if (f.w[q] != 0.f) a.out1[i] = fmaf(f.w[q] * P, c, o1[q]);
      P *= f.b[q];
      if (P != 0.f) a.out0[i] = fmaf(P, c, o0[q]);
    }
    base *= __shfl_sync(0xffffffffu, incl, 31);
    if (base == 0.f) break;  // uniform
  }
}

}  // namespace

namespace rls {

int vrows_finish_vtrace(const void* lpt, const void* lpb, const void* term, const void* trunc, int bf16, float* out0,
                        float* out1, int64_t M, int64_t S, float gamma, float rho_bar, float c_bar, float* seg_a,
                        float* seg_b, float* carry, int* seg_code, int64_t nseg, int64_t L, cudaStream_t s) {
  if (nseg > 6144) return RLS_EINVAL;  // callers keep nseg <= 6144
  VtraceFixArgs a{lpt, lpb, term, trunc, out0, out1, bf16, gamma, rho_bar, c_bar, M, S, L, nseg};
  if (int st = launch_dependent(vrows_carry, 1, kCarryThreads, 0, s, (const float*)seg_a, (const float*)seg_b, carry,
                                nseg, 1))
    return st;
  return launch_dependent(vrows_fixup_vtrace, (unsigned)((nseg + 3) / 4), 128, 0, s, a, seg_a, seg_b, carry,
                          seg_code);
}

int vrows_finish(int alg, const void* f0, const void* f1, int bf16, float* out, int64_t M, int64_t S, float coef,
                 int ends_at, float* seg_a, float* seg_b, float* carry, int* seg_code, int64_t nseg, int64_t L,
                 cudaStream_t s) {
  SegArgs a{};
  a.alg = alg;
  a.f0 = f0;
  a.f1 = f1;
  a.bf16 = bf16;
  a.out = out;
  a.N = M;
  a.S = S;
  a.coef = coef;
  a.ends_at = ends_at;
  a.halo = nullptr;
  a.backward = !(alg == RLS_ALG_ELIGIBILITY || alg == RLS_ALG_PREFIX || alg == RLS_ALG_SCAN_FWD);
  if (nseg > 6144) return RLS_EINVAL;  // callers keep nseg <= 6144
  if (int st = launch_dependent(vrows_carry, 1, kCarryThreads, 0, s, (const float*)seg_a, (const float*)seg_b, carry,
                                nseg, (int)a.backward))
    return st;
  return launch_dependent(vrows_fixup, (unsigned)nseg, kBlockWalk, 0, s, a, L, seg_a, seg_b, carry, seg_code);
}

}  // namespace rls

extern "C" {

int rls_segment_reduce(int alg, const void* flag0, const void* flag1, int in_dtype, const float* out,
                       float* seg_a, float* seg_b, int64_t num_envs, int64_t seq_len, float coef, int flags,
                       const rls_segment_t* seg, void* stream) {
  SegArgs a;
  int st = fill_args(alg, flag0, flag1, in_dtype, num_envs, seq_len, coef, flags, seg, a);
  if (st) return st;
  if (!out || !seg_a || !seg_b) return RLS_EINVAL;
  DeviceGuard guard{flag0, flag1, out, seg_a, seg_b, seg ? seg->halo : nullptr};
  if (guard.status()) return guard.status();
  a.out = const_cast<float*>(out);
  a.carry = nullptr;
  a.seg_a = seg_a;
  a.seg_b = seg_b;
  if (num_envs == 0) return RLS_OK;
  return launch_walk<0>(a, stream);
}

int rls_segment_fixup(int alg, const void* flag0, const void* flag1, int in_dtype, float* out, const float* carry,
                      int64_t num_envs, int64_t seq_len, float coef, int flags, const rls_segment_t* seg,
                      void* stream) {
  SegArgs a;
  int st = fill_args(alg, flag0, flag1, in_dtype, num_envs, seq_len, coef, flags, seg, a,
                     (flags & RLS_SEG_EXCLUSIVE) != 0);
  if (st) return st;
  if (!out || !carry) return RLS_EINVAL;
  DeviceGuard guard{flag0, flag1, out, carry, seg ? seg->halo : nullptr};
  if (guard.status()) return guard.status();
  a.out = out;
  a.carry = carry;
  a.seg_a = nullptr;
  a.seg_b = nullptr;
  if (num_envs == 0) return RLS_OK;
  return launch_walk<1>(a, stream);
}

int rls_segment_summary(int alg, const void* flag0, const void* flag1, const void* values, int in_dtype,
                        const float* out, float* summary, int64_t num_envs, int64_t seq_len, float gamma,
                        float coef, int flags, const rls_segment_t* seg, void* stream) {
  SegArgs a;
  int st = fill_args(alg, flag0, flag1, in_dtype, num_envs, seq_len, coef, flags | RLS_SEG_EXCLUSIVE, seg, a, true);
  if (st) return st;
  if (!out || !summary || (alg == RLS_ALG_GAE && !values)) return RLS_EINVAL;
  DeviceGuard guard{flag0, flag1, values, out, summary, seg ? seg->halo : nullptr};
  if (guard.status()) return guard.status();
  a.out = const_cast<float*>(out);
  a.carry = nullptr;
  a.summary = summary;
  a.seg_a = summary;
  a.seg_b = summary + num_envs;
  a.values = values;
  a.gamma = gamma;
  if (num_envs == 0) return RLS_OK;
  return launch_walk<0>(a, stream);
}

}  // extern "C"

namespace {
// One thread per row: the carry entering rank `rank`'s segment from the W
// summaries ([W][5][N], rank order).
__global__ void segment_compose(const float* sm, int rank, int world, int backward, int64_t N, float* carry) {
  const int64_t row = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= N) return;
  auto F = [&](int k, int f) { return sm[((int64_t)k * 5 + f) * N + row]; };
  float c = 0.f;
  if (backward) {
    if (rank < world - 1) {
      float s0 = F(world - 1, 0);  // state at the first column of the last segment
      for (int k = world - 2; k > rank; --k) {
        const float corr = fmaf(F(k, 3), s0, F(k, 2) * F(k + 1, 4));
        s0 = fmaf(F(k, 1), corr, F(k, 0));
      }
      c = fmaf(F(rank, 3), s0, F(rank, 2) * F(rank + 1, 4));
    }
  } else {
    for (int k = 0; k < rank; ++k) c = F(k, 2) * fmaf(F(k, 1), c, F(k, 0));
  }
  carry[row] = c;
}
}  // namespace

extern "C" int rls_segment_compose(const float* summaries, int rank, int world, int backward, int64_t num_envs,
                                   float* carry, void* stream) {
  if (!summaries || !carry || world < 1 || rank < 0 || rank >= world || num_envs < 0) return RLS_EINVAL;
  if (num_envs == 0) return RLS_OK;
  DeviceGuard guard{summaries, carry};
  if (guard.status()) return guard.status();
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  segment_compose<<<(unsigned)((num_envs + 255) / 256), 256, 0, s>>>(summaries, rank, world, backward, num_envs,
                                                                    carry);
  return cudaPeekAtLastError() == cudaSuccess ? RLS_OK : RLS_ECUDA;
}
