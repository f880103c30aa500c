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
      if (prev) flag = (col == 0) ? a.halo[row] : load_in(a.f0, a.bf16, i - 1);
      else flag = load_in(a.f0, a.bf16, i);
      const float k = (a.alg == RLS_ALG_ELIGIBILITY) ? a.coef : 1.f;
      return k * (1.f - flag);
    }
    default:  // generic scans: v
      return __ldg(reinterpret_cast<const float*>(a.f0) + i);
  }
}

// mode 0: reduce (seg_a, seg_b); mode 1: fix-up with carry.
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
      b = decay_at(a, row, col);
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
  }
}

constexpr int kBlockWalk = 512;   // threads of the block-per-row walk
constexpr int kBlockElems = 4;    // consecutive (walk-order) elements per thread

// Block-per-row version of segment_walk (same results up to the rounding of
// the decay products).
template <int MODE>
__global__ void __launch_bounds__(kBlockWalk) segment_walk_block(const SegArgs a) {
  constexpr int NW = kBlockWalk / 32;
  constexpr int STEP = kBlockWalk * kBlockElems;
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
    float b[kBlockElems];
    int64_t col[kBlockElems];
#pragma unroll
    for (int q = 0; q < kBlockElems; ++q) {
      const int64_t k = k0 + (int64_t)threadIdx.x * kBlockElems + q;
      col[q] = k < S ? (a.backward ? (S - 1 - k) : k) : -1;
      b[q] = col[q] >= 0 ? decay_at(a, row, col[q]) : 1.f;
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
    if (MODE == 1) {
#pragma unroll
      for (int q = 0; q < kBlockElems; ++q) {
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
  }
}

// Few rows: a block per row; many rows: a warp per row.
template <int MODE>
int launch_walk(const SegArgs& a, void* stream) {
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (a.N <= 64) segment_walk_block<MODE><<<(unsigned)a.N, kBlockWalk, 0, s>>>(a);
  else segment_walk<MODE><<<(unsigned)((a.N + 3) / 4), 128, 0, s>>>(a);
  return cudaPeekAtLastError() == cudaSuccess ? RLS_OK : RLS_ECUDA;
}

int fill_args(int alg, const void* flag0, const void* flag1, int in_dtype, int64_t N, int64_t S, float coef,
              int flags, const rls_segment_t* seg, SegArgs& a) {
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
  if (needs_halo && !a.halo && !a.global_edge) return RLS_EINVAL;
  return RLS_OK;
}

}  // namespace

extern "C" {

int rls_segment_reduce(int alg, const void* flag0, const void* flag1, int in_dtype, const float* out,
                       float* seg_a, float* seg_b, int64_t num_envs, int64_t seq_len, float coef, int flags,
                       const rls_segment_t* seg, void* stream) {
  SegArgs a;
  int st = fill_args(alg, flag0, flag1, in_dtype, num_envs, seq_len, coef, flags, seg, a);
  if (st) return st;
  if (!out || !seg_a || !seg_b) return RLS_EINVAL;
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
  int st = fill_args(alg, flag0, flag1, in_dtype, num_envs, seq_len, coef, flags, seg, a);
  if (st) return st;
  if (!out || !carry) return RLS_EINVAL;
  a.out = out;
  a.carry = carry;
  a.seg_a = nullptr;
  a.seg_b = nullptr;
  if (num_envs == 0) return RLS_OK;
  return launch_walk<1>(a, stream);
}

}  // extern "C"
