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
// One warp per row walks 32 elements per step from the edge inward with a
// shuffle product scan.
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
  const unsigned blocks = (unsigned)((num_envs + 3) / 4);
  segment_walk<0><<<blocks, 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(a);
  return cudaPeekAtLastError() == cudaSuccess ? RLS_OK : RLS_ECUDA;
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
  const unsigned blocks = (unsigned)((num_envs + 3) / 4);
  segment_walk<1><<<blocks, 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(a);
  return cudaPeekAtLastError() == cudaSuccess ? RLS_OK : RLS_ECUDA;
}

}  // extern "C"
