// common.cuh -- shared device helpers for the B200 return-estimation scans.
//
// Every estimator of the reference (simonsays1980/rl-triton) is a first-order
// affine recurrence  x[t] = a[t] + b[t] * x[t(+/-)1].  An element, a lane's run
// of elements, a warp, a tile and a whole segment are all summarised by the
// same object: the affine map  carry -> a + b * carry  (struct Pair).  The
// reference composes the same maps inside tl.associative_scan with the
// combine of src/rl_triton/kernels/scan.py:23-32.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include <initializer_list>

namespace rls {

// Affine map  c -> a + b*c  (state at the near end as a function of the carry
// entering at the far end).
struct Pair {
  float a, b;
};

__device__ __forceinline__ Pair pair_identity() { return Pair{0.f, 1.f}; }

// near(far(c)): `near` is the map closer to the output, `far` the one closer
// to where the carry enters.
__device__ __forceinline__ Pair compose(Pair near, Pair far) {
  return Pair{fmaf(near.b, far.a, near.a), near.b * far.b};
}

__device__ __forceinline__ float apply(Pair p, float c) { return fmaf(p.b, c, p.a); }

__device__ __forceinline__ Pair shfl_pair_down(Pair p, int d) {
  return Pair{__shfl_down_sync(0xffffffffu, p.a, d), __shfl_down_sync(0xffffffffu, p.b, d)};
}
__device__ __forceinline__ Pair shfl_pair_up(Pair p, int d) {
  return Pair{__shfl_up_sync(0xffffffffu, p.a, d), __shfl_up_sync(0xffffffffu, p.b, d)};
}
__device__ __forceinline__ Pair shfl_pair_idx(Pair p, int src) {
  return Pair{__shfl_sync(0xffffffffu, p.a, src), __shfl_sync(0xffffffffu, p.b, src)};
}

// ---- workspace ---------------------------------------------------------
// [ header 64 B | flags u32[ntiles] (padded to 16 B) | agg float2[ntiles] |
//   incl float2[ntiles] ]
// Zero-filled once by the owner.  The epoch (bumped by the last CTA of every
// launch) tags each tile flag, so no per-call clearing is needed.
struct WsHeader {
  unsigned ticket;    // dynamic tile ticket (reset by the last CTA)
  unsigned finished;  // CTAs finished in this launch (reset by the last CTA)
  unsigned epoch;     // launch counter, 30 bits
  unsigned error;     // latched error bits (1: look-back wait, 2: bulk-copy wait)
  unsigned pad[12];
};
static_assert(sizeof(WsHeader) == 64, "header is 64 bytes");

constexpr unsigned kFlagAgg = 1u;   // aggregate of the tile published
constexpr unsigned kFlagIncl = 2u;  // inclusive prefix of the tile published
constexpr unsigned kFlagSelf = 3u;  // inclusive prefix that needed no carry (product of b is 0)
constexpr unsigned kEpochMask = 0x3fffffffu;

struct Workspace {
  WsHeader* hdr;
  unsigned* flags;
  float2* agg;
  float2* incl;
};

__host__ __device__ inline size_t ws_bytes_for_tiles(int64_t ntiles) {
  size_t f = ((size_t)ntiles * 4 + 15) & ~(size_t)15;
  return 64 + f + (size_t)ntiles * 16;
}

// Tiles a workspace of `bytes` can describe.  The layout is carved by this
// capacity -- a property of the buffer, not of the launch -- so every launch on
// one buffer sees the flags, aggregates and inclusive values at the same
// places, and a stale aggregate can never be read as another launch's flag.
__host__ __device__ inline int64_t ws_capacity(size_t bytes) {
  if (bytes < 64 + 20) return 0;
  int64_t cap = (int64_t)((bytes - 64) / 20);
  while (cap > 0 && ws_bytes_for_tiles(cap) > bytes) --cap;
  return cap;
}

__host__ __device__ inline Workspace ws_carve(void* base, int64_t capacity) {
  char* p = (char*)base;
  Workspace w;
  w.hdr = (WsHeader*)p;
  w.flags = (unsigned*)(p + 64);
  size_t f = ((size_t)capacity * 4 + 15) & ~(size_t)15;
  w.agg = (float2*)(p + 64 + f);
  w.incl = w.agg + capacity;
  return w;
}

// ---- memory-model helpers (PTX) -----------------------------------------
__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_u32(unsigned* p, unsigned v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_relaxed_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// ---- streaming global loads / stores ------------------------------------
// Inputs are read exactly once: evict-first in L1 and L2.
__device__ __forceinline__ float4 ld_stream_f4(const float* p) {
  return __ldcs(reinterpret_cast<const float4*>(p));
}
__device__ __forceinline__ uint4 ld_stream_u4(const void* p) {
  return __ldcs(reinterpret_cast<const uint4*>(p));
}
__device__ __forceinline__ void st_stream_f4(float* p, float4 v) {
  __stcs(reinterpret_cast<float4*>(p), v);
}

__device__ __forceinline__ float bf16_bits_to_float(unsigned short h) {
  return __uint_as_float(((unsigned)h) << 16);
}

// Element type traits for the floating-point input streams.
template <class T>
struct InTraits;
template <>
struct InTraits<float> {
  static constexpr int kVec = 4;  // elements per 16-byte vector
  __device__ __forceinline__ static float scalar(const float* p, int64_t i) { return __ldg(p + i); }
  // Load kVec consecutive elements starting at i (16-byte aligned).
  __device__ __forceinline__ static void vec(const float* p, int64_t i, float* out) {
    float4 v = ld_stream_f4(p + i);
    out[0] = v.x; out[1] = v.y; out[2] = v.z; out[3] = v.w;
  }
};
template <>
struct InTraits<__nv_bfloat16> {
  static constexpr int kVec = 8;
  __device__ __forceinline__ static float scalar(const __nv_bfloat16* p, int64_t i) {
    unsigned short h = __ldg(reinterpret_cast<const unsigned short*>(p) + i);
    return bf16_bits_to_float(h);
  }
  __device__ __forceinline__ static void vec(const __nv_bfloat16* p, int64_t i, float* out) {
    uint4 v = ld_stream_u4(p + i);
    unsigned w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      out[2 * k] = __uint_as_float(w[k] << 16);
      out[2 * k + 1] = __uint_as_float(w[k] & 0xffff0000u);
    }
  }
};

// Load `n` (<= N) consecutive elements with bounds; pads the rest with `fill`.
template <class T, int N>
__device__ __forceinline__ void load_run(const T* p, int64_t i, int64_t M, bool full, float fill,
                                         float (&out)[N]) {
  static_assert(N % InTraits<T>::kVec == 0, "run is a whole number of vectors");
  if (full) {
#pragma unroll
    for (int k = 0; k < N; k += InTraits<T>::kVec) InTraits<T>::vec(p, i + k, out + k);
  } else {
#pragma unroll
    for (int k = 0; k < N; ++k) out[k] = (i + k < M) ? InTraits<T>::scalar(p, i + k) : fill;
  }
}

template <int N>
__device__ __forceinline__ void store_run(float* p, int64_t i, int64_t M, bool full,
                                          const float (&v)[N]) {
  if (full) {
#pragma unroll
    for (int k = 0; k < N; k += 4) st_stream_f4(p + i + k, make_float4(v[k], v[k + 1], v[k + 2], v[k + 3]));
  } else {
#pragma unroll
    for (int k = 0; k < N; ++k)
      if (i + k < M) p[i + k] = v[k];
  }
}

// Bounded spin limits.  A wait that runs out latches an error bit in the
// workspace and the kernel carries on with an identity carry, so a broken
// invariant shows up as a host-visible status, never as a hung GPU.
constexpr unsigned kSpinLimit = 1u << 22;  // ~0.3 s with the nanosleep back-off

// ---- programmatic dependent launch ------------------------------------------
// A kernel launched with cudaLaunchAttributeProgrammaticStreamSerialization may
// start while the kernel before it on the stream is still running.  It must
// execute pdl_wait() (griddepcontrol.wait: the preceding grid has completed and
// its memory is visible) before it reads anything that grid may have written
// and before its first store; pdl_trigger() lets the next such kernel launch.
// Both are no-ops for a kernel launched without the attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---- host: pointer placement and device guard ------------------------------
// Every entry point checks, before it enqueues anything, that each non-null
// array argument is memory of one CUDA device (device or managed memory, not
// pageable or pinned host memory), and runs the call with that device current,
// restoring the caller's device afterwards.  A host pointer handed to a kernel
// would fault the GPU; here it returns a status instead.
class DeviceGuard {
 public:
  // status(): 0 = ok; otherwise RLS_ENOTDEVICE (7) from rlscan.h.
  DeviceGuard(std::initializer_list<const void*> ptrs) {
    int dev = -1;
    for (const void* p : ptrs) {
      if (!p) continue;
      cudaPointerAttributes at;
      if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
        cudaGetLastError();  // clear the sticky-free error the query leaves
        status_ = 7;
        return;
      }
      if (at.type != cudaMemoryTypeDevice && at.type != cudaMemoryTypeManaged) { status_ = 7; return; }
      if (dev < 0) dev = at.device;
      else if (at.device != dev) { status_ = 7; return; }
    }
    if (dev < 0) return;
    if (cudaGetDevice(&prev_) != cudaSuccess) { cudaGetLastError(); prev_ = -1; }
    if (prev_ != dev) {
      if (cudaSetDevice(dev) != cudaSuccess) { status_ = 7; prev_ = -1; return; }
      switched_ = true;
    }
  }
  ~DeviceGuard() {
    if (switched_ && prev_ >= 0) cudaSetDevice(prev_);
  }
  int status() const { return status_; }
  DeviceGuard(const DeviceGuard&) = delete;
  DeviceGuard& operator=(const DeviceGuard&) = delete;

 private:
  int status_ = 0;
  int prev_ = -1;
  bool switched_ = false;
};

}  // namespace rls
