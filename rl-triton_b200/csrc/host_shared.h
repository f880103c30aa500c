// host_shared.h -- host-side state shared by the library's translation units.
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <initializer_list>
#include <mutex>
#include <utility>

#include "rlscan.h"

namespace rls {

// Every entry point enqueues its launches under this process-wide lock (a call
// may issue several launches that share the stream's workspace).
std::recursive_mutex& launch_mutex();

// Record layouts a workspace can hold; the first launch of one layout on a
// workspace last used by another clears the records (rlscan.cu).
enum : int { kLayoutNone = 0, kLayoutFlags = 1, kLayoutPacked = 2, kLayoutScratch = 3 };
int prepare_layout(void* ws, size_t wsb, int layout, cudaStream_t s);

// Programmatic dependent launch bookkeeping (rlscan.cu): the output ranges of
// the last early-triggering launch per stream, and whether a new launch's
// inputs may overlap them (1: wait before the first load) or not (2: the
// first loads may precede the wait).  Called under launch_mutex().
struct PdlIn {
  const void* p;
  size_t bytes;
};
int pdl_mode(cudaStream_t s, std::initializer_list<PdlIn> ins);
void pdl_record(cudaStream_t s, const void* out0, const void* out1, size_t bytes);
void pdl_record(cudaStream_t s, std::initializer_list<PdlIn> outs);  // up to 4 ranges

// Launch a kernel that triggers its dependents early: plainly when pdl_flag is
// 0, else with the programmatic-stream-serialization attribute; either way its
// outputs (out_elems fp32 each, out1 may be null) become the stream's record.
template <class... KArgs, class... Args>
inline int launch_rowk(void (*kern)(KArgs...), int64_t blocks, int threads, cudaStream_t s, int pdl_flag,
                       int64_t out_elems, const float* out0, const float* out1, Args&&... args) {
  if (blocks > 0x7fffffffLL) return RLS_EINVAL;
  if (pdl_flag == 0) {
    kern<<<(unsigned)blocks, threads, 0, s>>>(std::forward<Args>(args)...);
    if (cudaPeekAtLastError() != cudaSuccess) return RLS_ECUDA;
  } else {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)blocks);
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...) != cudaSuccess) return RLS_ECUDA;
  }
  pdl_record(s, out0, out1, (size_t)out_elems * sizeof(float));
  return RLS_OK;
}


}  // namespace rls
