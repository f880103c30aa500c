// host_shared.h -- host-side state shared by the library's translation units.
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <mutex>

namespace rls {

// Every entry point enqueues its launches under this process-wide lock (a call
// may issue several launches that share the stream's workspace).
std::recursive_mutex& launch_mutex();

// Record layouts a workspace can hold; the first launch of one layout on a
// workspace last used by another clears the records (rlscan.cu).
enum : int { kLayoutNone = 0, kLayoutFlags = 1, kLayoutPacked = 2, kLayoutScratch = 3 };
int prepare_layout(void* ws, size_t wsb, int layout, cudaStream_t s);

}  // namespace rls
