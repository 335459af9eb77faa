// Host-side helpers shared by the translation units of libsplat200: status
// reporting (splat_last_error), the launch counter (splat_launch_count) and
// argument checks.  Defined in splat200.cu.
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace splat {
namespace host {

// Records `what` as the calling thread's last error and returns `status`.
int fail(int status, const char* what);
// kOk, or kCudaError (recording the CUDA error) when a launch failed.
int check_launch(const char* what);
// Counts one kernel launch and returns its stream; every launch passes its
// stream through here.
cudaStream_t counted(cudaStream_t s);
// Streaming multiprocessors of the current device (148 on B200).
int sm_count();

inline unsigned blocks_for(long long n, int block) {
  return static_cast<unsigned>((n + block - 1) / block);
}

// float2/float4 rows and 16-byte async copies need 8/16-byte aligned
// addresses (NULL passes; it means "absent").
inline bool aligned(const void* p, uintptr_t a) {
  return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0;
}

}  // namespace host
}  // namespace splat
