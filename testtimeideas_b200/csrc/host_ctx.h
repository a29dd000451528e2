// Host-side identity of the CUDA context current on the calling thread, for
// caches of per-context resources (device addresses of __device__ symbols,
// library-owned streams and events). A device reset or a context other than
// the device's primary one yields another id, so nothing cached for one
// context is handed to another.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>

namespace ttt {

// Unique id (for the life of the process) of the current context; the current
// device's primary context is made current first if this thread has none yet.
// Returns false if no context can be made current or the driver lacks
// cuCtxGetId (CUDA < 12.0).
inline bool current_context_id(unsigned long long* id) {
  typedef CUresult (*GetCurrentFn)(CUcontext*);
  typedef CUresult (*GetIdFn)(CUcontext, unsigned long long*);
  static GetCurrentFn get_current = nullptr;
  static GetIdFn get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<GetCurrentFn>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<GetIdFn>(p);
  });
  if (get_current == nullptr || get_id == nullptr) return false;
  CUcontext ctx = nullptr;
  if (get_current(&ctx) != CUDA_SUCCESS) return false;
  if (ctx == nullptr) {
    // No context on this thread yet: since CUDA 12.0 cudaSetDevice makes the
    // device's primary context current (and allocates nothing).
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaSetDevice(dev) != cudaSuccess) return false;
    if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return false;
  }
  return get_id(ctx, id) == CUDA_SUCCESS;
}

}  // namespace ttt
