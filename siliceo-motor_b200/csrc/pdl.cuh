// Programmatic dependent launch for the decode chain.
//
// A kernel started with launch_pdl may begin while the previous kernel on the
// stream is still running. Before pdl_wait() it may only touch memory that
// kernel does not write (its weights, the KV cache of earlier positions, its
// own shared memory); pdl_wait() returns once the previous kernel has
// finished and its writes are visible. pdl_trigger() lets the next kernel of
// the stream start early. Both are no-ops for a kernel launched the ordinary
// way.
#pragma once
#include <cuda_runtime.h>

#include <utility>

namespace sm {

#ifdef __CUDACC__
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
#endif

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace sm
