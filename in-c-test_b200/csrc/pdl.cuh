#pragma once
// Programmatic dependent launch for the chains of small kernels of a decode
// step.  A kernel launched by launch_dependent() may be scheduled while the
// previous kernel on its stream is still running; it calls pdl_wait() before
// its first global memory access (read or write), which returns once that
// kernel has completed and its writes are visible.  pdl_trigger() lets the
// next dependent grid be scheduled; every kernel here calls it after its own
// pdl_wait(), so a dependent is never scheduled before its predecessor's
// predecessor has completed -- a dependent that reads an older kernel's
// output before its own wait (the attend's first query) stays correct.  When
// the launch had no programmatic predecessor both calls return at once.
#include <cuda_runtime.h>

#include <utility>

namespace kvl {

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... K, typename... A>
inline cudaError_t launch_dependent(void (*fn)(K...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                                    A &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, fn, std::forward<A>(args)...);
}

}  // namespace kvl
