// Programmatic dependent launch (sm_90 and later).  A kernel launched with
// the programmatic-stream-serialization attribute may start while the kernel
// ahead of it on the stream is still running: everything it does before
// pdl_wait() must read only data that no kernel still in flight writes (the
// small-batch kernels read their weights there), and pdl_wait() returns once
// that kernel has completed and its writes are visible.
// pdl_launch_dependents() lets the next such launch start as soon as every CTA
// of this grid has executed it.  Both are no-ops for a kernel launched without
// the attribute, and for a kernel with no such dependent.
#pragma once

#include <cuda_runtime.h>

namespace m3 {

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Launch kern<<<grid, block, smem, stream>>>(args...), as a programmatic
// dependent launch when pdl is set.
template <typename... KArgs, typename... Args>
cudaError_t launch_maybe_pdl(bool pdl, void (*kern)(KArgs...), dim3 grid, dim3 block,
                             size_t smem, cudaStream_t stream, Args&&... args) {
  if (!pdl) {
    kern<<<grid, block, smem, stream>>>(static_cast<Args&&>(args)...);
    return cudaGetLastError();
  }
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<Args&&>(args)...);
}

}  // namespace m3
