// pdl.cuh -- programmatic dependent launch (PDL) for the kernels of the forward.
//
// Every kernel of the forward is launched with programmatic stream
// serialisation: the next kernel in the stream may be scheduled before this
// one finishes, runs its prologue (barrier setup, TMEM allocation, descriptor
// prefetch, address arithmetic) and then blocks in griddepcontrol.wait until
// this grid has completed and its memory is visible. Each kernel therefore
// calls pdl_wait() before its first access to global memory that another
// kernel of the forward writes or reads, and pdl_launch() to let its
// successor be scheduled. Without the launch attribute both are no-ops.
#pragma once
#include <cuda_runtime.h>

#include <utility>

namespace mfb200 {

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Whether launches use the PDL attribute (default on; off for A/B timing).
bool pdl_enabled();
void set_pdl(bool enable);

// cudaLaunchKernelEx with the PDL attribute (when enabled) and an optional
// thread-block cluster of `cluster_x` CTAs.
template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                     int cluster_x, Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster_x > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = static_cast<unsigned>(cluster_x);
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace mfb200
