// sdg_launch.h — kernel launch with programmatic stream serialization.
#pragma once
#include <cuda_runtime.h>

#include <utility>

namespace sdg {

// Launch `k` on `s` allowing it to start before the previous kernel in the
// stream has finished (its pdl_wait() orders the memory accesses). Optional
// cluster dimension (x) for cluster kernels.
template <typename... KArgs, typename... Args>
cudaError_t launch_kernel(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, int cluster_x,
                          Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  int n = 0;
  attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[n].val.programmaticStreamSerializationAllowed = 1;
  ++n;
  if (cluster_x > 0) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster_x;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, k, std::forward<Args>(args)...);
}

}  // namespace sdg
