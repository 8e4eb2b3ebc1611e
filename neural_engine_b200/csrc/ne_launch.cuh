// ne_launch.cuh -- host-side kernel launch with programmatic dependent launch.
#pragma once
#include <cuda_runtime.h>

#include <cstdlib>

namespace ne {

// PDL is on unless the environment sets NE_PDL=0.
inline bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("NE_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

// Launch `kern` on `st`, allowing it to overlap its predecessor on the stream
// (the kernel itself calls pdl_wait() before reading what the predecessor wrote).
template <class Kern, class... Args>
cudaError_t launch_k(Kern kern, dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                     Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

// The same with thread-block clusters of `cluster_x` CTAs along x (the grid's x
// extent must be a multiple of it).
template <class Kern, class... Args>
cudaError_t launch_k_cluster(Kern kern, dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                             unsigned cluster_x, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster_x;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

}  // namespace ne
