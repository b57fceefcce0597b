// launch.cuh -- how the library launches its GEMM, GEMV and fix-up kernels.
//
// Each launch sets programmatic stream serialisation, so a kernel's CTAs can
// become resident and run their prologue (barrier init, TMEM allocation,
// descriptor prefetch) while the previous kernel on the stream drains; each
// kernel calls griddep_wait() (ptx.cuh) before its first global-memory access,
// so stream order is kept for every byte it reads or writes. A cluster shape
// other than 1 x 1 x 1 is added as the second attribute.
#pragma once
#include <cuda_runtime.h>

#include <utility>

namespace mmr {

template <typename... KArgs, typename... Args>
cudaError_t launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                          dim3 cluster, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  unsigned int n = 0;
  attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[n].val.programmaticStreamSerializationAllowed = 1;
  ++n;
  if (cluster.x * cluster.y * cluster.z > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster.x;
    attr[n].val.clusterDim.y = cluster.y;
    attr[n].val.clusterDim.z = cluster.z;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace mmr
