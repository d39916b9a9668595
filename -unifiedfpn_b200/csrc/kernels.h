// Internal include: the kernel launcher API lives in the public header.
#pragma once
#include "unified_fpn/kernels/interface.h"

#include <cuda_runtime.h>

#include <utility>

namespace ufpn {

// cudaLaunchKernelEx with an optional cluster of `cluster` CTAs along x and the launch
// options (programmatic stream serialisation, priority; see LaunchOpts).
template <typename... KArgs, typename... Args>
cudaError_t launch_ex(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                      cudaStream_t s, const LaunchOpts& opts, int cluster, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[3];
  unsigned n = 0;
  if (cluster > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = static_cast<unsigned>(cluster);
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  if (opts.pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (opts.priority != 0) {
    attr[n].id = cudaLaunchAttributePriority;
    attr[n].val.priority = opts.priority;
    ++n;
  }
  cfg.attrs = n ? attr : nullptr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace ufpn
