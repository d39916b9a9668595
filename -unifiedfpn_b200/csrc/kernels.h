// Internal include: the kernel launcher API lives in the public header.
#pragma once
#include "unified_fpn/kernels/interface.h"

#include <cuda_runtime.h>

#include <atomic>
#include <utility>

namespace ufpn {

// cudaLaunchKernelEx with an optional cluster of `cluster` CTAs along x and the launch
// options (programmatic stream serialisation, priority; see LaunchOpts).
// Runs `set` (e.g. a kernel's shared-memory opt-in, which belongs to the device's context)
// until it succeeds once for the current device; `done` is the call site's per-device record.
// Thread-safe; devices beyond the record's 64 entries run `set` every time.
template <typename F>
cudaError_t once_per_device(std::atomic<bool> (&done)[64], F&& set) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev >= 0 && dev < 64 && done[dev].load(std::memory_order_acquire)) return cudaSuccess;
  e = set();
  if (e == cudaSuccess && dev >= 0 && dev < 64) done[dev].store(true, std::memory_order_release);
  return e;
}

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
