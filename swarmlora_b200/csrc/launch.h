// Kernel launch helper shared by every product kernel: one cudaLaunchKernelEx
// carrying an optional cluster size and, unless switched off with
// swl_set_pdl(0), programmatic stream serialization, so a kernel's prologue
// (barrier setup, TMEM allocation, weight and adapter tile loads) overlaps the
// tail of the kernel before it. Every kernel launched this way calls
// ptx::grid_dep_wait() before its first global write and before reading
// anything the launch just ahead of it may write, and lets the next kernel
// start only after that wait; so when a kernel starts, every launch two or
// more places ahead of it on the stream has completed. The prologues use
// this to read, before their wait, data only such earlier launches write
// (weights, adapters, context lengths, block tables, the cos/sin cache).
#pragma once

#include <cuda_runtime.h>

#include <utility>

namespace swl {

bool pdl_enabled();

template <class... KArgs, class... Args>
cudaError_t launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                          cudaStream_t stream, unsigned cluster_x, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  unsigned n = 0;
  if (cluster_x > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster_x;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  if (pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace swl
