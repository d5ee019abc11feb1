// Host-side kernel launch through cudaLaunchKernelEx, with programmatic dependent launch when this
// thread's launch flags ask for it (aexrt_b200_set_launch_flags).  With it, a kernel's CTAs may be
// scheduled while the previous kernel on the stream still runs (each kernel's grid_dep_wait()
// orders its dependent memory accesses, ptx.cuh), so that launch latency and the set-up of a
// kernel (barrier init, TMEM allocation, weight and scale loads) overlap its predecessor.  This
// pays off when grids are small (one or a few images); at large batches the early CTAs would only
// hold SM resources.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <utility>

namespace aexrt {

constexpr uint32_t kLaunchProgrammatic = 1u;  // AEXRT_B200_LAUNCH_PROGRAMMATIC

uint32_t launch_flags();  // this thread's flags (capi.cu)

// The launch configuration of launch_kernel / launch_kernel_cluster (attr: room for two attributes).
inline cudaLaunchConfig_t launch_config(dim3 grid, dim3 block, size_t smem, cudaStream_t stream, unsigned cluster_x,
                                        cudaLaunchAttribute* attr) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  if (launch_flags() & kLaunchProgrammatic) {
    attr[cfg.numAttrs].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[cfg.numAttrs].val.programmaticStreamSerializationAllowed = 1;
    ++cfg.numAttrs;
  }
  if (cluster_x > 1) {
    attr[cfg.numAttrs].id = cudaLaunchAttributeClusterDimension;
    attr[cfg.numAttrs].val.clusterDim.x = cluster_x;
    attr[cfg.numAttrs].val.clusterDim.y = 1;
    attr[cfg.numAttrs].val.clusterDim.z = 1;
    ++cfg.numAttrs;
  }
  return cfg;
}

template <typename... KArgs, typename... Args>
cudaError_t launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                          Args&&... args) {
  cudaLaunchAttribute attr[2];
  const cudaLaunchConfig_t cfg = launch_config(grid, block, smem, stream, 1, attr);
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// launch_kernel with thread-block clusters of cluster_x CTAs along x (grid.x a multiple of it).
template <typename... KArgs, typename... Args>
cudaError_t launch_kernel_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                                  unsigned cluster_x, Args&&... args) {
  cudaLaunchAttribute attr[2];
  const cudaLaunchConfig_t cfg = launch_config(grid, block, smem, stream, cluster_x, attr);
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace aexrt
