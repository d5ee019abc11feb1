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

template <typename... KArgs, typename... Args>
cudaError_t launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                          Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  if (launch_flags() & kLaunchProgrammatic) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace aexrt
