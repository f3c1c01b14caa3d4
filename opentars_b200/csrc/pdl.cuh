// Programmatic dependent launch. The decode engine captures its step with every kernel launched
// with programmatic stream serialisation: a kernel may start while its predecessor drains; it
// calls griddep_wait() before it reads anything a predecessor wrote (or writes anything), which
// waits for the predecessor grids to complete and their memory to be visible. griddep_launch()
// lets the next kernel start early. Outside such launches both are no-ops.
#pragma once
#include <cuda_runtime.h>

#include <utility>

namespace tc {

#if defined(__CUDACC__)
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
#endif

// Host: whether launches made by this thread carry the programmatic-serialisation attribute
// (set by the engine while it captures a step).
bool& pdl_launches();

// cudaLaunchKernelEx with an optional cluster size and the programmatic attribute when enabled.
template <class... KArgs, class... Args>
cudaError_t launch_ex(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, int cluster,
                      Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (cluster > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  if (pdl_launches()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

}  // namespace tc
