// Kernel launches with programmatic dependent launch (PDL).
//
// Every decode kernel is launched with cudaLaunchAttributeProgrammatic-
// StreamSerialization, so the next kernel on the stream can start while this
// one runs.  Inside each kernel:
//   * before pdl_wait() it touches only data no kernel of the decode step
//     writes (packed weights, scales), or data written two or more launches
//     earlier (every kernel triggers its dependents only after its own wait,
//     so the launch before the previous one has completed);
//   * pdl_wait() blocks until the preceding grid has completed and its writes
//     are visible; pdl_trigger() then lets the next launch begin.
// Without the attribute (or under MAPLE_PDL=0) both are no-ops and launches
// serialise as usual.
#pragma once

#include <cuda_runtime.h>
#include <cstdlib>

namespace mb {

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }

inline bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("MAPLE_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
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
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

}  // namespace mb
