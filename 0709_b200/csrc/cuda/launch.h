// Host launch helper: every kernel goes through cudaLaunchKernelEx with
// programmatic stream serialization (PDL) unless ATLAS_PDL=0.
#pragma once

#include <cuda_runtime.h>

#include <cstdlib>
#include <utility>

namespace atlas {

inline bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("ATLAS_PDL");
    return v == nullptr || v[0] != '0';
  }();
  return on;
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                            Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

}  // namespace atlas
