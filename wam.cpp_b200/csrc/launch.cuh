// Kernel launch with programmatic dependent launch (PDL): the kernel may begin
// while its predecessor in the stream finishes; every engine kernel calls
// griddep_wait() before it touches memory the predecessor writes.
#pragma once

#include <cuda_runtime.h>

#include <cstdlib>
#include <utility>

namespace wamb {

inline bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("WAM_B200_DISABLE_PDL");
    return !(v && *v && *v != '0');
  }();
  return on;
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace wamb
