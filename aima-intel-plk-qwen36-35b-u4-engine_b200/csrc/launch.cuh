// launch.cuh — kernel launch with programmatic dependent launch (PDL).
//
// Every kernel of the library calls griddepcontrol.wait before touching data a
// predecessor may produce or read, so any launch may opt in to PDL: the next
// kernel's CTAs are scheduled while the current grid drains, hiding the launch
// gap between the ~10 dependent kernels of a decode sub-block (also inside a
// captured CUDA graph).
#pragma once

#include <cuda_runtime.h>

namespace iq36 {

bool pdl_enabled();

template <typename... KArgs, typename... Args>
cudaError_t launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                   cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace iq36
