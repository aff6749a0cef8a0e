// Host-side kernel launch with programmatic dependent launch (PDL).
//
// Every kernel of the library calls griddepcontrol.launch_dependents at its
// start and griddepcontrol.wait before it reads anything an earlier kernel
// wrote, and is launched through launch_pdl. A kernel's CTAs can then be
// scheduled (and do their set-up: barrier init, descriptor prefetch, weight
// prefetch) while the previous kernel is still finishing, which removes most
// of the launch gap between the ~10 short kernels of a decode layer inside a
// CUDA graph. Inside stream capture the attribute becomes a programmatic
// graph edge.
#pragma once

#include <cuda_runtime.h>

#include <cstdlib>
#include <stdexcept>
#include <string>
#include <utility>

namespace minisgl {

// MINISGL_NO_PDL=1 launches everything with plain stream order (a debugging
// and measurement switch; the kernels' griddepcontrol instructions are then
// no-ops).
inline bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("MINISGL_NO_PDL");
    return v == nullptr || v[0] == '\0' || v[0] == '0';
  }();
  return on;
}

template <typename... KArgs, typename... Args>
void launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
  if (e != cudaSuccess) throw std::runtime_error(std::string("minisgl: kernel launch failed: ") + cudaGetErrorString(e));
}

}  // namespace minisgl
