// Host side of programmatic dependent launch (PDL) for the kernels of one step
// (fused append -> decode -> split merge).  Each of them starts with
// ptx::grid_dependency_wait (it reads nothing before the previous kernel on
// its stream has completed and flushed) and then ptx::launch_dependents, so the
// next kernel's CTAs can be scheduled while this one drains: the launch gap
// between the kernels of a step disappears, the order of their memory effects
// does not change.  KCMM_PDL=0 (read once) launches in plain stream order.
#pragma once

#include <cuda_runtime.h>

#include <cstdlib>
#include <cstring>

namespace kcmm {
namespace dev {

inline bool pdl_enabled() {
  static const bool on = [] {
    const char *v = std::getenv("KCMM_PDL");
    return !(v && std::strcmp(v, "0") == 0);
  }();
  return on;
}

template <typename... Args>
cudaError_t launch_pdl(void (*kernel)(Args...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t stream, Args... args) {
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
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

}  // namespace dev
}  // namespace kcmm
