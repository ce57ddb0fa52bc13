// dw_launch.h -- kernel launches with programmatic dependent launch (PDL).
//
// Every engine kernel is launched with the programmatic stream-serialization
// attribute: it may start (barrier set-up, tensor-map prefetch) while the
// previous kernel of the stream drains, and waits in griddep_wait() before it
// touches global memory.  DWB_PDL=0 in the environment launches without the
// attribute (plain stream order), for comparisons.
#pragma once

#include <cuda_runtime.h>
#include <stdlib.h>

namespace dwb {

inline bool pdl_enabled() {
  static const bool on = [] {
    const char* v = getenv("DWB_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

inline cudaError_t launch_kernel(const void* fn, dim3 grid, dim3 block, void** args, size_t smem,
                                 cudaStream_t stream) {
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
  return cudaLaunchKernelExC(&cfg, fn, args);
}

}  // namespace dwb
