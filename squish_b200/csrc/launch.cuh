// launch.cuh — kernel launches with programmatic dependent launch (PDL).
//
// Every kernel of the model step is launched with programmatic stream serialisation, so
// the next kernel's CTAs can be scheduled while the previous kernel drains; each kernel
// calls pdl_wait() (griddepcontrol.wait) before it reads or writes memory a predecessor may
// touch, and pdl_trigger() (griddepcontrol.launch_dependents) once its own successor may
// start. The INT4 GEMM streams its (static) weights before waiting, which hides its launch,
// prologue and pipeline fill behind the previous kernel. SQ_NO_PDL=1 turns the attribute off.
#pragma once
#include <cuda_runtime.h>

#include <cstdlib>
#include <utility>

namespace sq {

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

inline bool pdl_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("SQ_NO_PDL");
    return !(e != nullptr && e[0] == '1');
  }();
  return on;
}

// Launch ``kern`` with PDL (and, when cluster_z > 1, a (1, 1, cluster_z) thread-block cluster).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                            unsigned cluster_z, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  unsigned n = 0;
  if (pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster_z > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = 1;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = cluster_z;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

}  // namespace sq

// launch with PDL; returns the launch error from the enclosing function
#define SQ_LAUNCH(...)                                      \
  do {                                                      \
    cudaError_t sq_launch_err_ = ::sq::launch_k(__VA_ARGS__); \
    if (sq_launch_err_ != cudaSuccess) return sq_launch_err_; \
  } while (0)
