// Programmatic dependent launch: every kernel of the step is launched with
// programmatic stream serialisation, so the next kernel's launch and its
// data-independent prologue overlap the previous one. Each kernel calls
// griddep_wait() before it touches global memory, which waits for the
// previous kernel to complete and its writes to be visible; since every kernel
// waits, completion is ordered transitively down the stream.
#pragma once
#include <cuda_runtime.h>

#include <utility>

namespace tb2 {

__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// griddep_wait, then let the next kernel launch: its CTAs are scheduled once
// every CTA of this grid has passed this point (so all of this grid's CTAs
// are already resident and none can be starved by the waiting ones), run
// their prologue on data no running kernel writes (weights) beside this one
// and block in their own wait until it completes. Used by the decode kernels,
// whose prologues load weight rows; in the training step the early-launched
// CTAs held shared memory the other stream's kernels needed and measured 2.5 %
// slower, so its kernels let the next one launch at their exit.
__device__ __forceinline__ void griddep_wait_release() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KParams, typename... Args>
int launch_pdl(void (*kernel)(KParams...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...) == cudaSuccess ? 0 : -3;
}

// The same launch with thread-block clusters of `cluster_x` CTAs along x.
template <typename... KParams, typename... Args>
int launch_pdl_cluster(void (*kernel)(KParams...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, int cluster_x,
                       Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = cluster_x;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...) == cudaSuccess ? 0 : -3;
}

}  // namespace tb2
