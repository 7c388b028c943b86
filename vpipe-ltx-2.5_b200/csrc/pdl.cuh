// pdl.cuh -- programmatic dependent launch (PDL) for the library's kernels.
//
// Every kernel here is launched with programmatic stream serialization, so
// the next kernel in the stream is scheduled while the current one drains:
// its prologue (mbarrier init, TMEM allocation, tensor-map prefetch) overlaps
// the previous kernel's tail instead of following its completion.  The
// contract inside each kernel:
//   * pdl_wait() before the first global read of data another kernel wrote
//     and before the first global write (it returns once every earlier
//     kernel of the stream has completed and its memory is visible);
//   * pdl_trigger() after the prologue's TMEM allocation, so that a
//     dependent grid launched early never holds TMEM a not-yet-allocated
//     CTA of this grid would wait for.
// A kernel launched without the attribute sees both as no-ops.  LTX25_PDL=0
// launches everything without it.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <cstdlib>
#include <utility>

namespace ltx {

__device__ __forceinline__ void pdl_wait()
{
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

__device__ __forceinline__ void pdl_trigger()
{
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

inline bool pdl_enabled()
{
  static const bool on = [] {
    const char* e = std::getenv("LTX25_PDL");
    return !(e != nullptr && e[0] == '0');
  }();
  return on;
}

// Raise a kernel's dynamic shared-memory limit once per device.  Function
// attributes belong to the device's context, so a process that drives several
// GPUs (one context per host thread) sets it on each; `done` is the call
// site's own mask, one bit per device ordinal.
template <typename... KArgs>
bool smem_limit_once(void (*kern)(KArgs...), int bytes, std::atomic<unsigned long long>& done)
{
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
  const unsigned long long bit = 1ull << dev;
  if ((done.load(std::memory_order_acquire) & bit) != 0) return true;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) !=
      cudaSuccess)
    return false;
  done.fetch_or(bit, std::memory_order_acq_rel);
  return true;
}

// cudaLaunchKernelEx with the PDL attribute (and a cluster size when > 1).
template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                     cudaStream_t s, int cluster, Args&&... args)
{
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  int n = 0;
  attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[n].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  ++n;
  if (cluster > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = (unsigned)cluster;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = (unsigned)n;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

}  // namespace ltx
