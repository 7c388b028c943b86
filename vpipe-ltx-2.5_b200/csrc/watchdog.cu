// watchdog.cu -- a self-test of the bounded-wait failure path.
//
// Every pipeline wait in the library gives up after a wall-clock bound,
// records a code in the context's error word and lets its CTA drain and
// exit, so a stalled pipeline becomes an error the host reads
// (ltx_ctx_check -> LTX_E_KERNEL) instead of a hung GPU.  This kernel
// exercises exactly that path on purpose, without faulting anything: it
// waits on an mbarrier that nothing will ever arrive at, with a short
// bound, and reports the timeout like the real kernels do.
#include <cuda_runtime.h>

#include "block_ops.h"
#include "kernels.h"
#include "ptx.cuh"

namespace ltx {

namespace {

constexpr int kWatchdogCode = 0x7E;

__global__ void watchdog_probe_kernel(int* err, unsigned long long bound_ns)
{
  __shared__ __align__(8) uint64_t bar;
  pdl_wait();
  pdl_trigger();
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);   // expects one arrival; none is ever made
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned long long t0 = globaltimer_ns();
    bool done = false;
    while (!done) {
      done = mbar_try_wait(&bar, 0);
      if (!done && globaltimer_ns() - t0 > bound_ns) break;
    }
    if (!done) atomicCAS(err, 0, kWatchdogCode);
  }
}

}  // namespace

int launch_watchdog_probe(int* err, int bound_ms, cudaStream_t s)
{
  if (bound_ms < 1 || bound_ms > 2000) return -2;
  launch_k(watchdog_probe_kernel, dim3(1), dim3(32), 0, s, 1, err,
           (unsigned long long)bound_ms * 1000000ull);
  return launched();
}

}  // namespace ltx
