// Watchdog self test: one block waits on an mbarrier that nothing ever arrives on, through the same
// bounded wait the fused kernel uses. The wait runs out after `limit_ns`, records kErrSelfTest in
// the error word and the kernel returns; the host sees the error status on its next
// synchronisation while the context stays usable. This is how a lost arrival (a dead peer, a
// copy that never lands) is reported instead of hanging the device.
#include <cuda_runtime.h>

#include "ptx.cuh"
#include "watchdog.cuh"

namespace ovvs {
namespace prim {
namespace {

__global__ void watchdog_selftest_kernel(int* err, uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    ptx::mbar_init(&bar, 1);
    abort_flag = 0;
    ptx::fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // Phase 0 of `bar` never completes: nothing arrives.
    (void)ptx::mbar_wait(&bar, 0, &abort_flag, err, kErrSelfTest, limit_ns);
  }
}

}  // namespace

cudaError_t launch_watchdog_selftest(int* err, uint64_t limit_ns, cudaStream_t stream) {
  watchdog_selftest_kernel<<<1, 32, 0, stream>>>(err, limit_ns);
  return cudaGetLastError();
}

}  // namespace prim
}  // namespace ovvs
