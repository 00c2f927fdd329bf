// Failure-detection self-test: one CTA waits on an mbarrier that nothing
// arrives at. The bounded wait must expire, set the timeout bit of the device
// status word and let the kernel return normally (no trap, no hang).
#include "common.cuh"
#include "kernels.h"

namespace fpv2 {

namespace {

__global__ void wait_selftest_kernel(int* status, long long budget) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bar), 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    WaitCtx wc{status, &abort_flag, budget};
    mbar_wait(smem_u32(&bar), 0, wc);   // phase 0 never completes
  }
  __syncthreads();
}

}  // namespace

cudaError_t launch_wait_selftest(const TcLaunch& L, cudaStream_t stream) {
  wait_selftest_kernel<<<1, 32, 0, stream>>>(L.status, L.budget);
  count_launch();
  return cudaGetLastError();
}

}  // namespace fpv2
