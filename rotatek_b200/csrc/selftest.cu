// rtk_selftest_wait_timeout: makes the library's bounded mbarrier wait run out,
// so that a test can check the error path every kernel here relies on -- the
// wait gives up, the abort flag stops the CTA's other waits, RTK_DEVICE_TIMEOUT
// lands in the status word that rtk_read_status reads, and the kernel returns
// with the context intact.
//
// One CTA of two warps waits on a shared-memory mbarrier that nothing arrives
// on: no TMA copy, no cp.async and no other thread is involved, so when the
// wait gives up nothing is left in flight.  Warp 0 waits with the caller's
// limit; warp 1 waits with the library's ordinary limit and leaves through the
// abort flag that warp 0's timeout sets.
#include <cuda_runtime.h>

#include "../../include/rotatek_b200.h"
#include "common.cuh"
#include "decode.h"

namespace rtk {
namespace {

__global__ void __launch_bounds__(64, 1) wait_timeout_kernel(unsigned int *status, unsigned long long limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  volatile int *abort = &abort_flag;
  if ((threadIdx.x & 31) == 0) {
    // phase 0 never completes: the only way out is the time limit or the abort flag
    mbar_wait_bounded(&bar, 0, abort, status, threadIdx.x == 0 ? limit_ns : kWaitLimitNs);
  }
  __syncwarp();
}

}  // namespace
}  // namespace rtk

extern "C" int rtk_selftest_wait_timeout(void *workspace, uint64_t limit_ns, void *stream) {
  if (workspace == nullptr) return rtk::report_error(RTK_ERR_INVALID, "workspace must be non-NULL");
  if (limit_ns == 0 || limit_ns > rtk::kWaitLimitNs)
    return rtk::report_error(RTK_ERR_INVALID, "limit_ns must be in (0, 2e9]");
  rtk::wait_timeout_kernel<<<1, 64, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<unsigned int *>(workspace), static_cast<unsigned long long>(limit_ns));
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return rtk::report_error(RTK_ERR_CUDA, cudaGetErrorString(e));
  return RTK_OK;
}
