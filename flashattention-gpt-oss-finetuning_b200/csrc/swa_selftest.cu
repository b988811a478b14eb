// swa_selftest.cu -- exercises the bounded-wait failure path without faulting the GPU.
//
// The kernel waits on an mbarrier that nothing ever arrives on, with a short time limit.  The
// wait gives up, the kernel records the error in the device error flag exactly as the
// attention kernels do, and returns; the host then sees SWA_ERR_DEVICE_TIMEOUT from
// swa_check_device and the context stays usable.
#include "sm100.cuh"
#include "swa_common.cuh"

namespace swa {
using namespace sm100;

__global__ void selftest_wait_timeout_kernel(int* err, unsigned long long limit_ns) {
  __shared__ uint64_t bar;
  __shared__ volatile int abort_sh;
  if (threadIdx.x == 0) {
    abort_sh = 0;
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0 && !mbar_wait_ns(&bar, 0, &abort_sh, limit_ns)) record_error(err, 1);
}

cudaError_t launch_selftest_wait_timeout(int* err, unsigned long long limit_ns, cudaStream_t st) {
  selftest_wait_timeout_kernel<<<1, 32, 0, st>>>(err, limit_ns);
  return cudaGetLastError();
}

}  // namespace swa
