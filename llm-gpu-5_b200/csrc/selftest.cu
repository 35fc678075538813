// Failure-detection self-test of the bounded waits (tc_common.cuh: mbar_wait).  One warp waits on
// an mbarrier that nothing ever arrives at, with a short limit; the wait gives up, records its
// site code in the library's device error word and the kernel returns.  Nothing faults, traps or
// hangs, and the context stays usable: a caller (or a test) reads the code with
// attn_device_error() and keeps launching work.
#include "tc_common.cuh"

namespace attn {

__global__ void __launch_bounds__(32, 1) wait_selftest_kernel(int* err, uint64_t limit_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);  // expects one arrival, which never comes
    fence_mbar_init();
  }
  __syncwarp();
  const bool ok = mbar_wait(&bar, 0, wait_err(err), ATTN_SELFTEST_SITE, limit_ns);
  (void)__all_sync(0xffffffffu, ok);
}

int wait_selftest(int limit_us, cudaStream_t s) {
  int* err = dev_error_ptr();
  if (!err) return ATTN_ERR_CUDA;
  wait_selftest_kernel<<<1, 32, 0, s>>>(err, (uint64_t)limit_us * 1000ull);
  count_launch();
  return check_launch("wait_selftest_kernel");
}

}  // namespace attn
