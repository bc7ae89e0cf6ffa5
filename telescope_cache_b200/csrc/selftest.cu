// Failure-detection self-test: a pipeline wait that can never complete must
// end by itself, report TC_DEV_WAIT_TIMEOUT in the device status word and
// leave the context usable.  One thread waits, through the same bounded
// mbarrier wait as the tensor-core kernels, on a barrier that nothing
// arrives at; no fault, trap or endless loop is involved.
#include "common.cuh"
#include "tc_ptx.cuh"

namespace {

__global__ void wait_timeout_kernel(int32_t* status) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x != 0) return;
  tc::ptx::mbar_init(&bar, 1);
  abort_flag = 0;
  tc::ptx::mbar_fence_init();
  // phase 0 never completes: the bounded wait gives up and records it
  (void)tc::ptx::mbar_wait(&bar, 0, &abort_flag, status);
}

}  // namespace

extern "C" int tc_selftest_wait_timeout(int32_t* dev_status, void* stream) {
  if (!dev_status) return TC_ERR_ARG;
  wait_timeout_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(dev_status);
  return tc::launch_status();
}
