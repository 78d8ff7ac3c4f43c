// Self-test of the bounded device waits that every pipelined kernel of the
// library relies on (TMA / tensor-core stages wait on mbarrier phases).  A
// wait on a phase that never completes gives up after its limit, flags
// CE_EW_TIMEOUT in the error word and lets the kernel run to its end; a
// waiter that polls the CTA's abort flag stops as soon as another warp gives
// up.  The failure is made by an mbarrier nothing arrives on, never by a
// trap, an assert or a bad address, so the context stays usable.
#include <cuda_runtime.h>

#include "ce_common.cuh"
#include "ce_host.h"

namespace ce {
namespace selftest {

// status[0]: warp 0's wait gave up; status[1]: warp 1 left its wait through
// the abort flag; status[2]: the block reached its end.
__global__ void wait_kernel(int complete, unsigned long long limit_ns, int32_t* err, int32_t* status) {
  __shared__ uint64_t bar;
  __shared__ int abort;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort = 0;
    fence_mbar_init();
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == 0) {
    if (complete && lane == 0) mbar_arrive(&bar);
    bool ok = true;
    if (lane == 0) ok = mbar_wait(&bar, 0, err, limit_ns);
    ok = __shfl_sync(0xffffffffu, ok, 0);
    if (!ok && lane == 0) {
      abort = 1;
      status[0] = 1;
    }
  } else if (warp == 1) {
    // a longer limit: this warp returns through warp 0's abort, not its own timeout
    const bool ok = warp_wait(&bar, 0, nullptr, &abort, lane);
    if (lane == 0) status[1] = ok ? 0 : 1;
  }
  __syncthreads();
  if (threadIdx.x == 0) status[2] = 1;
}

}  // namespace selftest
}  // namespace ce

using namespace ce;

extern "C" int ce_selftest_wait(int32_t complete, int64_t limit_ns, int32_t* err, int32_t* status,
                                void* stream) {
  if (!status) return host::fail(CE_ERR_ARG, "ce_selftest_wait: status is required");
  if (limit_ns < 1000 || limit_ns > static_cast<int64_t>(kWaitLimitNs))
    return host::fail(CE_ERR_ARG, "ce_selftest_wait: limit_ns must lie in [1 us, 2 s]");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(status, 0, 3 * sizeof(int32_t), st) != cudaSuccess)
    return host::fail_cuda("ce_selftest_wait memset");
  selftest::wait_kernel<<<1, 64, 0, st>>>(complete ? 1 : 0, static_cast<unsigned long long>(limit_ns), err,
                                          status);
  if (cudaPeekAtLastError() != cudaSuccess) return host::fail_cuda("ce_selftest_wait launch");
  return CE_OK;
}
