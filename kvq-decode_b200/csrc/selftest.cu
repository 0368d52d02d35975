// Self-test of the bounded pipeline wait: one CTA waits on an mbarrier phase that nothing
// completes, with a short budget, and must give up and report BPT_DEV_WAIT_TIMEOUT through the
// status word exactly as the decode kernels do. It faults nothing and leaves the context usable.
// No reference counterpart.
#include <cuda_runtime.h>

#include "common.cuh"

namespace bpt {
namespace {

__global__ void wait_timeout_selftest_kernel(unsigned* status, uint64_t budget_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);   // one expected arrival, which never comes
    fence_mbar_init();
  }
  __syncthreads();
  const bool ok = mbar_wait_for(&bar, 0u, budget_ns);
  if (!ok && threadIdx.x == 0) flag_device_error(status, BPT_DEV_WAIT_TIMEOUT);
}

}  // namespace
}  // namespace bpt

extern "C" int bpt_selftest_wait_timeout(unsigned* status, unsigned budget_us, void* stream) {
  if (!status || budget_us == 0 || budget_us > 1000000u) return BPT_ERR_INVALID_ARGUMENT;
  bpt::wait_timeout_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      status, uint64_t(budget_us) * 1000ull);
  return cudaGetLastError() == cudaSuccess ? BPT_OK : BPT_ERR_LAUNCH;
}
