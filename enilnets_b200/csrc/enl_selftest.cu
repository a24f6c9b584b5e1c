// Diagnostic: exercises the bounded-wait failure path of the kernels without
// faulting or hanging the GPU. One warp waits on an mbarrier that nothing
// arrives on; when the budget runs out the wait records kDevWaitTimeout in
// the device error word (info = the site below) and the kernel returns, so the
// context stays usable and the host reads the status with enl_device_error().
#include "enl_attn.h"
#include "enl_common.cuh"

namespace enl {

constexpr int kSelftestSite = 99;

__global__ void wait_timeout_probe(uint64_t budget_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0)
    mbar_wait_budget(&bar, 0, &abort_flag, kSelftestSite, budget_ns);  // nothing arrives
  __syncthreads();
}

}  // namespace enl

extern "C" int enl_selftest_wait_timeout(int64_t budget_ns, void* stream) {
  // Compiled in the same unit as enl_abi.cu, whose status helpers it uses.
  if (budget_ns < 1000 || budget_ns > 100ll * 1000 * 1000)
    return enl::fail(ENL_ERR_INVALID,
                     "enl_selftest_wait_timeout: budget_ns=%lld outside [1e3, 1e8]",
                     (long long)budget_ns);
  enl::wait_timeout_probe<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      (uint64_t)budget_ns);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? ENL_OK : enl::cuda_fail(e, "enl_selftest_wait_timeout launch");
}
