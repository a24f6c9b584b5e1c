// Diagnostics.
//
// enl_selftest_wait_timeout exercises the bounded-wait failure path of the
// kernels without faulting or hanging the GPU. One warp waits on an mbarrier
// that nothing arrives on; when the budget runs out the wait records
// kDevWaitTimeout in
// the device error word (info = the site below) and the kernel returns, so the
// context stays usable and the host reads the status with enl_device_error().
//
// enl_selftest_exp2 evaluates the FMA-pipe exponentials K1 takes a quarter
// of its softmax exponentials from (exp2_poly, exp2_poly2), next to CUDA's
// exp2f, so that their error bound can be checked on the host.
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

__global__ void exp2_probe(const float* __restrict__ x, float* __restrict__ y_poly,
                           float* __restrict__ y_poly2, float* __restrict__ y_ref, int n) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; 2 * i < n; i += gridDim.x * blockDim.x) {
    const float x0 = x[2 * i];
    const float x1 = 2 * i + 1 < n ? x[2 * i + 1] : 0.0f;
    float p0, p1;
    exp2_poly2(x0, x1, p0, p1);
    y_poly[2 * i] = exp2_poly(x0);
    y_poly2[2 * i] = p0;
    y_ref[2 * i] = exp2f(x0);
    if (2 * i + 1 < n) {
      y_poly[2 * i + 1] = exp2_poly(x1);
      y_poly2[2 * i + 1] = p1;
      y_ref[2 * i + 1] = exp2f(x1);
    }
  }
}

}  // namespace enl

extern "C" int enl_selftest_exp2(const float* x, float* y_poly, float* y_poly2, float* y_ref,
                                 int32_t n, void* stream) {
  if (!x || !y_poly || !y_poly2 || !y_ref || n < 0)
    return enl::fail(ENL_ERR_INVALID, "enl_selftest_exp2: NULL pointer or n < 0");
  if (n == 0) return ENL_OK;
  const int blocks = (int)std::min<long long>(((long long)n / 2 + 255) / 256 + 1, 4096);
  enl::exp2_probe<<<blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(x, y_poly,
                                                                                y_poly2, y_ref, n);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? ENL_OK : enl::cuda_fail(e, "enl_selftest_exp2 launch");
}

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
