// selftest.cu — exercises the kernel-side failure path without faulting the
// GPU: one CTA waits on an mbarrier that nothing arrives on, through the same
// bounded wait every pipeline stage uses (sm100.cuh). The wait gives up after
// the requested time, records a timeout in the device status word and the
// kernel returns normally, so the context stays usable.
#include "internal.h"
#include "sm100.cuh"

namespace choreo_impl {
namespace {

__global__ void selftest_wait_kernel(uint32_t* status, uint64_t timeout_ns) {
  using namespace choreo_sm100;
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bar), 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const WaitCtx w{status, timeout_ns, &abort_flag};
    // Phase 0 needs one arrival that never comes.
    mbar_wait(smem_u32(&bar), 0, w, kStatusTimeoutMma);
  }
  __syncthreads();
}

}  // namespace
}  // namespace choreo_impl

using namespace choreo_impl;

extern "C" int choreo_selftest_wait_timeout(double timeout_ms, void* stream) {
  if (!(timeout_ms > 0.0) || timeout_ms > 10000.0)
    return fail(CHOREO_ERR_INVALID_ARG, "selftest: timeout must be in (0, 10000] ms");
  uint32_t* status = status_word();
  if (status == nullptr) return CHOREO_ERR_CUDA;
  selftest_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      status, static_cast<uint64_t>(timeout_ms * 1e6));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "selftest launch");
  return ok();
}
