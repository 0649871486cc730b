// splitk.cu — the second pass of a split-K GEMM: sums the fp32 partial
// products of the K ranges and applies the epilogue.
//
// The first pass is the ordinary tcgen05 GEMM launch with the K splits as its
// batch items (TcProblem::split): partial s holds A[:, Ks*s : Ks*(s+1)] *
// B[Ks*s : Ks*(s+1), :] in fp32, laid out [split][m][n]. Splitting pays when
// few output tiles would leave most SMs idle over a long K; it also shortens
// every tensor-core accumulation chain, and the partials are summed here in
// IEEE fp32.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>

#include "internal.h"
#include "tc_kernel.cuh"

namespace choreo_impl {
namespace {

using choreo_sm100::from_f32;
using choreo_sm100::load_bias;
using choreo_sm100::to_f32;

// One thread per 4 consecutive columns of one row; partial rows are read as
// float4 when n is a multiple of 4 (16-byte aligned rows).
template <typename OutT>
__global__ void __launch_bounds__(256) splitk_reduce_kernel(const float* __restrict__ part, int64_t split, int64_t m,
                                                            int64_t n, OutT* __restrict__ c, int64_t ldc, float alpha,
                                                            float beta, const void* __restrict__ bias, int dtype_bias,
                                                            int relu) {
  choreo_sm100::griddep_wait();  // the first pass's partials are complete and visible
  const int64_t quads = (n + 3) / 4;
  const int64_t total = m * quads;
  const bool vec = (n % 4) == 0;
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t i = idx / quads;
    const int64_t j0 = (idx - i * quads) * 4;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int64_t s = 0; s < split; ++s) {
      const float* row = part + (s * m + i) * n;
      if (vec) {
        const float4 v = *reinterpret_cast<const float4*>(row + j0);
        acc[0] += v.x;
        acc[1] += v.y;
        acc[2] += v.z;
        acc[3] += v.w;
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (j0 + e < n) acc[e] += row[j0 + e];
      }
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int64_t j = j0 + e;
      if (j >= n) break;
      float v = alpha * acc[e];
      OutT* dst = c + i * ldc + j;
      if (beta != 0.f) v += beta * to_f32<OutT>(*dst);
      if (bias != nullptr) v += load_bias(bias, dtype_bias, static_cast<int>(j));
      if (relu) v = (v < 0.f) ? 0.f : v;  // NaN passes, like std::max(x, 0)
      *dst = from_f32<OutT>(v);
    }
  }
}

template <typename OutT>
int launch_typed(const float* part, int64_t split, int64_t m, int64_t n, void* c, int64_t ldc, float alpha, float beta,
                 const void* bias, int dtype_bias, int relu, cudaStream_t stream) {
  const int64_t total = m * ((n + 3) / 4);
  const int64_t blocks = std::min<int64_t>((total + 255) / 256, static_cast<int64_t>(current_sm_count()) * 16);
  const cudaError_t e = launch_pdl(splitk_reduce_kernel<OutT>, dim3(static_cast<unsigned>(blocks)), dim3(256), 0,
                                   stream, part, split, m, n, static_cast<OutT*>(c), ldc, alpha, beta, bias,
                                   dtype_bias, relu);
  return e == cudaSuccess ? CHOREO_OK : cuda_fail(e, "split-K reduction launch");
}

}  // namespace

int launch_splitk_reduce(const float* partials, int64_t split, int64_t m, int64_t n, void* c, int64_t ldc,
                         int dtype_c, float alpha, float beta, const void* bias, int dtype_bias, int relu,
                         cudaStream_t stream) {
  if (m == 0 || n == 0) return CHOREO_OK;
  switch (dtype_c) {
    case CHOREO_DTYPE_F16:
      return launch_typed<__half>(partials, split, m, n, c, ldc, alpha, beta, bias, dtype_bias, relu, stream);
    case CHOREO_DTYPE_BF16:
      return launch_typed<__nv_bfloat16>(partials, split, m, n, c, ldc, alpha, beta, bias, dtype_bias, relu, stream);
    case CHOREO_DTYPE_F32:
      return launch_typed<float>(partials, split, m, n, c, ldc, alpha, beta, bias, dtype_bias, relu, stream);
    default:
      return fail(CHOREO_ERR_UNSUPPORTED, "split-K reduction: unsupported output dtype %d", dtype_c);
  }
}

}  // namespace choreo_impl
