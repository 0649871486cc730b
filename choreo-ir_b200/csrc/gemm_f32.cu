// gemm_f32.cu — CUDA-core GEMM for Tensor<float> operands.
//
// The reference routes every device GEMM, fp32 included, through a 16 x 16
// shared-memory SIMT kernel (compute/cuda_core.hpp:93-146). fp32 is not a
// tensor-core type in this library (tf32 would change the results the
// reference's float path produces), so fp32 GEMMs run here: 64 x 64 output
// tiles, 256 threads each computing a 4 x 4 micro-tile, fp32 FMA accumulation,
// the same alpha/beta/bias/ReLU epilogue as the tensor-core path.
#include <algorithm>

#include "internal.h"

namespace choreo_impl {
namespace {

constexpr int TM = 64, TN = 64, TK = 16;

__global__ void __launch_bounds__(256) gemm_f32_kernel(choreo_gemm_desc d) {
  __shared__ float sA[TK][TM + 4];
  __shared__ float sB[TK][TN + 4];
  const float* A = static_cast<const float*>(d.a) + blockIdx.z * (d.batch > 1 ? d.stride_a : 0);
  const float* B = static_cast<const float*>(d.b) + blockIdx.z * (d.batch > 1 ? d.stride_b : 0);
  float* C = static_cast<float*>(d.c) + blockIdx.z * (d.batch > 1 ? d.stride_c : 0);
  const int64_t m0 = static_cast<int64_t>(blockIdx.y) * TM;
  const int64_t n0 = static_cast<int64_t>(blockIdx.x) * TN;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  float acc[4][4] = {};
  for (int64_t k0 = 0; k0 < d.k; k0 += TK) {
    for (int i = threadIdx.x; i < TK * TM; i += 256) {
      const int kk = i % TK, mm = i / TK;
      const int64_t gm = m0 + mm, gk = k0 + kk;
      float v = 0.f;
      if (gm < d.m && gk < d.k) v = d.trans_a ? A[gk * d.lda + gm] : A[gm * d.lda + gk];
      sA[kk][mm] = v;
    }
    for (int i = threadIdx.x; i < TK * TN; i += 256) {
      const int nn = i % TN, kk = i / TN;
      const int64_t gn = n0 + nn, gk = k0 + kk;
      float v = 0.f;
      if (gn < d.n && gk < d.k) v = d.trans_b ? B[gn * d.ldb + gk] : B[gk * d.ldb + gn];
      sB[kk][nn] = v;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < TK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = sA[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = sB[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t gm = m0 + ty * 4 + i;
    if (gm >= d.m) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t gn = n0 + tx * 4 + j;
      if (gn >= d.n) continue;
      float v = d.alpha * acc[i][j];
      if (d.beta != 0.f) v += d.beta * C[gm * d.ldc + gn];
      if (d.bias) v += static_cast<const float*>(d.bias)[gn];
      if (d.relu) v = (v < 0.f) ? 0.f : v;
      C[gm * d.ldc + gn] = v;
    }
  }
}

}  // namespace

int launch_gemm_f32(const choreo_gemm_desc& d, cudaStream_t stream) {
  if (d.batch > 65535) return fail(CHOREO_ERR_UNSUPPORTED, "f32 GEMM: batch > 65535");
  if ((d.m + TM - 1) / TM > 65535) return fail(CHOREO_ERR_UNSUPPORTED, "f32 GEMM: M too large");
  dim3 grid(static_cast<unsigned>((d.n + TN - 1) / TN), static_cast<unsigned>((d.m + TM - 1) / TM),
            static_cast<unsigned>(d.batch));
  gemm_f32_kernel<<<grid, 256, 0, stream>>>(d);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "f32 GEMM launch");
  return CHOREO_OK;
}

}  // namespace choreo_impl
