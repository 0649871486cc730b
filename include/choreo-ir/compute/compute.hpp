/**
 * @file compute.hpp
 * @brief GEMM configuration and entry points (the reference's
 *        compute/compute.hpp:22-119 declarations). Definitions are in
 *        compute/matmul.hpp.
 *
 * On sm_100a every f16/bf16 device GEMM runs on the tcgen05 tensor-core
 * kernel and every f32 device GEMM on the CUDA-core kernel; GEMMConfig's
 * backend field is informational (the reference's default CUDA_CORE
 * silently selected a 16x16 SIMT kernel with fp16 accumulation,
 * compute_impl.hpp:26-37).
 */
#ifndef CHOREO_IR_COMPUTE_COMPUTE_HPP
#define CHOREO_IR_COMPUTE_COMPUTE_HPP

#include <cuda_runtime.h>

#include "../core/config.hpp"
#include "../core/types.hpp"
#include "../tensor/tensor.hpp"
#include "validation.hpp"

namespace choreo_ir {
namespace compute {

enum class ComputeBackend {
  CUDA_CORE,  // f32 GEMM on CUDA cores
  WMMA,       // accepted for source compatibility; runs TCGEN05 on sm_100a
  MMA,        // accepted for source compatibility; runs TCGEN05 on sm_100a
  TCGEN05     // 5th-generation tensor cores (f16/bf16 in, f32 accumulate)
};

struct GEMMConfig {
  ComputeBackend backend = ComputeBackend::TCGEN05;
  bool use_tensor_core = true;
  cudaStream_t stream = nullptr;
  // Filled by get_optimal_gemm_config / auto_analyze from the dispatcher.
  dim_t tile_m = config::sm100::TILE_M;
  dim_t tile_n = 256;
  dim_t tile_k = config::sm100::TILE_K;
  dim_t stages = 4;
  // Fused epilogue applied by the kernel after alpha/beta.
  const void* bias = nullptr;         // N-vector on the device, or null
  DataType bias_dtype = DataType::FLOAT32;
  bool relu = false;
  // Synchronize the stream and check the kernel status word after the call.
  bool synchronize = false;

  GEMMConfig() = default;
  explicit GEMMConfig(ComputeBackend b) : backend(b) {}
};

/// C = alpha * A * B + beta * C (A: [..,M,K], B: [..,K,N], C: [..,M,N]).
template <typename T>
void gemm(const Tensor<T>& A, const Tensor<T>& B, Tensor<T>& C, T alpha = from_float<T>(1.0f),
          T beta = from_float<T>(0.0f), const GEMMConfig& config = GEMMConfig());

/// C = alpha * A * B, C allocated in A's memory type.
template <typename T>
Tensor<T> gemm(const Tensor<T>& A, const Tensor<T>& B, T alpha = from_float<T>(1.0f),
               const GEMMConfig& config = GEMMConfig());

template <typename T>
void matmul(const Tensor<T>& A, const Tensor<T>& B, Tensor<T>& C, const GEMMConfig& config = GEMMConfig());

template <typename T>
Tensor<T> matmul(const Tensor<T>& A, const Tensor<T>& B, const GEMMConfig& config = GEMMConfig());

template <typename T>
GEMMConfig get_optimal_gemm_config(const Tensor<T>& A, const Tensor<T>& B);

template <typename T>
bool can_use_tensor_core_gemm(const Tensor<T>& A, const Tensor<T>& B);

template <typename T>
bool can_use_wmma_gemm(const Tensor<T>& A, const Tensor<T>& B);

}  // namespace compute
}  // namespace choreo_ir

#include "matmul.hpp"

#endif  // CHOREO_IR_COMPUTE_COMPUTE_HPP
