/**
 * @file choreo-ir.hpp
 * @brief Umbrella header of the Choreo-IR API on B200: the reference's
 *        include/choreo-ir/choreo-ir.hpp surface (operator*, operator+,
 *        relu, initialize/finalize, type aliases) plus the documented-only
 *        pieces (+=, conv2d, batch_matmul, host_tensor/device_tensor,
 *        to_device/to_host, auto_analyze/launch).
 *
 * Device tensors compute through libchoreo_b200.so (link -lchoreo_b200);
 * host tensors keep the reference's host arithmetic.
 */
#ifndef CHOREO_IR_HPP
#define CHOREO_IR_HPP

#include <cuda_runtime.h>

#include <stdexcept>
#include <type_traits>

#include "compute/auto_analyze.hpp"
#include "compute/compute.hpp"
#include "compute/conv.hpp"
#include "compute/elementwise.hpp"
#include "compute/host_pipeline.hpp"
#include "compute/matmul.hpp"
#include "compute/validation.hpp"
#include "core/config.hpp"
#include "core/device.hpp"
#include "core/types.hpp"
#include "tensor/tensor.hpp"
#include "utils/cuda_utils.hpp"

namespace choreo_ir {

/// C = A * B (choreo-ir.hpp:53-104 of the reference). Device tensors run the
/// tcgen05 GEMM (f16/bf16, fp32 accumulation) or the CUDA-core f32 GEMM;
/// host tensors run the reference's host loop. A rank-3 A gives a batched
/// result [b, M, N].
template <typename T>
Tensor<T> operator*(const Tensor<T>& A, const Tensor<T>& B) {
  const index_t M = A.shape()[A.ndims() - 2];
  const index_t N = B.shape()[B.ndims() - 1];
  Tensor<T> C(A.ndims() == 3 ? Shape({A.shape()[0], M, N}) : Shape({M, N}), A.memory_type());
  compute::validate_matmul_contract(A, B, C, "Matrix multiplication");
  compute::matmul(A, B, C);
  return C;
}

/// Mixed element types: A is converted to B's type, then multiplied
/// (choreo-ir.hpp:109-145 of the reference; the conversion runs on the
/// device for device tensors instead of through the host).
template <typename T1, typename T2, typename = std::enable_if_t<!std::is_same_v<T1, T2>>>
Tensor<T2> operator*(const Tensor<T1>& A, const Tensor<T2>& B) {
  Tensor<T2> A2(A.shape(), A.memory_type());
  compute::convert_into(A, A2);
  return A2 * B;
}

/// Element-wise sum (choreo-ir.hpp:150-191): shapes must match
/// (std::runtime_error "Tensor shape mismatch for addition"); the result
/// lives where A lives.
template <typename T>
Tensor<T> operator+(const Tensor<T>& A, const Tensor<T>& B) {
  if (A.shape() != B.shape()) throw std::runtime_error("Tensor shape mismatch for addition");
  Tensor<T> C(A.shape(), A.memory_type());
  compute::add_into(A, B, C);
  return C;
}

/// C += X element-wise (so `C += A * B` accumulates a product; for a fused
/// accumulate use compute::gemm(A, B, C, 1, 1)).
template <typename T>
Tensor<T>& operator+=(Tensor<T>& C, const Tensor<T>& X) {
  if (C.shape() != X.shape()) throw std::runtime_error("Tensor shape mismatch for addition");
  compute::add_into(C, X, C);
  return C;
}

/// max(x, 0) element-wise (choreo-ir.hpp:196-222).
template <typename T>
Tensor<T> relu(const Tensor<T>& input) {
  Tensor<T> out(input.shape(), input.memory_type());
  compute::relu_into(input, out);
  return out;
}

template <typename T>
Tensor<T> batch_matmul(const Tensor<T>& A, const Tensor<T>& B) {
  return compute::batch_matmul(A, B);
}

using compute::matmul;

/// Selects the first sm_100 device (choreo-ir.hpp:228-230).
inline bool initialize() { return device::initialize(); }

/// Waits for outstanding work and forgets the device list. The reference
/// also destroyed a cuBLAS handle it never created and reset the device
/// (choreo-ir.hpp:235-251); nothing here owns a handle, and resetting a
/// device other components share would free their memory.
inline void finalize() {
  cudaDeviceSynchronize();
  device::finalize();
}

}  // namespace choreo_ir

#endif  // CHOREO_IR_HPP
