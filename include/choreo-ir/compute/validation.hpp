/**
 * @file validation.hpp
 * @brief Operation contracts (the reference's compute/validation.hpp:20-247:
 *        same checks, same order, same messages, all thrown as
 *        ValidationError, a std::runtime_error), plus the TMA contract the
 *        sm_100a kernels add.
 */
#ifndef CHOREO_IR_COMPUTE_VALIDATION_HPP
#define CHOREO_IR_COMPUTE_VALIDATION_HPP

#include <cstdint>
#include <stdexcept>
#include <string>
#include <type_traits>

#include "../core/types.hpp"
#include "../tensor/tensor.hpp"

namespace choreo_ir {
namespace compute {

class ValidationError : public std::runtime_error {
 public:
  explicit ValidationError(const std::string& message) : std::runtime_error(message) {}
};

namespace detail {
inline std::string dims(index_t a, index_t b) { return std::to_string(a) + "x" + std::to_string(b); }
}  // namespace detail

/// Matrix product contract: rank >= 2, inner extents equal, output M x N,
/// same memory type and dtype, non-null, non-empty, positive extents.
template <typename TA, typename TB, typename TC>
void validate_matmul_contract(const TA& A, const TB& B, const TC& C,
                              const std::string& op = "Matrix multiplication") {
  if (A.ndims() < 2 || B.ndims() < 2) throw ValidationError(op + ": Input tensors must be at least 2D");
  if (C.ndims() < 2) throw ValidationError(op + ": Output tensor must be at least 2D");
  const index_t M = A.shape()[A.ndims() - 2], K = A.shape()[A.ndims() - 1];
  const index_t K2 = B.shape()[B.ndims() - 2], N = B.shape()[B.ndims() - 1];
  const index_t Mo = C.shape()[C.ndims() - 2], No = C.shape()[C.ndims() - 1];
  if (K != K2)
    throw ValidationError(op + ": Matrix dimension mismatch: A(" + detail::dims(M, K) + ") * B(" + detail::dims(K2, N) + ")");
  if (M != Mo || N != No)
    throw ValidationError(op + ": Output shape mismatch: expected (" + detail::dims(M, N) + "), got (" +
                          detail::dims(Mo, No) + ")");
  if (A.memory_type() != B.memory_type() || A.memory_type() != C.memory_type())
    throw ValidationError(op + ": Memory type mismatch between input and output tensors");
  if (A.dtype() != B.dtype() || A.dtype() != C.dtype())
    throw ValidationError(op + ": Data type mismatch between input and output tensors");
  if (A.data() == nullptr) throw ValidationError(op + ": Input tensor A has null data pointer");
  if (B.data() == nullptr) throw ValidationError(op + ": Input tensor B has null data pointer");
  if (C.data() == nullptr) throw ValidationError(op + ": Output tensor C has null data pointer");
  if (A.numel() == 0) throw ValidationError(op + ": Input tensor A is empty");
  if (B.numel() == 0) throw ValidationError(op + ": Input tensor B is empty");
  if (C.numel() == 0) throw ValidationError(op + ": Output tensor C is empty");
  if (M <= 0 || N <= 0 || K <= 0)
    throw ValidationError(op + ": Invalid matrix dimensions: M=" + std::to_string(M) + ", N=" + std::to_string(N) +
                          ", K=" + std::to_string(K));
}

/// Mixed-precision variant: same checks except the output dtype may differ
/// (f16/bf16 inputs, f32 output).
template <typename TA, typename TB, typename TC>
void validate_mixed_matmul_contract(const TA& A, const TB& B, const TC& C,
                                    const std::string& op = "Mixed precision matmul") {
  if (A.ndims() < 2 || B.ndims() < 2) throw ValidationError(op + ": Input tensors must be at least 2D");
  const index_t M = A.shape()[A.ndims() - 2], K = A.shape()[A.ndims() - 1];
  const index_t K2 = B.shape()[B.ndims() - 2], N = B.shape()[B.ndims() - 1];
  if (K != K2)
    throw ValidationError(op + ": Matrix dimension mismatch: A(" + detail::dims(M, K) + ") * B(" + detail::dims(K2, N) + ")");
  if (C.ndims() < 2 || C.shape()[C.ndims() - 2] != M || C.shape()[C.ndims() - 1] != N)
    throw ValidationError(op + ": Output shape mismatch");
  if (A.dtype() != B.dtype()) throw ValidationError(op + ": Data type mismatch between input tensors");
  if (A.memory_type() != B.memory_type() || A.memory_type() != C.memory_type())
    throw ValidationError(op + ": Memory type mismatch between input and output tensors");
  if (A.data() == nullptr || B.data() == nullptr || C.data() == nullptr)
    throw ValidationError(op + ": Tensor has null data pointer");
}

template <typename T>
void validate_elementwise_contract(const Tensor<T>& A, const Tensor<T>& B, const Tensor<T>& C,
                                   const std::string& op = "Element-wise operation") {
  if (A.shape() != B.shape() || A.shape() != C.shape())
    throw ValidationError(op + ": Shape mismatch between input and output tensors");
  if (A.memory_type() != B.memory_type() || A.memory_type() != C.memory_type())
    throw ValidationError(op + ": Memory type mismatch between input and output tensors");
  if (A.dtype() != B.dtype() || A.dtype() != C.dtype())
    throw ValidationError(op + ": Data type mismatch between input and output tensors");
  if (A.data() == nullptr || B.data() == nullptr || C.data() == nullptr)
    throw ValidationError(op + ": Tensor has null data pointer");
  if (A.numel() == 0) throw ValidationError(op + ": Input tensors are empty");
}

/// Tensor-core contract on sm_100a: f16 or bf16 operands (f32 runs on CUDA
/// cores; f64 has no path), 16-byte aligned data. Extents need no padding:
/// ragged tails are handled by the TMA.
template <typename T>
void validate_tensor_core_contract(const Tensor<T>& A, const Tensor<T>& B, const Tensor<T>& C,
                                   const std::string& op = "Tensor core operation") {
  if constexpr (std::is_same_v<T, double>)
    throw ValidationError(op + ": Double precision not supported for tensor core operations");
  else if constexpr (!std::is_same_v<T, float16_t> && !std::is_same_v<T, bfloat16_t> && !std::is_same_v<T, float>)
    throw ValidationError(op + ": Data type not supported for tensor core operations");
  if (reinterpret_cast<std::uintptr_t>(A.data()) % 16 != 0) throw ValidationError(op + ": Tensor A data not 16-byte aligned");
  if (reinterpret_cast<std::uintptr_t>(B.data()) % 16 != 0) throw ValidationError(op + ": Tensor B data not 16-byte aligned");
  if (reinterpret_cast<std::uintptr_t>(C.data()) % 16 != 0) throw ValidationError(op + ": Tensor C data not 16-byte aligned");
}

/// True when the tcgen05 kernel reads this operand through TMA directly
/// (otherwise it is repacked into workspace first; both are correct).
template <typename View>
bool tma_direct(const View& t) {
  const MatrixStrides m = matrix_strides(t.shape(), t.stride());
  if (!m.valid) return false;
  const index_t batch = t.ndims() >= 3 ? t.shape()[t.ndims() - 3] : 1;
  return tma_addressable(t.data(), m.ld, m.batch_stride, batch, sizeof_dtype(t.dtype()));
}

}  // namespace compute
}  // namespace choreo_ir

#endif  // CHOREO_IR_COMPUTE_VALIDATION_HPP
