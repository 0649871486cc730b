/**
 * @file elementwise.hpp
 * @brief relu, add, fill and convert. The reference runs these as host loops
 *        (device tensors are copied to the host and back, choreo-ir.hpp:150-222);
 *        here device tensors use the library's vectorised kernels with the
 *        same per-element arithmetic (f16 through float, rounded back;
 *        relu = x < 0 ? 0 : x). Inside a GEMM or conv the same operations are
 *        fused into the epilogue instead (GEMMConfig::bias/relu,
 *        Conv2dParams::relu).
 */
#ifndef CHOREO_IR_COMPUTE_ELEMENTWISE_HPP
#define CHOREO_IR_COMPUTE_ELEMENTWISE_HPP

#include <algorithm>
#include <type_traits>

#include "../../choreo_b200.h"
#include "../tensor/tensor.hpp"
#include "validation.hpp"

namespace choreo_ir {
namespace compute {

template <typename T>
void relu_into(const Tensor<T>& in, Tensor<T>& out, cudaStream_t stream = nullptr) {
  if (in.shape() != out.shape()) throw ValidationError("ReLU: Shape mismatch between input and output tensors");
  if (in.memory_type() == MemoryType::HOST) {
    for (index_t i = 0; i < in.numel(); ++i) {
      if constexpr (std::is_same_v<T, float16_t>) {
        const float x = __half2float(in.data()[i]);
        out.data()[i] = __float2half(std::max(x, 0.0f));
      } else {
        out.data()[i] = std::max(in.data()[i], T(0));
      }
    }
    return;
  }
  constexpr int dt = choreo_ir::detail::abi_dtype<T>();
  static_assert(dt >= 0, "device relu supports float16, bfloat16 and float");
  choreo_ir::detail::status_check(choreo_relu(dt, in.data(), out.data(), in.numel(), stream));
  choreo_ir::detail::cuda_check(cudaStreamSynchronize(stream), "relu");
}

template <typename T>
void add_into(const Tensor<T>& a, const Tensor<T>& b, Tensor<T>& out, cudaStream_t stream = nullptr) {
  validate_elementwise_contract(a, b, out, "Addition");
  if (a.memory_type() == MemoryType::HOST) {
    for (index_t i = 0; i < a.numel(); ++i) {
      if constexpr (std::is_same_v<T, float16_t>)
        out.data()[i] = __float2half(__half2float(a.data()[i]) + __half2float(b.data()[i]));
      else
        out.data()[i] = a.data()[i] + b.data()[i];
    }
    return;
  }
  constexpr int dt = choreo_ir::detail::abi_dtype<T>();
  static_assert(dt >= 0, "device add supports float16, bfloat16 and float");
  choreo_ir::detail::status_check(choreo_add(dt, a.data(), b.data(), out.data(), a.numel(), stream));
  choreo_ir::detail::cuda_check(cudaStreamSynchronize(stream), "add");
}

/// dst = static_cast<TD>(src) element by element (f16/bf16/f32 pairs).
template <typename TS, typename TD>
void convert_into(const Tensor<TS>& src, Tensor<TD>& dst, cudaStream_t stream = nullptr) {
  if (src.shape() != dst.shape()) throw ValidationError("convert: Shape mismatch between input and output tensors");
  if (src.memory_type() == MemoryType::HOST) {
    for (index_t i = 0; i < src.numel(); ++i) dst.data()[i] = from_float<TD>(to_float(src.data()[i]));
    return;
  }
  choreo_ir::detail::status_check(choreo_convert(choreo_ir::detail::abi_dtype<TS>(), src.data(),
                                                 choreo_ir::detail::abi_dtype<TD>(), dst.data(), src.numel(), stream));
  choreo_ir::detail::cuda_check(cudaStreamSynchronize(stream), "convert");
}

}  // namespace compute
}  // namespace choreo_ir

#endif  // CHOREO_IR_COMPUTE_ELEMENTWISE_HPP
