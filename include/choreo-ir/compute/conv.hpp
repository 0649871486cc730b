/**
 * @file conv.hpp
 * @brief conv2d: the convolution the reference's benchmarks call
 *        (benchmark/performance/benchmark_suite.cpp:379) but never define,
 *        with the semantics of its only conv kernel
 *        (benchmark/kernels/gemm_example.cu:208-253: direct convolution with
 *        stride and zero padding), on NHWC activations and KRSC weights.
 *        Device tensors run the implicit-GEMM tcgen05 kernel
 *        (choreo_conv2d) with a fused bias + ReLU epilogue; host tensors
 *        run that reference loop, accumulating in T.
 */
#ifndef CHOREO_IR_COMPUTE_CONV_HPP
#define CHOREO_IR_COMPUTE_CONV_HPP

#include <type_traits>

#include "../../choreo_b200.h"
#include "../tensor/tensor.hpp"
#include "validation.hpp"

namespace choreo_ir {

struct Conv2dParams {
  int stride_h = 1, stride_w = 1;
  int pad_h = 0, pad_w = 0;
  int dil_h = 1, dil_w = 1;
  float alpha = 1.0f;
  bool relu = false;
  cudaStream_t stream = nullptr;
};

namespace detail {
inline index_t conv_out(index_t in, int pad, int dil, index_t k, int stride) {
  return (in + 2 * pad - dil * (k - 1) - 1) / stride + 1;
}
}  // namespace detail

/// output[n, p, q, k] = act(alpha * sum_{r,s,c} input[n, p*sh - ph + r*dh, q*sw - pw + s*dw, c]
///                          * weight[k, r, s, c] + bias[k]).
/// input NHWC, weight KRSC, output NHWC [n, P, Q, K]; bias optional ([K]).
template <typename T, typename TO, typename TB = TO>
void conv2d(const Tensor<T>& input, const Tensor<T>& weight, Tensor<TO>& output, const Conv2dParams& p,
            const Tensor<TB>* bias = nullptr) {
  using compute::ValidationError;
  if (input.ndims() != 4 || weight.ndims() != 4 || output.ndims() != 4)
    throw ValidationError("conv2d: input [N,H,W,C], weight [K,R,S,C] and output [N,P,Q,K] must be 4-D");
  const index_t N = input.shape()[0], H = input.shape()[1], W = input.shape()[2], Cc = input.shape()[3];
  const index_t K = weight.shape()[0], R = weight.shape()[1], S = weight.shape()[2];
  if (weight.shape()[3] != Cc) throw ValidationError("conv2d: weight channels differ from input channels");
  const index_t P = detail::conv_out(H, p.pad_h, p.dil_h, R, p.stride_h);
  const index_t Q = detail::conv_out(W, p.pad_w, p.dil_w, S, p.stride_w);
  if (output.shape() != Shape({N, P, Q, K})) throw ValidationError("conv2d: output shape mismatch");
  if (bias && bias->numel() != K) throw ValidationError("conv2d: bias must have K elements");
  if (input.memory_type() != weight.memory_type() || input.memory_type() != output.memory_type())
    throw ValidationError("conv2d: Memory type mismatch between input and output tensors");

  if (input.memory_type() == MemoryType::HOST) {
    for (index_t n = 0; n < N; ++n)
      for (index_t oh = 0; oh < P; ++oh)
        for (index_t ow = 0; ow < Q; ++ow)
          for (index_t k = 0; k < K; ++k) {
            T sum = from_float<T>(0.0f);
            for (index_t c = 0; c < Cc; ++c)
              for (index_t r = 0; r < R; ++r)
                for (index_t s = 0; s < S; ++s) {
                  const index_t hi = oh * p.stride_h - p.pad_h + r * p.dil_h;
                  const index_t wi = ow * p.stride_w - p.pad_w + s * p.dil_w;
                  if (hi >= 0 && hi < H && wi >= 0 && wi < W)
                    sum = from_float<T>(to_float(sum) + to_float(from_float<T>(
                                                            to_float(input(n, hi, wi, c)) * to_float(weight(k, r, s, c)))));
                }
            float v = p.alpha * to_float(sum) + (bias ? to_float((*bias)(k)) : 0.0f);
            if (p.relu && v < 0.0f) v = 0.0f;
            output(n, oh, ow, k) = from_float<TO>(v);
          }
    return;
  }
  static_assert(std::is_same_v<T, float16_t> || std::is_same_v<T, bfloat16_t>, "device conv2d needs f16 or bf16 inputs");
  if (!input.is_contiguous() || !weight.is_contiguous() || !output.is_contiguous())
    throw ValidationError("conv2d: device tensors must be contiguous");
  choreo_conv_desc d{};
  d.n = N; d.h = H; d.w = W; d.c = Cc;
  d.k = K; d.r = R; d.s = S;
  d.stride_h = p.stride_h; d.stride_w = p.stride_w;
  d.pad_h = p.pad_h; d.pad_w = p.pad_w;
  d.dil_h = p.dil_h; d.dil_w = p.dil_w;
  d.dtype = choreo_ir::detail::abi_dtype<T>();
  d.dtype_out = choreo_ir::detail::abi_dtype<TO>();
  d.input = input.data();
  d.weight = weight.data();
  d.output = output.data();
  d.bias = bias ? bias->data() : nullptr;
  d.dtype_bias = choreo_ir::detail::abi_dtype<TB>();
  d.relu = p.relu ? 1 : 0;
  d.alpha = p.alpha;
  choreo_ir::detail::status_check(choreo_conv2d(&d, nullptr, 0, p.stream));
}

/// Allocating form: conv2d(input, weight, stride, padding) as the reference's
/// benchmarks call it (square stride/padding, no bias, no activation).
template <typename T>
Tensor<T> conv2d(const Tensor<T>& input, const Tensor<T>& weight, int stride = 1, int padding = 0) {
  if (input.ndims() != 4 || weight.ndims() != 4)
    throw compute::ValidationError("conv2d: input [N,H,W,C] and weight [K,R,S,C] must be 4-D");
  Conv2dParams p;
  p.stride_h = p.stride_w = stride;
  p.pad_h = p.pad_w = padding;
  const index_t P = detail::conv_out(input.shape()[1], padding, 1, weight.shape()[1], stride);
  const index_t Q = detail::conv_out(input.shape()[2], padding, 1, weight.shape()[2], stride);
  Tensor<T> out(Shape({input.shape()[0], P, Q, weight.shape()[0]}), input.memory_type());
  conv2d<T, T, T>(input, weight, out, p, nullptr);
  return out;
}

}  // namespace choreo_ir

#endif  // CHOREO_IR_COMPUTE_CONV_HPP
