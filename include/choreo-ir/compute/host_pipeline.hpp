/**
 * @file host_pipeline.hpp
 * @brief GEMM and conv on HOST tensors with the transfers overlapped:
 *        the pipelined form of the reference's
 *        `A.to_device() * B.to_device()` ... `.to_host()` flow
 *        (tensor/tensor.hpp:568-598, README.md:86-94), over the C ABI's host
 *        plans (choreo_host_gemm_* / choreo_host_conv_*).
 *
 * A plan is made once per shape; it owns its device buffers, two copy streams
 * and its events. run() cuts A (or the image batch) into parts so that the
 * host->device copy of one part, the kernel of the previous one and the
 * device->host copy of the one before run at the same time, and returns with
 * all of it enqueued on the plan's stream (call synchronize(), or a stream
 * synchronize, before reading the output).
 *
 * Host tensors made with `new[]` (MemoryType::HOST) are pageable: the copies
 * still work but the driver stages them. Wrap them in a PinnedHost guard
 * (cudaHostRegister for the guard's lifetime) to get the overlap.
 */
#ifndef CHOREO_IR_COMPUTE_HOST_PIPELINE_HPP
#define CHOREO_IR_COMPUTE_HOST_PIPELINE_HPP

#include <cuda_runtime.h>

#include <utility>

#include "../../choreo_b200.h"
#include "../tensor/tensor.hpp"
#include "validation.hpp"

namespace choreo_ir {

/// Page-locks a host tensor's buffer for the guard's lifetime so copies
/// through a host plan overlap with the kernels (cudaHostRegister /
/// cudaHostUnregister). The tensor must outlive the guard.
class PinnedHost {
 public:
  template <typename T>
  explicit PinnedHost(const Tensor<T>& t) : ptr_(const_cast<T*>(t.data())) {
    if (t.memory_type() != MemoryType::HOST) throw compute::ValidationError("PinnedHost: host tensor required");
    if (ptr_ != nullptr)
      detail::cuda_check(cudaHostRegister(ptr_, t.bytes(), cudaHostRegisterDefault), "cudaHostRegister");
  }
  ~PinnedHost() {
    if (ptr_ != nullptr) cudaHostUnregister(ptr_);
  }
  PinnedHost(const PinnedHost&) = delete;
  PinnedHost& operator=(const PinnedHost&) = delete;

 private:
  void* ptr_;
};

namespace compute {

namespace detail {
/// Owns a choreo_host_plan.
class HostPlanHandle {
 public:
  HostPlanHandle() = default;
  explicit HostPlanHandle(choreo_host_plan* p) : p_(p) {}
  HostPlanHandle(HostPlanHandle&& o) noexcept : p_(std::exchange(o.p_, nullptr)) {}
  HostPlanHandle& operator=(HostPlanHandle&& o) noexcept {
    if (this != &o) {
      reset();
      p_ = std::exchange(o.p_, nullptr);
    }
    return *this;
  }
  ~HostPlanHandle() { reset(); }
  choreo_host_plan* get() const { return p_; }
  choreo_host_plan_info info() const {
    choreo_host_plan_info i{};
    choreo_ir::detail::status_check(choreo_host_plan_info_get(p_, &i));
    return i;
  }

 private:
  void reset() {
    if (p_) choreo_host_plan_destroy(p_);
    p_ = nullptr;
  }
  choreo_host_plan* p_ = nullptr;
};

template <typename T>
void require_host(const Tensor<T>& t, const char* what) {
  if (t.memory_type() == MemoryType::DEVICE)
    throw ValidationError(std::string("host pipeline: ") + what + " must be a host tensor");
}
}  // namespace detail

/// C = act(A * B + bias) for row-major HOST tensors A [M, K], B [K, N] and
/// C [M, N] (T = half or bfloat16_t; TC the output type).
template <typename T, typename TC = T>
class HostGemmPlan {
 public:
  HostGemmPlan(index_t M, index_t N, index_t K, bool has_bias = false, bool relu = false, int parts = 0,
               cudaStream_t stream = nullptr)
      : m_(M), n_(N), k_(K), has_bias_(has_bias), stream_(stream) {
    choreo_host_gemm_desc d{};
    d.m = M;
    d.n = N;
    d.k = K;
    d.dtype_ab = choreo_ir::detail::abi_dtype<T>();
    d.dtype_c = choreo_ir::detail::abi_dtype<TC>();
    d.alpha = 1.0f;
    d.has_bias = has_bias ? 1 : 0;
    d.dtype_bias = d.dtype_ab;
    d.relu = relu ? 1 : 0;
    d.parts = parts;
    int dev = 0;
    choreo_ir::detail::cuda_check(cudaGetDevice(&dev), "cudaGetDevice");
    d.device = dev;
    choreo_host_plan* p = nullptr;
    choreo_ir::detail::status_check(choreo_host_gemm_plan_create(&d, &p));
    plan_ = detail::HostPlanHandle(p);
  }

  /// Enqueues one product. bias: N elements, host (or, with a DEVICE bias and
  /// B, read in place from the device).
  void run(const Tensor<T>& A, const Tensor<T>& B, Tensor<TC>& C, const Tensor<T>* bias = nullptr) {
    detail::require_host(A, "A");
    detail::require_host(C, "C");
    if (A.shape() != Shape({m_, k_}) || B.shape() != Shape({k_, n_}) || C.shape() != Shape({m_, n_}))
      throw ValidationError("host pipeline: A, B and C must be [M,K], [K,N] and [M,N] of the plan");
    if ((bias != nullptr) != has_bias_) throw ValidationError("host pipeline: bias does not match the plan");
    const bool on_dev = B.memory_type() == MemoryType::DEVICE;
    if (bias && (bias->memory_type() == MemoryType::DEVICE) != on_dev)
      throw ValidationError("host pipeline: B and bias must both be host or both device tensors");
    choreo_ir::detail::status_check(choreo_host_gemm_run(plan_.get(), A.data(), B.data(),
                                                         bias ? bias->data() : nullptr, C.data(),
                                                         on_dev ? CHOREO_HOST_OPERANDS_ON_DEVICE : 0, stream_));
  }

  /// Waits for the enqueued runs and reports kernel-side failures.
  void synchronize() const { choreo_ir::detail::status_check(choreo_sync_status(stream_)); }

  choreo_host_plan_info info() const { return plan_.info(); }

 private:
  index_t m_, n_, k_;
  bool has_bias_;
  cudaStream_t stream_;
  detail::HostPlanHandle plan_;
};

/// conv2d on HOST tensors: input NHWC [N,H,W,C], weight KRSC [K,R,S,C],
/// output NHWC [N,P,Q,K], fused bias + ReLU (T = half or bfloat16_t).
template <typename T>
class HostConvPlan {
 public:
  HostConvPlan(const Shape& input, const Shape& weight, int stride = 1, int padding = 1, bool has_bias = false,
               bool relu = false, int parts = 0, cudaStream_t stream = nullptr)
      : has_bias_(has_bias), stream_(stream) {
    if (input.ndims() != 4 || weight.ndims() != 4 || weight[3] != input[3])
      throw ValidationError("host conv plan: input [N,H,W,C] and weight [K,R,S,C] expected");
    choreo_conv_desc d{};
    d.n = input[0];
    d.h = input[1];
    d.w = input[2];
    d.c = input[3];
    d.k = weight[0];
    d.r = weight[1];
    d.s = weight[2];
    d.stride_h = d.stride_w = stride;
    d.pad_h = d.pad_w = padding;
    d.dil_h = d.dil_w = 1;
    d.dtype = d.dtype_out = d.dtype_bias = choreo_ir::detail::abi_dtype<T>();
    d.bias = has_bias ? &d : nullptr;  // non-null marks a plan with a bias; the pointer is not used
    d.relu = relu ? 1 : 0;
    d.alpha = 1.0f;
    const index_t P = (d.h + 2 * padding - d.r) / stride + 1, Q = (d.w + 2 * padding - d.s) / stride + 1;
    in_ = input;
    w_ = weight;
    out_ = Shape({d.n, P, Q, d.k});
    int dev = 0;
    choreo_ir::detail::cuda_check(cudaGetDevice(&dev), "cudaGetDevice");
    choreo_host_plan* p = nullptr;
    choreo_ir::detail::status_check(choreo_host_conv_plan_create(&d, parts, dev, &p));
    plan_ = detail::HostPlanHandle(p);
  }

  const Shape& output_shape() const { return out_; }

  void run(const Tensor<T>& input, const Tensor<T>& weight, Tensor<T>& output, const Tensor<T>* bias = nullptr) {
    detail::require_host(input, "input");
    detail::require_host(output, "output");
    if (input.shape() != in_ || weight.shape() != w_ || output.shape() != out_)
      throw ValidationError("host conv plan: tensor shapes differ from the plan's");
    if ((bias != nullptr) != has_bias_) throw ValidationError("host conv plan: bias does not match the plan");
    const bool on_dev = weight.memory_type() == MemoryType::DEVICE;
    choreo_ir::detail::status_check(choreo_host_conv_run(plan_.get(), input.data(), weight.data(),
                                                         bias ? bias->data() : nullptr, output.data(),
                                                         on_dev ? CHOREO_HOST_OPERANDS_ON_DEVICE : 0, stream_));
  }

  void synchronize() const { choreo_ir::detail::status_check(choreo_sync_status(stream_)); }

 private:
  bool has_bias_;
  cudaStream_t stream_;
  Shape in_, w_, out_;
  detail::HostPlanHandle plan_;
};

}  // namespace compute
}  // namespace choreo_ir

#endif  // CHOREO_IR_COMPUTE_HOST_PIPELINE_HPP
