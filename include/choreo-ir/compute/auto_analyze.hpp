/**
 * @file auto_analyze.hpp
 * @brief auto_analyze(A, B, C) -> LaunchConfig and config.launch(), the
 *        automatic configuration the reference documents
 *        (README.md:122-128, examples/ideal_matmul_example.cu:244-290) but
 *        never defines.
 *
 * auto_analyze asks the dispatcher (choreo_gemm_query) which sm_100a kernel,
 * tile, pipeline depth, grid and shared memory a product of these tensors
 * gets. LaunchConfig::launch() runs exactly that GEMM; launch(kernel, args...)
 * launches a caller's own kernel with the analysed grid / block / dynamic
 * shared memory, as the reference's example does.
 */
#ifndef CHOREO_IR_COMPUTE_AUTO_ANALYZE_HPP
#define CHOREO_IR_COMPUTE_AUTO_ANALYZE_HPP

#include <cuda_runtime.h>

#include <array>
#include <tuple>
#include <type_traits>
#include <utility>

#include "../../choreo_b200.h"
#include "matmul.hpp"

namespace choreo_ir {

class LaunchConfig;
template <typename T>
LaunchConfig auto_analyze(const Tensor<T>& A, const Tensor<T>& B, const Tensor<T>& C, cudaStream_t stream = nullptr);

class LaunchConfig {
 public:
  dim3 grid_dim{1, 1, 1};
  dim3 block_dim{1, 1, 1};
  size_t shared_memory = 0;
  int tmem_columns = 0;
  dim3 tile_sizes{0, 0, 0};   // (tile_m, tile_n, tile_k)
  int stages = 0;
  int cluster_m = 1;
  int64_t tiles = 0;
  size_t workspace_bytes = 0;  // scratch of the fastest plan (K-split partials, repacks)
  int split_k = 1;             // K ranges computed in parallel and summed in fp32
  bool use_tensor_cores = false;
  cudaStream_t stream = nullptr;

  /// Runs the analysed GEMM (C = A * B with the tensors given to auto_analyze).
  void launch() const {
    compute::detail::run_gemm(desc_, stream, false);
  }

  /// Launches `kernel` with this configuration's grid, block and dynamic
  /// shared memory (the kernel's own arguments are passed through).
  template <typename... KArgs, typename... Args>
  void launch(void (*kernel)(KArgs...), Args&&... args) const {
    static_assert(sizeof...(KArgs) == sizeof...(Args), "launch: argument count differs from the kernel's");
    if (shared_memory > 0)
      choreo_ir::detail::cuda_check(
          cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(shared_memory)),
          "cudaFuncSetAttribute");
    // cudaLaunchKernel reads each argument as the kernel's parameter type.
    std::tuple<std::decay_t<KArgs>...> values(std::forward<Args>(args)...);
    std::array<void*, sizeof...(KArgs) + 1> params{};
    std::apply([&params](auto&... v) {
      size_t i = 0;
      ((params[i++] = static_cast<void*>(&v)), ...);
    }, values);
    choreo_ir::detail::cuda_check(cudaLaunchKernel(reinterpret_cast<const void*>(kernel), grid_dim, block_dim,
                                                   params.data(), shared_memory, stream),
                                  "LaunchConfig::launch");
  }

  const choreo_gemm_desc& descriptor() const { return desc_; }

 private:
  template <typename T>
  friend LaunchConfig auto_analyze(const Tensor<T>&, const Tensor<T>&, const Tensor<T>&, cudaStream_t);
  choreo_gemm_desc desc_{};
};

/// Analyses C = A * B for device tensors A [.., M, K], B [.., K, N], C [.., M, N].
template <typename T>
LaunchConfig auto_analyze(const Tensor<T>& A, const Tensor<T>& B, const Tensor<T>& C, cudaStream_t stream) {
  compute::validate_matmul_contract(A, B, C, "auto_analyze");
  if (A.memory_type() == MemoryType::HOST) throw compute::ValidationError("auto_analyze: device tensors required");
  const compute::detail::Operand a = compute::detail::operand_of(A, "A");
  const compute::detail::Operand b = compute::detail::operand_of(B, "B");
  const compute::detail::Operand c = compute::detail::operand_of(C, "C");
  LaunchConfig lc;
  choreo_gemm_desc& d = lc.desc_;
  d.m = A.shape()[A.ndims() - 2];
  d.k = A.shape()[A.ndims() - 1];
  d.n = B.shape()[B.ndims() - 1];
  d.dtype_ab = d.dtype_c = choreo_ir::detail::abi_dtype<T>();
  d.a = a.ptr; d.lda = a.ld; d.trans_a = a.trans;
  d.b = b.ptr; d.ldb = b.ld; d.trans_b = b.trans;
  d.c = C.data(); d.ldc = c.ld;
  d.alpha = 1.0f;
  d.beta = 0.0f;
  d.batch = c.batch;
  d.stride_a = a.batch == 1 ? 0 : a.batch_stride;
  d.stride_b = b.batch == 1 ? 0 : b.batch_stride;
  d.stride_c = c.batch_stride;
  choreo_launch_config q;
  choreo_ir::detail::status_check(choreo_gemm_query(&d, &q));
  lc.grid_dim = dim3(static_cast<unsigned>(q.grid_x), static_cast<unsigned>(q.grid_y), static_cast<unsigned>(q.grid_z));
  lc.block_dim = dim3(static_cast<unsigned>(q.block_x), 1, 1);
  lc.shared_memory = static_cast<size_t>(q.smem_bytes);
  lc.tmem_columns = q.tmem_cols;
  lc.tile_sizes = dim3(static_cast<unsigned>(q.tile_m), static_cast<unsigned>(q.tile_n), static_cast<unsigned>(q.tile_k));
  lc.stages = q.stages;
  lc.cluster_m = q.cluster_m;
  lc.tiles = q.tiles;
  lc.workspace_bytes = static_cast<size_t>(q.workspace_bytes);
  lc.split_k = static_cast<int>(q.split_k);
  lc.use_tensor_cores = q.kernel == 1;
  lc.stream = stream;
  return lc;
}

}  // namespace choreo_ir

#endif  // CHOREO_IR_COMPUTE_AUTO_ANALYZE_HPP
