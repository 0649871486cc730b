/**
 * @file matmul.hpp
 * @brief GEMM / matmul / batch_matmul definitions over the C ABI
 *        (include/choreo_b200.h). Device tensors run choreo_gemm (tcgen05 for
 *        f16/bf16 with fp32 accumulation, CUDA cores for f32); host tensors
 *        keep the reference's host loop (choreo-ir.hpp:71-101: i-j-k order,
 *        fp16 rounded back after every k, other types accumulated in T).
 *
 * Operand layout comes from the tensors' strides: each of A and B may be
 * row- or column-major (a transpose() view is read in place, never copied),
 * batched operands are rank 3, and a rank-2 B against a rank-3 A is
 * broadcast over the batch.
 */
#ifndef CHOREO_IR_COMPUTE_MATMUL_HPP
#define CHOREO_IR_COMPUTE_MATMUL_HPP

#include <cuda_runtime.h>

#include <string>
#include <type_traits>

#include "../../choreo_b200.h"
#include "compute.hpp"
#include "validation.hpp"

namespace choreo_ir {
namespace compute {
namespace detail {

using choreo_ir::detail::abi_dtype;
using choreo_ir::detail::cuda_check;
using choreo_ir::detail::status_check;

struct Operand {
  const void* ptr = nullptr;
  bool trans = false;     // stored with the second-to-last dimension contiguous
  index_t ld = 0;
  index_t batch = 1;
  index_t batch_stride = 0;
};

template <typename View>
Operand operand_of(const View& t, const char* name) {
  const MatrixStrides m = matrix_strides(t.shape(), t.stride());
  if (!m.valid)
    throw ValidationError(std::string("GEMM operation: ") + name +
                          " needs a contiguous row or column dimension (stride 1)");
  if (t.ndims() > 3) throw ValidationError(std::string("GEMM operation: ") + name + " has more than 3 dimensions");
  Operand o;
  o.ptr = t.data();
  o.trans = m.transposed;
  o.ld = m.ld;
  o.batch = t.ndims() == 3 ? t.shape()[0] : 1;
  o.batch_stride = t.ndims() == 3 ? m.batch_stride : 0;
  return o;
}

/// Validates, queries, allocates the workspace if the dispatcher needs one
/// (stream-ordered), launches, and frees the workspace.
inline void run_gemm(const choreo_gemm_desc& d, cudaStream_t stream, bool sync) {
  choreo_launch_config q;
  status_check(choreo_gemm_query(&d, &q));
  void* ws = nullptr;
  if (q.workspace_bytes > 0)
    cuda_check(cudaMallocAsync(&ws, static_cast<size_t>(q.workspace_bytes), stream), "GEMM workspace");
  const int rc = choreo_gemm(&d, ws, static_cast<size_t>(q.workspace_bytes), stream);
  if (ws) cudaFreeAsync(ws, stream);
  status_check(rc);
  if (sync) status_check(choreo_sync_status(stream));
}

/// Device GEMM on views: C = alpha * op(A) op(B) + beta * C (+ bias, ReLU).
template <typename TAB, typename TC, typename VA, typename VB, typename VC>
void device_gemm(const VA& A, const VB& B, const VC& C, float alpha, float beta, const GEMMConfig& cfg) {
  constexpr int dab = abi_dtype<TAB>();
  constexpr int dc = abi_dtype<TC>();
  static_assert(dab >= 0 && dc >= 0, "device GEMM supports float16, bfloat16 and float");
  const Operand a = operand_of(A, "A"), b = operand_of(B, "B"), c = operand_of(C, "C");
  if (c.trans) throw ValidationError("GEMM operation: output C must be row-major (last dimension contiguous)");
  const index_t batch = c.batch;
  if ((a.batch != batch && a.batch != 1) || (b.batch != batch && b.batch != 1))
    throw ValidationError("GEMM operation: batch sizes of A, B and C differ");
  choreo_gemm_desc d{};
  d.m = A.shape()[A.ndims() - 2];
  d.k = A.shape()[A.ndims() - 1];
  d.n = B.shape()[B.ndims() - 1];
  d.dtype_ab = dab;
  d.dtype_c = dc;
  d.a = a.ptr;
  d.lda = a.ld;
  d.trans_a = a.trans ? 1 : 0;
  d.b = b.ptr;
  d.ldb = b.ld;
  d.trans_b = b.trans ? 1 : 0;
  d.c = const_cast<void*>(static_cast<const void*>(C.data()));
  d.ldc = c.ld;
  d.alpha = alpha;
  d.beta = beta;
  d.bias = cfg.bias;
  d.dtype_bias = static_cast<int32_t>(cfg.bias_dtype);
  d.relu = cfg.relu ? 1 : 0;
  d.batch = batch;
  d.stride_a = a.batch == 1 ? 0 : a.batch_stride;
  d.stride_b = b.batch == 1 ? 0 : b.batch_stride;
  d.stride_c = c.batch_stride;
  run_gemm(d, cfg.stream, cfg.synchronize);
}

/// The reference's host loop for one (batch item of a) product, generalised
/// with alpha/beta: for alpha = 1, beta = 0 the result is bit-identical to
/// the reference's operator* host branch.
template <typename T>
void host_gemm(const Tensor<T>& A, const Tensor<T>& B, Tensor<T>& C, T alpha, T beta) {
  const index_t M = A.shape()[A.ndims() - 2], K = A.shape()[A.ndims() - 1], N = B.shape()[B.ndims() - 1];
  const index_t batch = C.ndims() == 3 ? C.shape()[0] : 1;
  const bool plain = to_float(alpha) == 1.0f && to_float(beta) == 0.0f;
  for (index_t bi = 0; bi < batch; ++bi) {
    const T* a = A.data() + (A.ndims() == 3 ? bi * M * K : 0);
    const T* b = B.data() + (B.ndims() == 3 ? bi * K * N : 0);
    T* c = C.data() + bi * M * N;
    for (index_t i = 0; i < M; ++i) {
      for (index_t j = 0; j < N; ++j) {
        T acc = from_float<T>(0.0f);
        for (index_t k = 0; k < K; ++k) {
          if constexpr (std::is_same_v<T, float16_t>) {
            acc = __float2half(__half2float(acc) + __half2float(a[i * K + k]) * __half2float(b[k * N + j]));
          } else {
            acc += a[i * K + k] * b[k * N + j];
          }
        }
        if (plain) {
          c[i * N + j] = acc;
        } else {
          c[i * N + j] = from_float<T>(to_float(alpha) * to_float(acc) + to_float(beta) * to_float(c[i * N + j]));
        }
      }
    }
  }
}

}  // namespace detail

template <typename T>
void gemm(const Tensor<T>& A, const Tensor<T>& B, Tensor<T>& C, T alpha, T beta, const GEMMConfig& config) {
  validate_matmul_contract(A, B, C, "GEMM operation");
  if (A.memory_type() == MemoryType::HOST) {
    detail::host_gemm(A, B, C, alpha, beta);
    return;
  }
  detail::device_gemm<T, T>(A, B, C, to_float(alpha), to_float(beta), config);
}

template <typename T>
Tensor<T> gemm(const Tensor<T>& A, const Tensor<T>& B, T alpha, const GEMMConfig& config) {
  Tensor<T> C(Shape({A.shape()[A.ndims() - 2], B.shape()[B.ndims() - 1]}), A.memory_type());
  gemm(A, B, C, alpha, from_float<T>(0.0f), config);
  return C;
}

template <typename T>
void matmul(const Tensor<T>& A, const Tensor<T>& B, Tensor<T>& C, const GEMMConfig& config) {
  validate_matmul_contract(A, B, C, "Matrix multiplication");
  gemm(A, B, C, from_float<T>(1.0f), from_float<T>(0.0f), config);
}

template <typename T>
Tensor<T> matmul(const Tensor<T>& A, const Tensor<T>& B, const GEMMConfig& config) {
  Tensor<T> C(Shape({A.shape()[A.ndims() - 2], B.shape()[B.ndims() - 1]}), A.memory_type());
  matmul(A, B, C, config);
  return C;
}

/// Mixed precision: f16/bf16 inputs, f32 output, fp32 accumulation
/// (docs/TESTING_AND_BENCHMARKS.md:172-178 of the reference). Device only.
template <typename TIn, std::enable_if_t<std::is_same_v<TIn, float16_t> || std::is_same_v<TIn, bfloat16_t>, int> = 0>
void matmul(const Tensor<TIn>& A, const Tensor<TIn>& B, Tensor<float>& C, const GEMMConfig& config = GEMMConfig()) {
  validate_mixed_matmul_contract(A, B, C);
  if (A.memory_type() == MemoryType::HOST) throw ValidationError("Mixed precision matmul: device tensors required");
  detail::device_gemm<TIn, float>(A, B, C, 1.0f, 0.0f, config);
}

/// GEMM on views (e.g. transpose() or tile(offset, shape) windows): all
/// three views must be device memory.
template <typename T, typename TC>
void matmul(const TensorView<T>& A, const TensorView<T>& B, const TensorView<TC>& C, float alpha = 1.0f,
            float beta = 0.0f, const GEMMConfig& config = GEMMConfig()) {
  detail::device_gemm<T, TC>(A, B, C, alpha, beta, config);
}

/// Batched product [b, m, k] x [b, k, n] (or a shared [k, n]) -> [b, m, n]
/// (benchmark_suite.cpp:333-362 of the reference).
template <typename T>
Tensor<T> batch_matmul(const Tensor<T>& A, const Tensor<T>& B, const GEMMConfig& config = GEMMConfig()) {
  if (A.ndims() != 3 || (B.ndims() != 3 && B.ndims() != 2))
    throw ValidationError("Batch matmul: A must be [b, m, k] and B [b, k, n] or [k, n]");
  if (B.ndims() == 3 && B.shape()[0] != A.shape()[0]) throw ValidationError("Batch matmul: batch sizes differ");
  Tensor<T> C(Shape({A.shape()[0], A.shape()[1], B.shape()[B.ndims() - 1]}), A.memory_type());
  validate_matmul_contract(A, B, C, "Batch matmul");
  gemm(A, B, C, from_float<T>(1.0f), from_float<T>(0.0f), config);
  return C;
}

template <typename T>
GEMMConfig get_optimal_gemm_config(const Tensor<T>& A, const Tensor<T>& B) {
  GEMMConfig cfg;
  cfg.backend = can_use_tensor_core_gemm(A, B) ? ComputeBackend::TCGEN05 : ComputeBackend::CUDA_CORE;
  cfg.use_tensor_core = cfg.backend == ComputeBackend::TCGEN05;
  if (A.memory_type() != MemoryType::DEVICE || B.memory_type() != MemoryType::DEVICE) return cfg;
  if constexpr (detail::abi_dtype<T>() >= 0) {
    choreo_gemm_desc d{};
    const detail::Operand a = detail::operand_of(A, "A"), b = detail::operand_of(B, "B");
    d.m = A.shape()[A.ndims() - 2];
    d.k = A.shape()[A.ndims() - 1];
    d.n = B.shape()[B.ndims() - 1];
    d.dtype_ab = d.dtype_c = detail::abi_dtype<T>();
    d.a = a.ptr;
    d.lda = a.ld;
    d.trans_a = a.trans;
    d.b = b.ptr;
    d.ldb = b.ld;
    d.trans_b = b.trans;
    d.c = const_cast<void*>(static_cast<const void*>(A.data()));  // only validated, never written
    d.ldc = d.n;
    d.alpha = 1.0f;
    d.batch = 1;
    choreo_launch_config q;
    if (choreo_gemm_query(&d, &q) == CHOREO_OK) {
      cfg.tile_m = q.tile_m;
      cfg.tile_n = q.tile_n;
      cfg.tile_k = q.tile_k;
      cfg.stages = q.stages;
    }
  }
  return cfg;
}

template <typename T>
bool can_use_tensor_core_gemm(const Tensor<T>& A, const Tensor<T>& B) {
  if (!std::is_same_v<T, float16_t> && !std::is_same_v<T, bfloat16_t>) return false;
  return A.memory_type() == MemoryType::DEVICE && B.memory_type() == MemoryType::DEVICE;
}

template <typename T>
bool can_use_wmma_gemm(const Tensor<T>& A, const Tensor<T>& B) {
  return can_use_tensor_core_gemm(A, B);
}

}  // namespace compute
}  // namespace choreo_ir

#endif  // CHOREO_IR_COMPUTE_MATMUL_HPP
