/*
 * oracle/ref_entry.cu — C entry points around the reference's own host code
 * (include/choreo-ir/choreo-ir.hpp from the reference, compiled unmodified
 * with oracle/ref_shim.h force-included). Built by oracle/build.py into
 * oracle/_ref/libchoreo_ref.so.
 *
 * TEST INFRASTRUCTURE ONLY: the pin for the oracle's restatement, and the
 * "reference" CPU baseline bench.py may time. Host tensors only; no GPU call
 * is made.
 */
#include <cstdint>
#include <exception>
#include <thread>
#include <vector>

#include "choreo-ir/choreo-ir.hpp"

using namespace choreo_ir;

namespace {

// C = A * B through the reference's operator* (host branch, choreo-ir.hpp:71-101).
template <typename T>
int host_matmul(const void* a, const void* b, void* c, int64_t M, int64_t N, int64_t K) {
  try {
    Tensor<T> A(Shape({M, K}), MemoryType::HOST);
    Tensor<T> B(Shape({K, N}), MemoryType::HOST);
    A.copy_from_host(static_cast<const T*>(a));
    B.copy_from_host(static_cast<const T*>(b));
    Tensor<T> C = A * B;
    C.copy_to_host(static_cast<T*>(c));
    return 0;
  } catch (const std::exception&) {
    return -1;
  }
}

// Rows [row0, row1) of C = A * B: the reference operator* applied to the row
// slab of A (each row of C depends only on that row of A), split over
// nthreads host threads.
template <typename T>
int host_matmul_rows(const void* a, const void* b, void* c, int64_t M, int64_t N, int64_t K,
                     int64_t row0, int64_t row1, int nthreads) {
  (void)M;
  if (nthreads < 1) nthreads = 1;
  const int64_t rows = row1 - row0;
  if (rows <= 0) return 0;
  std::vector<std::thread> th;
  std::vector<int> rc(nthreads, 0);
  const int64_t per = (rows + nthreads - 1) / nthreads;
  for (int t = 0; t < nthreads; ++t) {
    const int64_t r0 = row0 + t * per;
    const int64_t r1 = std::min(row1, r0 + per);
    if (r0 >= r1) break;
    th.emplace_back([=, &rc] {
      rc[t] = host_matmul<T>(static_cast<const T*>(a) + r0 * K, b, static_cast<T*>(c) + r0 * N, r1 - r0,
                             N, K);
    });
  }
  for (auto& x : th) x.join();
  for (int v : rc)
    if (v) return v;
  return 0;
}

template <typename T>
int host_relu(const void* in, void* out, int64_t n) {
  try {
    Tensor<T> X(Shape({n}), MemoryType::HOST);
    X.copy_from_host(static_cast<const T*>(in));
    Tensor<T> Y = relu(X);
    Y.copy_to_host(static_cast<T*>(out));
    return 0;
  } catch (const std::exception&) {
    return -1;
  }
}

// operator+ (choreo-ir.hpp:150-191) on host tensors of different lengths:
// the reference throws std::runtime_error at its shape check (:152-154)
// before it allocates anything. Returns -2 when it throws, 0 if it did not.
// (Equal shapes are not exercised: the output is constructed with the default
// DEVICE memory type at :156 while the host branch writes it through
// C.data() at :183.)
template <typename T>
int host_add_mismatch(int64_t n_a, int64_t n_b) {
  if (n_a == n_b) return -3;
  try {
    Tensor<T> A(Shape({n_a}), MemoryType::HOST);
    Tensor<T> B(Shape({n_b}), MemoryType::HOST);
    Tensor<T> C = A + B;
    (void)C;
    return 0;
  } catch (const std::runtime_error&) {
    return -2;
  }
}

// operator* with K mismatch (tests/test_end2end.cpp:342-347): -2 if it throws.
template <typename T>
int host_matmul_mismatch(int64_t M, int64_t K, int64_t K2, int64_t N) {
  try {
    Tensor<T> A(Shape({M, K}), MemoryType::HOST);
    Tensor<T> B(Shape({K2, N}), MemoryType::HOST);
    Tensor<T> C = A * B;
    (void)C;
    return 0;
  } catch (const std::runtime_error&) {
    return -2;
  }
}

}  // namespace

// The reference's cuda_core_gemm_kernel declares `extern __shared__ T
// shared_mem[]` (compute/cuda_core.hpp:99), which cannot be instantiated for
// two element types in one translation unit; oracle/build.py therefore
// compiles this file once per type with CHOREO_REF_TYPE = 1 (f16), 2 (bf16)
// or 3 (f32).
extern "C" {

#if CHOREO_REF_TYPE == 1
int choreo_ref_matmul_f16(const void* a, const void* b, void* c, int64_t M, int64_t N, int64_t K) {
  return host_matmul<__half>(a, b, c, M, N, K);
}
int choreo_ref_matmul_f16_rows(const void* a, const void* b, void* c, int64_t M, int64_t N, int64_t K,
                               int64_t row0, int64_t row1, int nthreads) {
  return host_matmul_rows<__half>(a, b, c, M, N, K, row0, row1, nthreads);
}
int choreo_ref_relu_f16(const void* in, void* out, int64_t n) { return host_relu<__half>(in, out, n); }
#elif CHOREO_REF_TYPE == 2
int choreo_ref_matmul_bf16(const void* a, const void* b, void* c, int64_t M, int64_t N, int64_t K) {
  return host_matmul<__nv_bfloat16>(a, b, c, M, N, K);
}
int choreo_ref_matmul_bf16_rows(const void* a, const void* b, void* c, int64_t M, int64_t N, int64_t K,
                                int64_t row0, int64_t row1, int nthreads) {
  return host_matmul_rows<__nv_bfloat16>(a, b, c, M, N, K, row0, row1, nthreads);
}
#elif CHOREO_REF_TYPE == 3
int choreo_ref_matmul_f32(const void* a, const void* b, void* c, int64_t M, int64_t N, int64_t K) {
  return host_matmul<float>(a, b, c, M, N, K);
}
int choreo_ref_relu_f32(const void* in, void* out, int64_t n) { return host_relu<float>(in, out, n); }
int choreo_ref_add_mismatch_f32(int64_t n_a, int64_t n_b) { return host_add_mismatch<float>(n_a, n_b); }
int choreo_ref_matmul_mismatch_f32(int64_t M, int64_t K, int64_t K2, int64_t N) {
  return host_matmul_mismatch<float>(M, K, K2, N);
}
#else
#error "define CHOREO_REF_TYPE to 1, 2 or 3"
#endif

}  // extern "C"
