/*
 * oracle/ref_shim.h — forced-include prelude that lets the reference's umbrella
 * header (include/choreo-ir/choreo-ir.hpp) compile with nvcc 12.9 so its host
 * operator*, relu and operator+ can be called as the oracle's pin.
 *
 * TEST INFRASTRUCTURE ONLY (used by oracle/build.py for oracle/_ref).
 *
 * What it works around (none of it touches the host code being pinned):
 *  - tensor/shape.hpp uses std::invalid_argument without <stdexcept>;
 *    utils/profiler.hpp-style headers miss <iomanip>/<fstream>.
 *  - compute/wmma.hpp and compute/mma.hpp do not compile (tag types used as
 *    values at wmma.hpp:32-41, a <<<>>> launch of a __device__ function at
 *    wmma.hpp:149, a non-existent nvcuda::mma namespace at mma.hpp:105-112).
 *    Their include guards are pre-defined so they are skipped, and the four
 *    names compute_impl.hpp uses from them are declared here; the device
 *    backends are never reached from host tensors.
 *  - choreo-ir.hpp:240 calls detail::get_cublas_handle(), defined nowhere.
 */
#pragma once
#include <stdexcept>
#include <vector>
#include <iomanip>
#include <fstream>
#include <cublas_v2.h>

#define CHOREO_IR_COMPUTE_WMMA_HPP
#define CHOREO_IR_COMPUTE_MMA_HPP

namespace choreo_ir {
template <typename T> class Tensor;
namespace compute {
struct WMMAConfig {};
struct MMAConfig {};
template <typename T>
void wmma_gemm(const Tensor<T>&, const Tensor<T>&, Tensor<T>&, T, T, const WMMAConfig&) {
  throw std::runtime_error("WMMA backend does not compile in the reference");
}
template <typename T>
void mma_gemm(const Tensor<T>&, const Tensor<T>&, Tensor<T>&, T, T, const MMAConfig&) {
  throw std::runtime_error("MMA backend is declared but never defined in the reference");
}
}  // namespace compute
namespace detail {
inline cublasHandle_t& get_cublas_handle() {
  static cublasHandle_t h = nullptr;
  return h;
}
}  // namespace detail
}  // namespace choreo_ir
