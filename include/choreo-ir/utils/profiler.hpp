/**
 * @file profiler.hpp
 * @brief Event timing and the FLOP formulas the reference's profiler uses
 *        (utils/profiler.hpp:42-83 GPUTimer, :306-335 TFLOP/s helpers).
 */
#ifndef CHOREO_IR_UTILS_PROFILER_HPP
#define CHOREO_IR_UTILS_PROFILER_HPP

#include <cuda_runtime.h>

#include "cuda_utils.hpp"

namespace choreo_ir {
namespace utils {

/// CUDA-event timer on one stream.
class GPUTimer {
 public:
  explicit GPUTimer(cudaStream_t s = nullptr) : stream_(s) {}
  void start() { begin_.record(stream_); }
  /// Records the end event, waits for it, returns milliseconds since start().
  float stop() {
    end_.record(stream_);
    end_.synchronize();
    return end_.elapsed_since(begin_);
  }

 private:
  cudaStream_t stream_;
  CudaEvent begin_, end_;
};

/// 2*M*N*K FLOP over `ms` milliseconds, in TFLOP/s.
inline double calculate_matmul_tflops(long long m, long long n, long long k, double ms) {
  return 2.0 * static_cast<double>(m) * n * k / (ms * 1e-3) / 1e12;
}

/// 2*N*K*P*Q*C*R*S FLOP over `ms` milliseconds, in TFLOP/s.
inline double calculate_conv_tflops(long long n, long long c, long long p, long long q, long long k, long long r,
                                    long long s, double ms) {
  return 2.0 * static_cast<double>(n) * k * p * q * c * r * s / (ms * 1e-3) / 1e12;
}

}  // namespace utils
}  // namespace choreo_ir

#endif  // CHOREO_IR_UTILS_PROFILER_HPP
