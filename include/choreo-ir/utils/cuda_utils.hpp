/**
 * @file cuda_utils.hpp
 * @brief CUDA error checks and RAII stream/event handles (the reference's
 *        utils/cuda_utils.hpp:26-82, 319-400 names; no cuBLAS/cuDNN
 *        dependency, since no library GEMM sits on this path).
 */
#ifndef CHOREO_IR_UTILS_CUDA_UTILS_HPP
#define CHOREO_IR_UTILS_CUDA_UTILS_HPP

#include <cuda_runtime.h>

#include <stdexcept>
#include <string>

#define CUDA_CHECK(call)                                                                              \
  do {                                                                                                \
    cudaError_t choreo_err_ = (call);                                                                 \
    if (choreo_err_ != cudaSuccess)                                                                   \
      throw std::runtime_error(std::string("CUDA error at ") + __FILE__ + ":" + std::to_string(__LINE__) + \
                               ": " + cudaGetErrorString(choreo_err_));                               \
  } while (0)

namespace choreo_ir {
namespace utils {

class CudaStream {
 public:
  CudaStream() { CUDA_CHECK(cudaStreamCreateWithFlags(&s_, cudaStreamNonBlocking)); }
  ~CudaStream() {
    if (s_) cudaStreamDestroy(s_);
  }
  CudaStream(const CudaStream&) = delete;
  CudaStream& operator=(const CudaStream&) = delete;
  cudaStream_t get() const { return s_; }
  operator cudaStream_t() const { return s_; }
  void synchronize() const { CUDA_CHECK(cudaStreamSynchronize(s_)); }

 private:
  cudaStream_t s_ = nullptr;
};

class CudaEvent {
 public:
  CudaEvent() { CUDA_CHECK(cudaEventCreate(&e_)); }
  ~CudaEvent() {
    if (e_) cudaEventDestroy(e_);
  }
  CudaEvent(const CudaEvent&) = delete;
  CudaEvent& operator=(const CudaEvent&) = delete;
  void record(cudaStream_t s = nullptr) { CUDA_CHECK(cudaEventRecord(e_, s)); }
  void synchronize() const { CUDA_CHECK(cudaEventSynchronize(e_)); }
  /// Milliseconds from `start` to this event.
  float elapsed_since(const CudaEvent& start) const {
    float ms = 0.f;
    CUDA_CHECK(cudaEventElapsedTime(&ms, start.e_, e_));
    return ms;
  }
  cudaEvent_t get() const { return e_; }

 private:
  cudaEvent_t e_ = nullptr;
};

}  // namespace utils
}  // namespace choreo_ir

#endif  // CHOREO_IR_UTILS_CUDA_UTILS_HPP
