/**
 * @file tensor.hpp
 * @brief Owning Tensor<T> and non-owning TensorView<T> (the reference's
 *        tensor/tensor.hpp:28-736 interface and behaviour), plus the API the
 *        reference documents but never defines: host_tensor<T>/device_tensor<T>
 *        factories with random(), to_device()/to_host(), and tile(offset, shape)
 *        windows.
 *
 * Ownership as in the reference: a Tensor owns its buffer (HOST: new[],
 * DEVICE: cudaMalloc, UNIFIED: cudaMallocManaged), deep-copies on copy and
 * steals on move; views never own. Transfers (copy_from_host/copy_to_host,
 * to_device/to_host) are synchronous cudaMemcpy, as in the reference. A
 * non-zero device fill() runs a device kernel (choreo_fill) instead of
 * staging a host vector (reference tensor.hpp:545-559).
 */
#ifndef CHOREO_IR_TENSOR_TENSOR_HPP
#define CHOREO_IR_TENSOR_TENSOR_HPP

#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <random>
#include <stdexcept>
#include <string>
#include <type_traits>
#include <vector>

#include "../../choreo_b200.h"
#include "../core/config.hpp"
#include "../core/types.hpp"
#include "layout.hpp"

namespace choreo_ir {

enum class MemorySpace { GLOBAL, SHARED, LOCAL, TEXTURE, CONSTANT };

namespace detail {
inline void cuda_check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}
inline void status_check(int rc) {
  if (rc != CHOREO_OK) throw std::runtime_error(choreo_last_error());
}
/// C ABI dtype code of T, or -1 if the library has no kernel for T.
template <typename T>
constexpr int abi_dtype() {
  return std::is_same_v<T, float16_t> ? CHOREO_DTYPE_F16
       : std::is_same_v<T, bfloat16_t> ? CHOREO_DTYPE_BF16
       : std::is_same_v<T, float> ? CHOREO_DTYPE_F32 : -1;
}
}  // namespace detail

template <typename T>
class TensorView {
 public:
  TensorView(T* data, const Layout& layout, MemorySpace space = MemorySpace::GLOBAL)
      : data_(data), layout_(layout), space_(space) {}

  T* data() const { return data_; }
  const Layout& layout() const { return layout_; }
  const Shape& shape() const { return layout_.shape(); }
  const Stride& stride() const { return layout_.stride(); }
  MemorySpace memory_space() const { return space_; }
  dim_t ndims() const { return layout_.ndims(); }
  index_t numel() const { return layout_.numel(); }
  DataType dtype() const { return get_dtype<T>(); }
  bool is_contiguous() const { return layout_.is_contiguous(); }
  bool is_coalesced() const { return layout_.is_coalesced(); }

  template <typename... Args>
  T& operator()(Args... idx) const {
    return data_[layout_.offset(idx...)];
  }

  TensorView slice(dim_t start, dim_t end) const { return TensorView(data_, layout_.slice(start, end), space_); }
  TensorView transpose() const { return TensorView(data_, layout_.transpose(), space_); }
  /// Reference contract: same rank required, the view itself is returned.
  TensorView tile(const Shape& tile_shape) const { return TensorView(data_, layout_.tile(tile_shape), space_); }
  /// The window [offset, offset + tile_shape) clipped at the tensor's edge.
  /// Kernels reading a window through TMA see zeros past the edge.
  TensorView tile(const std::vector<index_t>& offset, const Shape& tile_shape) const {
    return TensorView(data_ + layout_.offset(offset), layout_.window(offset, tile_shape), space_);
  }
  TensorView reshape(const Shape& s) const { return TensorView(data_, layout_.reshape(s), space_); }

 private:
  T* data_;
  Layout layout_;
  MemorySpace space_;
};

template <typename T>
class Tensor {
 public:
  Tensor() : data_(nullptr), memory_type_(MemoryType::DEVICE) {}
  explicit Tensor(const Shape& shape, MemoryType mt = MemoryType::DEVICE) : layout_(shape), memory_type_(mt) {
    allocate();
  }
  explicit Tensor(const Layout& layout, MemoryType mt = MemoryType::DEVICE) : layout_(layout), memory_type_(mt) {
    allocate();
  }
  Tensor(const Tensor& o) : layout_(o.layout_), memory_type_(o.memory_type_) {
    allocate();
    copy_from(o);
  }
  Tensor(Tensor&& o) noexcept : data_(o.data_), layout_(std::move(o.layout_)), memory_type_(o.memory_type_) {
    o.data_ = nullptr;
  }
  ~Tensor() { deallocate(); }

  Tensor& operator=(const Tensor& o) {
    if (this != &o) {
      deallocate();
      layout_ = o.layout_;
      memory_type_ = o.memory_type_;
      allocate();
      copy_from(o);
    }
    return *this;
  }
  Tensor& operator=(Tensor&& o) noexcept {
    if (this != &o) {
      deallocate();
      data_ = o.data_;
      layout_ = std::move(o.layout_);
      memory_type_ = o.memory_type_;
      o.data_ = nullptr;
    }
    return *this;
  }

  T* data() const { return data_; }
  const Layout& layout() const { return layout_; }
  const Shape& shape() const { return layout_.shape(); }
  const Stride& stride() const { return layout_.stride(); }
  dim_t ndims() const { return layout_.ndims(); }
  index_t numel() const { return layout_.numel(); }
  DataType dtype() const { return get_dtype<T>(); }
  MemoryType memory_type() const { return memory_type_; }
  bool empty() const { return data_ == nullptr || layout_.numel() == 0; }
  bool is_contiguous() const { return layout_.is_contiguous(); }
  bool is_coalesced() const { return layout_.is_coalesced(); }

  /// Element access (host or unified memory).
  template <typename... Args>
  T& operator()(Args... idx) const {
    return data_[layout_.offset(idx...)];
  }

  TensorView<T> view() const { return TensorView<T>(data_, layout_, MemorySpace::GLOBAL); }
  TensorView<T> slice(dim_t start, dim_t end) const { return view().slice(start, end); }
  TensorView<T> transpose() const { return view().transpose(); }
  TensorView<T> tile(const Shape& s) const { return view().tile(s); }
  TensorView<T> tile(const std::vector<index_t>& offset, const Shape& s) const { return view().tile(offset, s); }
  TensorView<T> reshape(const Shape& s) const { return view().reshape(s); }

  void resize(const Shape& s) {
    if (s.numel() != layout_.numel()) {
      deallocate();
      layout_ = Layout(s);
      allocate();
    } else {
      layout_ = Layout(s);
    }
  }

  void fill(T value) {
    if (data_ == nullptr || layout_.numel() == 0) return;
    if (memory_type_ == MemoryType::HOST) {
      std::fill_n(data_, layout_.numel(), value);
      return;
    }
    constexpr int dt = detail::abi_dtype<T>();
    if constexpr (dt >= 0) {
      detail::status_check(choreo_fill(dt, data_, static_cast<double>(to_float(value)), layout_.numel(), nullptr));
      detail::cuda_check(cudaStreamSynchronize(nullptr), "Tensor::fill");
    } else {
      std::vector<T> h(static_cast<size_t>(layout_.numel()), value);
      detail::cuda_check(cudaMemcpy(data_, h.data(), bytes(), cudaMemcpyHostToDevice), "Tensor::fill");
    }
  }

  void copy_from_host(const T* host) {
    if (data_ == nullptr || host == nullptr || layout_.numel() == 0) return;
    if (memory_type_ == MemoryType::HOST)
      std::memcpy(data_, host, bytes());
    else
      detail::cuda_check(cudaMemcpy(data_, host, bytes(), cudaMemcpyHostToDevice), "copy_from_host");
  }

  void copy_to_host(T* host) const {
    if (data_ == nullptr || host == nullptr || layout_.numel() == 0) return;
    if (memory_type_ == MemoryType::HOST)
      std::memcpy(host, data_, bytes());
    else
      detail::cuda_check(cudaMemcpy(host, data_, bytes(), cudaMemcpyDeviceToHost), "copy_to_host");
  }

  /// A DEVICE copy of this tensor (a copy of a device tensor too).
  Tensor to_device() const { return copy_as(MemoryType::DEVICE); }
  /// A HOST copy of this tensor.
  Tensor to_host() const { return copy_as(MemoryType::HOST); }

  static Tensor host(const Shape& s) { return Tensor(s, MemoryType::HOST); }
  static Tensor device(const Shape& s) { return Tensor(s, MemoryType::DEVICE); }
  static Tensor zeros(const Shape& s, MemoryType mt = MemoryType::DEVICE) {
    Tensor t(s, mt);
    if (mt == MemoryType::HOST)
      t.fill(from_float<T>(0.0f));
    else if (t.data_)
      detail::cuda_check(cudaMemset(t.data_, 0, t.bytes()), "Tensor::zeros");
    return t;
  }
  static Tensor ones(const Shape& s, MemoryType mt = MemoryType::DEVICE) {
    Tensor t(s, mt);
    t.fill(from_float<T>(1.0f));
    return t;
  }
  /// Elements drawn from std::mt19937_64(seed) with a uniform [lo, hi)
  /// distribution in float, then rounded to T.
  static Tensor random(const Shape& s, MemoryType mt = MemoryType::HOST, float lo = -1.0f, float hi = 1.0f,
                       uint64_t seed = 42) {
    std::vector<T> h(static_cast<size_t>(s.numel()));
    std::mt19937_64 gen(seed);
    std::uniform_real_distribution<float> dist(lo, hi);
    for (auto& v : h) v = from_float<T>(dist(gen));
    Tensor t(s, mt);
    t.copy_from_host(h.data());
    return t;
  }

  size_t bytes() const { return static_cast<size_t>(layout_.numel()) * sizeof(T); }

 private:
  Tensor copy_as(MemoryType mt) const {
    Tensor t(layout_, mt);
    t.copy_from(*this);
    return t;
  }

  void allocate() {
    data_ = nullptr;
    if (layout_.numel() == 0) return;
    if (memory_type_ == MemoryType::HOST) {
      data_ = new T[static_cast<size_t>(layout_.numel())];
      return;
    }
    cudaError_t e = memory_type_ == MemoryType::DEVICE ? cudaMalloc(reinterpret_cast<void**>(&data_), bytes())
                                                        : cudaMallocManaged(reinterpret_cast<void**>(&data_), bytes());
    if (e != cudaSuccess) {
      data_ = nullptr;
      cudaGetLastError();
      std::fprintf(stderr, "[Tensor] allocate: %s failed for %zu bytes: %s\n",
                   memory_type_ == MemoryType::DEVICE ? "cudaMalloc" : "cudaMallocManaged", bytes(),
                   cudaGetErrorString(e));
      throw std::runtime_error(memory_type_ == MemoryType::DEVICE ? "Tensor::allocate: cudaMalloc failed"
                                                                  : "Tensor::allocate: cudaMallocManaged failed");
    }
  }

  void deallocate() {
    if (data_ == nullptr) return;
    if (memory_type_ == MemoryType::HOST)
      delete[] data_;
    else
      cudaFree(data_);
    data_ = nullptr;
  }

  void copy_from(const Tensor& o) {
    if (data_ == nullptr || o.data_ == nullptr || layout_.numel() != o.layout_.numel()) return;
    if (memory_type_ == MemoryType::HOST && o.memory_type_ == MemoryType::HOST) {
      std::memcpy(data_, o.data_, bytes());
      return;
    }
    cudaMemcpyKind kind = cudaMemcpyDefault;
    if (memory_type_ == MemoryType::HOST && o.memory_type_ == MemoryType::DEVICE) kind = cudaMemcpyDeviceToHost;
    else if (memory_type_ == MemoryType::DEVICE && o.memory_type_ == MemoryType::HOST) kind = cudaMemcpyHostToDevice;
    else if (memory_type_ == MemoryType::DEVICE && o.memory_type_ == MemoryType::DEVICE) kind = cudaMemcpyDeviceToDevice;
    detail::cuda_check(cudaMemcpy(data_, o.data_, bytes(), kind), "Tensor copy");
  }

  T* data_ = nullptr;
  Layout layout_;
  MemoryType memory_type_;
};

/// Factories the reference's README and examples use (README.md:83-94).
template <typename T>
struct host_tensor {
  static Tensor<T> random(const Shape& s, float lo = -1.0f, float hi = 1.0f, uint64_t seed = 42) {
    return Tensor<T>::random(s, MemoryType::HOST, lo, hi, seed);
  }
  static Tensor<T> zeros(const Shape& s) { return Tensor<T>::zeros(s, MemoryType::HOST); }
  static Tensor<T> ones(const Shape& s) { return Tensor<T>::ones(s, MemoryType::HOST); }
  static Tensor<T> empty(const Shape& s) { return Tensor<T>(s, MemoryType::HOST); }
};

template <typename T>
struct device_tensor {
  static Tensor<T> random(const Shape& s, float lo = -1.0f, float hi = 1.0f, uint64_t seed = 42) {
    return Tensor<T>::random(s, MemoryType::DEVICE, lo, hi, seed);
  }
  static Tensor<T> zeros(const Shape& s) { return Tensor<T>::zeros(s, MemoryType::DEVICE); }
  static Tensor<T> ones(const Shape& s) { return Tensor<T>::ones(s, MemoryType::DEVICE); }
  static Tensor<T> empty(const Shape& s) { return Tensor<T>(s, MemoryType::DEVICE); }
};

using TensorF32 = Tensor<float32_t>;
using TensorF16 = Tensor<float16_t>;
using TensorBF16 = Tensor<bfloat16_t>;
using TensorI32 = Tensor<int32_t>;
using TensorI8 = Tensor<int8_t>;
using TensorViewF32 = TensorView<float32_t>;
using TensorViewF16 = TensorView<float16_t>;
using TensorViewBF16 = TensorView<bfloat16_t>;
using TensorViewI32 = TensorView<int32_t>;
using TensorViewI8 = TensorView<int8_t>;

}  // namespace choreo_ir

#endif  // CHOREO_IR_TENSOR_TENSOR_HPP
