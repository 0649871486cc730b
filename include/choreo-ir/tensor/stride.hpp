/**
 * @file stride.hpp
 * @brief Element strides of a tensor (the reference's tensor/stride.hpp:23-327
 *        interface and behaviour), plus the TMA view of a strided matrix:
 *        which dimension is contiguous, its leading dimension in elements and
 *        in bytes, and whether a tensor-memory-accelerator descriptor can
 *        address it directly (16-byte aligned base, leading stride and batch
 *        stride).
 */
#ifndef CHOREO_IR_TENSOR_STRIDE_HPP
#define CHOREO_IR_TENSOR_STRIDE_HPP

#include <array>
#include <cstdint>
#include <initializer_list>
#include <stdexcept>
#include <vector>

#include "../core/config.hpp"
#include "../core/types.hpp"
#include "shape.hpp"

namespace choreo_ir {

class Stride {
 public:
  Stride() : ndims_(0), s_{} {}
  Stride(std::initializer_list<index_t> s) : Stride(s.begin(), static_cast<size_t>(s.size())) {}
  explicit Stride(const std::vector<index_t>& s) : Stride(s.data(), s.size()) {}
  Stride(const index_t* s, dim_t ndims) : Stride(s, static_cast<size_t>(ndims < 0 ? 0 : ndims)) {}

  static Stride from_shape_row_major(const Shape& shape) {
    Stride st;
    st.ndims_ = shape.ndims();
    index_t acc = 1;
    for (dim_t i = st.ndims_ - 1; i >= 0; --i) {
      st.s_[i] = acc;
      acc *= shape[i];
    }
    return st;
  }

  static Stride from_shape_col_major(const Shape& shape) {
    Stride st;
    st.ndims_ = shape.ndims();
    index_t acc = 1;
    for (dim_t i = 0; i < st.ndims_; ++i) {
      st.s_[i] = acc;
      acc *= shape[i];
    }
    return st;
  }

  dim_t ndims() const { return ndims_; }
  index_t operator[](dim_t i) const { return s_[check(i)]; }
  index_t& operator[](dim_t i) { return s_[check(i)]; }
  index_t at(dim_t i) const { return s_[check(i)]; }

  template <typename... Args>
  index_t offset(Args... idx) const {
    const index_t v[] = {static_cast<index_t>(idx)...};
    if (static_cast<dim_t>(sizeof...(Args)) != ndims_)
      throw std::invalid_argument("Number of indices must match number of dimensions");
    index_t off = 0;
    for (dim_t i = 0; i < ndims_; ++i) off += v[i] * s_[i];
    return off;
  }

  index_t offset(const std::vector<index_t>& idx) const {
    if (static_cast<dim_t>(idx.size()) != ndims_)
      throw std::invalid_argument("Number of indices must match number of dimensions");
    index_t off = 0;
    for (dim_t i = 0; i < ndims_; ++i) off += idx[i] * s_[i];
    return off;
  }

  bool is_contiguous(const Shape& shape) const { return *this == from_shape_row_major(shape) && ndims_ == shape.ndims(); }
  bool is_contiguous_col_major(const Shape& shape) const {
    return ndims_ == shape.ndims() && *this == from_shape_col_major(shape);
  }
  bool is_coalesced() const { return ndims_ > 0 && s_[ndims_ - 1] == 1; }

  Stride transpose() const {
    Stride t = *this;
    if (ndims_ >= 2) std::swap(t.s_[ndims_ - 1], t.s_[ndims_ - 2]);
    return t;
  }

  Stride slice(dim_t start, dim_t end) const {
    if (start < 0 || start >= ndims_ || end > ndims_ || end <= start) throw std::out_of_range("Invalid slice range");
    return Stride(s_.data() + start, static_cast<size_t>(end - start));
  }

  bool operator==(const Stride& o) const {
    if (ndims_ != o.ndims_) return false;
    for (dim_t i = 0; i < ndims_; ++i)
      if (s_[i] != o.s_[i]) return false;
    return true;
  }
  bool operator!=(const Stride& o) const { return !(*this == o); }

  const index_t* begin() const { return s_.data(); }
  const index_t* end() const { return s_.data() + ndims_; }
  std::vector<index_t> to_vector() const { return std::vector<index_t>(begin(), end()); }

 private:
  Stride(const index_t* s, size_t n) : ndims_(0), s_{} {
    if (n > static_cast<size_t>(config::MAX_TENSOR_DIMS)) throw std::invalid_argument("Too many dimensions");
    ndims_ = static_cast<dim_t>(n);
    for (size_t i = 0; i < n; ++i) s_[i] = s[i];
  }
  dim_t check(dim_t i) const {
    if (i < 0 || i >= ndims_) throw std::out_of_range("Dimension index out of range");
    return i;
  }
  dim_t ndims_;
  std::array<index_t, config::MAX_TENSOR_DIMS> s_;
};

template <typename... Args>
Stride make_stride(Args... s) {
  return Stride({static_cast<index_t>(s)...});
}

/// How the last two dimensions of a strided tensor map onto a GEMM operand:
/// one of them must be contiguous (stride 1); the other stride is the leading
/// dimension. `transposed` means the second-to-last dimension is the
/// contiguous one (the matrix is stored column-major / "T").
struct MatrixStrides {
  bool valid = false;
  bool transposed = false;
  index_t ld = 0;          // leading dimension, elements
  index_t batch_stride = 0;
};

inline MatrixStrides matrix_strides(const Shape& shape, const Stride& stride) {
  MatrixStrides m;
  const dim_t n = shape.ndims();
  if (n < 2 || stride.ndims() != n) return m;
  const index_t rows = shape[n - 2], cols = shape[n - 1];
  const index_t s_row = stride[n - 2], s_col = stride[n - 1];
  if (s_col == 1 && (s_row >= cols || rows == 1)) {
    m.valid = true;
    m.ld = rows == 1 ? cols : s_row;
  } else if (s_row == 1 && (s_col >= rows || cols == 1)) {
    m.valid = true;
    m.transposed = true;
    m.ld = cols == 1 ? rows : s_col;
  }
  m.batch_stride = n >= 3 ? stride[n - 3] : 0;
  return m;
}

/// True when a TMA descriptor can address the operand without a repack:
/// 16-byte aligned base, leading stride and (for batches) batch stride.
inline bool tma_addressable(const void* base, index_t ld, index_t batch_stride, index_t batch,
                            size_t elem_bytes) {
  const auto a = static_cast<index_t>(config::sm100::TMA_ALIGNMENT);
  if (reinterpret_cast<std::uintptr_t>(base) % static_cast<std::uintptr_t>(a) != 0) return false;
  if ((ld * static_cast<index_t>(elem_bytes)) % a != 0) return false;
  if (batch > 1 && (batch_stride <= 0 || (batch_stride * static_cast<index_t>(elem_bytes)) % a != 0)) return false;
  return true;
}

}  // namespace choreo_ir

#endif  // CHOREO_IR_TENSOR_STRIDE_HPP
