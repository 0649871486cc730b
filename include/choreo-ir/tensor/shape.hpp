/**
 * @file shape.hpp
 * @brief Tensor shape (interface and behaviour of the reference's
 *        tensor/shape.hpp:24-249: up to MAX_TENSOR_DIMS extents, scalar
 *        numel 1, out_of_range on bad indices, invalid_argument "Too many
 *        dimensions", transpose swapping the last two extents).
 */
#ifndef CHOREO_IR_TENSOR_SHAPE_HPP
#define CHOREO_IR_TENSOR_SHAPE_HPP

#include <array>
#include <initializer_list>
#include <stdexcept>
#include <vector>

#include "../core/config.hpp"
#include "../core/types.hpp"

namespace choreo_ir {

class Shape {
 public:
  Shape() : ndims_(0), dims_{} {}

  Shape(std::initializer_list<index_t> dims) : Shape(dims.begin(), static_cast<size_t>(dims.size())) {}

  explicit Shape(const std::vector<index_t>& dims) : Shape(dims.data(), dims.size()) {}

  Shape(const index_t* dims, dim_t ndims) : Shape(dims, static_cast<size_t>(ndims < 0 ? 0 : ndims)) {}

  dim_t ndims() const { return ndims_; }

  index_t operator[](dim_t i) const { return dims_[check(i)]; }
  index_t& operator[](dim_t i) { return dims_[check(i)]; }
  index_t at(dim_t i) const { return dims_[check(i)]; }

  index_t numel() const {
    index_t n = 1;
    for (dim_t i = 0; i < ndims_; ++i) n *= dims_[i];
    return n;
  }

  bool empty() const {
    for (dim_t i = 0; i < ndims_; ++i)
      if (dims_[i] == 0) return true;
    return false;
  }

  bool is_scalar() const { return ndims_ == 0; }
  bool is_vector() const { return ndims_ == 1; }
  bool is_matrix() const { return ndims_ == 2; }

  index_t last_dim() const { return ndims_ >= 1 ? dims_[ndims_ - 1] : 1; }
  index_t second_last_dim() const { return ndims_ >= 2 ? dims_[ndims_ - 2] : 1; }

  Shape reshape(const Shape& to) const {
    if (to.numel() != numel()) throw std::invalid_argument("Cannot reshape: element count mismatch");
    return to;
  }

  Shape transpose() const {
    Shape t = *this;
    if (ndims_ >= 2) std::swap(t.dims_[ndims_ - 1], t.dims_[ndims_ - 2]);
    return t;
  }

  /// Extents [start, end).
  Shape slice(dim_t start, dim_t end) const {
    if (start < 0 || start >= ndims_ || end > ndims_ || end <= start)
      throw std::out_of_range("Invalid slice range");
    return Shape(dims_.data() + start, static_cast<size_t>(end - start));
  }

  bool operator==(const Shape& o) const {
    if (ndims_ != o.ndims_) return false;
    for (dim_t i = 0; i < ndims_; ++i)
      if (dims_[i] != o.dims_[i]) return false;
    return true;
  }
  bool operator!=(const Shape& o) const { return !(*this == o); }

  const index_t* begin() const { return dims_.data(); }
  const index_t* end() const { return dims_.data() + ndims_; }
  std::vector<index_t> to_vector() const { return std::vector<index_t>(begin(), end()); }

 private:
  Shape(const index_t* dims, size_t n) : ndims_(0), dims_{} {
    if (n > static_cast<size_t>(config::MAX_TENSOR_DIMS)) throw std::invalid_argument("Too many dimensions");
    ndims_ = static_cast<dim_t>(n);
    for (size_t i = 0; i < n; ++i) dims_[i] = dims[i];
  }
  dim_t check(dim_t i) const {
    if (i < 0 || i >= ndims_) throw std::out_of_range("Dimension index out of range");
    return i;
  }

  dim_t ndims_;
  std::array<index_t, config::MAX_TENSOR_DIMS> dims_;
};

template <typename... Args>
Shape make_shape(Args... dims) {
  return Shape({static_cast<index_t>(dims)...});
}

}  // namespace choreo_ir

#endif  // CHOREO_IR_TENSOR_SHAPE_HPP
