/**
 * @file layout.hpp
 * @brief Shape + stride layouts (the reference's tensor/layout.hpp:21-336
 *        interface and behaviour), and the swizzled shared-memory tile
 *        layouts the sm_100a kernels stage operands in.
 *
 * `Layout::tile(Shape)` keeps the reference's contract (same rank required,
 * the layout itself is returned, tests/test_layout.cpp:168-177); sub-windows
 * are taken with TensorView::tile(offset, shape). Boundary handling of a
 * window that runs past the tensor is done by the kernels' TMA loads, which
 * read zeros outside the tensor.
 *
 * SmemTileLayout describes a 128-byte-swizzled operand tile exactly as the
 * TMA writes it (SWIZZLE_128B) and as the tcgen05 shared-memory matrix
 * descriptor reads it: rows of 64 16-bit elements (128 bytes), 8-row atoms
 * of 1024 bytes in which the 16-byte chunk index is XORed with the row index.
 */
#ifndef CHOREO_IR_TENSOR_LAYOUT_HPP
#define CHOREO_IR_TENSOR_LAYOUT_HPP

#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <stdexcept>
#include <vector>

#include "../core/config.hpp"
#include "../core/types.hpp"
#include "shape.hpp"
#include "stride.hpp"

namespace choreo_ir {

enum class LayoutType { ROW_MAJOR, COLUMN_MAJOR, STRIDED, BLOCKED };

class Layout {
 public:
  Layout() : layout_type_(LayoutType::ROW_MAJOR) {}
  explicit Layout(const Shape& shape)
      : shape_(shape), stride_(Stride::from_shape_row_major(shape)), layout_type_(LayoutType::ROW_MAJOR) {}
  Layout(const Shape& shape, LayoutType type) : shape_(shape), layout_type_(type) {
    stride_ = type == LayoutType::COLUMN_MAJOR ? Stride::from_shape_col_major(shape)
                                               : Stride::from_shape_row_major(shape);
  }
  Layout(const Shape& shape, const Stride& stride)
      : shape_(shape), stride_(stride), layout_type_(LayoutType::STRIDED) {
    if (shape.ndims() != stride.ndims()) throw std::invalid_argument("Shape and stride dimensions must match");
  }

  const Shape& shape() const { return shape_; }
  const Stride& stride() const { return stride_; }
  LayoutType layout_type() const { return layout_type_; }
  dim_t ndims() const { return shape_.ndims(); }
  index_t numel() const { return shape_.numel(); }
  size_t memory_size(DataType dtype) const { return static_cast<size_t>(numel()) * sizeof_dtype(dtype); }

  bool is_contiguous() const {
    return layout_type_ == LayoutType::COLUMN_MAJOR ? stride_.is_contiguous_col_major(shape_)
                                                    : stride_.is_contiguous(shape_);
  }
  bool is_coalesced() const { return stride_.is_coalesced(); }

  template <typename... Args>
  index_t offset(Args... idx) const {
    return stride_.offset(idx...);
  }
  index_t offset(const std::vector<index_t>& idx) const { return stride_.offset(idx); }

  Layout transpose() const { return Layout(shape_.transpose(), stride_.transpose()); }

  Layout reshape(const Shape& to) const {
    if (!is_contiguous()) throw std::runtime_error("Cannot reshape non-contiguous tensor");
    if (to.numel() != numel()) throw std::invalid_argument("Cannot reshape: element count mismatch");
    return Layout(to, layout_type_);
  }

  Layout slice(dim_t start, dim_t end) const { return Layout(shape_.slice(start, end), stride_.slice(start, end)); }

  Layout tile(const Shape& tile_shape) const {
    if (tile_shape.ndims() != shape_.ndims()) throw std::invalid_argument("Tile shape must have same number of dimensions");
    return *this;
  }

  /// Layout of the window [offset, offset + tile_shape) clipped to the tensor:
  /// the window's shape with this layout's strides.
  Layout window(const std::vector<index_t>& offset, const Shape& tile_shape) const {
    if (tile_shape.ndims() != shape_.ndims() || static_cast<dim_t>(offset.size()) != shape_.ndims())
      throw std::invalid_argument("Tile shape must have same number of dimensions");
    std::vector<index_t> ext(tile_shape.ndims());
    for (dim_t i = 0; i < tile_shape.ndims(); ++i) {
      if (offset[i] < 0 || offset[i] > shape_[i]) throw std::out_of_range("Tile offset out of range");
      ext[i] = std::min(tile_shape[i], shape_[i] - offset[i]);
    }
    return Layout(Shape(ext), stride_);
  }

  /// A 2-D (or batched) layout the tensor-core GEMM can consume: last two
  /// extents multiples of 8 (16-byte rows for 16-bit types) and one of the
  /// last two dimensions contiguous.
  bool is_tensor_core_compatible() const {
    if (shape_.ndims() < 2) return false;
    const MatrixStrides m = matrix_strides(shape_, stride_);
    return m.valid && shape_.second_last_dim() % 16 == 0 && shape_.last_dim() % 16 == 0;
  }

  dim3 get_optimal_block_size() const {
    if (shape_.ndims() == 0) return dim3(1, 1, 1);
    if (shape_.ndims() == 1)
      return dim3(static_cast<unsigned>(std::min<index_t>(config::DEFAULT_BLOCK_SIZE, std::max<index_t>(shape_[0], 1))), 1, 1);
    if (shape_.ndims() == 2) {
      const index_t bx = std::min<index_t>(config::WARP_SIZE, std::max<index_t>(shape_[1], 1));
      const index_t by = std::min<index_t>(config::DEFAULT_BLOCK_SIZE / bx, std::max<index_t>(shape_[0], 1));
      return dim3(static_cast<unsigned>(bx), static_cast<unsigned>(by), 1);
    }
    return dim3(config::DEFAULT_BLOCK_SIZE, 1, 1);
  }

  dim3 get_grid_size() const {
    const dim3 b = get_optimal_block_size();
    if (shape_.ndims() == 0) return dim3(1, 1, 1);
    if (shape_.ndims() == 1) return dim3(static_cast<unsigned>((shape_[0] + b.x - 1) / b.x), 1, 1);
    if (shape_.ndims() == 2)
      return dim3(static_cast<unsigned>((shape_[1] + b.x - 1) / b.x), static_cast<unsigned>((shape_[0] + b.y - 1) / b.y), 1);
    const index_t per = static_cast<index_t>(b.x) * b.y * b.z;
    return dim3(static_cast<unsigned>((numel() + per - 1) / per), 1, 1);
  }

  bool operator==(const Layout& o) const { return shape_ == o.shape_ && stride_ == o.stride_; }
  bool operator!=(const Layout& o) const { return !(*this == o); }

 private:
  Shape shape_;
  Stride stride_;
  LayoutType layout_type_;
};

inline Layout make_row_major_layout(const Shape& shape) { return Layout(shape, LayoutType::ROW_MAJOR); }
inline Layout make_col_major_layout(const Shape& shape) { return Layout(shape, LayoutType::COLUMN_MAJOR); }
inline Layout make_strided_layout(const Shape& shape, const Stride& stride) { return Layout(shape, stride); }

// ---------------------------------------------------------------------------
// Shared-memory operand tiles (sm_100a)

enum class Swizzle : uint8_t { NONE = 0, B32 = 32, B64 = 64, B128 = 128 };
enum class OperandMajor : uint8_t { K = 0, MN = 1 };

/// One operand tile in shared memory as the tcgen05 kernels hold it.
///   K-major  : `rows` = M (or N) rows of 64 K-elements each.
///   MN-major : `rows` = 64 K rows; the MN extent is split in 64-element
///              chunks stored one after another (`mn_chunks` of them).
struct SmemTileLayout {
  OperandMajor major = OperandMajor::K;
  int rows = 128;             // K-major: MN rows; MN-major: K rows (64)
  int mn_chunks = 1;          // MN-major only
  int elem_bytes = 2;
  Swizzle swizzle = Swizzle::B128;

  static constexpr int kRowBytes = 128;
  static constexpr int kAtomBytes = 1024;

  int chunk_bytes() const { return rows * kRowBytes; }
  int bytes() const { return major == OperandMajor::K ? rows * kRowBytes : mn_chunks * chunk_bytes(); }

  /// Byte offset of element (mn, k) of the tile (MN index, K index).
  uint32_t offset(int mn, int k) const {
    uint32_t linear;
    if (major == OperandMajor::K) {
      linear = static_cast<uint32_t>(mn * kRowBytes + k * elem_bytes);
    } else {
      const int chunk = mn / 64, in = mn % 64;
      linear = static_cast<uint32_t>(chunk * chunk_bytes() + k * kRowBytes + in * elem_bytes);
    }
    return swizzle_128b(linear);
  }

  /// The 128-byte swizzle: bits [4,7) (16-byte chunk within a 128-byte row)
  /// XOR bits [7,10) (row within the 1024-byte atom).
  static uint32_t swizzle_128b(uint32_t linear) { return linear ^ (((linear >> 7) & 7u) << 4); }

  /// Leading / stride byte offsets of the tcgen05 shared-memory descriptor.
  uint32_t lbo() const { return major == OperandMajor::K ? 16u : static_cast<uint32_t>(chunk_bytes()); }
  uint32_t sbo() const { return kAtomBytes; }
  /// Descriptor start-address advance per 16-element UMMA K step.
  uint32_t k_step_bytes() const { return major == OperandMajor::K ? 32u : 16u * kRowBytes; }

  /// TMA box (innermost first) that fills one tile, or one MN chunk of it.
  std::vector<uint32_t> tma_box() const {
    if (major == OperandMajor::K) return {64u, static_cast<uint32_t>(rows)};
    return {64u, static_cast<uint32_t>(rows)};
  }
};

}  // namespace choreo_ir

#endif  // CHOREO_IR_TENSOR_LAYOUT_HPP
