/**
 * @file device_tile.hpp
 * @brief Device-side tile movement for user kernels: the building blocks the
 *        GEMM mainloop uses, in the reference's `shared = global.tile(...)`
 *        form (reference: tensor/tensor.hpp:164-254, TensorView::
 *        copy_to_shared / copy_to_local / async_copy_to_shared and the
 *        global -> shared operator=).
 *
 * Host side:
 *   GlobalMatrix<T> g = global_matrix(view);        // a 2-D row-major view, passed by value
 *   TmaTileMap<T, R, C> tm = TmaTileMap<T, R, C>::make(view);   // TMA map for R x C tiles
 * Device side (one CTA):
 *   SharedTile<T, R, C> s(smem);                     // dense row-major R x C tile in shared memory
 *   s = g.tile(row0, col0);                          // block-cooperative copy (cp.async 16 B),
 *                                                    // zeros past the matrix edge; ends in __syncthreads
 *   s.store(g.tile(row0, col0));                     // block-cooperative store back, clipped
 *   TileBarrier bar(&mbar);  bar.init(1);            // one thread, then __syncthreads
 *   tma_load(tm, s, bar, row0, col0);                // one thread: a bulk tensor copy, zero fill at edges
 *   bar.wait(phase);                                 // every thread that reads the tile
 *
 * TMA coordinates: the innermost one (col0) times sizeof(T) must be a multiple
 * of 16 bytes and the shared tile 128-byte aligned; tma_load checks both and
 * returns false without issuing the copy when they do not hold. Waits are
 * bounded (TileBarrier::wait returns false after its time limit).
 */
#ifndef CHOREO_IR_TENSOR_DEVICE_TILE_HPP
#define CHOREO_IR_TENSOR_DEVICE_TILE_HPP

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <stdexcept>
#include <string>

#include "../../choreo_b200.h"
#include "tensor.hpp"

namespace choreo_ir {
namespace device {

template <typename T>
struct TileRef;

/// A 2-D row-major global matrix with unit inner stride, passed to kernels by value.
template <typename T>
struct GlobalMatrix {
  T* data;
  int64_t rows, cols, ld;  // ld: elements between row starts
  /// The window of a tile whose top-left element is (row0, col0).
  __host__ __device__ TileRef<T> tile(int64_t row0, int64_t col0) const { return TileRef<T>{*this, row0, col0}; }
};

template <typename T>
struct TileRef {
  GlobalMatrix<T> m;
  int64_t row0, col0;
};

/// GlobalMatrix of a 2-D TensorView (innermost stride 1).
template <typename T>
GlobalMatrix<T> global_matrix(const TensorView<T>& v) {
  if (v.ndims() != 2) throw std::invalid_argument("global_matrix: the view must be 2-D");
  if (v.stride()[1] != 1) throw std::invalid_argument("global_matrix: the innermost stride must be 1");
  return GlobalMatrix<T>{v.data(), static_cast<int64_t>(v.shape()[0]), static_cast<int64_t>(v.shape()[1]),
                         static_cast<int64_t>(v.stride()[0])};
}

/// Dense row-major R x C tile in shared memory.
template <typename T, int R, int C>
struct SharedTile {
  static_assert(R > 0 && C > 0, "tile extents must be positive");
  T* data;
  __device__ explicit SharedTile(T* p) : data(p) {}
  __device__ T& operator()(int r, int c) const { return data[r * C + c]; }
  static constexpr int kBytes = R * C * static_cast<int>(sizeof(T));

#if defined(__CUDACC__)
  /// shared = global.tile(row0, col0): every thread of the block takes part.
  /// 16-byte cp.async copies where a chunk is aligned and inside the matrix,
  /// element copies at the ragged edge, zeros past it; ends with
  /// __syncthreads(), so the tile is visible to the whole block.
  __device__ SharedTile& operator=(const TileRef<T>& src) {
    constexpr int kVec = 16 / static_cast<int>(sizeof(T));
    const GlobalMatrix<T>& g = src.m;
    const bool vec_ok = (C % kVec == 0) && (reinterpret_cast<uintptr_t>(g.data) % 16 == 0) &&
                        (g.ld % kVec == 0) && (src.col0 % kVec == 0) &&
                        (static_cast<uint32_t>(__cvta_generic_to_shared(data)) % 16 == 0);
    if (vec_ok) {
      constexpr int kChunks = R * C / kVec;
      for (int i = threadIdx.x; i < kChunks; i += blockDim.x) {
        const int r = i / (C / kVec);
        const int c = (i % (C / kVec)) * kVec;
        const int64_t gr = src.row0 + r, gc = src.col0 + c;
        T* dst = data + r * C + c;
        if (gr >= 0 && gr < g.rows && gc >= 0 && gc + kVec <= g.cols) {
          const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
          asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(g.data + gr * g.ld + gc) : "memory");
        } else {
          for (int e = 0; e < kVec; ++e) {
            const bool in = gr >= 0 && gr < g.rows && gc + e >= 0 && gc + e < g.cols;
            dst[e] = in ? g.data[gr * g.ld + gc + e] : T(0.0f);
          }
        }
      }
      asm volatile("cp.async.wait_all;" ::: "memory");
    } else {
      for (int i = threadIdx.x; i < R * C; i += blockDim.x) {
        const int r = i / C, c = i % C;
        const int64_t gr = src.row0 + r, gc = src.col0 + c;
        const bool in = gr >= 0 && gr < g.rows && gc >= 0 && gc < g.cols;
        data[i] = in ? g.data[gr * g.ld + gc] : T(0.0f);
      }
    }
    __syncthreads();
    return *this;
  }

  /// global.tile(row0, col0) = shared: every thread of the block takes part;
  /// elements past the matrix edge are not written. Starts with
  /// __syncthreads() so writes to the tile made by other threads are seen.
  __device__ void store(const TileRef<T>& dst) const {
    __syncthreads();
    const GlobalMatrix<T>& g = dst.m;
    for (int i = threadIdx.x; i < R * C; i += blockDim.x) {
      const int r = i / C, c = i % C;
      const int64_t gr = dst.row0 + r, gc = dst.col0 + c;
      if (gr >= 0 && gr < g.rows && gc >= 0 && gc < g.cols) g.data[gr * g.ld + gc] = data[i];
    }
  }

  /// copy_to_local: this thread's `N` consecutive elements starting at
  /// element `first` of the tile (row-major), into registers.
  template <int N>
  __device__ void copy_to_local(T (&local)[N], int first) const {
#pragma unroll
    for (int i = 0; i < N; ++i) local[i] = (first + i < R * C) ? data[first + i] : T(0.0f);
  }
#endif
};

/// A TMA tensor map for R x C tiles of a 2-D matrix (no swizzle: the tile
/// lands dense and row-major, as SharedTile<T, R, C> expects). Build on the
/// host, pass to the kernel as a `const __grid_constant__` parameter.
template <typename T, int R, int C>
struct alignas(64) TmaTileMap {
  static_assert(R >= 1 && R <= 256 && C >= 1 && C <= 256, "TMA box extents are 1..256");
  static_assert((C * sizeof(T)) % 16 == 0, "a TMA tile row must be a multiple of 16 bytes");
  CUtensorMap map;

  static TmaTileMap make(const GlobalMatrix<T>& g) {
    TmaTileMap t;
    const int64_t dims[2] = {g.cols, g.rows};
    const int64_t strides[1] = {g.ld * static_cast<int64_t>(sizeof(T))};
    const uint32_t box[2] = {static_cast<uint32_t>(C), static_cast<uint32_t>(R)};
    const int rc = choreo_tensor_map_encode(&t.map, static_cast<int32_t>(get_dtype<T>()), 2, g.data, dims,
                                            strides, box, 0);
    if (rc != CHOREO_OK) throw std::runtime_error(std::string("TmaTileMap: ") + choreo_last_error());
    return t;
  }
  static TmaTileMap make(const TensorView<T>& v) { return make(global_matrix(v)); }
};

#if defined(__CUDACC__)
/// An mbarrier in shared memory that counts the bytes of TMA tile copies.
struct TileBarrier {
  uint64_t* bar;
  __device__ explicit TileBarrier(uint64_t* b) : bar(b) {}
  __device__ uint32_t addr() const { return static_cast<uint32_t>(__cvta_generic_to_shared(bar)); }
  /// One thread, before any use; then __syncthreads().
  __device__ void init(uint32_t arrivals = 1) const {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(addr()), "r"(arrivals) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __device__ void arrive_expect_tx(uint32_t bytes) const {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(addr()), "r"(bytes) : "memory");
  }
  __device__ bool try_wait(uint32_t parity) const {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(addr()), "r"(parity)
        : "memory");
    return ok != 0;
  }
  /// Waits for the phase with this parity to complete; false after
  /// `timeout_ns` (default 1 s) without it.
  __device__ bool wait(uint32_t parity, uint64_t timeout_ns = 1000000000ull) const {
    if (try_wait(parity)) return true;
    uint64_t t0;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    for (;;) {
      if (try_wait(parity)) return true;
      uint64_t t;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
      if (t - t0 > timeout_ns) return false;
    }
  }
};

/// One thread: copies the R x C tile at (row0, col0) of the map's matrix into
/// `dst` with one bulk tensor copy (zeros past the edges; row0 and col0 may
/// be negative) and arms `bar` with its byte count. Returns false, issuing
/// nothing, when col0 * sizeof(T) is not a multiple of 16 bytes or `dst` is
/// not 128-byte aligned.
template <typename T, int R, int C>
__device__ bool tma_load(const TmaTileMap<T, R, C>& tm, const SharedTile<T, R, C>& dst, const TileBarrier& bar,
                         int32_t row0, int32_t col0) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(dst.data));
  if (((static_cast<int64_t>(col0) * static_cast<int64_t>(sizeof(T))) & 15) != 0 || (s & 127u) != 0) return false;
  bar.arrive_expect_tx(static_cast<uint32_t>(SharedTile<T, R, C>::kBytes));
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(s),
      "l"(reinterpret_cast<uint64_t>(&tm.map)), "r"(bar.addr()), "r"(col0), "r"(row0)
      : "memory");
  return true;
}
#endif

}  // namespace device
}  // namespace choreo_ir

#endif  // CHOREO_IR_TENSOR_DEVICE_TILE_HPP
