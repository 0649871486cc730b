/**
 * @file config.hpp
 * @brief Compile-time constants of the Choreo-IR API. The reference's names
 *        (core/config.hpp:15-76) are kept; the B200 tile geometry the
 *        tcgen05 kernels use is added under `config::sm100`.
 */
#ifndef CHOREO_IR_CORE_CONFIG_HPP
#define CHOREO_IR_CORE_CONFIG_HPP

#include "types.hpp"

namespace choreo_ir {
namespace config {

constexpr int VERSION_MAJOR = 1;
constexpr int VERSION_MINOR = 0;
constexpr int VERSION_PATCH = 0;

constexpr dim_t MAX_TENSOR_DIMS = 8;
constexpr size_t DEFAULT_ALIGNMENT = 256;

constexpr int DEFAULT_BLOCK_SIZE = 256;
constexpr int MAX_BLOCK_SIZE = 1024;
constexpr int WARP_SIZE = 32;

constexpr size_t MAX_SHARED_MEMORY_PER_BLOCK = 227 * 1024;  // opt-in limit on sm_100
constexpr size_t SHARED_MEMORY_BANK_SIZE = 32;

// Fragment shape of the reference's WMMA path; kept for source compatibility.
constexpr int WMMA_M = 16;
constexpr int WMMA_N = 16;
constexpr int WMMA_K = 16;

constexpr float PERFORMANCE_TOLERANCE = 0.05f;

#ifdef CHOREO_IR_DEBUG
constexpr bool DEBUG_MODE = true;
#else
constexpr bool DEBUG_MODE = false;
#endif
#ifdef CHOREO_IR_PROFILE
constexpr bool PROFILE_MODE = true;
#else
constexpr bool PROFILE_MODE = false;
#endif

constexpr DataType DEFAULT_DTYPE = DataType::FLOAT16;

enum class LayoutPreference { ROW_MAJOR, COLUMN_MAJOR, AUTO };
constexpr LayoutPreference DEFAULT_LAYOUT = LayoutPreference::AUTO;

constexpr ComputeCapability MIN_COMPUTE_CAPABILITY = ComputeCapability::SM_100;

constexpr bool ENABLE_CUDA_ERROR_CHECKING = true;
constexpr bool ENABLE_ASSERTIONS = DEBUG_MODE;
constexpr bool ENABLE_FAST_MATH = false;
constexpr bool ENABLE_TENSOR_CORE = true;
constexpr bool ENABLE_ASYNC_EXECUTION = true;

/// Geometry of the sm_100a tcgen05 kernels (choreo-ir_b200/csrc/tc_kernel.cuh).
namespace sm100 {
constexpr int TILE_M = 128;            // UMMA M per CTA (TMEM lanes)
constexpr int TILE_K = 64;             // K per pipeline stage: one 128-byte swizzle row of f16/bf16
constexpr int UMMA_K = 16;             // K per tcgen05.mma kind::f16
constexpr int TILE_N_CHOICES[3] = {256, 128, 64};
constexpr int THREADS = 320;           // producer warp, MMA warp, 8 epilogue warps
constexpr int TMEM_COLUMNS = 512;      // per SM
constexpr int SWIZZLE_BYTES = 128;
constexpr int SWIZZLE_ATOM_BYTES = 1024;  // 8 rows x 128 bytes
constexpr int TMA_ALIGNMENT = 16;      // base, strides and innermost coordinate, in bytes
}  // namespace sm100

}  // namespace config
}  // namespace choreo_ir

#endif  // CHOREO_IR_CORE_CONFIG_HPP
