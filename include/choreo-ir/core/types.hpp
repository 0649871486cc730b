/**
 * @file types.hpp
 * @brief Element, memory and architecture types of the Choreo-IR API
 *        (same names and values as the reference's core/types.hpp:20-149,
 *        with SM_100 added).
 */
#ifndef CHOREO_IR_CORE_TYPES_HPP
#define CHOREO_IR_CORE_TYPES_HPP

#include <cstddef>
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace choreo_ir {

using int8_t = std::int8_t;
using int16_t = std::int16_t;
using int32_t = std::int32_t;
using int64_t = std::int64_t;
using uint8_t = std::uint8_t;
using uint16_t = std::uint16_t;
using uint32_t = std::uint32_t;
using uint64_t = std::uint64_t;

using float32_t = float;
using float64_t = double;
using float16_t = __half;
using bfloat16_t = __nv_bfloat16;
using half = __half;

using index_t = int64_t;
using dim_t = int32_t;
using size_t = std::size_t;

/// Element types; the numeric values are also the C ABI's dtype codes.
enum class DataType : uint8_t {
  INT8 = 0,
  INT16 = 1,
  INT32 = 2,
  INT64 = 3,
  UINT8 = 4,
  UINT16 = 5,
  UINT32 = 6,
  UINT64 = 7,
  FLOAT16 = 8,
  FLOAT32 = 9,
  FLOAT64 = 10,
  BFLOAT16 = 11
};

constexpr size_t sizeof_dtype(DataType dtype) {
  switch (dtype) {
    case DataType::INT8: case DataType::UINT8: return 1;
    case DataType::INT16: case DataType::UINT16: case DataType::FLOAT16: case DataType::BFLOAT16: return 2;
    case DataType::INT32: case DataType::UINT32: case DataType::FLOAT32: return 4;
    case DataType::INT64: case DataType::UINT64: case DataType::FLOAT64: return 8;
  }
  return 0;
}

template <typename T> struct type_to_dtype;
template <> struct type_to_dtype<int8_t> { static constexpr DataType value = DataType::INT8; };
template <> struct type_to_dtype<int16_t> { static constexpr DataType value = DataType::INT16; };
template <> struct type_to_dtype<int32_t> { static constexpr DataType value = DataType::INT32; };
template <> struct type_to_dtype<int64_t> { static constexpr DataType value = DataType::INT64; };
template <> struct type_to_dtype<uint8_t> { static constexpr DataType value = DataType::UINT8; };
template <> struct type_to_dtype<uint16_t> { static constexpr DataType value = DataType::UINT16; };
template <> struct type_to_dtype<uint32_t> { static constexpr DataType value = DataType::UINT32; };
template <> struct type_to_dtype<uint64_t> { static constexpr DataType value = DataType::UINT64; };
template <> struct type_to_dtype<float16_t> { static constexpr DataType value = DataType::FLOAT16; };
template <> struct type_to_dtype<float32_t> { static constexpr DataType value = DataType::FLOAT32; };
template <> struct type_to_dtype<float64_t> { static constexpr DataType value = DataType::FLOAT64; };
template <> struct type_to_dtype<bfloat16_t> { static constexpr DataType value = DataType::BFLOAT16; };

template <typename T>
constexpr DataType get_dtype() {
  return type_to_dtype<T>::value;
}

enum class MemoryType : uint8_t { HOST = 0, DEVICE = 1, UNIFIED = 2 };

/// Compute capabilities. SM_100 (B200) is the only one this build's kernels
/// target; the older values remain so code written against the reference
/// still compiles.
enum class ComputeCapability : uint8_t {
  SM_70 = 70,
  SM_75 = 75,
  SM_80 = 80,
  SM_86 = 86,
  SM_89 = 89,
  SM_90 = 90,
  SM_100 = 100
};

/// float <-> element conversions usable from host code.
template <typename T> inline T from_float(float v) { return static_cast<T>(v); }
template <> inline __half from_float<__half>(float v) { return __float2half_rn(v); }
template <> inline __nv_bfloat16 from_float<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <typename T> inline float to_float(T v) { return static_cast<float>(v); }
template <> inline float to_float<__half>(__half v) { return __half2float(v); }
template <> inline float to_float<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

}  // namespace choreo_ir

#endif  // CHOREO_IR_CORE_TYPES_HPP
