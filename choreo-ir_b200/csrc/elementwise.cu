// elementwise.cu — device kernels for the reference's elementwise operations,
// which the reference runs as host loops over device data copied back to the
// host (relu: choreo-ir.hpp:196-222, operator+: choreo-ir.hpp:150-191, fill:
// tensor/tensor.hpp:530-562). HBM-bound: 16-byte vector loads/stores over a
// grid sized as a multiple of the SM count, scalar tail.
//
// Arithmetic matches the reference's host code: f16 values go through float
// and are rounded back (RNE), f32 stays f32; relu is (x < 0 ? 0 : x), so a
// NaN passes through as std::max(x, 0) lets it.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>

#include "internal.h"

namespace choreo_impl {
namespace {

template <typename T> __device__ __forceinline__ float ld_f(const T* p, int64_t i);
template <> __device__ __forceinline__ float ld_f<__half>(const __half* p, int64_t i) { return __half2float(p[i]); }
template <> __device__ __forceinline__ float ld_f<__nv_bfloat16>(const __nv_bfloat16* p, int64_t i) { return __bfloat162float(p[i]); }
template <> __device__ __forceinline__ float ld_f<float>(const float* p, int64_t i) { return p[i]; }

template <typename T> __device__ __forceinline__ T cvt(float v);
template <> __device__ __forceinline__ __half cvt<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 cvt<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <> __device__ __forceinline__ float cvt<float>(float v) { return v; }

struct OpRelu {
  __device__ __forceinline__ float operator()(float x, float) const { return x < 0.f ? 0.f : x; }
};
struct OpAdd {
  __device__ __forceinline__ float operator()(float x, float y) const { return x + y; }
};

// Elementwise map over n elements: vector part in 16-byte chunks when every
// pointer is 16-byte aligned, scalar remainder.
template <typename T, class Op, bool BINARY>
__global__ void map_kernel(const T* __restrict__ a, const T* __restrict__ b, T* __restrict__ out,
                           int64_t n, bool vec) {
  constexpr int V = 16 / sizeof(T);
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t nthreads = static_cast<int64_t>(gridDim.x) * blockDim.x;
  Op op;
  int64_t start_scalar = 0;
  if (vec) {
    const int64_t nv = n / V;
    const uint4* av = reinterpret_cast<const uint4*>(a);
    const uint4* bv = reinterpret_cast<const uint4*>(b);
    uint4* ov = reinterpret_cast<uint4*>(out);
    for (int64_t i = tid; i < nv; i += nthreads) {
      uint4 x = av[i];
      uint4 y = BINARY ? bv[i] : x;
      const T* xs = reinterpret_cast<const T*>(&x);
      const T* ys = reinterpret_cast<const T*>(&y);
      uint4 r;
      T* rs = reinterpret_cast<T*>(&r);
#pragma unroll
      for (int j = 0; j < V; ++j) rs[j] = cvt<T>(op(ld_f<T>(xs, j), BINARY ? ld_f<T>(ys, j) : 0.f));
      ov[i] = r;
    }
    start_scalar = nv * V;
  }
  for (int64_t i = start_scalar + tid; i < n; i += nthreads)
    out[i] = cvt<T>(op(ld_f<T>(a, i), BINARY ? ld_f<T>(b, i) : 0.f));
}

template <typename T>
__global__ void fill_kernel(T* __restrict__ out, T v, int64_t n) {
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t nthreads = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = tid; i < n; i += nthreads) out[i] = v;
}

template <typename S, typename D>
__global__ void convert_kernel(const S* __restrict__ src, D* __restrict__ dst, int64_t n) {
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t nthreads = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = tid; i < n; i += nthreads) dst[i] = cvt<D>(ld_f<S>(src, i));
}

int grid_for(int64_t work) {
  const int sms = current_sm_count();
  const int64_t want = (work + 255) / 256;
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, static_cast<int64_t>(sms) * 8)));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

template <class Op, bool BINARY>
int launch_map(int dtype, const void* a, const void* b, void* out, int64_t n, cudaStream_t s) {
  const bool vec = aligned16(a) && aligned16(out) && (!BINARY || aligned16(b));
  const int eb = dtype_bytes(dtype);
  if (eb == 0) return fail(CHOREO_ERR_UNSUPPORTED, "elementwise: unsupported dtype %d", dtype);
  const int grid = grid_for(vec ? n / (16 / eb) + 1 : n);
  switch (dtype) {
    case CHOREO_DTYPE_F16:
      map_kernel<__half, Op, BINARY><<<grid, 256, 0, s>>>(static_cast<const __half*>(a), static_cast<const __half*>(b), static_cast<__half*>(out), n, vec);
      break;
    case CHOREO_DTYPE_BF16:
      map_kernel<__nv_bfloat16, Op, BINARY><<<grid, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(a), static_cast<const __nv_bfloat16*>(b), static_cast<__nv_bfloat16*>(out), n, vec);
      break;
    default:
      map_kernel<float, Op, BINARY><<<grid, 256, 0, s>>>(static_cast<const float*>(a), static_cast<const float*>(b), static_cast<float*>(out), n, vec);
      break;
  }
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? CHOREO_OK : cuda_fail(e, "elementwise launch");
}

template <typename S>
int convert_from(const S* src, int ddst, void* dst, int64_t n, cudaStream_t s) {
  const int grid = grid_for(n);
  switch (ddst) {
    case CHOREO_DTYPE_F16: convert_kernel<S, __half><<<grid, 256, 0, s>>>(src, static_cast<__half*>(dst), n); break;
    case CHOREO_DTYPE_BF16: convert_kernel<S, __nv_bfloat16><<<grid, 256, 0, s>>>(src, static_cast<__nv_bfloat16*>(dst), n); break;
    case CHOREO_DTYPE_F32: convert_kernel<S, float><<<grid, 256, 0, s>>>(src, static_cast<float*>(dst), n); break;
    default: return fail(CHOREO_ERR_UNSUPPORTED, "convert: unsupported destination dtype %d", ddst);
  }
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? CHOREO_OK : cuda_fail(e, "convert launch");
}

}  // namespace

int launch_relu(int dtype, const void* in, void* out, int64_t n, cudaStream_t s) {
  return launch_map<OpRelu, false>(dtype, in, nullptr, out, n, s);
}
int launch_add(int dtype, const void* a, const void* b, void* out, int64_t n, cudaStream_t s) {
  return launch_map<OpAdd, true>(dtype, a, b, out, n, s);
}
int launch_fill(int dtype, void* dst, double v, int64_t n, cudaStream_t s) {
  const int grid = grid_for(n);
  switch (dtype) {
    case CHOREO_DTYPE_F16: fill_kernel<__half><<<grid, 256, 0, s>>>(static_cast<__half*>(dst), __float2half_rn(static_cast<float>(v)), n); break;
    case CHOREO_DTYPE_BF16: fill_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(static_cast<__nv_bfloat16*>(dst), __float2bfloat16_rn(static_cast<float>(v)), n); break;
    case CHOREO_DTYPE_F32: fill_kernel<float><<<grid, 256, 0, s>>>(static_cast<float*>(dst), static_cast<float>(v), n); break;
    default: return fail(CHOREO_ERR_UNSUPPORTED, "fill: unsupported dtype %d", dtype);
  }
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? CHOREO_OK : cuda_fail(e, "fill launch");
}
int launch_convert(int dsrc, const void* src, int ddst, void* dst, int64_t n, cudaStream_t s) {
  switch (dsrc) {
    case CHOREO_DTYPE_F16: return convert_from(static_cast<const __half*>(src), ddst, dst, n, s);
    case CHOREO_DTYPE_BF16: return convert_from(static_cast<const __nv_bfloat16*>(src), ddst, dst, n, s);
    case CHOREO_DTYPE_F32: return convert_from(static_cast<const float*>(src), ddst, dst, n, s);
    default: return fail(CHOREO_ERR_UNSUPPORTED, "convert: unsupported source dtype %d", dsrc);
  }
}

}  // namespace choreo_impl
