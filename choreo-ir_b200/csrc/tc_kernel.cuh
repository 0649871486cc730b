// tc_kernel.cuh — the persistent, warp-specialised tcgen05 mainloop shared by
// the GEMM and the implicit-GEMM convolution.
//
// CTA = 10 warps (320 threads), one CTA per SM, grid = min(tiles, SMs):
//   warp 0       TMA producer: fills a STAGES-deep ring of shared-memory
//                stages (A tile 128 x 64, B tile BN x 64, 128-byte swizzle).
//   warp 1       allocates 2*BN TMEM columns (two fp32 accumulators), and one
//                elected lane issues tcgen05.mma (128 x BN x 16 per
//                instruction, 4 per stage), releasing each stage with
//                tcgen05.commit and signalling a finished accumulator.
//   warps 2..9   epilogue, two warps per TMEM lane quarter (warp w reads TMEM
//                lanes 32*(w%4)..+31 = tile rows; warps 2..5 take the first
//                half of the columns, 6..9 the second): tcgen05.ld the
//                accumulator, hand it back to the MMA issuer, apply
//                alpha/beta/bias/ReLU, cast, and store through a 4 KB staging
//                buffer with bulk tensor stores (16-byte vector stores when C
//                is not TMA-addressable). Accumulators are double buffered so
//                the epilogue of tile i overlaps the MMAs of i+1.
// Tiles are walked in groups of `group_m` M-tiles so concurrently running
// CTAs share A and B panels in L2.
//
// Every mbarrier wait is bounded (see sm100.cuh): a stuck pipeline records an
// error in the device status word and the kernel returns.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "sm100.cuh"

namespace choreo_sm100 {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kThreads = 320;
constexpr int kEpiWarps = 8;
// Epilogue staging: one 4 KB buffer (32 rows x 128 bytes) per epilogue warp.
constexpr int kStagingBytes = kEpiWarps * 4096;

// Everything the kernel needs besides the two tensor maps.
struct TcParams {
  int32_t m, n;            // output rows / columns (per batch item)
  int32_t num_k_blocks;    // K / 64 rounded up (conv: R*S*ceil(C/64)); per split when split_kb > 0
  int32_t split_kb;        // > 0: the batch index is a K split of split_kb k-blocks (GEMM loader)
  int32_t num_m_blocks, num_n_blocks;
  int32_t batch;
  int64_t num_tiles;
  int32_t group_m;
  int32_t ab_bf16;
  int32_t l2_policy_a, l2_policy_b;  // 0 evict_normal, 1 evict_last, 2 evict_first
  // epilogue
  void* c;
  int64_t ldc, stride_c;   // elements
  int32_t c_vec_ok;        // 16-byte vector stores are legal for C
  int32_t c_tma;           // C is TMA-addressable: the epilogues store through staging tiles
  float alpha, beta;
  const void* bias;
  int32_t dtype_bias;      // 8 f16, 9 f32, 11 bf16
  int32_t relu;
  // convolution geometry (loader-specific)
  int32_t conv_c_blocks;   // ceil(C / 64)
  int32_t conv_s;          // filter width
  int32_t conv_q, conv_p;  // output width / height
  int32_t conv_pad_w, conv_pad_h;
  int32_t conv_stride_w, conv_stride_h;
  int32_t conv_dil_w, conv_dil_h;
  // failure reporting
  uint32_t* status;
  uint64_t timeout_ns;
  // wide tile: k-blocks one accumulator half runs alone at each hand-over
  // (0 = library choice; see wide_head_kb)
  int32_t handover_kb;
  // measurement hook (null = off): CTA 0 adds the SM clock cycles and the
  // %globaltimer nanoseconds of its lifetime to [0] and [1], and 1 to [2]
  unsigned long long* clock_probe;
};

// Start / end stamps of the clock probe, kept in the CTA's barrier block.
__device__ __forceinline__ void probe_start(const TcParams& p, uint64_t* slot) {
  if (p.clock_probe != nullptr && blockIdx.x == 0) {
    slot[0] = static_cast<uint64_t>(clock64());
    slot[1] = globaltimer_ns();
  }
}
__device__ __forceinline__ void probe_end(const TcParams& p, const uint64_t* slot) {
  if (p.clock_probe != nullptr && blockIdx.x == 0 && threadIdx.x == 0) {
    const uint64_t ns = globaltimer_ns();
    const uint64_t clk = static_cast<uint64_t>(clock64());
    atomicAdd(p.clock_probe, static_cast<unsigned long long>(clk - slot[0]));
    atomicAdd(p.clock_probe + 1, static_cast<unsigned long long>(ns - slot[1]));
    atomicAdd(p.clock_probe + 2, 1ull);
  }
}

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }

__device__ __forceinline__ uint32_t pack2(float a, float b, __half*) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t pack2(float a, float b, __nv_bfloat16*) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ float load_bias(const void* bias, int dt, int idx) {
  if (dt == 9) return __ldg(static_cast<const float*>(bias) + idx);
  if (dt == 11) return __bfloat162float(static_cast<const __nv_bfloat16*>(bias)[idx]);
  return __half2float(static_cast<const __half*>(bias)[idx]);
}

// Bias values one epilogue warp needs for a tile, loaded before it waits for
// the accumulator so the load latency hides behind the wait: lane j holds
// column n_first + 32 c + j for chunk c (0 past N or without a bias).
template <int kCols>
struct BiasRegs {
  float v[kCols / 32];
};
template <int kCols>
__device__ __forceinline__ void bias_prefetch(BiasRegs<kCols>& br, int n_first, const TcParams& p, int lane) {
#pragma unroll
  for (int c = 0; c < kCols / 32; ++c) {
    const int n = n_first + 32 * c + lane;
    br.v[c] = (p.bias != nullptr && n < p.n) ? load_bias(p.bias, p.dtype_bias, n) : 0.f;
  }
}

__device__ __forceinline__ uint64_t l2_policy(int code) {
  return code == 1 ? l2_policy_evict_last() : (code == 2 ? l2_policy_evict_first() : l2_policy_evict_normal());
}

// Maps a linear tile index to (batch item, M tile, N tile) with grouped
// rasterisation.
__device__ __forceinline__ void tile_coords(int64_t t, const TcParams& p, int& b, int& mb, int& nb) {
  const int64_t per_batch = static_cast<int64_t>(p.num_m_blocks) * p.num_n_blocks;
  b = static_cast<int>(t / per_batch);
  const int r = static_cast<int>(t - static_cast<int64_t>(b) * per_batch);
  const int tiles_per_group = p.group_m * p.num_n_blocks;
  const int g = r / tiles_per_group;
  const int first_m = g * p.group_m;
  const int gm = min(p.num_m_blocks - first_m, p.group_m);
  const int in = r - g * tiles_per_group;
  mb = first_m + in % gm;
  nb = in / gm;
}

__device__ __forceinline__ void unpack2(uint32_t u, float& a, float& b, __half*) {
  const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&u));
  a = f.x;
  b = f.y;
}
__device__ __forceinline__ void unpack2(uint32_t u, float& a, float& b, __nv_bfloat16*) {
  const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u));
  a = f.x;
  b = f.y;
}

// alpha * acc + beta * C + bias, then ReLU, for one 32-column chunk of one row.
// Called by all 32 lanes of a warp together (lane = row within the warp's
// slab): the chunk's bias is read once, lane j fetching column n_base + j, and
// broadcast with shuffles.
template <typename OutT>
__device__ __forceinline__ void epilogue_values(const uint32_t (&r)[32], float (&v)[32], const OutT* crow,
                                                int n_base, const TcParams& p, bool row_ok, int lane) {
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]) * p.alpha;
  const bool full = (n_base + 32 <= p.n);
  if (p.beta != 0.f && row_ok) {
    if (full && p.c_vec_ok) {
      if constexpr (sizeof(OutT) == 2) {
        const uint4* src = reinterpret_cast<const uint4*>(crow + n_base);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint4 q = src[j];
          const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            float a, b;
            unpack2(w[e], a, b, static_cast<OutT*>(nullptr));
            v[8 * j + 2 * e] += p.beta * a;
            v[8 * j + 2 * e + 1] += p.beta * b;
          }
        }
      } else {
        const float4* src = reinterpret_cast<const float4*>(crow + n_base);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float4 q = src[j];
          v[4 * j + 0] += p.beta * q.x;
          v[4 * j + 1] += p.beta * q.y;
          v[4 * j + 2] += p.beta * q.z;
          v[4 * j + 3] += p.beta * q.w;
        }
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (full || n_base + i < p.n) v[i] += p.beta * to_f32<OutT>(crow[n_base + i]);
    }
  }
  if (p.bias != nullptr) {
    const float bl = (n_base + lane < p.n) ? load_bias(p.bias, p.dtype_bias, n_base + lane) : 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] += __shfl_sync(0xffffffffu, bl, i);
  }
  if (p.relu) {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = (v[i] < 0.f) ? 0.f : v[i];  // NaN passes, like std::max(x, 0)
  }
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}

// Writes 32 converted values of this thread's row into a 128-byte-swizzled
// staging row (the layout a SWIZZLE_128B TMA store reads), starting at
// 16-byte chunk `chunk0` of the row. Lanes 8 apart share a chunk position, so
// each 8-lane phase of the warp's stores hits 32 distinct banks.
template <typename OutT>
__device__ __forceinline__ void stage_row_32(const float (&v)[32], uint32_t row_addr, int lane, int chunk0) {
  const int sw = lane & 7;
  if constexpr (sizeof(OutT) == 2) {
#pragma unroll
    for (int j = 0; j < 4; ++j)
      st_shared_v4(row_addr + (((chunk0 + j) ^ sw) << 4), pack2(v[8 * j + 0], v[8 * j + 1], static_cast<OutT*>(nullptr)),
                   pack2(v[8 * j + 2], v[8 * j + 3], static_cast<OutT*>(nullptr)),
                   pack2(v[8 * j + 4], v[8 * j + 5], static_cast<OutT*>(nullptr)),
                   pack2(v[8 * j + 6], v[8 * j + 7], static_cast<OutT*>(nullptr)));
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j)
      st_shared_v4(row_addr + (((chunk0 + j) ^ sw) << 4), __float_as_uint(v[4 * j + 0]), __float_as_uint(v[4 * j + 1]),
                   __float_as_uint(v[4 * j + 2]), __float_as_uint(v[4 * j + 3]));
  }
}

__device__ __forceinline__ float4 ld_shared_v4_f32(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
  return v;
}

__device__ __forceinline__ void st_shared_f32(uint32_t addr, float v) {
  asm volatile("st.shared.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

// (d0, d1) = (a0, a1) * s + (c0, c1) with one packed fp32 FMA (one rounding
// per element).
__device__ __forceinline__ void fma2(float& d0, float& d1, float a0, float a1, float s, float c0, float c1) {
  uint64_t a, b, c, d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(a) : "f"(a0), "f"(a1));
  asm("mov.b64 %0, {%1, %1};" : "=l"(b) : "f"(s));
  asm("mov.b64 %0, {%1, %2};" : "=l"(c) : "f"(c0), "f"(c1));
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(d0), "=f"(d1) : "l"(d));
}

// Round a pair to 16 bits with ReLU folded into the conversion (cvt .relu:
// negative results become 0, NaN stays NaN); a lands in the low half.
__device__ __forceinline__ uint32_t pack2_relu(float a, float b, __half*) {
  uint32_t r;
  asm("cvt.rn.relu.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(b), "f"(a));
  return r;
}
__device__ __forceinline__ uint32_t pack2_relu(float a, float b, __nv_bfloat16*) {
  uint32_t r;
  asm("cvt.rn.relu.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(b), "f"(a));
  return r;
}

// One 32-column chunk of the 16-bit epilogue: alpha * acc + bias (bias read
// as broadcasts from `bias_s`, the chunk's 32 values; none when null),
// rounded to 16-bit pairs, with ReLU folded into the rounding when RELU.
template <typename OutT, bool RELU>
__device__ __forceinline__ void convert_chunk(const uint32_t (&r)[32], float alpha, uint32_t bias_s, bool has_bias,
                                              uint32_t (&q)[16]) {
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float4 bv = has_bias ? ld_shared_v4_f32(bias_s + static_cast<uint32_t>(4 * j) * 4u)
                               : make_float4(0.f, 0.f, 0.f, 0.f);
    float v0, v1, v2, v3;
    fma2(v0, v1, __uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]), alpha, bv.x, bv.y);
    fma2(v2, v3, __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]), alpha, bv.z, bv.w);
    if constexpr (RELU) {
      q[2 * j] = pack2_relu(v0, v1, static_cast<OutT*>(nullptr));
      q[2 * j + 1] = pack2_relu(v2, v3, static_cast<OutT*>(nullptr));
    } else {
      q[2 * j] = pack2(v0, v1, static_cast<OutT*>(nullptr));
      q[2 * j + 1] = pack2(v2, v3, static_cast<OutT*>(nullptr));
    }
  }
}

// Writes 32 values of this thread's row, already packed as 16 16-bit pairs,
// into the 128-byte-swizzled staging row at 16-byte chunk `chunk0`.
__device__ __forceinline__ void stage_packed_32(const uint32_t (&q)[16], uint32_t row_addr, int lane, int chunk0) {
  const int sw = lane & 7;
#pragma unroll
  for (int j = 0; j < 4; ++j)
    st_shared_v4(row_addr + (((chunk0 + j) ^ sw) << 4), q[4 * j + 0], q[4 * j + 1], q[4 * j + 2], q[4 * j + 3]);
}

// Epilogue for one 32-column chunk of one row held by this thread (direct
// global stores: 16-byte vectors where legal, scalars at ragged edges).
template <typename OutT>
__device__ __forceinline__ void epilogue_chunk(const uint32_t (&r)[32], OutT* crow, int n_base,
                                               const TcParams& p, bool row_ok, int lane) {
  float v[32];
  epilogue_values<OutT>(r, v, crow, n_base, p, row_ok, lane);
  const bool full = (n_base + 32 <= p.n);
  if (!row_ok) return;
  if constexpr (sizeof(OutT) == 2) {
    if (full && p.c_vec_ok) {
      uint4* dst = reinterpret_cast<uint4*>(crow + n_base);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint4 q;
        q.x = pack2(v[8 * j + 0], v[8 * j + 1], static_cast<OutT*>(nullptr));
        q.y = pack2(v[8 * j + 2], v[8 * j + 3], static_cast<OutT*>(nullptr));
        q.z = pack2(v[8 * j + 4], v[8 * j + 5], static_cast<OutT*>(nullptr));
        q.w = pack2(v[8 * j + 6], v[8 * j + 7], static_cast<OutT*>(nullptr));
        dst[j] = q;
      }
      return;
    }
  } else {
    if (full && p.c_vec_ok) {
      float4* dst = reinterpret_cast<float4*>(crow + n_base);
#pragma unroll
      for (int j = 0; j < 8; ++j)
        dst[j] = make_float4(v[4 * j + 0], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
      return;
    }
  }
#pragma unroll
  for (int i = 0; i < 32; ++i)
    if (n_base + i < p.n) crow[n_base + i] = from_f32<OutT>(v[i]);
}

// Epilogue of one warp: 32 accumulator rows (the TMEM lanes of the warp's
// quarter) x kCols columns at TMEM address `taddr`, written to output rows
// row0 .. row0 + 31 and columns n_first .. n_first + kCols of batch item b.
// `release` hands the accumulator back to the MMA issuer, which waits for it
// before the next tile's MMAs into the same columns, so the work before it is
// on the MMA pipe's critical path.
//  - 16-bit output through the TMA store without a beta * C term (the common
//    case): every column is read from TMEM, scaled, biased (bias prefetched in
//    `br`), clamped and packed to 16-bit pairs in registers, then the
//    accumulator is released, and only then are the rows staged in the warp's
//    4 KB buffer and sent as bulk tensor stores of 128-byte rows (clipped by
//    the tensor map at the matrix edges).
//  - otherwise columns are read in batches of 64 (two tcgen05.ld per wait),
//    the accumulator is released once the last batch is in registers, and the
//    arithmetic and stores follow batch by batch (staging + bulk tensor stores
//    when C is TMA-addressable, else 16-byte vector stores).
template <int kCols, typename OutT, typename Release>
__device__ __forceinline__ void epilogue_warp(uint32_t taddr, int n_first, int row0, int b, const TcParams& p,
                                              const CUtensorMap* tma_c, uint32_t stage_buf, int lane,
                                              const BiasRegs<kCols>& br, Release&& release) {
  constexpr int kBatch = kCols < 64 ? kCols / 32 : 2;  // 32-column chunks per tcgen05.wait::ld
  constexpr int kBatches = kCols / 32 / kBatch;
  constexpr int E = 128 / static_cast<int>(sizeof(OutT));  // columns per 128-byte staging row
  constexpr int kCpg = E / 32;                              // chunks per staging row
  constexpr bool kTmaOk = (kBatch * 32) % E == 0;
  // Batches holding at least one valid column, for a warp with at least one valid row.
  int valid = 0;
  if (row0 < p.m && n_first < p.n) {
    valid = (p.n - n_first + kBatch * 32 - 1) / (kBatch * 32);
    if (valid > kBatches) valid = kBatches;
  }
  if (valid == 0) {
    release();
    return;
  }
  const bool use_tma = kTmaOk && p.c_tma != 0;
  if constexpr (sizeof(OutT) == 2 && kTmaOk) {
    if (use_tma && p.beta == 0.f) {
      constexpr int kChunks = kCols / 32;
      const bool has_bias = p.bias != nullptr;
      if (has_bias) {
        // The warp's kCols bias values go to the head of its staging buffer
        // (free until the stores below) and are read back as broadcast
        // vector loads: no cross-lane shuffles in the arithmetic.
        if (lane == 0) bulk_wait_read_all();  // the warp's previous store has read the buffer
        __syncwarp();
#pragma unroll
        for (int c = 0; c < kChunks; ++c) st_shared_f32(stage_buf + static_cast<uint32_t>(c * 32 + lane) * 4u, br.v[c]);
        __syncwarp();
      }
      // Every chunk's TMEM read is in flight at once and waited for once; the
      // accumulator goes back to the MMA issuer before the arithmetic.
      // Columns past N are read and converted too (TMEM holds them; the
      // tensor map clips them from the stores).
      uint32_t r[kChunks][32];
#pragma unroll
      for (int c = 0; c < kChunks; ++c) tmem_ld_32x32b_x32(taddr + c * 32, r[c]);
      tmem_wait_ld();
      release();
      uint32_t q[kChunks][16];
#pragma unroll
      for (int c = 0; c < kChunks; ++c) {
        const uint32_t bias_s = stage_buf + static_cast<uint32_t>(c * 32) * 4u;
        if (p.relu)
          convert_chunk<OutT, true>(r[c], p.alpha, bias_s, has_bias, q[c]);
        else
          convert_chunk<OutT, false>(r[c], p.alpha, bias_s, has_bias, q[c]);
      }
      const uint32_t row_addr = stage_buf + static_cast<uint32_t>(lane) * 128u;
#pragma unroll
      for (int g = 0; g < kChunks / kCpg; ++g) {
        const int n_base = n_first + g * E;
        if (n_base >= p.n) break;  // warp-uniform
        if (lane == 0) bulk_wait_read_all();  // the warp's previous store has read the buffer
        __syncwarp();
#pragma unroll
        for (int c = 0; c < kCpg; ++c) stage_packed_32(q[g * kCpg + c], row_addr, lane, c * 4);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_3d(tma_c, stage_buf, n_base, row0, b);
          bulk_commit_group();
        }
      }
      return;
    }
  }
  const int row = row0 + lane;
  const bool row_ok = row < p.m;
  OutT* crow = static_cast<OutT*>(p.c) + static_cast<int64_t>(b) * p.stride_c +
               static_cast<int64_t>(row_ok ? row : 0) * p.ldc;
#pragma unroll 1
  for (int bi = 0; bi < kBatches; ++bi) {
    if (bi >= valid) break;  // warp-uniform
    uint32_t r[kBatch][32];
#pragma unroll
    for (int j = 0; j < kBatch; ++j) tmem_ld_32x32b_x32(taddr + (bi * kBatch + j) * 32, r[j]);
    tmem_wait_ld();
    if (bi == valid - 1) release();
    const int n_batch = n_first + bi * kBatch * 32;
    if constexpr (kTmaOk) {
      if (use_tma) {
#pragma unroll
        for (int g = 0; g < kBatch / kCpg; ++g) {
          const int n_base = n_batch + g * E;
          if (n_base >= p.n) break;  // warp-uniform
          if (lane == 0) bulk_wait_read_all();  // the warp's previous store has read the buffer
          __syncwarp();
#pragma unroll
          for (int c = 0; c < kCpg; ++c) {
            float v[32];
            epilogue_values<OutT>(r[g * kCpg + c], v, crow, n_base + c * 32, p, row_ok, lane);
            stage_row_32<OutT>(v, stage_buf + static_cast<uint32_t>(lane) * 128u, lane,
                               c * (32 * static_cast<int>(sizeof(OutT)) / 16));
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_3d(tma_c, stage_buf, n_base, row0, b);
            bulk_commit_group();
          }
        }
        continue;
      }
    }
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      const int n_base = n_batch + j * 32;
      if (n_base < p.n) epilogue_chunk<OutT>(r[j], crow, n_base, p, row_ok, lane);
    }
  }
}

// Shared-memory bookkeeping beyond the stage ring.
template <int STAGES>
struct alignas(8) TcBarriers {
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t drain;
  uint64_t probe[2];
  uint32_t tmem_base;
  int32_t abort;
};

template <int BN, int STAGES>
constexpr int tc_smem_bytes() {
  return STAGES * (kBM * kBK * 2 + BN * kBK * 2) + kStagingBytes + 1024 /*alignment slack*/ +
         static_cast<int>(sizeof(TcBarriers<STAGES>));
}

// Loader contract:
//   static constexpr bool kAMn, kBMn;          operand majorness in shared memory
//   __device__ static void issue(const CUtensorMap* ta, const CUtensorMap* tb, const TcParams&,
//                                int b, int m0, int n0, int kb, uint32_t dst_a, uint32_t dst_b,
//                                uint32_t bar, uint64_t pol_a, uint64_t pol_b);
// loads this CTA's A rows [m0, m0 + 128) and B columns [n0, n0 + B width) for
// k-block kb of batch item b into the stage at dst_a / dst_b, counted on bar.
// The wide tile's producer uses a per-tile cursor instead:
//   struct WideCursor;  static WideCursor wide_cursor(const TcParams&, int b, int m0, int n0);
//   static void issue_wide(ta, tb, p, WideCursor&, int kb, dst_a, dst_b, bar, pol_a, pol_b);
// called for k-blocks 0, 1, ... of one tile in order (this CTA's 256 A rows).
template <int BN, int STAGES, class Loader, typename OutT>
__global__ void __launch_bounds__(kThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                   const __grid_constant__ CUtensorMap tma_c, const TcParams p) {
  constexpr uint32_t kAStage = kBM * kBK * 2;
  constexpr uint32_t kBStage = BN * kBK * 2;
  constexpr uint32_t kStageBytes = kAStage + kBStage;
  constexpr uint32_t kTmemCols = 2 * BN;
  static_assert(BN == 64 || BN == 128 || BN == 256, "BN must be 64, 128 or 256");

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* s_a = smem;
  uint8_t* s_b = smem + STAGES * kAStage;
  uint8_t* s_stage = s_b + STAGES * kBStage;  // 1024-aligned: every stage is a multiple of 1 KB
  auto* bars = reinterpret_cast<TcBarriers<STAGES>*>(s_stage + kStagingBytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&bars->full[s]), 1);
      mbar_init(smem_u32(&bars->empty[s]), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&bars->tmem_full[i]), 1);
      mbar_init(smem_u32(&bars->tmem_empty[i]), kEpiWarps);
    }
    if (p.c_tma) tma_prefetch_desc(&tma_c);
    mbar_init(smem_u32(&bars->drain), 1);
    bars->abort = 0;
    probe_start(p, bars->probe);
    fence_mbar_init();
    tma_prefetch_desc(&tma_a);
    tma_prefetch_desc(&tma_b);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&bars->tmem_base), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = bars->tmem_base;
  const WaitCtx wctx{p.status, p.timeout_ns, &bars->abort};

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      griddep_wait();  // the previous kernel's writes to A and B are visible
      const uint64_t pol_a = l2_policy(p.l2_policy_a);
      const uint64_t pol_b = l2_policy(p.l2_policy_b);
      uint32_t stage = 0, phase = 0, issued = 0;
      bool ok = true;
      for (int64_t t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x) {
        int b, mb, nb;
        tile_coords(t, p, b, mb, nb);
        for (int kb = 0; kb < p.num_k_blocks; ++kb) {
          if (!mbar_wait(smem_u32(&bars->empty[stage]), phase ^ 1, wctx, kStatusTimeoutProducer)) {
            ok = false;
            break;
          }
          const uint32_t fb = smem_u32(&bars->full[stage]);
          mbar_arrive_expect_tx(fb, kStageBytes);
          Loader::issue(&tma_a, &tma_b, p, b, mb * kBM, nb * BN, kb, smem_u32(s_a + stage * kAStage),
                        smem_u32(s_b + stage * kBStage), fb, pol_a, pol_b);
          ++issued;
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      griddep_launch_dependents();  // every load is issued: the next kernel may start launching
      if (!ok) {
        // Let the loads already in flight land before the CTA exits.
        const uint32_t inflight = issued < STAGES ? issued : STAGES;
        uint32_t s = stage, ph = phase;
        for (uint32_t i = 0; i < inflight; ++i) {
          if (s == 0) { s = STAGES - 1; ph ^= 1; } else { --s; }
          mbar_wait(smem_u32(&bars->full[s]), ph, wctx, kStatusTimeoutDrain, false);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(kBM, BN, p.ab_bf16 != 0, Loader::kAMn, Loader::kBMn);
      uint32_t stage = 0, phase = 0, local = 0;
      bool ok = true;
      for (int64_t t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x, ++local) {
        const uint32_t buf = local & 1;
        const uint32_t tph = (local >> 1) & 1;
        if (!mbar_wait(smem_u32(&bars->tmem_empty[buf]), tph ^ 1, wctx, kStatusTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        for (int kb = 0; kb < p.num_k_blocks; ++kb) {
          if (!mbar_wait(smem_u32(&bars->full[stage]), phase, wctx, kStatusTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(s_a + stage * kAStage);
          const uint32_t b0 = smem_u32(s_b + stage * kBStage);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            const uint64_t ad = Loader::kAMn ? smem_desc_sw128(a0 + k * 2048, 8192, 1024)
                                             : smem_desc_sw128(a0 + k * 32, 16, 1024);
            const uint64_t bd = Loader::kBMn ? smem_desc_sw128(b0 + k * 2048, 8192, 1024)
                                             : smem_desc_sw128(b0 + k * 32, 16, 1024);
            umma_f16(d_tmem, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit(smem_u32(&bars->empty[stage]));
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        umma_commit(smem_u32(&bars->tmem_full[buf]));
      }
      // All MMAs must have finished before TMEM is released.
      umma_commit(smem_u32(&bars->drain));
      mbar_wait(smem_u32(&bars->drain), 0, wctx, kStatusTimeoutDrain, false);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;       // TMEM lanes this warp may read
    const int col_half = (warp - 2) >> 2;  // which half of the columns
    const uint32_t stage_buf = smem_u32(s_stage) + static_cast<uint32_t>(warp - 2) * 4096u;
    griddep_wait();  // the previous kernel is done with C
    uint32_t local = 0;
    for (int64_t t = blockIdx.x; t < p.num_tiles; t += gridDim.x, ++local) {
      const uint32_t buf = local & 1;
      const uint32_t tph = (local >> 1) & 1;
      int b, mb, nb;
      tile_coords(t, p, b, mb, nb);
      const int n_first = nb * BN + col_half * (BN / 2);
      BiasRegs<BN / 2> br;
      bias_prefetch(br, n_first, p, lane);
      int ready = 0;
      if (lane == 0)
        ready = mbar_wait(smem_u32(&bars->tmem_full[buf]), tph, wctx, kStatusTimeoutEpilogue) ? 1 : 0;
      ready = __shfl_sync(0xffffffffu, ready, 0);
      if (!ready) break;
      tc_fence_after();
      const uint32_t taddr =
          tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + buf * BN + col_half * (BN / 2);
      epilogue_warp<BN / 2, OutT>(taddr, n_first, mb * kBM + quarter * 32, b, p, &tma_c, stage_buf, lane, br, [&] {
                                    tc_fence_before();
                                    __syncwarp();
                                    if (lane == 0) mbar_arrive(smem_u32(&bars->tmem_empty[buf]));
                                  });
    }
    // The staged stores have read their shared-memory source before the CTA's
    // shared memory goes away; their global writes drain on their own.
    if (lane == 0) bulk_wait_read_all();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  probe_end(p, bars->probe);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// CTA-pair variant: a cluster of 2 CTAs on the two SMs of a TPC computes one
// 256 x BN output tile with tcgen05 cta_group::2 MMAs (M = 256 per
// instruction). Each CTA stages its own 128 A rows and BN/2 B columns per
// k-block (A split by M, B split by N across the pair), so a pair moves
// (256 + BN) x 64 operand elements per k-block for a 256 x BN tile — a third
// less L2->SM traffic per FLOP than two independent 128 x BN CTAs. Each
// CTA's TMEM holds its 128 accumulator rows; each CTA's epilogue stores them.
//   - both producers' TMA loads count their bytes on the LEADER's (rank 0)
//     full barrier, which the leader's producer arms with both CTAs' bytes;
//   - the leader's MMA thread releases a stage / publishes an accumulator by
//     committing to the barrier in each CTA (two plain commits);
//   - the leader's accumulator-empty barrier takes 16 arrivals: 8 local
//     epilogue warps and 8 of the peer's (remote mbarrier arrive).
template <int BN, int STAGES>
constexpr int tc_pair_smem_bytes() {
  return STAGES * (kBM * kBK * 2 + (BN / 2) * kBK * 2) + kStagingBytes + 1024 +
         static_cast<int>(sizeof(TcBarriers<STAGES>));
}

template <int BN, int STAGES, class Loader, typename OutT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    tc_gemm_pair_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                        const __grid_constant__ CUtensorMap tma_c, const TcParams p) {
  constexpr int BNL = BN / 2;  // B columns this CTA stages
  constexpr uint32_t kAStage = kBM * kBK * 2;
  constexpr uint32_t kBStage = BNL * kBK * 2;
  constexpr uint32_t kStageBytes = kAStage + kBStage;
  constexpr uint32_t kTmemCols = 2 * BN;
  static_assert(BN == 128 || BN == 256, "pair tile N must be 128 or 256");

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* s_a = smem;
  uint8_t* s_b = smem + STAGES * kAStage;
  uint8_t* s_stage = s_b + STAGES * kBStage;  // 1024-aligned: every stage is a multiple of 1 KB
  auto* bars = reinterpret_cast<TcBarriers<STAGES>*>(s_stage + kStagingBytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int64_t cluster_id = blockIdx.x >> 1;
  const int64_t num_clusters = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&bars->full[s]), 1);
      mbar_init(smem_u32(&bars->empty[s]), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&bars->tmem_full[i]), 1);
      mbar_init(smem_u32(&bars->tmem_empty[i]), 2 * kEpiWarps);
    }
    if (p.c_tma) tma_prefetch_desc(&tma_c);
    mbar_init(smem_u32(&bars->drain), 1);
    bars->abort = 0;
    probe_start(p, bars->probe);
    fence_mbar_init();
    tma_prefetch_desc(&tma_a);
    tma_prefetch_desc(&tma_b);
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(&bars->tmem_base), kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised before any remote use
  tc_fence_after();
  const uint32_t tmem_base = bars->tmem_base;
  const WaitCtx wctx{p.status, p.timeout_ns, &bars->abort};

  if (warp == 0) {
    // ------------------------------------------------------------ producers (both CTAs)
    if (lane == 0) {
      griddep_wait();  // the previous kernel's writes to A and B are visible
      const uint64_t pol_a = l2_policy(p.l2_policy_a);
      const uint64_t pol_b = l2_policy(p.l2_policy_b);
      uint32_t stage = 0, phase = 0, issued = 0;
      bool ok = true;
      for (int64_t t = cluster_id; t < p.num_tiles && ok; t += num_clusters) {
        int b, mb, nb;
        tile_coords(t, p, b, mb, nb);
        const int m0 = mb * (2 * kBM) + static_cast<int>(rank) * kBM;
        const int n0 = nb * BN + static_cast<int>(rank) * BNL;
        for (int kb = 0; kb < p.num_k_blocks; ++kb) {
          if (!mbar_wait(smem_u32(&bars->empty[stage]), phase ^ 1, wctx, kStatusTimeoutProducer)) {
            ok = false;
            break;
          }
          const uint32_t own_full = smem_u32(&bars->full[stage]);
          if (leader) mbar_arrive_expect_tx(own_full, 2 * kStageBytes);
          Loader::issue(&tma_a, &tma_b, p, b, m0, n0, kb, smem_u32(s_a + stage * kAStage),
                        smem_u32(s_b + stage * kBStage), mapa_shared(own_full, 0), pol_a, pol_b);
          ++issued;
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      griddep_launch_dependents();  // every load is issued: the next kernel may start launching
      if (!ok) {
        if (leader) {
          const uint32_t inflight = issued < STAGES ? issued : STAGES;
          uint32_t s = stage, ph = phase;
          for (uint32_t i = 0; i < inflight; ++i) {
            if (s == 0) { s = STAGES - 1; ph ^= 1; } else { --s; }
            mbar_wait(smem_u32(&bars->full[s]), ph, wctx, kStatusTimeoutDrain, false);
          }
        } else {
          // The peer's loads count on the leader's barriers: give them time to land.
          const uint64_t t0 = globaltimer_ns();
          while (globaltimer_ns() - t0 < 200000ull) {
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader only)
    if (leader && lane == 0) {
      const uint32_t idesc = idesc_f16(2 * kBM, BN, p.ab_bf16 != 0, Loader::kAMn, Loader::kBMn);
      uint32_t stage = 0, phase = 0, local = 0;
      bool ok = true;
      for (int64_t t = cluster_id; t < p.num_tiles && ok; t += num_clusters, ++local) {
        const uint32_t buf = local & 1;
        const uint32_t tph = (local >> 1) & 1;
        if (!mbar_wait(smem_u32(&bars->tmem_empty[buf]), tph ^ 1, wctx, kStatusTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        for (int kb = 0; kb < p.num_k_blocks; ++kb) {
          if (!mbar_wait(smem_u32(&bars->full[stage]), phase, wctx, kStatusTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(s_a + stage * kAStage);
          const uint32_t b0 = smem_u32(s_b + stage * kBStage);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            const uint64_t ad = Loader::kAMn ? smem_desc_sw128(a0 + k * 2048, 8192, 1024)
                                             : smem_desc_sw128(a0 + k * 32, 16, 1024);
            const uint64_t bd = Loader::kBMn ? smem_desc_sw128(b0 + k * 2048, 8192, 1024)
                                             : smem_desc_sw128(b0 + k * 32, 16, 1024);
            umma_f16_pair(d_tmem, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          const uint32_t eb = smem_u32(&bars->empty[stage]);
          umma_commit_pair(eb);
          umma_commit_pair(mapa_shared(eb, 1));
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        const uint32_t fb = smem_u32(&bars->tmem_full[buf]);
        umma_commit_pair(fb);
        umma_commit_pair(mapa_shared(fb, 1));
      }
      umma_commit_pair(smem_u32(&bars->drain));
      mbar_wait(smem_u32(&bars->drain), 0, wctx, kStatusTimeoutDrain, false);
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int quarter = warp & 3;
    const int col_half = (warp - 2) >> 2;
    const uint32_t stage_buf = smem_u32(s_stage) + static_cast<uint32_t>(warp - 2) * 4096u;
    griddep_wait();  // the previous kernel is done with C
    uint32_t local = 0;
    for (int64_t t = cluster_id; t < p.num_tiles; t += num_clusters, ++local) {
      const uint32_t buf = local & 1;
      const uint32_t tph = (local >> 1) & 1;
      int b, mb, nb;
      tile_coords(t, p, b, mb, nb);
      const int n_first = nb * BN + col_half * (BN / 2);
      BiasRegs<BN / 2> br;
      bias_prefetch(br, n_first, p, lane);
      int ready = 0;
      if (lane == 0)
        ready = mbar_wait(smem_u32(&bars->tmem_full[buf]), tph, wctx, kStatusTimeoutEpilogue) ? 1 : 0;
      ready = __shfl_sync(0xffffffffu, ready, 0);
      if (!ready) break;
      tc_fence_after();
      const uint32_t taddr =
          tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + buf * BN + col_half * (BN / 2);
      epilogue_warp<BN / 2, OutT>(taddr, n_first, mb * (2 * kBM) + static_cast<int>(rank) * kBM + quarter * 32, b,
                                  p, &tma_c, stage_buf, lane, br, [&] {
                                    tc_fence_before();
                                    __syncwarp();
                                    if (lane == 0) {
                                      const uint32_t eb = smem_u32(&bars->tmem_empty[buf]);
                                      if (leader)
                                        mbar_arrive(eb);
                                      else
                                        mbar_arrive_cluster(mapa_shared(eb, 0));
                                    }
                                  });
    }
    // The staged stores have read their shared-memory source before the CTA's
    // shared memory goes away; their global writes drain on their own.
    if (lane == 0) bulk_wait_read_all();
    __syncwarp();
  }

  tc_fence_before();
  cluster_sync();  // both CTAs done (MMAs drained, epilogues finished) before TMEM is freed
  probe_end(p, bars->probe);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// Wide CTA-pair variant: the pair computes a 512 x 256 tile as two M = 256
// halves that share every B k-block (two cta_group::2 MMAs per k-step). CTA r
// owns tile rows [256 r, 256 r + 256), staged per k-block as one 256-row A
// box, plus 128 B columns; half h of the tile is rows [128 h, 128 h + 128) of
// each CTA. Each CTA keeps its 256 x 256 fp32 accumulator (128 rows of each
// half) in all 512 TMEM columns: a quarter less L2 -> SM operand traffic per
// FLOP than 256 x 256 tiles. With no room for a second accumulator, overlap
// comes from handing the accumulator over in halves: a tile's first D
// k-blocks run for half 0 alone while the epilogue reads the previous tile's
// half 1 out; then both halves run over k-blocks D .. K-1, half 0 is published,
// and half 1 finishes over k-blocks 0 .. D-1, which the producer loads a
// second time, while the epilogue reads half 0 out. No stage is held across a
// hand-over, so the ring keeps streaming over tile boundaries (holding the
// window's stages instead left the 4-stage ring to refill twice per tile).
// Tiles no longer than the window hold their stages and replay them.
template <int STAGES>
struct alignas(8) TcWideBarriers {
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tmem_full[2];   // accumulator half h of this tile is complete (leader commit, count 1)
  uint64_t tmem_empty[2];  // accumulator half h read out by the pair's 16 epilogue warps (leader's, count 16)
  uint64_t drain;
  uint64_t probe[2];
  uint32_t tmem_base;
  int32_t abort;
};

// The wide tile's hand-over window D: k-blocks half 0 runs alone at the head
// of a tile (and half 1 at its end). choreo_tuning::handover_kb when in
// 1 .. 16, else the ring depth, one less for tiles under 64 k-blocks. A tile
// of no more k-blocks than that holds its stages (D = K) when they fit the
// ring, and otherwise streams with D = the ring depth. Producer and MMA issuer
// both use it.
__device__ __forceinline__ int wide_head_kb(const TcParams& p, int stages) {
  const int w = p.handover_kb > 0 && p.handover_kb <= 16
                    ? p.handover_kb
                    : (p.num_k_blocks < 64 && stages > 2 ? stages - 1 : stages);
  if (p.num_k_blocks > w) return w;
  return p.num_k_blocks <= stages ? p.num_k_blocks : stages;
}

template <int STAGES>
constexpr int tc_wide_smem_bytes() {
  return STAGES * (2 * kBM * kBK * 2 + 128 * kBK * 2) + kStagingBytes + 1024 +
         static_cast<int>(sizeof(TcWideBarriers<STAGES>));
}

template <int STAGES, class Loader, typename OutT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    tc_gemm_pair_wide_kernel(const __grid_constant__ CUtensorMap tma_a,
                             const __grid_constant__ CUtensorMap tma_b,
                             const __grid_constant__ CUtensorMap tma_c, const TcParams p) {
  constexpr int BN = 256;
  constexpr int BNL = 128;
  constexpr uint32_t kAHalf = kBM * kBK * 2;   // 128 rows x 64 (16 KB)
  constexpr uint32_t kAStage = 2 * kAHalf;
  constexpr uint32_t kBStage = BNL * kBK * 2;  // 16 KB
  constexpr uint32_t kStageBytes = kAStage + kBStage;
  constexpr uint32_t kTmemCols = 512;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* s_a = smem;
  uint8_t* s_b = smem + STAGES * kAStage;
  uint8_t* s_stage = s_b + STAGES * kBStage;  // 1024-aligned: every stage is a multiple of 1 KB
  auto* bars = reinterpret_cast<TcWideBarriers<STAGES>*>(s_stage + kStagingBytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int64_t cluster_id = blockIdx.x >> 1;
  const int64_t num_clusters = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&bars->full[s]), 1);
      mbar_init(smem_u32(&bars->empty[s]), 1);
    }
    if (p.c_tma) tma_prefetch_desc(&tma_c);
    mbar_init(smem_u32(&bars->tmem_full[0]), 1);
    mbar_init(smem_u32(&bars->tmem_full[1]), 1);
    mbar_init(smem_u32(&bars->tmem_empty[0]), 2 * kEpiWarps);
    mbar_init(smem_u32(&bars->tmem_empty[1]), 2 * kEpiWarps);
    mbar_init(smem_u32(&bars->drain), 1);
    bars->abort = 0;
    probe_start(p, bars->probe);
    fence_mbar_init();
    tma_prefetch_desc(&tma_a);
    tma_prefetch_desc(&tma_b);
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(&bars->tmem_base), kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = bars->tmem_base;
  const WaitCtx wctx{p.status, p.timeout_ns, &bars->abort};

  if (warp == 0) {
    // ------------------------------------------------------------ producers (both CTAs)
    if (lane == 0) {
      griddep_wait();  // the previous kernel's writes to A and B are visible
      const uint64_t pol_a = l2_policy(p.l2_policy_a);
      const uint64_t pol_b = l2_policy(p.l2_policy_b);
      uint32_t stage = 0, phase = 0, issued = 0;
      bool ok = true;
      for (int64_t t = cluster_id; t < p.num_tiles && ok; t += num_clusters) {
        int b, mb, nb;
        tile_coords(t, p, b, mb, nb);
        const int m0 = mb * (4 * kBM) + static_cast<int>(rank) * (2 * kBM);  // this CTA's 256 rows
        const int n0 = nb * BN + static_cast<int>(rank) * BNL;
        // k-blocks 0 .. K-1, then 0 .. D-1 again for half 1 when the tile is
        // longer than the hand-over window (see the MMA issuer)
        const int D = wide_head_kb(p, STAGES);
        const int loads = p.num_k_blocks + (D < p.num_k_blocks ? D : 0);
        auto cur = Loader::wide_cursor(p, b, m0, n0);  // per-tile load state; k-blocks in order
        for (int i = 0; i < loads; ++i) {
          if (i == p.num_k_blocks) cur = Loader::wide_cursor(p, b, m0, n0);
          const int kb = i < p.num_k_blocks ? i : i - p.num_k_blocks;
          if (!mbar_wait(smem_u32(&bars->empty[stage]), phase ^ 1, wctx, kStatusTimeoutProducer)) {
            ok = false;
            break;
          }
          const uint32_t own_full = smem_u32(&bars->full[stage]);
          if (leader) mbar_arrive_expect_tx(own_full, 2 * kStageBytes);
          const uint32_t bar = mapa_shared(own_full, 0);
          Loader::issue_wide(&tma_a, &tma_b, p, cur, kb, smem_u32(s_a + stage * kAStage),
                             smem_u32(s_b + stage * kBStage), bar, pol_a, pol_b);
          ++issued;
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      griddep_launch_dependents();  // every load is issued: the next kernel may start launching
      if (!ok) {
        if (leader) {
          const uint32_t inflight = issued < STAGES ? issued : STAGES;
          uint32_t s = stage, ph = phase;
          for (uint32_t i = 0; i < inflight; ++i) {
            if (s == 0) { s = STAGES - 1; ph ^= 1; } else { --s; }
            mbar_wait(smem_u32(&bars->full[s]), ph, wctx, kStatusTimeoutDrain, false);
          }
        } else {
          const uint64_t t0 = globaltimer_ns();
          while (globaltimer_ns() - t0 < 200000ull) {
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader only)
    if (leader && lane == 0) {
      const uint32_t idesc = idesc_f16(2 * kBM, BN, p.ab_bf16 != 0, Loader::kAMn, Loader::kBMn);
      // The MMAs of one accumulator half for one stage; `first` starts the sum.
      auto issue_half = [&](int h, uint32_t st, bool first) {
        const uint32_t ah = smem_u32(s_a + st * kAStage) + h * kAHalf;
        const uint32_t b0 = smem_u32(s_b + st * kBStage);
#pragma unroll
        for (int k = 0; k < kBK / 16; ++k) {
          const uint64_t ad = Loader::kAMn ? smem_desc_sw128(ah + k * 2048, 8192, 1024)
                                           : smem_desc_sw128(ah + k * 32, 16, 1024);
          const uint64_t bd = Loader::kBMn ? smem_desc_sw128(b0 + k * 2048, 8192, 1024)
                                           : smem_desc_sw128(b0 + k * 32, 16, 1024);
          umma_f16_pair(tmem_base + h * BN, ad, bd, idesc, (first && k == 0) ? 0u : 1u);
        }
      };
      auto release = [&](uint32_t st) {
        const uint32_t eb = smem_u32(&bars->empty[st]);
        umma_commit_pair(eb);
        umma_commit_pair(mapa_shared(eb, 1));
      };
      uint32_t stage = 0, phase = 0, local = 0;
      bool ok = true;
      auto publish = [&](int h) {  // half h of the tile is complete once its MMAs finish
        const uint32_t fb = smem_u32(&bars->tmem_full[h]);
        umma_commit_pair(fb);
        umma_commit_pair(mapa_shared(fb, 1));
      };
      auto wait_full = [&](uint32_t st, uint32_t ph) {
        if (!mbar_wait(smem_u32(&bars->full[st]), ph, wctx, kStatusTimeoutMma)) return false;
        tc_fence_after();
        return true;
      };
      auto advance = [&] {
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      };
      const int K = p.num_k_blocks;
      const int D = wide_head_kb(p, STAGES);
      for (int64_t t = cluster_id; t < p.num_tiles && ok; t += num_clusters, ++local) {
        const uint32_t tph = local & 1;
        if (!mbar_wait(smem_u32(&bars->tmem_empty[0]), tph ^ 1, wctx, kStatusTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (D == K) {
          // The whole tile fits the window: its stages are held after the
          // half-0 MMAs, replayed for half 1 once the epilogue has read the
          // previous tile's half 1, and released then.
          uint32_t st = stage, ph = phase;
          for (int kb = 0; kb < K; ++kb) {
            if (!wait_full(st, ph)) {
              ok = false;
              break;
            }
            issue_half(0, st, kb == 0);
            if (++st == STAGES) { st = 0; ph ^= 1; }
          }
          if (!ok) break;
          publish(0);
          if (!mbar_wait(smem_u32(&bars->tmem_empty[1]), tph ^ 1, wctx, kStatusTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          for (int kb = 0; kb < K; ++kb) {
            issue_half(1, stage, kb == 0);
            release(stage);
            advance();
          }
          publish(1);
          continue;
        }
        // Head: k-blocks 0 .. D-1 for half 0 while the epilogue reads the
        // previous tile's half 1 out. Each stage is released at once, so the
        // ring keeps streaming across the tile boundary; the producer loads
        // these k-blocks again after the tile's last one, for half 1.
        for (int kb = 0; kb < D; ++kb) {
          if (!wait_full(stage, phase)) {
            ok = false;
            break;
          }
          issue_half(0, stage, kb == 0);
          release(stage);
          advance();
        }
        if (!ok) break;
        if (!mbar_wait(smem_u32(&bars->tmem_empty[1]), tph ^ 1, wctx, kStatusTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // Body: both halves per stage; half 1's sum starts at k-block D.
        for (int kb = D; kb < K; ++kb) {
          if (!wait_full(stage, phase)) {
            ok = false;
            break;
          }
          issue_half(0, stage, false);
          issue_half(1, stage, kb == D);
          release(stage);
          advance();
        }
        if (!ok) break;
        publish(0);  // read out by the epilogue during the replay below
        // Replay: k-blocks 0 .. D-1 again, for half 1.
        for (int kb = 0; kb < D; ++kb) {
          if (!wait_full(stage, phase)) {
            ok = false;
            break;
          }
          issue_half(1, stage, false);
          release(stage);
          advance();
        }
        if (!ok) break;
        publish(1);
      }
      umma_commit_pair(smem_u32(&bars->drain));
      mbar_wait(smem_u32(&bars->drain), 0, wctx, kStatusTimeoutDrain, false);
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int quarter = warp & 3;
    const int col_half = (warp - 2) >> 2;
    const uint32_t stage_buf = smem_u32(s_stage) + static_cast<uint32_t>(warp - 2) * 4096u;
    griddep_wait();  // the previous kernel is done with C
    uint32_t local = 0;
    bool ok = true;
    for (int64_t t = cluster_id; t < p.num_tiles && ok; t += num_clusters, ++local) {
      int b, mb, nb;
      tile_coords(t, p, b, mb, nb);
      const int n_first = nb * BN + col_half * (BN / 2);  // the same columns for both halves
      BiasRegs<BN / 2> br;
      bias_prefetch(br, n_first, p, lane);
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        int ready = 0;
        if (lane == 0)
          ready = mbar_wait(smem_u32(&bars->tmem_full[h]), local & 1, wctx, kStatusTimeoutEpilogue) ? 1 : 0;
        ready = __shfl_sync(0xffffffffu, ready, 0);
        if (!ready) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t taddr =
            tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + h * BN + col_half * (BN / 2);
        epilogue_warp<BN / 2, OutT>(taddr, n_first,
                                    mb * (4 * kBM) + static_cast<int>(rank) * (2 * kBM) + h * kBM + quarter * 32,
                                    b, p, &tma_c, stage_buf, lane, br, [&] {
                                      tc_fence_before();
                                      __syncwarp();
                                      if (lane == 0) {
                                        const uint32_t eb = smem_u32(&bars->tmem_empty[h]);
                                        if (leader)
                                          mbar_arrive(eb);
                                        else
                                          mbar_arrive_cluster(mapa_shared(eb, 0));
                                      }
                                    });
      }
    }
    // The staged stores have read their shared-memory source before the CTA's
    // shared memory goes away; their global writes drain on their own.
    if (lane == 0) bulk_wait_read_all();
    __syncwarp();
  }

  tc_fence_before();
  cluster_sync();
  probe_end(p, bars->probe);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

}  // namespace choreo_sm100
