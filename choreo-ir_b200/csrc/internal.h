// internal.h — declarations shared by the translation units of libchoreo_b200.so.
// Not installed; the public surface is include/choreo_b200.h.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <atomic>
#include <utility>
#include <cstdint>
#include <cstddef>

#include "../../include/choreo_b200.h"

namespace choreo_impl {

// Records `msg` as this host thread's last error and returns `code`.
int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
// Clears the last error and returns CHOREO_OK.
int ok();
// Converts a CUDA runtime error into CHOREO_ERR_CUDA with context.
int cuda_fail(cudaError_t e, const char* what);

// Raises a kernel's dynamic shared-memory limit once per device: `done` is
// the caller's per-kernel record (bit d set once device d has it).
template <typename Kernel>
int set_smem_limit_once(Kernel kern, int smem, std::atomic<uint64_t>& done, const char* what) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  const uint64_t bit = dev < 64 ? (uint64_t{1} << dev) : 0;
  if (bit != 0 && (done.load(std::memory_order_acquire) & bit) != 0) return CHOREO_OK;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return cuda_fail(e, what);
  done.fetch_or(bit, std::memory_order_release);
  return CHOREO_OK;
}

// Launches `kern` with programmatic stream serialization: the grid may start
// while the previous kernel in the stream is finishing; the kernel's
// griddep_wait() orders its global accesses after that kernel.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// Device status word of the current device (kernel-side failure record).
uint32_t* status_word();
// Per-wait time limit handed to kernels, in nanoseconds.
uint64_t wait_timeout_ns();
// This host thread's clock-probe buffer (choreo_clock_probe_set), or null.
unsigned long long* clock_probe();
// SM count and opt-in shared memory of the current device (cached).
int current_sm_count();
int current_smem_optin();

// 16-bit element tensor-map encoding (TMA, SWIZZLE_128B, zero OOB fill).
// dims/strides follow cuTensorMapEncodeTiled: dims[0] innermost; strides in
// bytes for dims[1..rank-1].
int encode_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base,
                const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                CUtensorMapSwizzle swizzle);

// The settings choreo_tuning_set installed (defaults unless a test or a
// tuning sweep changed them), with a generation number that changes on
// every set so cached plans can tell they are stale.
struct Tuning {
  choreo_tuning t;
  uint64_t generation;
};
Tuning tuning();

// L2 eviction policy codes handed to the kernels (A operand, B operand) and
// the tile rasterisation group: defaults, or the tuning overrides
// (choreo_tuning::l2_policy_a/b, group_m).
struct L2Plan {
  int policy_a, policy_b;
  int group_rows;   // rows of A walked together (group = group_rows / tile rows M tiles)
  int group_m;      // > 0: explicit group in M tiles (tuning override)
};
inline int group_tiles(const L2Plan& p, int tile_rows, int num_m_blocks) {
  int g = p.group_m > 0 ? p.group_m : p.group_rows / tile_rows;
  if (g < 1) g = 1;
  return g < num_m_blocks ? g : num_m_blocks;
}

L2Plan l2_plan();

// ---------------------------------------------------------------- GEMM
// Threads per CTA of every tcgen05 kernel (producer warp, MMA warp, 8
// epilogue warps).
constexpr int kTcThreads = 320;

// Tile configurations of the tcgen05 GEMM (BM = 128, BK = 64).
struct TcConfig {
  bool pair;    // CTA pair (cluster of 2, tcgen05 cta_group::2): 256-row tiles
  bool wide;    // CTA pair with two M halves per CTA: 512 x 256 tiles
  int bn;       // tile N: 64, 128 or 256 (pairs: 128 or 256; wide: 256)
  int stages;   // shared-memory pipeline depth
  int smem;     // dynamic shared memory bytes per CTA
  int group_m;  // rasterisation group (M tiles walked together for L2 reuse)
};
TcConfig select_tc_config(int64_t m, int64_t n, int64_t k, int64_t batch, int sm_count);
inline int tile_rows_of(const TcConfig& c) { return c.wide ? 512 : (c.pair ? 256 : 128); }
// Same choice from the K-block count (the convolution's K is R*S*ceil(C/64) blocks).
TcConfig select_tile_config(int64_t m, int64_t n, int64_t k_blocks, int64_t batch, int sm_count);
// The tile shape and, with allow_split (batch 1), the number of K splits with
// the lowest estimated time; out_bytes is the size of one output element.
struct TilePlan {
  TcConfig cfg{};
  int64_t split = 1;
  double est_us = 0;
};
TilePlan plan_tiles(int64_t m, int64_t n, int64_t k_blocks, int64_t batch, int sm_count, bool allow_split,
                    int out_bytes);

// A GEMM with every operand already TMA-legal (16-byte aligned base, ld and
// batch stride), in the orientation it is stored.
struct TcProblem {
  int64_t m, n, k, batch;
  bool bf16;                 // A/B are bf16 (else f16)
  const void* a; int64_t lda; int64_t stride_a; bool a_mn;   // a_mn: A stored K x M
  const void* b; int64_t ldb; int64_t stride_b; bool b_mn;   // b_mn: B stored K x N
  void* c; int64_t ldc; int64_t stride_c; int dtype_c;
  float alpha, beta;
  const void* bias; int dtype_bias;
  int relu;
  // > 1: K is cut into `split` equal ranges of whole k-blocks, computed as the
  // batch items of one launch (batch must be 1); C is then the fp32 partial
  // buffer [split][m][n] and the epilogue fields must be the identity.
  int64_t split = 1;
};
int launch_gemm_tc(const TcProblem& p, const TcConfig& cfg, cudaStream_t stream);

// Sums `split` fp32 partials [split][m][n] and applies the epilogue
// (alpha, beta * C, bias, ReLU, cast) into C.
int launch_splitk_reduce(const float* partials, int64_t split, int64_t m, int64_t n, void* c, int64_t ldc,
                         int dtype_c, float alpha, float beta, const void* bias, int dtype_bias, int relu,
                         cudaStream_t stream);

// CUDA-core f32 GEMM (A/B/C f32), any strides.
int launch_gemm_f32(const choreo_gemm_desc& d, cudaStream_t stream);

// Strided copy of a batch of rows x cols 16-bit matrices (used to repack an
// operand whose leading dimension or base is not 16-byte aligned).
int launch_repack16(const void* src, int64_t ld_src, int64_t stride_src, void* dst,
                    int64_t ld_dst, int64_t stride_dst, int64_t rows, int64_t cols,
                    int64_t batch, cudaStream_t stream);

// ---------------------------------------------------------------- conv
int conv_query(const choreo_conv_desc& d, choreo_launch_config* out);
int launch_conv_tc(const choreo_conv_desc& d, cudaStream_t stream);

// ---------------------------------------------------------------- elementwise
int launch_relu(int dtype, const void* in, void* out, int64_t n, cudaStream_t s);
int launch_add(int dtype, const void* a, const void* b, void* out, int64_t n, cudaStream_t s);
int launch_fill(int dtype, void* dst, double v, int64_t n, cudaStream_t s);
int launch_convert(int dsrc, const void* src, int ddst, void* dst, int64_t n, cudaStream_t s);

inline int dtype_bytes(int dt) {
  switch (dt) {
    case CHOREO_DTYPE_F16: case CHOREO_DTYPE_BF16: return 2;
    case CHOREO_DTYPE_F32: return 4;
    default: return 0;
  }
}

}  // namespace choreo_impl
