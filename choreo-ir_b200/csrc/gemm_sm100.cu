// gemm_sm100.cu — tcgen05 GEMM: the TMA loader for (batched) row-major
// operands in any of the NN / NT / TN / TT orientations, the tile
// configuration choice, and the host launch.
//
// Orientation is handled entirely by the TMA descriptors and the UMMA
// majorness bits, never by a transpose pass:
//   A stored M x K (K contiguous)  -> K-major tile, one 64 x 128 box
//   A stored K x M (M contiguous)  -> MN-major tile, two 64 x 64 boxes
//   B stored N x K (K contiguous)  -> K-major tile, one 64 x BN box
//   B stored K x N (N contiguous)  -> MN-major tile, BN/64 boxes of 64 x 64
// Out-of-range rows/columns/K of a ragged problem read as zero (TMA OOB fill)
// and the epilogue predicates its stores, which is how the reference's
// tile() boundary handling (tensor/layout.hpp:201-209) is realised here.
#include <algorithm>
#include <cstdio>

#include "internal.h"
#include "tc_kernel.cuh"

namespace choreo_sm100 {

template <bool A_MN, bool B_MN, int BN>
struct GemmLoader {
  static constexpr bool kAMn = A_MN;
  static constexpr bool kBMn = B_MN;
  __device__ __forceinline__ static void issue(const CUtensorMap* ta, const CUtensorMap* tb,
                                               const TcParams&, int b, int mb, int nb, int kb,
                                               uint32_t dst_a, uint32_t dst_b, uint32_t bar,
                                               uint64_t pol_a, uint64_t pol_b) {
    const int k0 = kb * kBK;
    if constexpr (!A_MN) {
      tma_load_3d(dst_a, ta, bar, k0, mb * kBM, b, pol_a);
    } else {
      tma_load_3d(dst_a, ta, bar, mb * kBM, k0, b, pol_a);
      tma_load_3d(dst_a + 8192, ta, bar, mb * kBM + 64, k0, b, pol_a);
    }
    if constexpr (!B_MN) {
      tma_load_3d(dst_b, tb, bar, k0, nb * BN, b, pol_b);
    } else {
#pragma unroll
      for (int j = 0; j < BN / 64; ++j) tma_load_3d(dst_b + j * 8192, tb, bar, nb * BN + j * 64, k0, b, pol_b);
    }
  }
};

}  // namespace choreo_sm100

namespace choreo_impl {
using namespace choreo_sm100;

namespace {

constexpr int stages_for(int bn) { return bn == 256 ? 4 : (bn == 128 ? 6 : 8); }

template <int BN, bool A_MN, bool B_MN, typename OutT>
int launch_one(const CUtensorMap& ta, const CUtensorMap& tb, const TcParams& kp, int grid,
               cudaStream_t stream) {
  constexpr int STAGES = stages_for(BN);
  constexpr int smem = tc_smem_bytes<BN, STAGES>();
  auto kern = tc_gemm_kernel<BN, STAGES, GemmLoader<A_MN, B_MN, BN>, OutT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(gemm)");
  kern<<<grid, kThreads, smem, stream>>>(ta, tb, kp);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "tcgen05 GEMM launch");
  return CHOREO_OK;
}

template <int BN, typename OutT>
int dispatch_major(bool a_mn, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb,
                   const TcParams& kp, int grid, cudaStream_t s) {
  if (!a_mn && !b_mn) return launch_one<BN, false, false, OutT>(ta, tb, kp, grid, s);
  if (!a_mn && b_mn) return launch_one<BN, false, true, OutT>(ta, tb, kp, grid, s);
  if (a_mn && !b_mn) return launch_one<BN, true, false, OutT>(ta, tb, kp, grid, s);
  return launch_one<BN, true, true, OutT>(ta, tb, kp, grid, s);
}

template <typename OutT>
int dispatch_bn(int bn, bool a_mn, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb,
                const TcParams& kp, int grid, cudaStream_t s) {
  switch (bn) {
    case 256: return dispatch_major<256, OutT>(a_mn, b_mn, ta, tb, kp, grid, s);
    case 128: return dispatch_major<128, OutT>(a_mn, b_mn, ta, tb, kp, grid, s);
    default: return dispatch_major<64, OutT>(a_mn, b_mn, ta, tb, kp, grid, s);
  }
}

}  // namespace

TcConfig select_tc_config(int64_t m, int64_t n, int64_t k, int64_t batch, int sm_count) {
  // Relative cost of one 128-row output tile: a 128 x BN x 16 UMMA reads
  // (16 KB/4) of A plus BN*32 B of B from shared memory per 128*BN/... cycles;
  // at BN = 64 shared-memory bandwidth caps the tensor pipe at ~2/3 of peak,
  // at BN = 128 it is borderline, at 256 it is not limiting.
  const int bns[3] = {256, 128, 64};
  const double eff[3] = {1.0, 0.92, 0.66};
  const int64_t mt = (m + kBM - 1) / kBM;
  const int64_t kt = (k + kBK - 1) / kBK;
  double best = 1e300;
  int best_bn = 256;
  for (int i = 0; i < 3; ++i) {
    const int bn = bns[i];
    const int64_t nt = (n + bn - 1) / bn;
    const int64_t tiles = mt * nt * batch;
    const int64_t waves = (tiles + sm_count - 1) / sm_count;
    // per-tile time ~ (pipeline fill + k blocks) at this tile's efficiency
    const double per_tile = (static_cast<double>(kt) + 4.0) * bn / eff[i];
    const double t = static_cast<double>(waves) * per_tile;
    if (t < best * 0.97) { best = t; best_bn = bn; }
  }
  TcConfig c;
  c.bn = best_bn;
  c.stages = stages_for(best_bn);
  c.smem = best_bn == 256 ? tc_smem_bytes<256, stages_for(256)>()
         : best_bn == 128 ? tc_smem_bytes<128, stages_for(128)>()
                          : tc_smem_bytes<64, stages_for(64)>();
  c.group_m = 16;
  return c;
}

int launch_gemm_tc(const TcProblem& p, const TcConfig& cfg, cudaStream_t stream) {
  const CUtensorMapDataType tdt =
      p.bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap ta, tb;
  {
    // A: inner dim is K (K-major) or M (MN-major).
    const uint64_t inner = p.a_mn ? p.m : p.k;
    const uint64_t outer = p.a_mn ? p.k : p.m;
    const uint64_t dims[3] = {inner, outer, static_cast<uint64_t>(p.batch)};
    const uint64_t bstride = p.batch > 1 ? p.stride_a * 2 : outer * p.lda * 2;
    const uint64_t strides[2] = {static_cast<uint64_t>(p.lda) * 2, bstride};
    const uint32_t box[3] = {64, p.a_mn ? 64u : 128u, 1};
    int rc = encode_tmap(&ta, tdt, 3, p.a, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  {
    const uint64_t inner = p.b_mn ? p.n : p.k;
    const uint64_t outer = p.b_mn ? p.k : p.n;
    const uint64_t dims[3] = {inner, outer, static_cast<uint64_t>(p.batch)};
    const uint64_t bstride = p.batch > 1 ? p.stride_b * 2 : outer * p.ldb * 2;
    const uint64_t strides[2] = {static_cast<uint64_t>(p.ldb) * 2, bstride};
    const uint32_t box[3] = {64, p.b_mn ? 64u : static_cast<uint32_t>(cfg.bn), 1};
    int rc = encode_tmap(&tb, tdt, 3, p.b, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }

  TcParams kp{};
  kp.m = static_cast<int32_t>(p.m);
  kp.n = static_cast<int32_t>(p.n);
  kp.num_k_blocks = static_cast<int32_t>((p.k + kBK - 1) / kBK);
  kp.num_m_blocks = static_cast<int32_t>((p.m + kBM - 1) / kBM);
  kp.num_n_blocks = static_cast<int32_t>((p.n + cfg.bn - 1) / cfg.bn);
  kp.batch = static_cast<int32_t>(p.batch);
  kp.num_tiles = static_cast<int64_t>(kp.num_m_blocks) * kp.num_n_blocks * p.batch;
  kp.group_m = std::max(1, std::min(cfg.group_m, kp.num_m_blocks));
  kp.ab_bf16 = p.bf16 ? 1 : 0;
  kp.c = p.c;
  kp.ldc = p.ldc;
  kp.stride_c = p.stride_c;
  const int cb = dtype_bytes(p.dtype_c);
  kp.c_vec_ok = ((reinterpret_cast<uintptr_t>(p.c) & 15u) == 0 && (p.ldc * cb) % 16 == 0 &&
                 (p.batch == 1 || (p.stride_c * cb) % 16 == 0))
                    ? 1
                    : 0;
  kp.alpha = p.alpha;
  kp.beta = p.beta;
  kp.bias = p.bias;
  kp.dtype_bias = p.dtype_bias;
  kp.relu = p.relu;
  kp.status = status_word();
  kp.timeout_ns = wait_timeout_ns();
  if (kp.status == nullptr) return CHOREO_ERR_CUDA;

  const int sms = current_sm_count();
  const int grid = static_cast<int>(std::min<int64_t>(kp.num_tiles, sms));
  switch (p.dtype_c) {
    case CHOREO_DTYPE_F16: return dispatch_bn<__half>(cfg.bn, p.a_mn, p.b_mn, ta, tb, kp, grid, stream);
    case CHOREO_DTYPE_BF16:
      return dispatch_bn<__nv_bfloat16>(cfg.bn, p.a_mn, p.b_mn, ta, tb, kp, grid, stream);
    case CHOREO_DTYPE_F32: return dispatch_bn<float>(cfg.bn, p.a_mn, p.b_mn, ta, tb, kp, grid, stream);
    default: return fail(CHOREO_ERR_UNSUPPORTED, "unsupported output dtype %d", p.dtype_c);
  }
}

// ------------------------------------------------------------------ repack
namespace {
__global__ void repack16_kernel(const uint16_t* __restrict__ src, int64_t ld_src, int64_t stride_src,
                                uint16_t* __restrict__ dst, int64_t ld_dst, int64_t stride_dst,
                                int64_t rows, int64_t cols) {
  const int64_t b = blockIdx.z;
  const uint16_t* s = src + b * stride_src;
  uint16_t* d = dst + b * stride_dst;
  for (int64_t r = blockIdx.y; r < rows; r += gridDim.y) {
    for (int64_t c = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; c < ld_dst;
         c += static_cast<int64_t>(gridDim.x) * blockDim.x) {
      d[r * ld_dst + c] = c < cols ? s[r * ld_src + c] : uint16_t(0);
    }
  }
}
}  // namespace

int launch_repack16(const void* src, int64_t ld_src, int64_t stride_src, void* dst, int64_t ld_dst,
                    int64_t stride_dst, int64_t rows, int64_t cols, int64_t batch,
                    cudaStream_t stream) {
  if (batch > 65535) return fail(CHOREO_ERR_UNSUPPORTED, "repack: batch %lld > 65535", (long long)batch);
  dim3 block(256);
  dim3 grid(static_cast<unsigned>(std::min<int64_t>((ld_dst + 255) / 256, 64)),
            static_cast<unsigned>(std::min<int64_t>(rows, 65535)), static_cast<unsigned>(batch));
  repack16_kernel<<<grid, block, 0, stream>>>(static_cast<const uint16_t*>(src), ld_src, stride_src,
                                              static_cast<uint16_t*>(dst), ld_dst, stride_dst, rows,
                                              cols);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "repack launch");
  return CHOREO_OK;
}

}  // namespace choreo_impl
