// conv_sm100.cu — implicit-GEMM 2-D convolution on the tcgen05 mainloop.
//
// GEMM view (NHWC activations, KRSC weights, NHWC output):
//   M = N*P*Q output pixels, N_gemm = K output channels, K_gemm = R*S*C.
// K is walked as (r, s, 64-channel block). For each k-block:
//   A tile (128 pixels x 64 channels) comes from one im2col-mode TMA load:
//     the tensor map's bounding box is the set of filter base positions
//     (lower corner -pad, upper corner pad - (filter-1)*dilation), the load
//     starts at the tile's first output pixel and walks 128 pixels through
//     that box (wrapping rows and images), each pixel shifted by the filter
//     offset (s*dil_w, r*dil_h). Out-of-image pixels and channels >= C read
//     as zero, which is the zero padding of the convolution.
//   B tile (BN output channels x 64 channels) is a 3-D tiled load of the
//     weights viewed as [K][R*S][C].
// Both land as K-major 128-byte-swizzled tiles, exactly like a row-major GEMM,
// so the MMA issuer and the fused bias/ReLU epilogue are the GEMM's.
//
// Semantics follow the reference's only convolution code,
// benchmark/kernels/gemm_example.cu:208-253 (direct conv with stride and
// zero padding, KCRS weights, NCHW), restated for NHWC/KRSC.
#include <algorithm>

#include "internal.h"
#include "tc_kernel.cuh"

namespace choreo_sm100 {

__device__ __forceinline__ void tma_load_im2col_4d(uint32_t dst, const CUtensorMap* map,
                                                   uint32_t bar, int32_t c, int32_t w, int32_t h,
                                                   int32_t n, uint16_t off_w, uint16_t off_h,
                                                   uint64_t cache_hint) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.im2col.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%3, %4, %5, %6}], [%2], {%7, %8}, %9;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c), "r"(w), "r"(h), "r"(n),
      "h"(off_w), "h"(off_h), "l"(cache_hint)
      : "memory");
}

template <int BN>
struct ConvLoader {
  static constexpr bool kAMn = false;
  static constexpr bool kBMn = false;
  __device__ __forceinline__ static void issue(const CUtensorMap* ta, const CUtensorMap* tb,
                                               const TcParams& p, int, int mb, int nb, int kb,
                                               uint32_t dst_a, uint32_t dst_b, uint32_t bar,
                                               uint64_t pol_a, uint64_t pol_b) {
    const int rs = kb / p.conv_c_blocks;
    const int cb = kb - rs * p.conv_c_blocks;
    const int r = rs / p.conv_s;
    const int s = rs - r * p.conv_s;
    const int m0 = mb * kBM;
    const int pq = p.conv_p * p.conv_q;
    const int img = m0 / pq;
    const int rem = m0 - img * pq;
    const int op = rem / p.conv_q;
    const int oq = rem - op * p.conv_q;
    tma_load_im2col_4d(dst_a, ta, bar, cb * 64, oq * p.conv_stride_w - p.conv_pad_w,
                       op * p.conv_stride_h - p.conv_pad_h, img,
                       static_cast<uint16_t>(s * p.conv_dil_w), static_cast<uint16_t>(r * p.conv_dil_h),
                       pol_a);
    tma_load_3d(dst_b, tb, bar, cb * 64, rs, nb * BN, pol_b);
  }
};

}  // namespace choreo_sm100

namespace choreo_impl {
using namespace choreo_sm100;

int encode_tmap_im2col(CUtensorMap* map, CUtensorMapDataType dtype, const void* base,
                       const uint64_t* dims, const uint64_t* strides_bytes, const int* lower,
                       const int* upper, uint32_t channels, uint32_t pixels,
                       const uint32_t* elem_strides);

namespace {

struct ConvGeom {
  int64_t p, q, m, kblocks, c_blocks;
};

ConvGeom geom(const choreo_conv_desc& d) {
  ConvGeom g;
  g.p = (d.h + 2 * d.pad_h - d.dil_h * (d.r - 1) - 1) / d.stride_h + 1;
  g.q = (d.w + 2 * d.pad_w - d.dil_w * (d.s - 1) - 1) / d.stride_w + 1;
  g.m = d.n * g.p * g.q;
  g.c_blocks = (d.c + 63) / 64;
  g.kblocks = d.r * d.s * g.c_blocks;
  return g;
}

int pick_bn(const choreo_conv_desc& d, const ConvGeom& g, int sms) {
  // Same wave-quantisation model as the GEMM; K <= 64 or 128 caps BN.
  const int bns[3] = {256, 128, 64};
  const double eff[3] = {1.0, 0.92, 0.66};
  const int64_t mt = (g.m + kBM - 1) / kBM;
  double best = 1e300;
  int best_bn = 128;
  for (int i = 0; i < 3; ++i) {
    const int bn = bns[i];
    const int64_t nt = (d.k + bn - 1) / bn;
    const int64_t tiles = mt * nt;
    const int64_t waves = (tiles + sms - 1) / sms;
    const double t = static_cast<double>(waves) * (static_cast<double>(g.kblocks) + 4.0) * bn / eff[i];
    if (t < best * 0.97) { best = t; best_bn = bn; }
  }
  return best_bn;
}

constexpr int conv_stages(int bn) { return bn == 256 ? 4 : (bn == 128 ? 6 : 8); }

template <int BN, typename OutT>
int launch_conv_one(const CUtensorMap& ta, const CUtensorMap& tb, const TcParams& kp, int grid,
                    cudaStream_t stream) {
  constexpr int STAGES = conv_stages(BN);
  constexpr int smem = tc_smem_bytes<BN, STAGES>();
  auto kern = tc_gemm_kernel<BN, STAGES, ConvLoader<BN>, OutT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(conv)");
  kern<<<grid, kThreads, smem, stream>>>(ta, tb, kp);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "tcgen05 conv launch");
  return CHOREO_OK;
}

template <typename OutT>
int conv_dispatch_bn(int bn, const CUtensorMap& ta, const CUtensorMap& tb, const TcParams& kp,
                     int grid, cudaStream_t s) {
  switch (bn) {
    case 256: return launch_conv_one<256, OutT>(ta, tb, kp, grid, s);
    case 128: return launch_conv_one<128, OutT>(ta, tb, kp, grid, s);
    default: return launch_conv_one<64, OutT>(ta, tb, kp, grid, s);
  }
}

}  // namespace

int conv_query(const choreo_conv_desc& d, choreo_launch_config* out) {
  const ConvGeom g = geom(d);
  const int sms = current_sm_count();
  const int bn = pick_bn(d, g, sms);
  out->kernel = 3;
  out->tile_m = kBM;
  out->tile_n = bn;
  out->tile_k = kBK;
  out->stages = conv_stages(bn);
  out->cluster_m = 1;
  out->tiles = ((g.m + kBM - 1) / kBM) * ((d.k + bn - 1) / bn);
  out->grid_x = static_cast<int32_t>(std::min<int64_t>(out->tiles, sms));
  out->grid_y = 1;
  out->grid_z = 1;
  out->block_x = kThreads;
  out->smem_bytes = bn == 256 ? tc_smem_bytes<256, conv_stages(256)>()
                  : bn == 128 ? tc_smem_bytes<128, conv_stages(128)>()
                              : tc_smem_bytes<64, conv_stages(64)>();
  out->tmem_cols = 2 * bn;
  out->workspace_bytes = 0;
  return CHOREO_OK;
}

int launch_conv_tc(const choreo_conv_desc& d, cudaStream_t stream) {
  const ConvGeom g = geom(d);
  choreo_launch_config lc{};
  conv_query(d, &lc);
  const int bn = lc.tile_n;
  const CUtensorMapDataType tdt = d.dtype == CHOREO_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                               : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap ta, tb;
  {
    const uint64_t dims[4] = {static_cast<uint64_t>(d.c), static_cast<uint64_t>(d.w),
                              static_cast<uint64_t>(d.h), static_cast<uint64_t>(d.n)};
    const uint64_t strides[3] = {static_cast<uint64_t>(d.c) * 2, static_cast<uint64_t>(d.w * d.c) * 2,
                                 static_cast<uint64_t>(d.h * d.w * d.c) * 2};
    const int lower[2] = {-d.pad_w, -d.pad_h};
    const int upper[2] = {static_cast<int>(d.pad_w - (d.s - 1) * d.dil_w),
                          static_cast<int>(d.pad_h - (d.r - 1) * d.dil_h)};
    const uint32_t estr[4] = {1, static_cast<uint32_t>(d.stride_w), static_cast<uint32_t>(d.stride_h), 1};
    int rc = encode_tmap_im2col(&ta, tdt, d.input, dims, strides, lower, upper, 64, kBM, estr);
    if (rc) return rc;
  }
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(d.c), static_cast<uint64_t>(d.r * d.s),
                              static_cast<uint64_t>(d.k)};
    const uint64_t strides[2] = {static_cast<uint64_t>(d.c) * 2, static_cast<uint64_t>(d.r * d.s * d.c) * 2};
    const uint32_t box[3] = {64, 1, static_cast<uint32_t>(bn)};
    int rc = encode_tmap(&tb, tdt, 3, d.weight, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  TcParams kp{};
  kp.m = static_cast<int32_t>(g.m);
  kp.n = static_cast<int32_t>(d.k);
  kp.num_k_blocks = static_cast<int32_t>(g.kblocks);
  kp.num_m_blocks = static_cast<int32_t>((g.m + kBM - 1) / kBM);
  kp.num_n_blocks = static_cast<int32_t>((d.k + bn - 1) / bn);
  kp.batch = 1;
  kp.num_tiles = static_cast<int64_t>(kp.num_m_blocks) * kp.num_n_blocks;
  kp.group_m = std::max(1, std::min(16, kp.num_m_blocks));
  kp.ab_bf16 = d.dtype == CHOREO_DTYPE_BF16 ? 1 : 0;
  kp.c = d.output;
  kp.ldc = d.k;
  kp.stride_c = 0;
  const int ob = dtype_bytes(d.dtype_out);
  kp.c_vec_ok = ((reinterpret_cast<uintptr_t>(d.output) & 15u) == 0 && (d.k * ob) % 16 == 0) ? 1 : 0;
  kp.alpha = d.alpha;
  kp.beta = 0.f;
  kp.bias = d.bias;
  kp.dtype_bias = d.dtype_bias;
  kp.relu = d.relu;
  kp.conv_c_blocks = static_cast<int32_t>(g.c_blocks);
  kp.conv_s = static_cast<int32_t>(d.s);
  kp.conv_q = static_cast<int32_t>(g.q);
  kp.conv_p = static_cast<int32_t>(g.p);
  kp.conv_pad_w = d.pad_w;
  kp.conv_pad_h = d.pad_h;
  kp.conv_stride_w = d.stride_w;
  kp.conv_stride_h = d.stride_h;
  kp.conv_dil_w = d.dil_w;
  kp.conv_dil_h = d.dil_h;
  kp.status = status_word();
  kp.timeout_ns = wait_timeout_ns();
  if (kp.status == nullptr) return CHOREO_ERR_CUDA;
  const int grid = lc.grid_x;
  switch (d.dtype_out) {
    case CHOREO_DTYPE_F16: return conv_dispatch_bn<__half>(bn, ta, tb, kp, grid, stream);
    case CHOREO_DTYPE_BF16: return conv_dispatch_bn<__nv_bfloat16>(bn, ta, tb, kp, grid, stream);
    case CHOREO_DTYPE_F32: return conv_dispatch_bn<float>(bn, ta, tb, kp, grid, stream);
    default: return fail(CHOREO_ERR_UNSUPPORTED, "conv: unsupported output dtype %d", d.dtype_out);
  }
}

}  // namespace choreo_impl
