// conv_sm100.cu — implicit-GEMM 2-D convolution on the tcgen05 mainloop.
//
// GEMM view (NHWC activations, KRSC weights, NHWC output):
//   M = N*P*Q output pixels, N_gemm = K output channels, K_gemm = R*S*C.
// K is walked as (r, s, 64-channel block). For each k-block:
//   A tile (128 pixels x 64 channels; 256 for a wide tile's CTA) comes from one
//     im2col-mode TMA load:
//     the tensor map's bounding box is the set of filter base positions
//     (lower corner -pad, upper corner pad - (filter-1)*dilation), the load
//     starts at the tile's first output pixel and walks 128 (256) pixels through
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
#include <cstring>

#include "internal.h"
#include "tc_kernel.cuh"

namespace choreo_sm100 {

// BNL = output channels one CTA stages per k-block; PAIR selects the
// CTA-pair TMA form (bytes counted on the pair leader's barrier).
template <int BNL, bool PAIR>
struct ConvLoader {
  static constexpr bool kAMn = false;
  static constexpr bool kBMn = false;
  // 128 output pixels starting at pixel m0 (NHW order) for k-block kb = (r, s, channel block).
  __device__ __forceinline__ static void issue_a(const CUtensorMap* ta, const TcParams& p, int, int m0, int kb,
                                                 uint32_t dst_a, uint32_t bar, uint64_t pol_a) {
    const int rs = kb / p.conv_c_blocks;
    const int cb = kb - rs * p.conv_c_blocks;
    const int r = rs / p.conv_s;
    const int s = rs - r * p.conv_s;
    const int pq = p.conv_p * p.conv_q;
    const int img = m0 / pq;
    const int rem = m0 - img * pq;
    const int op = rem / p.conv_q;
    const int oq = rem - op * p.conv_q;
    const int w0 = oq * p.conv_stride_w - p.conv_pad_w;
    const int h0 = op * p.conv_stride_h - p.conv_pad_h;
    const uint16_t off_w = static_cast<uint16_t>(s * p.conv_dil_w);
    const uint16_t off_h = static_cast<uint16_t>(r * p.conv_dil_h);
    if constexpr (PAIR)
      tma_load_im2col_4d_pair(dst_a, ta, bar, cb * 64, w0, h0, img, off_w, off_h, pol_a);
    else
      tma_load_im2col_4d(dst_a, ta, bar, cb * 64, w0, h0, img, off_w, off_h, pol_a);
  }
  // Output channels [n0, n0 + BNL) of the weights for k-block kb.
  __device__ __forceinline__ static void issue_b(const CUtensorMap* tb, const TcParams& p, int, int n0, int kb,
                                                 uint32_t dst_b, uint32_t bar, uint64_t pol_b) {
    const int rs = kb / p.conv_c_blocks;
    const int cb = kb - rs * p.conv_c_blocks;
    if constexpr (PAIR)
      tma_load_3d_pair(dst_b, tb, bar, cb * 64, rs, n0, pol_b);
    else
      tma_load_3d(dst_b, tb, bar, cb * 64, rs, n0, pol_b);
  }
  // The wide tile's 256 rows of one CTA: one im2col load, its tensor map
  // encoded with 256 pixels per column for the wide tile (the 128-byte
  // swizzle repeats every 8 rows, so the rows land as two 128-row halves would).
  __device__ __forceinline__ static void issue_a_256(const CUtensorMap* ta, const TcParams& p, int b, int m0,
                                                     int kb, uint32_t dst_a, uint32_t bar, uint64_t pol_a) {
    issue_a(ta, p, b, m0, kb, dst_a, bar, pol_a);
  }
  __device__ __forceinline__ static void issue(const CUtensorMap* ta, const CUtensorMap* tb,
                                               const TcParams& p, int b, int m0, int n0, int kb,
                                               uint32_t dst_a, uint32_t dst_b, uint32_t bar,
                                               uint64_t pol_a, uint64_t pol_b) {
    issue_a(ta, p, b, m0, kb, dst_a, bar, pol_a);
    issue_b(tb, p, b, n0, kb, dst_b, bar, pol_b);
  }
  // The wide tile's per-tile load state: the first output pixel's image and
  // input corner, decomposed once per tile, and the filter tap and channel
  // block of the next k-block, stepped as the producer walks k-blocks 0, 1, ...
  // (channel blocks of one tap, then the next tap) with no division per stage.
  struct WideCursor {
    int img, h0, w0, n0;
    int r, s, cb;
  };
  __device__ __forceinline__ static WideCursor wide_cursor(const TcParams& p, int, int m0, int n0) {
    const int pq = p.conv_p * p.conv_q;
    const int img = m0 / pq;
    const int rem = m0 - img * pq;
    const int op = rem / p.conv_q;
    const int oq = rem - op * p.conv_q;
    return WideCursor{img, op * p.conv_stride_h - p.conv_pad_h, oq * p.conv_stride_w - p.conv_pad_w, n0, 0, 0, 0};
  }
  __device__ __forceinline__ static void issue_wide(const CUtensorMap* ta, const CUtensorMap* tb, const TcParams& p,
                                                    WideCursor& c, int, uint32_t dst_a, uint32_t dst_b,
                                                    uint32_t bar, uint64_t pol_a, uint64_t pol_b) {
    const uint16_t off_w = static_cast<uint16_t>(c.s * p.conv_dil_w);
    const uint16_t off_h = static_cast<uint16_t>(c.r * p.conv_dil_h);
    const int rs = c.r * p.conv_s + c.s;
    if constexpr (PAIR) {
      tma_load_im2col_4d_pair(dst_a, ta, bar, c.cb * 64, c.w0, c.h0, c.img, off_w, off_h, pol_a);
      tma_load_3d_pair(dst_b, tb, bar, c.cb * 64, rs, c.n0, pol_b);
    } else {
      tma_load_im2col_4d(dst_a, ta, bar, c.cb * 64, c.w0, c.h0, c.img, off_w, off_h, pol_a);
      tma_load_3d(dst_b, tb, bar, c.cb * 64, rs, c.n0, pol_b);
    }
    if (++c.cb == p.conv_c_blocks) {
      c.cb = 0;
      if (++c.s == p.conv_s) {
        c.s = 0;
        ++c.r;
      }
    }
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

constexpr int conv_stages(int bn) { return bn == 256 ? 4 : (bn == 128 ? 6 : 8); }
constexpr int conv_pair_stages(int bn) { return bn == 256 ? 6 : 8; }
constexpr int kConvWideStages = 4;

template <typename OutT>
int launch_conv_wide(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const TcParams& kp,
                     int grid, cudaStream_t stream) {
  constexpr int smem = tc_wide_smem_bytes<kConvWideStages>();
  auto kern = tc_gemm_pair_wide_kernel<kConvWideStages, ConvLoader<128, true>, OutT>;
  static std::atomic<uint64_t> attr_done{0};
  if (int rc = set_smem_limit_once(kern, smem, attr_done, "cudaFuncSetAttribute(conv wide)")) return rc;
  cudaError_t e;
  e = launch_pdl(kern, dim3(grid), dim3(kThreads), smem, stream, ta, tb, tc, kp);
  if (e != cudaSuccess) return cuda_fail(e, "tcgen05 wide CTA-pair conv launch");
  return CHOREO_OK;
}

template <int BN, typename OutT>
int launch_conv_one(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const TcParams& kp,
                    int grid, cudaStream_t stream) {
  constexpr int STAGES = conv_stages(BN);
  constexpr int smem = tc_smem_bytes<BN, STAGES>();
  auto kern = tc_gemm_kernel<BN, STAGES, ConvLoader<BN, false>, OutT>;
  static std::atomic<uint64_t> attr_done{0};
  if (int rc = set_smem_limit_once(kern, smem, attr_done, "cudaFuncSetAttribute(conv)")) return rc;
  cudaError_t e;
  e = launch_pdl(kern, dim3(grid), dim3(kThreads), smem, stream, ta, tb, tc, kp);
  if (e != cudaSuccess) return cuda_fail(e, "tcgen05 conv launch");
  return CHOREO_OK;
}

template <int BN, typename OutT>
int launch_conv_pair(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const TcParams& kp,
                     int grid, cudaStream_t stream) {
  constexpr int STAGES = conv_pair_stages(BN);
  constexpr int smem = tc_pair_smem_bytes<BN, STAGES>();
  auto kern = tc_gemm_pair_kernel<BN, STAGES, ConvLoader<BN / 2, true>, OutT>;
  static std::atomic<uint64_t> attr_done{0};
  if (int rc = set_smem_limit_once(kern, smem, attr_done, "cudaFuncSetAttribute(conv pair)")) return rc;
  cudaError_t e;
  e = launch_pdl(kern, dim3(grid), dim3(kThreads), smem, stream, ta, tb, tc, kp);
  if (e != cudaSuccess) return cuda_fail(e, "tcgen05 CTA-pair conv launch");
  return CHOREO_OK;
}

template <typename OutT>
int conv_dispatch(const TcConfig& cfg, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc,
                  const TcParams& kp, int grid, cudaStream_t s) {
  if (cfg.wide) return launch_conv_wide<OutT>(ta, tb, tc, kp, grid, s);
  if (cfg.pair) {
    if (cfg.bn == 256) return launch_conv_pair<256, OutT>(ta, tb, tc, kp, grid, s);
    return launch_conv_pair<128, OutT>(ta, tb, tc, kp, grid, s);
  }
  switch (cfg.bn) {
    case 256: return launch_conv_one<256, OutT>(ta, tb, tc, kp, grid, s);
    case 128: return launch_conv_one<128, OutT>(ta, tb, tc, kp, grid, s);
    default: return launch_conv_one<64, OutT>(ta, tb, tc, kp, grid, s);
  }
}

TcConfig conv_config(const choreo_conv_desc& d, const ConvGeom& g) {
  TcConfig c = select_tile_config(g.m, d.k, g.kblocks, 1, current_sm_count());
  c.stages = c.wide ? kConvWideStages : (c.pair ? conv_pair_stages(c.bn) : conv_stages(c.bn));
  return c;
}

int conv_grid(const TcConfig& c, int64_t tiles) {
  const int sms = current_sm_count();
  return c.pair ? 2 * static_cast<int>(std::min<int64_t>(tiles, sms / 2))
                : static_cast<int>(std::min<int64_t>(tiles, sms));
}

}  // namespace

int conv_query(const choreo_conv_desc& d, choreo_launch_config* out) {
  const ConvGeom g = geom(d);
  const TcConfig c = conv_config(d, g);
  const int64_t rows = tile_rows_of(c);
  out->kernel = 3;
  out->tile_m = static_cast<int32_t>(rows);
  out->tile_n = c.bn;
  out->tile_k = kBK;
  out->stages = c.stages;
  out->cluster_m = c.pair ? 2 : 1;
  out->tiles = ((g.m + rows - 1) / rows) * ((d.k + c.bn - 1) / c.bn);
  out->grid_x = conv_grid(c, out->tiles);
  out->grid_y = 1;
  out->grid_z = 1;
  out->block_x = kThreads;
  out->smem_bytes = c.smem;
  out->tmem_cols = 2 * c.bn;
  out->workspace_bytes = 0;
  out->workspace_min_bytes = 0;
  out->split_k = 1;
  return CHOREO_OK;
}

int launch_conv_tc(const choreo_conv_desc& d, cudaStream_t stream) {
  const ConvGeom g = geom(d);
  const TcConfig cfg = conv_config(d, g);
  const int bn = cfg.bn;
  const int64_t tile_rows = tile_rows_of(cfg);
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
    // pixels per load: the wide tile's CTA takes its 256 rows in one load
    const uint32_t pixels = cfg.wide ? 2 * kBM : kBM;
    int rc = encode_tmap_im2col(&ta, tdt, d.input, dims, strides, lower, upper, 64, pixels, estr);
    if (rc) return rc;
  }
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(d.c), static_cast<uint64_t>(d.r * d.s),
                              static_cast<uint64_t>(d.k)};
    const uint64_t strides[2] = {static_cast<uint64_t>(d.c) * 2, static_cast<uint64_t>(d.r * d.s * d.c) * 2};
    const uint32_t box[3] = {64, 1, static_cast<uint32_t>(cfg.pair ? bn / 2 : bn)};
    int rc = encode_tmap(&tb, tdt, 3, d.weight, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  TcParams kp{};
  kp.m = static_cast<int32_t>(g.m);
  kp.n = static_cast<int32_t>(d.k);
  kp.num_k_blocks = static_cast<int32_t>(g.kblocks);
  kp.num_m_blocks = static_cast<int32_t>((g.m + tile_rows - 1) / tile_rows);
  kp.num_n_blocks = static_cast<int32_t>((d.k + bn - 1) / bn);
  kp.batch = 1;
  kp.num_tiles = static_cast<int64_t>(kp.num_m_blocks) * kp.num_n_blocks;
  const L2Plan l2 = l2_plan();
  kp.group_m = group_tiles(l2, static_cast<int>(tile_rows), kp.num_m_blocks);
  kp.l2_policy_a = l2.policy_a;
  kp.l2_policy_b = l2.policy_b;
  kp.ab_bf16 = d.dtype == CHOREO_DTYPE_BF16 ? 1 : 0;
  kp.c = d.output;
  kp.ldc = d.k;
  kp.stride_c = 0;
  const int ob = dtype_bytes(d.dtype_out);
  kp.c_vec_ok = ((reinterpret_cast<uintptr_t>(d.output) & 15u) == 0 && (d.k * ob) % 16 == 0) ? 1 : 0;
  kp.alpha = d.alpha;
  kp.beta = 0.f;
  CUtensorMap tc;
  std::memset(&tc, 0, sizeof(tc));
  kp.c_tma = 0;
  if (kp.c_vec_ok) {
    const uint64_t elem = static_cast<uint64_t>(ob);
    const uint64_t dims[3] = {static_cast<uint64_t>(d.k), static_cast<uint64_t>(g.m), 1};
    const uint64_t strides[2] = {static_cast<uint64_t>(d.k) * elem, static_cast<uint64_t>(g.m) * d.k * elem};
    const uint32_t box[3] = {static_cast<uint32_t>(128 / elem), 32, 1};
    const CUtensorMapDataType cdt = d.dtype_out == CHOREO_DTYPE_F32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                  : d.dtype_out == CHOREO_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                                    : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    int rc = encode_tmap(&tc, cdt, 3, d.output, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    kp.c_tma = 1;
  }
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
  kp.clock_probe = clock_probe();
  kp.handover_kb = tuning().t.handover_kb;
  if (kp.status == nullptr) return CHOREO_ERR_CUDA;
  const int grid = conv_grid(cfg, kp.num_tiles);
  switch (d.dtype_out) {
    case CHOREO_DTYPE_F16: return conv_dispatch<__half>(cfg, ta, tb, tc, kp, grid, stream);
    case CHOREO_DTYPE_BF16: return conv_dispatch<__nv_bfloat16>(cfg, ta, tb, tc, kp, grid, stream);
    case CHOREO_DTYPE_F32: return conv_dispatch<float>(cfg, ta, tb, tc, kp, grid, stream);
    default: return fail(CHOREO_ERR_UNSUPPORTED, "conv: unsupported output dtype %d", d.dtype_out);
  }
}

}  // namespace choreo_impl
