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
#include <cstdlib>
#include <cstring>

#include "internal.h"
#include "tc_kernel.cuh"

namespace choreo_sm100 {

// 3-D tiled load through the single-CTA or the CTA-pair form.
template <bool PAIR>
__device__ __forceinline__ void load3(uint32_t dst, const CUtensorMap* map, uint32_t bar, int32_t c0, int32_t c1,
                                      int32_t c2, uint64_t pol) {
  if constexpr (PAIR)
    tma_load_3d_pair(dst, map, bar, c0, c1, c2, pol);
  else
    tma_load_3d(dst, map, bar, c0, c1, c2, pol);
}

// BNL = B columns one CTA stages per k-block (the tile's N for a single CTA,
// half of it for a CTA pair).
template <bool A_MN, bool B_MN, int BNL, bool PAIR>
struct GemmLoader {
  static constexpr bool kAMn = A_MN;
  static constexpr bool kBMn = B_MN;
  // With a K split (p.split_kb > 0) the batch index b selects k-blocks
  // [b * split_kb, (b + 1) * split_kb) of the single operand pair.
  __device__ __forceinline__ static int k_origin(const TcParams& p, int b, int kb) {
    return (p.split_kb > 0 ? b * p.split_kb + kb : kb) * kBK;
  }
  __device__ __forceinline__ static int batch_of(const TcParams& p, int b) { return p.split_kb > 0 ? 0 : b; }
  // A rows [m0, m0 + 128) of k-block kb.
  __device__ __forceinline__ static void issue_a(const CUtensorMap* ta, const TcParams& p, int b0, int m0, int kb,
                                                 uint32_t dst_a, uint32_t bar, uint64_t pol_a) {
    const int k0 = k_origin(p, b0, kb);
    const int b = batch_of(p, b0);
    if constexpr (!A_MN) {
      load3<PAIR>(dst_a, ta, bar, k0, m0, b, pol_a);
    } else {
      load3<PAIR>(dst_a, ta, bar, m0, k0, b, pol_a);
      load3<PAIR>(dst_a + 8192, ta, bar, m0 + 64, k0, b, pol_a);
    }
  }
  // A rows [m0, m0 + 256) of k-block kb (the wide tile's two halves of one
  // CTA): one 256-row box when K-major, four 64-row chunks when MN-major.
  __device__ __forceinline__ static void issue_a_256(const CUtensorMap* ta, const TcParams& p, int b0, int m0,
                                                     int kb, uint32_t dst_a, uint32_t bar, uint64_t pol_a) {
    const int k0 = k_origin(p, b0, kb);
    const int b = batch_of(p, b0);
    if constexpr (!A_MN) {
      load3<PAIR>(dst_a, ta, bar, k0, m0, b, pol_a);
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) load3<PAIR>(dst_a + j * 8192, ta, bar, m0 + j * 64, k0, b, pol_a);
    }
  }
  // B columns [n0, n0 + BNL) of k-block kb.
  __device__ __forceinline__ static void issue_b(const CUtensorMap* tb, const TcParams& p, int b0, int n0, int kb,
                                                 uint32_t dst_b, uint32_t bar, uint64_t pol_b) {
    const int k0 = k_origin(p, b0, kb);
    const int b = batch_of(p, b0);
    if constexpr (!B_MN) {
      load3<PAIR>(dst_b, tb, bar, k0, n0, b, pol_b);
    } else {
#pragma unroll
      for (int j = 0; j < BNL / 64; ++j) load3<PAIR>(dst_b + j * 8192, tb, bar, n0 + j * 64, k0, b, pol_b);
    }
  }
  __device__ __forceinline__ static void issue(const CUtensorMap* ta, const CUtensorMap* tb,
                                               const TcParams& p, int b, int m0, int n0, int kb,
                                               uint32_t dst_a, uint32_t dst_b, uint32_t bar,
                                               uint64_t pol_a, uint64_t pol_b) {
    issue_a(ta, p, b, m0, kb, dst_a, bar, pol_a);
    issue_b(tb, p, b, n0, kb, dst_b, bar, pol_b);
  }
  // The wide tile's per-tile load state: the tile's coordinates.
  struct WideCursor {
    int b, m0, n0;
  };
  __device__ __forceinline__ static WideCursor wide_cursor(const TcParams&, int b, int m0, int n0) {
    return WideCursor{b, m0, n0};
  }
  // k-block kb of a wide tile: this CTA's 256 A rows and its B columns.
  __device__ __forceinline__ static void issue_wide(const CUtensorMap* ta, const CUtensorMap* tb, const TcParams& p,
                                                    WideCursor& c, int kb, uint32_t dst_a, uint32_t dst_b,
                                                    uint32_t bar, uint64_t pol_a, uint64_t pol_b) {
    issue_a_256(ta, p, c.b, c.m0, kb, dst_a, bar, pol_a);
    issue_b(tb, p, c.b, c.n0, kb, dst_b, bar, pol_b);
  }
};

}  // namespace choreo_sm100

namespace choreo_impl {
using namespace choreo_sm100;
static_assert(kThreads == kTcThreads, "launch width and reported block size must agree");

namespace {

constexpr int stages_for(int bn) { return bn == 256 ? 4 : (bn == 128 ? 6 : 8); }
constexpr int pair_stages_for(int bn) { return bn == 256 ? 6 : 8; }
constexpr int kWideStages = 4;

template <int BN, bool A_MN, bool B_MN, typename OutT>
int launch_one(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const TcParams& kp, int grid,
               cudaStream_t stream) {
  constexpr int STAGES = stages_for(BN);
  constexpr int smem = tc_smem_bytes<BN, STAGES>();
  auto kern = tc_gemm_kernel<BN, STAGES, GemmLoader<A_MN, B_MN, BN, false>, OutT>;
  static std::atomic<uint64_t> attr_done{0};
  if (int rc = set_smem_limit_once(kern, smem, attr_done, "cudaFuncSetAttribute(gemm)")) return rc;
  cudaError_t e;
  e = launch_pdl(kern, dim3(grid), dim3(kThreads), smem, stream, ta, tb, tc, kp);
  if (e != cudaSuccess) return cuda_fail(e, "tcgen05 GEMM launch");
  return CHOREO_OK;
}

template <int BN, bool A_MN, bool B_MN, typename OutT>
int launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const TcParams& kp, int grid,
                cudaStream_t stream) {
  constexpr int STAGES = pair_stages_for(BN);
  constexpr int smem = tc_pair_smem_bytes<BN, STAGES>();
  auto kern = tc_gemm_pair_kernel<BN, STAGES, GemmLoader<A_MN, B_MN, BN / 2, true>, OutT>;
  static std::atomic<uint64_t> attr_done{0};
  if (int rc = set_smem_limit_once(kern, smem, attr_done, "cudaFuncSetAttribute(gemm pair)")) return rc;
  cudaError_t e;
  e = launch_pdl(kern, dim3(grid), dim3(kThreads), smem, stream, ta, tb, tc, kp);
  if (e != cudaSuccess) return cuda_fail(e, "tcgen05 CTA-pair GEMM launch");
  return CHOREO_OK;
}

template <bool A_MN, bool B_MN, typename OutT>
int launch_wide(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const TcParams& kp,
                int grid, cudaStream_t stream) {
  constexpr int smem = tc_wide_smem_bytes<kWideStages>();
  auto kern = tc_gemm_pair_wide_kernel<kWideStages, GemmLoader<A_MN, B_MN, 128, true>, OutT>;
  static std::atomic<uint64_t> attr_done{0};
  if (int rc = set_smem_limit_once(kern, smem, attr_done, "cudaFuncSetAttribute(gemm wide)")) return rc;
  cudaError_t e;
  e = launch_pdl(kern, dim3(grid), dim3(kThreads), smem, stream, ta, tb, tc, kp);
  if (e != cudaSuccess) return cuda_fail(e, "tcgen05 wide CTA-pair GEMM launch");
  return CHOREO_OK;
}

template <typename OutT>
int dispatch_wide(bool a_mn, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc,
                  const TcParams& kp, int grid, cudaStream_t s) {
  if (!a_mn && !b_mn) return launch_wide<false, false, OutT>(ta, tb, tc, kp, grid, s);
  if (!a_mn && b_mn) return launch_wide<false, true, OutT>(ta, tb, tc, kp, grid, s);
  if (a_mn && !b_mn) return launch_wide<true, false, OutT>(ta, tb, tc, kp, grid, s);
  return launch_wide<true, true, OutT>(ta, tb, tc, kp, grid, s);
}

template <bool PAIR, int BN, typename OutT>
int dispatch_major(bool a_mn, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc,
                   const TcParams& kp, int grid, cudaStream_t s) {
  if constexpr (PAIR) {
    if (!a_mn && !b_mn) return launch_pair<BN, false, false, OutT>(ta, tb, tc, kp, grid, s);
    if (!a_mn && b_mn) return launch_pair<BN, false, true, OutT>(ta, tb, tc, kp, grid, s);
    if (a_mn && !b_mn) return launch_pair<BN, true, false, OutT>(ta, tb, tc, kp, grid, s);
    return launch_pair<BN, true, true, OutT>(ta, tb, tc, kp, grid, s);
  } else {
    if (!a_mn && !b_mn) return launch_one<BN, false, false, OutT>(ta, tb, tc, kp, grid, s);
    if (!a_mn && b_mn) return launch_one<BN, false, true, OutT>(ta, tb, tc, kp, grid, s);
    if (a_mn && !b_mn) return launch_one<BN, true, false, OutT>(ta, tb, tc, kp, grid, s);
    return launch_one<BN, true, true, OutT>(ta, tb, tc, kp, grid, s);
  }
}

template <typename OutT>
int dispatch_bn(const TcConfig& cfg, bool a_mn, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb,
                const CUtensorMap& tc, const TcParams& kp, int grid, cudaStream_t s) {
  if (cfg.wide) return dispatch_wide<OutT>(a_mn, b_mn, ta, tb, tc, kp, grid, s);
  if (cfg.pair) {
    if (cfg.bn == 256) return dispatch_major<true, 256, OutT>(a_mn, b_mn, ta, tb, tc, kp, grid, s);
    return dispatch_major<true, 128, OutT>(a_mn, b_mn, ta, tb, tc, kp, grid, s);
  }
  switch (cfg.bn) {
    case 256: return dispatch_major<false, 256, OutT>(a_mn, b_mn, ta, tb, tc, kp, grid, s);
    case 128: return dispatch_major<false, 128, OutT>(a_mn, b_mn, ta, tb, tc, kp, grid, s);
    default: return dispatch_major<false, 64, OutT>(a_mn, b_mn, ta, tb, tc, kp, grid, s);
  }
}

}  // namespace

TcConfig select_tc_config(int64_t m, int64_t n, int64_t k, int64_t batch, int sm_count) {
  return select_tile_config(m, n, (k + kBK - 1) / kBK, batch, sm_count);
}

namespace {
TcConfig make_config(bool pair, bool wide, int bn) {
  TcConfig c{};
  c.pair = pair;
  c.wide = wide;
  c.bn = bn;
  if (c.wide) {
    c.stages = kWideStages;
    c.smem = tc_wide_smem_bytes<kWideStages>();
  } else if (c.pair) {
    c.stages = pair_stages_for(c.bn);
    c.smem = c.bn == 256 ? tc_pair_smem_bytes<256, pair_stages_for(256)>()
                         : tc_pair_smem_bytes<128, pair_stages_for(128)>();
  } else {
    c.stages = stages_for(c.bn);
    c.smem = c.bn == 256 ? tc_smem_bytes<256, stages_for(256)>()
           : c.bn == 128 ? tc_smem_bytes<128, stages_for(128)>()
                         : tc_smem_bytes<64, stages_for(64)>();
  }
  c.group_m = 0;
  return c;
}
}  // namespace

TilePlan plan_tiles(int64_t m, int64_t n, int64_t k_blocks, int64_t batch, int sm_count, bool allow_split,
                    int out_bytes) {
  // Candidates: wide CTA pairs (512 x 256 tiles on 2 SMs), CTA pairs
  // (256 x BN) and single CTAs (128 x BN). A tile puts rows_per_sm x BN
  // outputs on each SM, `area` = rows_per_sm * BN / (128 * 256) slabs. One
  // k-block of a 128 x 256 slab takes kSlabUs / eff on one SM; `fixed` is the
  // per-tile pipeline fill in k-blocks and `epi` the time to drain, convert
  // and store one slab, in k-blocks. Accumulators go back to the MMA issuer as
  // soon as they are read, so mainloop and epilogue overlap: a tile costs the
  // larger of the two, the launch costs waves * that plus kLaunchUs. The
  // constants are a least-squares fit (rms log error 0.08) to forced-tile
  // timings on B200 of every candidate at ten shapes: 16384 x 16384 x {64,
  // 128, 256}, 8192 x 8192 x {512, 2048}, 2048^3, 4096^3, 4097 x 3000 x 1536,
  // 1024 x 1024 x 512, 3072 x 3072 x 1024 (operand bytes per FLOP from L2
  // set eff; the pair tiles' epilogue is cheap since the peer CTA hands its
  // accumulator back with a CTA-scope arrive).
  //
  // With allow_split (one batch item), K may also be cut into `split` equal
  // ranges of whole k-blocks (at least 8 each) run as the batch items of one
  // launch, the partials (fp32) then summed by a second pass that costs its
  // bytes at about 5 TB/s plus a launch. The cheapest (tile, split) wins.
  struct Cand { const char* name; bool pair, wide; int bn; double eff, fixed, epi; };
  const Cand cands[6] = {{"wide256", true, true, 256, 1.21, 3.3, 4.1},
                         {"pair256", true, false, 256, 1.01, 2.3, 4.4},
                         {"single256", false, false, 256, 0.89, 2.5, 2.2},
                         {"pair128", true, false, 128, 0.55, 1.3, 5.7},
                         {"single128", false, false, 128, 0.61, 1.4, 5.6},
                         {"single64", false, false, 64, 0.33, 0.9, 11.4}};
  constexpr double kSlabUs = 0.435;          // one k-block of a 128 x 256 slab at eff 1
  constexpr double kLaunchUs = 6.0;          // launch, ramp and the last tile's drain
  constexpr double kReduceBytesPerUs = 5.0e6;
  constexpr double kReduceLaunchUs = 3.0;
  const Tuning tu = tuning();  // forced tile name / split count (tests and tuning sweeps)
  const char* force = tu.t.tile[0] != 0 ? tu.t.tile : nullptr;
  const int64_t want_split = tu.t.split_k;
  TilePlan best{};
  best.est_us = 1e300;
  for (const Cand& cd : cands) {
    if (force && std::strcmp(force, cd.name) != 0) continue;
    const int64_t rows = cd.wide ? 4 * kBM : (cd.pair ? 2 * kBM : kBM);
    const int64_t rows_per_sm = cd.wide ? 2 * kBM : kBM;
    const int64_t slots = cd.pair ? sm_count / 2 : sm_count;
    const int64_t tiles1 = ((m + rows - 1) / rows) * ((n + cd.bn - 1) / cd.bn) * batch;
    const double area = static_cast<double>(rows_per_sm * cd.bn) / (kBM * 256.0);
    for (int64_t split = 1; split <= 64; ++split) {
      if (split > 1 && (!allow_split || batch != 1 || k_blocks % split != 0 || k_blocks / split < 8)) continue;
      if (want_split > 0 && split != want_split) continue;
      const int64_t tiles = tiles1 * split;
      const int64_t waves = (tiles + slots - 1) / slots;
      const double kb = static_cast<double>(k_blocks / split);
      const double mainloop = (kb + cd.fixed) / cd.eff;
      const double epi = split > 1 ? cd.epi * 4.0 / out_bytes : cd.epi;  // fp32 partials
      double t = kLaunchUs + static_cast<double>(waves) * area * (mainloop > epi ? mainloop : epi) * kSlabUs;
      if (split > 1)
        t += static_cast<double>(m) * static_cast<double>(n) * (4.0 * split + out_bytes) / kReduceBytesPerUs +
             kReduceLaunchUs;
      if (t < best.est_us * 0.97) {
        best.est_us = t;
        best.cfg = make_config(cd.pair, cd.wide, cd.bn);
        best.split = split;
      }
    }
  }
  if (best.est_us == 1e300) {  // unknown forced name or split: default choice
    best.cfg = make_config(true, false, 256);
    best.split = 1;
  }
  return best;
}

TcConfig select_tile_config(int64_t m, int64_t n, int64_t k_blocks, int64_t batch, int sm_count) {
  return plan_tiles(m, n, k_blocks, batch, sm_count, false, 2).cfg;
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
    const uint32_t box[3] = {64, p.a_mn ? 64u : (cfg.wide ? 256u : 128u), 1};
    int rc = encode_tmap(&ta, tdt, 3, p.a, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  {
    const uint64_t inner = p.b_mn ? p.n : p.k;
    const uint64_t outer = p.b_mn ? p.k : p.n;
    const uint64_t dims[3] = {inner, outer, static_cast<uint64_t>(p.batch)};
    const uint64_t bstride = p.batch > 1 ? p.stride_b * 2 : outer * p.ldb * 2;
    const uint64_t strides[2] = {static_cast<uint64_t>(p.ldb) * 2, bstride};
    const uint32_t bnl = static_cast<uint32_t>(cfg.pair ? cfg.bn / 2 : cfg.bn);
    const uint32_t box[3] = {64, p.b_mn ? 64u : bnl, 1};
    int rc = encode_tmap(&tb, tdt, 3, p.b, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }

  TcParams kp{};
  kp.m = static_cast<int32_t>(p.m);
  kp.n = static_cast<int32_t>(p.n);
  const int64_t kblocks = (p.k + kBK - 1) / kBK;
  const int64_t items = p.split > 1 ? p.split : p.batch;  // scheduler batch: K splits or batch items
  if (p.split > 1 && (p.batch != 1 || kblocks % p.split != 0))
    return fail(CHOREO_ERR_INVALID_ARG, "split-K launch: batch %lld, %lld k-blocks over %lld splits",
                (long long)p.batch, (long long)kblocks, (long long)p.split);
  kp.num_k_blocks = static_cast<int32_t>(kblocks / (p.split > 1 ? p.split : 1));
  kp.split_kb = p.split > 1 ? kp.num_k_blocks : 0;
  const int64_t tile_rows = tile_rows_of(cfg);
  kp.num_m_blocks = static_cast<int32_t>((p.m + tile_rows - 1) / tile_rows);
  kp.num_n_blocks = static_cast<int32_t>((p.n + cfg.bn - 1) / cfg.bn);
  kp.batch = static_cast<int32_t>(items);
  kp.num_tiles = static_cast<int64_t>(kp.num_m_blocks) * kp.num_n_blocks * items;
  const L2Plan l2 = l2_plan();
  kp.group_m = group_tiles(l2, static_cast<int>(tile_rows), kp.num_m_blocks);
  kp.l2_policy_a = l2.policy_a;
  kp.l2_policy_b = l2.policy_b;
  kp.ab_bf16 = p.bf16 ? 1 : 0;
  kp.c = p.c;
  kp.ldc = p.ldc;
  kp.stride_c = p.stride_c;
  const int cb = dtype_bytes(p.dtype_c);
  kp.c_vec_ok = ((reinterpret_cast<uintptr_t>(p.c) & 15u) == 0 && (p.ldc * cb) % 16 == 0 &&
                 (items == 1 || (p.stride_c * cb) % 16 == 0))
                    ? 1
                    : 0;
  kp.alpha = p.alpha;
  kp.beta = p.beta;
  kp.bias = p.bias;
  kp.dtype_bias = p.dtype_bias;
  kp.relu = p.relu;
  // The kernels store C through a staging tile and bulk tensor stores when C
  // is TMA-addressable (16-byte aligned base, leading dimension and batch stride).
  CUtensorMap tc;
  std::memset(&tc, 0, sizeof(tc));
  kp.c_tma = 0;
  if (kp.c_vec_ok) {
    const uint64_t elem = static_cast<uint64_t>(cb);
    const uint64_t dims[3] = {static_cast<uint64_t>(p.n), static_cast<uint64_t>(p.m), static_cast<uint64_t>(items)};
    const uint64_t bstride = items > 1 ? static_cast<uint64_t>(p.stride_c) * elem
                                         : static_cast<uint64_t>(p.m) * static_cast<uint64_t>(p.ldc) * elem;
    const uint64_t strides[2] = {static_cast<uint64_t>(p.ldc) * elem, bstride};
    const uint32_t box[3] = {static_cast<uint32_t>(128 / elem), 32, 1};
    const CUtensorMapDataType cdt = p.dtype_c == CHOREO_DTYPE_F32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                  : p.dtype_c == CHOREO_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                                   : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    int rc = encode_tmap(&tc, cdt, 3, p.c, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    kp.c_tma = 1;
  }
  kp.status = status_word();
  kp.timeout_ns = wait_timeout_ns();
  kp.clock_probe = clock_probe();
  kp.handover_kb = tuning().t.handover_kb;
  if (kp.status == nullptr) return CHOREO_ERR_CUDA;

  const int sms = current_sm_count();
  const int grid = cfg.pair ? 2 * static_cast<int>(std::min<int64_t>(kp.num_tiles, sms / 2))
                            : static_cast<int>(std::min<int64_t>(kp.num_tiles, sms));
  switch (p.dtype_c) {
    case CHOREO_DTYPE_F16: return dispatch_bn<__half>(cfg, p.a_mn, p.b_mn, ta, tb, tc, kp, grid, stream);
    case CHOREO_DTYPE_BF16:
      return dispatch_bn<__nv_bfloat16>(cfg, p.a_mn, p.b_mn, ta, tb, tc, kp, grid, stream);
    case CHOREO_DTYPE_F32: return dispatch_bn<float>(cfg, p.a_mn, p.b_mn, ta, tb, tc, kp, grid, stream);
    default: return fail(CHOREO_ERR_UNSUPPORTED, "unsupported output dtype %d", p.dtype_c);
  }
}

// ------------------------------------------------------------------ repack
namespace {
// dst rows are ld_dst (a multiple of 8) elements, 16-byte aligned: each
// thread writes 8 elements with one 16-byte store; the source rows may sit at
// any 2-byte alignment, so they are read element by element (coalesced across
// the warp, served from L1).
__global__ void repack16_kernel(const uint16_t* __restrict__ src, int64_t ld_src, int64_t stride_src,
                                uint16_t* __restrict__ dst, int64_t ld_dst, int64_t stride_dst,
                                int64_t rows, int64_t cols) {
  griddep_launch_dependents();  // the GEMM that reads the repack may start its prologue
  const int64_t b = blockIdx.z;
  const uint16_t* s = src + b * stride_src;
  uint16_t* d = dst + b * stride_dst;
  const int64_t chunks = ld_dst / 8;
  const int64_t total = rows * chunks;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / chunks;
    const int64_t c0 = (i - r * chunks) * 8;
    const uint16_t* srow = s + r * ld_src;
    uint32_t w[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const uint32_t lo = c0 + 2 * e < cols ? srow[c0 + 2 * e] : 0u;
      const uint32_t hi = c0 + 2 * e + 1 < cols ? srow[c0 + 2 * e + 1] : 0u;
      w[e] = lo | (hi << 16);
    }
    *reinterpret_cast<uint4*>(d + r * ld_dst + c0) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}
}  // namespace

int launch_repack16(const void* src, int64_t ld_src, int64_t stride_src, void* dst, int64_t ld_dst,
                    int64_t stride_dst, int64_t rows, int64_t cols, int64_t batch,
                    cudaStream_t stream) {
  if (batch > 65535) return fail(CHOREO_ERR_UNSUPPORTED, "repack: batch %lld > 65535", (long long)batch);
  if (ld_dst % 8 != 0) return fail(CHOREO_ERR_INVALID_ARG, "repack: destination ld %lld not a multiple of 8",
                                   (long long)ld_dst);
  dim3 block(256);
  const int64_t work = rows * (ld_dst / 8);
  dim3 grid(static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>((work + 255) / 256,
                                                                         int64_t{8} * current_sm_count()))),
            1, static_cast<unsigned>(batch));
  repack16_kernel<<<grid, block, 0, stream>>>(static_cast<const uint16_t*>(src), ld_src, stride_src,
                                              static_cast<uint16_t*>(dst), ld_dst, stride_dst, rows,
                                              cols);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "repack launch");
  return CHOREO_OK;
}

}  // namespace choreo_impl
