// capi.cu — the extern "C" surface of libchoreo_b200.so: argument contracts,
// dispatch, workspace planning, tensor-map encoding, the per-device status
// word, and the row-sharded multi-GPU driver.
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "internal.h"

// Kernel-side failure record, one per device context (see sm100.cuh).
__device__ uint32_t g_choreo_status_word;

namespace choreo_impl {

namespace {
thread_local std::string g_last_error;
constexpr int kMaxDevices = 64;

struct DeviceCache {
  std::mutex mu;
  uint32_t* status[kMaxDevices] = {};
  int sm_count[kMaxDevices] = {};
  int smem_optin[kMaxDevices] = {};
};
DeviceCache& cache() {
  static DeviceCache c;
  return c;
}

int current_device_or(int fallback) {
  int dev = fallback;
  if (cudaGetDevice(&dev) != cudaSuccess) return fallback;
  return dev;
}

PFN_cuTensorMapEncodeTiled_v12000 g_encode_tiled = nullptr;
PFN_cuTensorMapEncodeIm2col_v12000 g_encode_im2col = nullptr;
std::once_flag g_encode_once;

int load_encoders() {
  std::call_once(g_encode_once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess && q == cudaDriverEntryPointSuccess)
      g_encode_tiled = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    p = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeIm2col", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess && q == cudaDriverEntryPointSuccess)
      g_encode_im2col = reinterpret_cast<PFN_cuTensorMapEncodeIm2col_v12000>(p);
  });
  if (!g_encode_tiled || !g_encode_im2col)
    return fail(CHOREO_ERR_CUDA, "could not resolve cuTensorMapEncode* from the CUDA driver");
  return CHOREO_OK;
}
}  // namespace

int fail(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int ok() {
  g_last_error.clear();
  return CHOREO_OK;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(CHOREO_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

uint32_t* status_word() {
  const int dev = current_device_or(0);
  if (dev < 0 || dev >= kMaxDevices) {
    fail(CHOREO_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
    return nullptr;
  }
  DeviceCache& c = cache();
  std::lock_guard<std::mutex> lk(c.mu);
  if (c.status[dev] == nullptr) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_choreo_status_word);
    if (e != cudaSuccess) {
      cuda_fail(e, "cudaGetSymbolAddress(status word)");
      return nullptr;
    }
    c.status[dev] = static_cast<uint32_t*>(p);
  }
  return c.status[dev];
}

namespace {
// Process-wide tuning settings. Readers keep a per-thread copy and refresh it
// only when the generation moves, so the common path takes no lock.
std::mutex g_tuning_mu;
choreo_tuning g_tuning = {{0}, 0, 0, -1, -1, 0.0, 0, 0};
std::atomic<uint64_t> g_tuning_gen{1};

bool known_tile(const char* s) {
  static const char* const names[] = {"wide256", "pair256", "pair128", "single256", "single128", "single64"};
  for (const char* n : names)
    if (std::strcmp(s, n) == 0) return true;
  return false;
}
}  // namespace

Tuning tuning() {
  thread_local Tuning cached{{{0}, 0, 0, -1, -1, 0.0, 0, 0}, 0};
  const uint64_t gen = g_tuning_gen.load(std::memory_order_acquire);
  if (cached.generation != gen) {
    std::lock_guard<std::mutex> lk(g_tuning_mu);
    cached.t = g_tuning;
    cached.generation = g_tuning_gen.load(std::memory_order_relaxed);
  }
  return cached;
}

L2Plan l2_plan() {
  // Tiles walk N inside a group of M tiles covering 4096 rows: the group's A
  // panels are reused by every later tile of the group, so A is kept in L2
  // (evict_last); B k-blocks are shared by the tiles of one wave at about the
  // same time (evict_normal: evict_first doubles DRAM reads). Measured on the
  // fp16 8192^3 GEMM with 512 x 256 tiles under the power cap, against
  // cuBLAS on the same box: 96.2 % of its throughput with 4096-row groups,
  // 95.3 % with 2048, 93-94 % with 1024 or 8192 rows; the other eviction
  // hints were 0.5-1.5 % slower.
  L2Plan p{1, 0, 4096, 0};
  const Tuning t = tuning();
  if (t.t.l2_policy_a >= 0) p.policy_a = t.t.l2_policy_a;
  if (t.t.l2_policy_b >= 0) p.policy_b = t.t.l2_policy_b;
  if (t.t.group_m > 0) p.group_m = t.t.group_m;
  return p;
}

uint64_t wait_timeout_ns() {
  const double ms = tuning().t.wait_timeout_ms;
  return static_cast<uint64_t>((ms > 0 ? ms : 2000.0) * 1e6);
}

namespace {
thread_local unsigned long long* g_clock_probe = nullptr;
}  // namespace

unsigned long long* clock_probe() { return g_clock_probe; }

namespace {
void fill_device_cache(int dev) {
  DeviceCache& c = cache();
  std::lock_guard<std::mutex> lk(c.mu);
  if (c.sm_count[dev] == 0) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    c.sm_count[dev] = v > 0 ? v : 148;
    v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    c.smem_optin[dev] = v;
  }
}
}  // namespace

int current_sm_count() {
  const int dev = current_device_or(0);
  if (dev < 0 || dev >= kMaxDevices) return 148;
  fill_device_cache(dev);
  return cache().sm_count[dev];
}

int current_smem_optin() {
  const int dev = current_device_or(0);
  if (dev < 0 || dev >= kMaxDevices) return 0;
  fill_device_cache(dev);
  return cache().smem_optin[dev];
}

int encode_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base,
                const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                CUtensorMapSwizzle swizzle) {
  int rc = load_encoders();
  if (rc) return rc;
  cuuint64_t gd[5];
  cuuint64_t gs[4];
  cuuint32_t bx[5];
  cuuint32_t es[5];
  for (int i = 0; i < rank; ++i) {
    gd[i] = dims[i];
    bx[i] = box[i];
    es[i] = 1;
    if (i + 1 < rank) gs[i] = strides_bytes[i];
  }
  CUresult r = g_encode_tiled(map, dtype, static_cast<cuuint32_t>(rank), const_cast<void*>(base), gd, gs,
                              bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(CHOREO_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d): rank %d dims[0]=%llu box[0]=%u",
                static_cast<int>(r), rank, static_cast<unsigned long long>(dims[0]), box[0]);
  return CHOREO_OK;
}

int encode_tmap_im2col(CUtensorMap* map, CUtensorMapDataType dtype, const void* base,
                       const uint64_t* dims, const uint64_t* strides_bytes, const int* lower,
                       const int* upper, uint32_t channels, uint32_t pixels,
                       const uint32_t* elem_strides) {
  int rc = load_encoders();
  if (rc) return rc;
  cuuint64_t gd[4] = {dims[0], dims[1], dims[2], dims[3]};
  cuuint64_t gs[3] = {strides_bytes[0], strides_bytes[1], strides_bytes[2]};
  cuuint32_t es[4] = {elem_strides[0], elem_strides[1], elem_strides[2], elem_strides[3]};
  CUresult r = g_encode_im2col(map, dtype, 4, const_cast<void*>(base), gd, gs, lower, upper, channels,
                               pixels, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(CHOREO_ERR_CUDA, "cuTensorMapEncodeIm2col failed (%d)", static_cast<int>(r));
  return CHOREO_OK;
}

// ------------------------------------------------------------------ GEMM planning
namespace {

bool is_tc_type(int dt) { return dt == CHOREO_DTYPE_F16 || dt == CHOREO_DTYPE_BF16; }
bool is_float_type(int dt) { return is_tc_type(dt) || dt == CHOREO_DTYPE_F32; }
int64_t round_up(int64_t x, int64_t a) { return (x + a - 1) / a * a; }

// Confirms `p` is memory the current device can read (device, or managed).
int check_device_ptr(const void* p, const char* name) {
  cudaPointerAttributes attr{};
  cudaError_t e = cudaPointerGetAttributes(&attr, p);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(CHOREO_ERR_INVALID_ARG, "%s: not a CUDA allocation (%s)", name, cudaGetErrorString(e));
  }
  if (attr.type == cudaMemoryTypeManaged) return CHOREO_OK;
  if (attr.type != cudaMemoryTypeDevice)
    return fail(CHOREO_ERR_INVALID_ARG, "%s: pointer is host memory; device memory required", name);
  const int dev = current_device_or(-1);
  if (attr.device != dev)
    return fail(CHOREO_ERR_INVALID_ARG, "%s: pointer belongs to device %d, current device is %d", name,
                attr.device, dev);
  return CHOREO_OK;
}

int validate_gemm(const choreo_gemm_desc* d) {
  if (d == nullptr) return fail(CHOREO_ERR_INVALID_ARG, "GEMM: null descriptor");
  if (d->m <= 0 || d->n <= 0 || d->k <= 0)
    return fail(CHOREO_ERR_INVALID_ARG, "GEMM: Invalid matrix dimensions: M=%lld, N=%lld, K=%lld",
                (long long)d->m, (long long)d->n, (long long)d->k);
  if (d->m > INT32_MAX || d->n > INT32_MAX || d->k > INT32_MAX)
    return fail(CHOREO_ERR_UNSUPPORTED, "GEMM: dimensions above 2^31-1 are not supported");
  if (d->batch < 1) return fail(CHOREO_ERR_INVALID_ARG, "GEMM: batch must be >= 1");
  if (d->batch > INT32_MAX) return fail(CHOREO_ERR_UNSUPPORTED, "GEMM: batch above 2^31-1 is not supported");
  if (d->a == nullptr) return fail(CHOREO_ERR_INVALID_ARG, "GEMM: Input tensor A has null data pointer");
  if (d->b == nullptr) return fail(CHOREO_ERR_INVALID_ARG, "GEMM: Input tensor B has null data pointer");
  if (d->c == nullptr) return fail(CHOREO_ERR_INVALID_ARG, "GEMM: Output tensor C has null data pointer");
  if (!is_float_type(d->dtype_ab))
    return fail(CHOREO_ERR_UNSUPPORTED, "GEMM: unsupported input dtype %d", d->dtype_ab);
  if (!is_float_type(d->dtype_c))
    return fail(CHOREO_ERR_UNSUPPORTED, "GEMM: unsupported output dtype %d", d->dtype_c);
  if (d->dtype_ab == CHOREO_DTYPE_F32 && d->dtype_c != CHOREO_DTYPE_F32)
    return fail(CHOREO_ERR_UNSUPPORTED, "GEMM: f32 inputs need an f32 output");
  const int64_t a_inner = d->trans_a ? d->m : d->k;
  const int64_t b_inner = d->trans_b ? d->k : d->n;
  if (d->lda < a_inner)
    return fail(CHOREO_ERR_INVALID_ARG, "GEMM: lda=%lld smaller than %lld", (long long)d->lda, (long long)a_inner);
  if (d->ldb < b_inner)
    return fail(CHOREO_ERR_INVALID_ARG, "GEMM: ldb=%lld smaller than %lld", (long long)d->ldb, (long long)b_inner);
  if (d->ldc < d->n)
    return fail(CHOREO_ERR_INVALID_ARG, "GEMM: ldc=%lld smaller than N=%lld", (long long)d->ldc, (long long)d->n);
  if (d->batch > 1 && (d->stride_a < 0 || d->stride_b < 0 || d->stride_c < 0))
    return fail(CHOREO_ERR_INVALID_ARG, "GEMM: negative batch stride");
  if (d->batch > 1 && d->stride_c < d->m * d->ldc)
    return fail(CHOREO_ERR_INVALID_ARG, "GEMM: batch items of C overlap (stride_c < M*ldc)");
  if (d->bias != nullptr) {
    if (!is_float_type(d->dtype_bias))
      return fail(CHOREO_ERR_UNSUPPORTED, "GEMM: unsupported bias dtype %d", d->dtype_bias);
    if (d->dtype_ab == CHOREO_DTYPE_F32 && d->dtype_bias != CHOREO_DTYPE_F32)
      return fail(CHOREO_ERR_UNSUPPORTED, "GEMM: f32 GEMM needs an f32 bias");
  }
  int rc;
  if ((rc = check_device_ptr(d->a, "GEMM A"))) return rc;
  if ((rc = check_device_ptr(d->b, "GEMM B"))) return rc;
  if ((rc = check_device_ptr(d->c, "GEMM C"))) return rc;
  if (d->bias && (rc = check_device_ptr(d->bias, "GEMM bias"))) return rc;
  return CHOREO_OK;
}

// An operand the TMA cannot address directly gets repacked into the workspace.
struct OperandPlan {
  bool repack = false;
  int64_t outer = 0, inner = 0, ld_pad = 0;
  int64_t bytes = 0, offset = 0;
};

OperandPlan plan_operand(const void* ptr, int64_t ld, int64_t stride, int64_t batch, int64_t outer,
                         int64_t inner) {
  OperandPlan o;
  o.outer = outer;
  o.inner = inner;
  const bool legal = (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0 && (ld * 2) % 16 == 0 &&
                     (batch == 1 || (stride > 0 && (stride * 2) % 16 == 0));
  if (!legal) {
    o.repack = true;
    o.ld_pad = round_up(inner, 8);
    o.bytes = round_up(batch * outer * o.ld_pad * 2, 256);
  }
  return o;
}

struct GemmPlan {
  OperandPlan a, b;
  int64_t workspace = 0;    // required: operand repacks
  TcConfig cfg{};
  // The fastest plan may cut K into `split` ranges computed in parallel
  // (split_cfg) and summed by a second pass; it needs split_bytes of fp32
  // partials in the workspace and runs only when the caller provides them.
  int64_t split = 1;
  TcConfig split_cfg{};
  int64_t split_bytes = 0;
};

int64_t tile_count(const TcConfig& c, int64_t m, int64_t n, int64_t items) {
  const int64_t rows = tile_rows_of(c);
  return ((m + rows - 1) / rows) * ((n + c.bn - 1) / c.bn) * items;
}

GemmPlan plan_tc(const choreo_gemm_desc& d) {
  GemmPlan g;
  g.a = plan_operand(d.a, d.lda, d.stride_a, d.batch, d.trans_a ? d.k : d.m, d.trans_a ? d.m : d.k);
  g.b = plan_operand(d.b, d.ldb, d.stride_b, d.batch, d.trans_b ? d.n : d.k, d.trans_b ? d.k : d.n);
  g.a.offset = 0;
  g.b.offset = g.a.bytes;
  g.workspace = g.a.bytes + g.b.bytes;
  const int sms = current_sm_count();
  const int64_t kb = (d.k + 63) / 64;
  // The fastest plan, possibly with K split, and the unsplit fallback for a
  // caller whose workspace holds no partials; the last shapes planned on
  // this host thread are remembered (the cost model depends on nothing else).
  struct Entry {
    int64_t m, n, kb, batch;
    int out_bytes, sms;
    uint64_t tuning_gen;   // the tuning settings the plan was made under
    TilePlan best;
    TcConfig unsplit;
  };
  thread_local Entry cache[32];
  thread_local int cache_used = 0, cache_next = 0;
  const int out_bytes = dtype_bytes(d.dtype_c);
  const uint64_t gen = tuning().generation;
  const Entry* hit = nullptr;
  for (int i = 0; i < cache_used; ++i) {
    const Entry& e = cache[i];
    if (e.m == d.m && e.n == d.n && e.kb == kb && e.batch == d.batch && e.out_bytes == out_bytes && e.sms == sms &&
        e.tuning_gen == gen) {
      hit = &e;
      break;
    }
  }
  if (hit == nullptr) {
    Entry e{d.m, d.n, kb, d.batch, out_bytes, sms, gen, {}, {}};
    e.best = plan_tiles(d.m, d.n, kb, d.batch, sms, d.batch == 1, out_bytes);
    e.unsplit = e.best.split > 1 ? plan_tiles(d.m, d.n, kb, d.batch, sms, false, out_bytes).cfg : e.best.cfg;
    cache[cache_next] = e;
    hit = &cache[cache_next];
    cache_next = (cache_next + 1) % 32;
    if (cache_used < 32) ++cache_used;
  }
  const TilePlan best = hit->best;
  g.cfg = hit->unsplit;
  if (best.split > 1) {
    g.split = best.split;
    g.split_cfg = best.cfg;
    g.split_bytes = round_up(g.split * d.m * d.n * 4, 256);
  }
  return g;
}

}  // namespace
}  // namespace choreo_impl

using namespace choreo_impl;

extern "C" {

int choreo_version(void) { return 1 * 10000 + 0 * 100 + 0; }

const char* choreo_last_error(void) { return g_last_error.c_str(); }

int choreo_device_props_get(int device, choreo_device_props* out) {
  if (out == nullptr) return fail(CHOREO_ERR_INVALID_ARG, "device props: null output");
  cudaDeviceProp prop{};
  cudaError_t e = cudaGetDeviceProperties(&prop, device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceProperties");
  std::memset(out, 0, sizeof(*out));
  out->device = device;
  out->cc_major = prop.major;
  out->cc_minor = prop.minor;
  out->sm_count = prop.multiProcessorCount;
  out->max_smem_optin = static_cast<int32_t>(prop.sharedMemPerBlockOptin);
  int cl = 0;
  cudaDeviceGetAttribute(&cl, cudaDevAttrClusterLaunch, device);
  out->cluster_launch = cl;
  out->total_mem = static_cast<int64_t>(prop.totalGlobalMem);
  std::snprintf(out->name, sizeof(out->name), "%s", prop.name);
  return ok();
}

int choreo_sync_status(void* stream) {
  cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
  uint32_t* w = status_word();
  if (w == nullptr) return CHOREO_ERR_CUDA;
  uint32_t v = 0;
  e = cudaMemcpy(&v, w, sizeof(v), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "reading the status word");
  if (v != 0) {
    const uint32_t zero = 0;
    cudaMemcpy(w, &zero, sizeof(zero), cudaMemcpyHostToDevice);
    return fail(CHOREO_ERR_TIMEOUT, "a kernel pipeline wait expired (status 0x%x)", v);
  }
  return ok();
}

int choreo_tuning_set(const choreo_tuning* t) {
  choreo_tuning v = {{0}, 0, 0, -1, -1, 0.0, 0, 0};
  if (t != nullptr) {
    v = *t;
    v.tile[sizeof(v.tile) - 1] = 0;
    if (v.tile[0] != 0 && !known_tile(v.tile))
      return fail(CHOREO_ERR_INVALID_ARG, "tuning: unknown tile \"%s\"", v.tile);
    if (v.split_k < 0 || v.split_k > 64) return fail(CHOREO_ERR_INVALID_ARG, "tuning: split_k %d outside 0..64", v.split_k);
    if (v.group_m < 0 || v.group_m > 1024)
      return fail(CHOREO_ERR_INVALID_ARG, "tuning: group_m %d outside 0..1024", v.group_m);
    if (v.l2_policy_a < -1 || v.l2_policy_a > 2 || v.l2_policy_b < -1 || v.l2_policy_b > 2)
      return fail(CHOREO_ERR_INVALID_ARG, "tuning: L2 policy codes are -1, 0, 1 or 2");
    if (!(v.wait_timeout_ms >= 0.0) || v.wait_timeout_ms > 3.6e6)
      return fail(CHOREO_ERR_INVALID_ARG, "tuning: wait_timeout_ms outside 0..3.6e6");
    if (v.handover_kb < 0 || v.handover_kb > 16)
      return fail(CHOREO_ERR_INVALID_ARG, "tuning: handover_kb %d outside 0..16", v.handover_kb);
    v.reserved = 0;
  }
  {
    std::lock_guard<std::mutex> lk(g_tuning_mu);
    g_tuning = v;
    g_tuning_gen.fetch_add(1, std::memory_order_release);
  }
  return ok();
}

int choreo_tuning_get(choreo_tuning* out) {
  if (out == nullptr) return fail(CHOREO_ERR_INVALID_ARG, "tuning: null output");
  *out = tuning().t;
  return ok();
}

int choreo_clock_probe_set(void* probe) {
  if (probe != nullptr) {
    if (reinterpret_cast<uintptr_t>(probe) & 7u)
      return fail(CHOREO_ERR_INVALID_ARG, "clock probe: the buffer must be 8-byte aligned");
    int rc = check_device_ptr(probe, "clock probe");
    if (rc) return rc;
  }
  g_clock_probe = static_cast<unsigned long long*>(probe);
  return ok();
}

int choreo_gemm_query(const choreo_gemm_desc* d, choreo_launch_config* out) {
  int rc = validate_gemm(d);
  if (rc) return rc;
  if (out == nullptr) return fail(CHOREO_ERR_INVALID_ARG, "GEMM query: null output");
  std::memset(out, 0, sizeof(*out));
  const int sms = current_sm_count();
  if (d->dtype_ab == CHOREO_DTYPE_F32) {
    out->kernel = 2;
    out->tile_m = 64;
    out->tile_n = 64;
    out->tile_k = 16;
    out->stages = 1;
    out->cluster_m = 1;
    out->grid_x = static_cast<int32_t>((d->n + 63) / 64);
    out->grid_y = static_cast<int32_t>((d->m + 63) / 64);
    out->grid_z = static_cast<int32_t>(d->batch);
    out->block_x = 256;
    out->smem_bytes = 2 * 16 * 68 * 4;
    out->tiles = static_cast<int64_t>(out->grid_x) * out->grid_y * out->grid_z;
    out->split_k = 1;
    return ok();
  }
  GemmPlan g = plan_tc(*d);
  const TcConfig& c = g.split > 1 ? g.split_cfg : g.cfg;
  out->kernel = 1;
  out->tile_m = static_cast<int32_t>(tile_rows_of(c));
  out->tile_n = c.bn;
  out->tile_k = 64;
  out->stages = c.stages;
  out->cluster_m = c.pair ? 2 : 1;
  out->tiles = tile_count(c, d->m, d->n, g.split > 1 ? g.split : d->batch);
  out->grid_x = c.pair ? 2 * static_cast<int32_t>(std::min<int64_t>(out->tiles, sms / 2))
                       : static_cast<int32_t>(std::min<int64_t>(out->tiles, sms));
  out->grid_y = 1;
  out->grid_z = 1;
  out->block_x = kTcThreads;
  out->smem_bytes = c.smem;
  out->tmem_cols = 2 * c.bn;
  out->workspace_bytes = g.workspace + g.split_bytes;
  out->workspace_min_bytes = g.workspace;
  out->split_k = g.split;
  return ok();
}

int choreo_gemm(const choreo_gemm_desc* d, void* workspace, size_t workspace_bytes, void* stream) {
  int rc = validate_gemm(d);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (d->dtype_ab == CHOREO_DTYPE_F32) {
    rc = launch_gemm_f32(*d, s);
    return rc ? rc : ok();
  }
  GemmPlan g = plan_tc(*d);
  if (g.workspace > 0) {
    if (workspace == nullptr || workspace_bytes < static_cast<size_t>(g.workspace))
      return fail(CHOREO_ERR_WORKSPACE,
                  "GEMM: an operand is not 16-byte aligned (base, leading dimension or batch stride); "
                  "it is repacked into a workspace of %lld bytes, got %zu",
                  (long long)g.workspace, workspace_bytes);
  }
  // The K split runs only when the caller's workspace also holds its partials.
  const bool split = g.split > 1 && workspace != nullptr &&
                     workspace_bytes >= static_cast<size_t>(g.workspace + g.split_bytes);
  if (g.workspace > 0 || split) {
    if ((rc = check_device_ptr(workspace, "GEMM workspace"))) return rc;
    if (reinterpret_cast<uintptr_t>(workspace) & 255u)
      return fail(CHOREO_ERR_WORKSPACE, "GEMM: workspace must be 256-byte aligned");
  }
  TcProblem p{};
  p.m = d->m;
  p.n = d->n;
  p.k = d->k;
  p.batch = d->batch;
  p.bf16 = d->dtype_ab == CHOREO_DTYPE_BF16;
  p.a = d->a;
  p.lda = d->lda;
  p.stride_a = d->stride_a;
  p.a_mn = d->trans_a != 0;
  p.b = d->b;
  p.ldb = d->ldb;
  p.stride_b = d->stride_b;
  p.b_mn = d->trans_b == 0;  // B stored K x N is N-contiguous: MN-major
  if (g.a.repack) {
    void* dst = static_cast<char*>(workspace) + g.a.offset;
    rc = launch_repack16(d->a, d->lda, d->stride_a, dst, g.a.ld_pad, g.a.outer * g.a.ld_pad, g.a.outer,
                         g.a.inner, d->batch, s);
    if (rc) return rc;
    p.a = dst;
    p.lda = g.a.ld_pad;
    p.stride_a = g.a.outer * g.a.ld_pad;
  }
  if (g.b.repack) {
    void* dst = static_cast<char*>(workspace) + g.b.offset;
    rc = launch_repack16(d->b, d->ldb, d->stride_b, dst, g.b.ld_pad, g.b.outer * g.b.ld_pad, g.b.outer,
                         g.b.inner, d->batch, s);
    if (rc) return rc;
    p.b = dst;
    p.ldb = g.b.ld_pad;
    p.stride_b = g.b.outer * g.b.ld_pad;
  }
  if (split) {
    // First pass: fp32 partials [split][m][n] after the repacked operands.
    float* partials = reinterpret_cast<float*>(static_cast<char*>(workspace) + g.workspace);
    p.split = g.split;
    p.c = partials;
    p.ldc = d->n;
    p.stride_c = d->m * d->n;
    p.dtype_c = CHOREO_DTYPE_F32;
    p.alpha = 1.f;
    p.beta = 0.f;
    p.bias = nullptr;
    p.dtype_bias = CHOREO_DTYPE_F32;
    p.relu = 0;
    if ((rc = launch_gemm_tc(p, g.split_cfg, s))) return rc;
    rc = launch_splitk_reduce(partials, g.split, d->m, d->n, d->c, d->ldc, d->dtype_c, d->alpha, d->beta, d->bias,
                              d->dtype_bias, d->relu, s);
    return rc ? rc : ok();
  }
  p.c = d->c;
  p.ldc = d->ldc;
  p.stride_c = d->stride_c;
  p.dtype_c = d->dtype_c;
  p.alpha = d->alpha;
  p.beta = d->beta;
  p.bias = d->bias;
  p.dtype_bias = d->dtype_bias;
  p.relu = d->relu;
  rc = launch_gemm_tc(p, g.cfg, s);
  return rc ? rc : ok();
}

int choreo_shard_rows(int64_t m, int nshards, int rank, int64_t* row0, int64_t* rows) {
  if (m < 0 || nshards < 1 || rank < 0 || rank >= nshards || row0 == nullptr || rows == nullptr)
    return fail(CHOREO_ERR_INVALID_ARG, "shard_rows: bad arguments (m=%lld nshards=%d rank=%d)",
                (long long)m, nshards, rank);
  const int64_t tiles = (m + 127) / 128;
  const int64_t base = tiles / nshards;
  const int64_t extra = tiles % nshards;
  const int64_t t0 = rank * base + std::min<int64_t>(rank, extra);
  const int64_t nt = base + (rank < extra ? 1 : 0);
  const int64_t r0 = std::min<int64_t>(t0 * 128, m);
  const int64_t r1 = std::min<int64_t>((t0 + nt) * 128, m);
  *row0 = r0;
  *rows = r1 - r0;
  return ok();
}

int choreo_gemm_rowsharded(const choreo_gemm_desc* descs, int ngpu, const int* devices,
                           void* const* streams, float* ms_out) {
  if (descs == nullptr || devices == nullptr || ngpu < 1)
    return fail(CHOREO_ERR_INVALID_ARG, "rowsharded GEMM: bad arguments");
  std::vector<int> rcs(ngpu, CHOREO_OK);
  std::vector<std::string> msgs(ngpu);
  std::vector<std::thread> workers;
  workers.reserve(ngpu);
  for (int i = 0; i < ngpu; ++i) {
    workers.emplace_back([&, i] {
      cudaError_t e = cudaSetDevice(devices[i]);
      if (e != cudaSuccess) {
        rcs[i] = cuda_fail(e, "cudaSetDevice");
        msgs[i] = g_last_error;
        return;
      }
      cudaStream_t s = streams ? static_cast<cudaStream_t>(streams[i]) : nullptr;
      if (ms_out == nullptr) {
        rcs[i] = choreo_gemm(&descs[i], nullptr, 0, s);
        msgs[i] = g_last_error;
        return;
      }
      // Timed: ms_out[i] is the shard's device time, or -1 if none was measured.
      ms_out[i] = -1.f;
      cudaEvent_t e0 = nullptr, e1 = nullptr;
      if ((e = cudaEventCreate(&e0)) != cudaSuccess || (e = cudaEventCreate(&e1)) != cudaSuccess) {
        rcs[i] = cuda_fail(e, "cudaEventCreate");
      } else if ((e = cudaEventRecord(e0, s)) != cudaSuccess) {
        rcs[i] = cuda_fail(e, "cudaEventRecord");
      } else {
        rcs[i] = choreo_gemm(&descs[i], nullptr, 0, s);
        if (rcs[i] == CHOREO_OK) {
          float ms = 0.f;
          if ((e = cudaEventRecord(e1, s)) != cudaSuccess)
            rcs[i] = cuda_fail(e, "cudaEventRecord");
          else if ((e = cudaEventSynchronize(e1)) != cudaSuccess)
            rcs[i] = cuda_fail(e, "cudaEventSynchronize");
          else if ((e = cudaEventElapsedTime(&ms, e0, e1)) != cudaSuccess)
            rcs[i] = cuda_fail(e, "cudaEventElapsedTime");
          else
            ms_out[i] = ms;
        }
      }
      if (e0) cudaEventDestroy(e0);
      if (e1) cudaEventDestroy(e1);
      msgs[i] = g_last_error;
    });
  }
  for (auto& t : workers) t.join();
  for (int i = 0; i < ngpu; ++i)
    if (rcs[i] != CHOREO_OK)
      return fail(rcs[i], "rowsharded GEMM: shard %d (device %d): %s", i, devices[i], msgs[i].c_str());
  return ok();
}

// ------------------------------------------------------------------ conv
static int validate_conv(const choreo_conv_desc* d) {
  if (d == nullptr) return fail(CHOREO_ERR_INVALID_ARG, "conv2d: null descriptor");
  if (d->n <= 0 || d->h <= 0 || d->w <= 0 || d->c <= 0 || d->k <= 0 || d->r <= 0 || d->s <= 0)
    return fail(CHOREO_ERR_INVALID_ARG, "conv2d: non-positive dimension");
  if (d->stride_h < 1 || d->stride_w < 1 || d->dil_h < 1 || d->dil_w < 1 || d->pad_h < 0 || d->pad_w < 0)
    return fail(CHOREO_ERR_INVALID_ARG, "conv2d: stride/dilation must be >= 1 and padding >= 0");
  if (d->input == nullptr || d->weight == nullptr || d->output == nullptr)
    return fail(CHOREO_ERR_INVALID_ARG, "conv2d: null data pointer");
  if (!is_tc_type(d->dtype))
    return fail(CHOREO_ERR_UNSUPPORTED, "conv2d: input dtype must be f16 or bf16");
  if (!is_float_type(d->dtype_out)) return fail(CHOREO_ERR_UNSUPPORTED, "conv2d: unsupported output dtype");
  if (d->bias && !is_float_type(d->dtype_bias)) return fail(CHOREO_ERR_UNSUPPORTED, "conv2d: unsupported bias dtype");
  const int64_t p = (d->h + 2 * d->pad_h - d->dil_h * (d->r - 1) - 1) / d->stride_h + 1;
  const int64_t q = (d->w + 2 * d->pad_w - d->dil_w * (d->s - 1) - 1) / d->stride_w + 1;
  if (p <= 0 || q <= 0) return fail(CHOREO_ERR_INVALID_ARG, "conv2d: empty output");
  if (d->c % 8 != 0)
    return fail(CHOREO_ERR_UNSUPPORTED, "conv2d: C=%lld must be a multiple of 8 (16-byte pixel rows)", (long long)d->c);
  if (d->pad_h > 127 || d->pad_w > 127 || d->stride_h > 8 || d->stride_w > 8 ||
      (d->r - 1) * d->dil_h > 255 || (d->s - 1) * d->dil_w > 255)
    return fail(CHOREO_ERR_UNSUPPORTED, "conv2d: padding/stride/filter extent outside the im2col TMA range");
  if (reinterpret_cast<uintptr_t>(d->input) & 15u || reinterpret_cast<uintptr_t>(d->weight) & 15u)
    return fail(CHOREO_ERR_INVALID_ARG, "conv2d: input and weight must be 16-byte aligned");
  if (d->n * p * q > INT32_MAX) return fail(CHOREO_ERR_UNSUPPORTED, "conv2d: too many output pixels");
  int rc;
  if ((rc = check_device_ptr(d->input, "conv2d input"))) return rc;
  if ((rc = check_device_ptr(d->weight, "conv2d weight"))) return rc;
  if ((rc = check_device_ptr(d->output, "conv2d output"))) return rc;
  if (d->bias && (rc = check_device_ptr(d->bias, "conv2d bias"))) return rc;
  return CHOREO_OK;
}

int choreo_conv2d_query(const choreo_conv_desc* d, choreo_launch_config* out) {
  int rc = validate_conv(d);
  if (rc) return rc;
  if (out == nullptr) return fail(CHOREO_ERR_INVALID_ARG, "conv2d query: null output");
  std::memset(out, 0, sizeof(*out));
  rc = conv_query(*d, out);
  return rc ? rc : ok();
}

int choreo_conv2d(const choreo_conv_desc* d, void* workspace, size_t workspace_bytes, void* stream) {
  (void)workspace;
  (void)workspace_bytes;
  int rc = validate_conv(d);
  if (rc) return rc;
  rc = launch_conv_tc(*d, static_cast<cudaStream_t>(stream));
  return rc ? rc : ok();
}

// ------------------------------------------------------------------ elementwise
static int check_elementwise(int32_t dtype, int64_t numel, std::initializer_list<const void*> ptrs) {
  if (dtype_bytes(dtype) == 0) return fail(CHOREO_ERR_UNSUPPORTED, "elementwise: unsupported dtype %d", dtype);
  if (numel < 0) return fail(CHOREO_ERR_INVALID_ARG, "elementwise: negative element count");
  int idx = 0;
  for (const void* p : ptrs) {
    if (p == nullptr) return fail(CHOREO_ERR_INVALID_ARG, "elementwise: Tensor has null data pointer");
    int rc = check_device_ptr(p, idx == 0 ? "elementwise operand 0" : "elementwise operand");
    if (rc) return rc;
    ++idx;
  }
  return CHOREO_OK;
}

int choreo_relu(int32_t dtype, const void* in, void* out, int64_t numel, void* stream) {
  int rc = check_elementwise(dtype, numel, {in, out});
  if (rc) return rc;
  if (numel == 0) return ok();
  rc = launch_relu(dtype, in, out, numel, static_cast<cudaStream_t>(stream));
  return rc ? rc : ok();
}

int choreo_add(int32_t dtype, const void* a, const void* b, void* out, int64_t numel, void* stream) {
  int rc = check_elementwise(dtype, numel, {a, b, out});
  if (rc) return rc;
  if (numel == 0) return ok();
  rc = launch_add(dtype, a, b, out, numel, static_cast<cudaStream_t>(stream));
  return rc ? rc : ok();
}

int choreo_fill(int32_t dtype, void* dst, double value, int64_t numel, void* stream) {
  int rc = check_elementwise(dtype, numel, {dst});
  if (rc) return rc;
  if (numel == 0) return ok();
  rc = launch_fill(dtype, dst, value, numel, static_cast<cudaStream_t>(stream));
  return rc ? rc : ok();
}

int choreo_convert(int32_t dtype_src, const void* src, int32_t dtype_dst, void* dst, int64_t numel,
                   void* stream) {
  int rc = check_elementwise(dtype_src, numel, {src, dst});
  if (rc) return rc;
  if (dtype_bytes(dtype_dst) == 0) return fail(CHOREO_ERR_UNSUPPORTED, "convert: unsupported dtype %d", dtype_dst);
  if (numel == 0) return ok();
  rc = launch_convert(dtype_src, src, dtype_dst, dst, numel, static_cast<cudaStream_t>(stream));
  return rc ? rc : ok();
}

int choreo_tensor_map_encode(void* map, int32_t dtype, int32_t rank, const void* base, const int64_t* dims,
                             const int64_t* strides_bytes, const uint32_t* box, int32_t swizzle_bytes) {
  const int eb = dtype_bytes(dtype);
  if (map == nullptr || base == nullptr || dims == nullptr || box == nullptr)
    return fail(CHOREO_ERR_INVALID_ARG, "tensor map: null argument");
  if ((reinterpret_cast<uintptr_t>(map) & 63u) != 0)
    return fail(CHOREO_ERR_INVALID_ARG, "tensor map: the map must be 64-byte aligned");
  if (eb == 0) return fail(CHOREO_ERR_UNSUPPORTED, "tensor map: unsupported dtype %d", dtype);
  if (rank < 1 || rank > 5) return fail(CHOREO_ERR_INVALID_ARG, "tensor map: rank %d outside 1..5", rank);
  if (rank > 1 && strides_bytes == nullptr) return fail(CHOREO_ERR_INVALID_ARG, "tensor map: null strides");
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0)
    return fail(CHOREO_ERR_INVALID_ARG, "tensor map: base address is not 16-byte aligned");
  for (int i = 0; i < rank; ++i) {
    if (dims[i] < 1 || dims[i] > (int64_t{1} << 32))
      return fail(CHOREO_ERR_INVALID_ARG, "tensor map: dims[%d] = %lld outside 1..2^32", i,
                  static_cast<long long>(dims[i]));
    if (box[i] < 1 || box[i] > 256)
      return fail(CHOREO_ERR_INVALID_ARG, "tensor map: box[%d] = %u outside 1..256", i, box[i]);
    if (i + 1 < rank && (strides_bytes[i] <= 0 || strides_bytes[i] % 16 != 0))
      return fail(CHOREO_ERR_INVALID_ARG, "tensor map: strides_bytes[%d] = %lld is not a positive multiple of 16", i,
                  static_cast<long long>(strides_bytes[i]));
  }
  const int64_t inner = static_cast<int64_t>(box[0]) * eb;
  if (inner % 16 != 0)
    return fail(CHOREO_ERR_INVALID_ARG, "tensor map: box[0] * element size = %lld bytes is not a multiple of 16",
                static_cast<long long>(inner));
  CUtensorMapSwizzle sw;
  switch (swizzle_bytes) {
    case 0: sw = CU_TENSOR_MAP_SWIZZLE_NONE; break;
    case 32: sw = CU_TENSOR_MAP_SWIZZLE_32B; break;
    case 64: sw = CU_TENSOR_MAP_SWIZZLE_64B; break;
    case 128: sw = CU_TENSOR_MAP_SWIZZLE_128B; break;
    default: return fail(CHOREO_ERR_INVALID_ARG, "tensor map: swizzle_bytes %d not 0, 32, 64 or 128", swizzle_bytes);
  }
  if (swizzle_bytes != 0 && inner > swizzle_bytes)
    return fail(CHOREO_ERR_INVALID_ARG, "tensor map: a %lld-byte box row exceeds the %d-byte swizzle span",
                static_cast<long long>(inner), swizzle_bytes);
  const CUtensorMapDataType tdt = dtype == CHOREO_DTYPE_F32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                  : dtype == CHOREO_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                               : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  uint64_t d[5], st[4];
  for (int i = 0; i < rank; ++i) {
    d[i] = static_cast<uint64_t>(dims[i]);
    if (i + 1 < rank) st[i] = static_cast<uint64_t>(strides_bytes[i]);
  }
  int rc = encode_tmap(static_cast<CUtensorMap*>(map), tdt, rank, base, d, st, box, sw);
  return rc ? rc : ok();
}

}  // extern "C"
