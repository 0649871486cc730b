/*
 * choreo_b200.h — C ABI of the B200 (sm_100a) dense-contraction library.
 *
 * Plain pointers, sizes and status codes only: no CUDA, C++ or Python types
 * appear in the signatures (streams are passed as `void*`, i.e. a
 * cudaStream_t or NULL for the legacy default stream). The library never owns
 * caller memory: every device pointer below is allocated and freed by the
 * caller, who keeps ownership.
 *
 * The reference (codes1gn/choreo-ir) is a header-only C++ library with no C
 * ABI; each entry point names the reference interface it stands behind. The
 * C++ front end in include/choreo-ir/ calls these functions and rethrows
 * non-zero status codes as std::runtime_error with the message from
 * choreo_last_error(), which is what the reference's callers expect.
 *
 * Error convention: 0 = success, negative = failure (see choreo_status).
 * Launch-time checks are synchronous; failures inside a kernel (a pipeline
 * wait that ran out of time) are recorded in a per-device status word and
 * reported by choreo_sync_status().
 */
#ifndef CHOREO_B200_H
#define CHOREO_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
typedef enum choreo_status {
  CHOREO_OK = 0,
  CHOREO_ERR_INVALID_ARG = -1,  /* shape/dtype/pointer contract violated */
  CHOREO_ERR_UNSUPPORTED = -2,  /* valid request this build does not implement */
  CHOREO_ERR_CUDA = -3,         /* a CUDA runtime/driver call failed */
  CHOREO_ERR_TIMEOUT = -4,      /* a kernel pipeline wait expired (see choreo_sync_status) */
  CHOREO_ERR_WORKSPACE = -5     /* workspace missing or smaller than the queried size */
} choreo_status;

/* Element types. Values equal the reference's DataType enum
 * (include/choreo-ir/core/types.hpp:58-71) so the C++ front end can pass
 * Tensor<T>::dtype() straight through. */
typedef enum choreo_dtype {
  CHOREO_DTYPE_F16 = 8,
  CHOREO_DTYPE_F32 = 9,
  CHOREO_DTYPE_BF16 = 11
} choreo_dtype;

/* One (optionally batched) GEMM:
 *   C[b] = act(alpha * op(A[b]) * op(B[b]) + beta * C[b] + bias)
 * op(A) is M x K: trans_a == 0 -> A stored M x K row-major with leading
 * dimension lda (>= K); trans_a == 1 -> A stored K x M row-major (lda >= M).
 * op(B) is K x N: trans_b == 0 -> B stored K x N row-major (ldb >= N);
 * trans_b == 1 -> B stored N x K row-major (ldb >= K).
 * C is M x N row-major with leading dimension ldc (>= N).
 * bias (optional, may be NULL) is an N-vector broadcast over rows.
 * act is ReLU when relu != 0, identity otherwise.
 * batch >= 1; stride_* are element strides between consecutive batch items
 * (ignored when batch == 1).
 * Supported types: A/B f16 or bf16 (tensor cores, fp32 accumulation) with C
 * f16, bf16 or f32; or A/B/C all f32 (CUDA cores, fp32 accumulation). */
typedef struct choreo_gemm_desc {
  int64_t m, n, k;
  int32_t dtype_ab;
  int32_t dtype_c;
  const void* a;
  int64_t lda;
  int32_t trans_a;
  const void* b;
  int64_t ldb;
  int32_t trans_b;
  void* c;
  int64_t ldc;
  float alpha;
  float beta;
  const void* bias;
  int32_t dtype_bias;
  int32_t relu;
  int64_t batch;
  int64_t stride_a, stride_b, stride_c;
} choreo_gemm_desc;

/* The kernel configuration the dispatcher picks for a request (backs the
 * reference's get_optimal_gemm_config, compute/compute_impl.hpp:74-91, and the
 * auto_analyze() of examples/ideal_matmul_example.cu:244-290). */
typedef struct choreo_launch_config {
  int32_t kernel;          /* 1 = tcgen05 tile GEMM, 2 = CUDA-core f32 GEMM, 3 = tcgen05 conv */
  int32_t tile_m, tile_n, tile_k;
  int32_t stages;          /* shared-memory pipeline depth */
  int32_t cluster_m;       /* CTAs per cluster along M (1 = no cluster) */
  int32_t grid_x, grid_y, grid_z;
  int32_t block_x;         /* threads per CTA */
  int32_t smem_bytes;      /* dynamic shared memory per CTA */
  int32_t tmem_cols;       /* tensor-memory columns per CTA */
  int64_t tiles;           /* output tiles (all batch items, all K splits) */
  int64_t workspace_bytes; /* device scratch for the fastest plan (0 = none) */
  int64_t workspace_min_bytes; /* scratch the call cannot run without (operand repacks);
                                  between this and workspace_bytes the call runs without
                                  splitting K */
  int64_t split_k;         /* K ranges computed in parallel and summed in fp32 (1 = none) */
} choreo_launch_config;

/* Implicit-GEMM 2-D convolution, NHWC activations, KRSC weights:
 *   out[n,p,q,k] = act(alpha * sum_{r,s,c} in[n, p*stride_h - pad_h + r*dil_h,
 *                                              q*stride_w - pad_w + s*dil_w, c]
 *                                         * w[k,r,s,c] + bias[k])
 * with zero padding. out is NHWC [n, P, Q, k_out]. */
typedef struct choreo_conv_desc {
  int64_t n, h, w, c;          /* input NHWC */
  int64_t k, r, s;             /* output channels, filter height, width */
  int32_t stride_h, stride_w;
  int32_t pad_h, pad_w;
  int32_t dil_h, dil_w;
  int32_t dtype;               /* input/weight type: f16 or bf16 */
  int32_t dtype_out;           /* f16, bf16 or f32 */
  const void* input;
  const void* weight;
  void* output;
  const void* bias;            /* optional K-vector */
  int32_t dtype_bias;
  int32_t relu;
  float alpha;
} choreo_conv_desc;

/* Device properties the dispatcher uses (backs core/device.hpp:233-269). */
typedef struct choreo_device_props {
  int32_t device;
  int32_t cc_major, cc_minor;
  int32_t sm_count;
  int32_t max_smem_optin;      /* bytes of shared memory a CTA may opt into */
  int32_t cluster_launch;      /* 1 if thread-block clusters are supported */
  int64_t total_mem;
  char name[256];
} choreo_device_props;

/* ---- library / device ------------------------------------------------- */

/* Library version as major*10000 + minor*100 + patch. */
int choreo_version(void);

/* Message of the last failing call on this host thread ("" if none). */
const char* choreo_last_error(void);

/* Fills *out for `device`. Replaces DeviceManager::query_device_info
 * (core/device.hpp:233-269), which maps sm_100 to SM_70. */
int choreo_device_props_get(int device, choreo_device_props* out);

/* Synchronizes `stream` and reports kernel-side failures recorded since the
 * last call (CHOREO_ERR_TIMEOUT), clearing the record; CHOREO_ERR_CUDA if the
 * stream itself reports an error. */
int choreo_sync_status(void* stream);

/* Process-wide overrides of the dispatcher's choices, for tests and tuning
 * sweeps. A zeroed struct with l2_policy_a/b = -1 (what choreo_tuning_set(NULL)
 * installs) leaves every decision to the library; production callers never
 * need to touch it. Nothing is read from the environment. The reference
 * exposes the same kind of knob as GEMMConfig::tile_m/n/k and backend
 * (compute/compute.hpp:32-44), which its dispatcher ignores. */
typedef struct choreo_tuning {
  char tile[16];            /* "" = cost model; else force "wide256", "pair256", "pair128",
                               "single256", "single128" or "single64" (GEMM and conv) */
  int32_t split_k;          /* 0 = cost model; n >= 1 = only plans with exactly n K ranges
                               (where K divides into them; else the unsplit plan) */
  int32_t group_m;          /* 0 = rasterise tiles in groups of 4096 rows of A;
                               n >= 1 = groups of n M tiles */
  int32_t l2_policy_a;      /* -1 = default (evict_last); 0 normal, 1 evict_last, 2 evict_first */
  int32_t l2_policy_b;      /* -1 = default (normal); same codes */
  double wait_timeout_ms;   /* 0 = default 2000: limit of every bounded pipeline wait */
  int32_t handover_kb;      /* 512 x 256 tiles: k-blocks the MMA issuer runs for one accumulator
                               half alone while the other is handed over, at each end of a
                               tile (1..16; 0 = the pipeline depth, one less for tiles of
                               fewer than 64 k-blocks) */
  int32_t reserved;
} choreo_tuning;

/* Installs *t for every later call from any host thread (NULL restores the
 * defaults). CHOREO_ERR_INVALID_ARG for an unknown tile name or an out-of-range
 * field, leaving the previous settings in place. */
int choreo_tuning_set(const choreo_tuning* t);

/* Copies the settings in force into *out. */
int choreo_tuning_get(choreo_tuning* out);

/* Measurement hook: while `probe` is set (non-NULL) on this host thread,
 * every tensor-core GEMM and conv launched from the thread adds, from its
 * first CTA, the SM clock cycles (%clock64) and the global-timer nanoseconds
 * (%globaltimer) between that CTA's start and its end to probe[0] and
 * probe[1], and 1 to probe[2]: probe[0] / probe[1] is the effective SM clock
 * in GHz during those kernels. `probe` is three 8-byte-aligned uint64 in
 * device memory of the device the kernels run on, zeroed by the caller.
 * NULL turns it off. Reads clocks only; changes no setting. No counterpart in
 * the reference (its utils/profiler.hpp times with CUDA events only). */
int choreo_clock_probe_set(void* probe);

/* Launches one CTA that waits, through the bounded wait every kernel
 * pipeline uses, on an mbarrier nothing arrives on. The wait gives up after
 * timeout_ms, records a timeout in the status word and the kernel returns:
 * the next choreo_sync_status() reports CHOREO_ERR_TIMEOUT and the context
 * stays usable. Exercises the failure path without faulting the GPU. The
 * reference has no failure detection (errors are host exceptions only,
 * compute/validation.hpp:20-23, utils/cuda_utils.hpp:26-32). */
int choreo_selftest_wait_timeout(double timeout_ms, void* stream);

/* ---- GEMM ------------------------------------------------------------- */

/* Validates `d` and reports the kernel configuration and workspace size.
 * Replaces compute::get_optimal_gemm_config (compute/compute_impl.hpp:74-91). */
int choreo_gemm_query(const choreo_gemm_desc* d, choreo_launch_config* out);

/* Enqueues the GEMM on `stream`. Replaces compute::gemm
 * (compute/compute_impl.hpp:19-38, declared compute/compute.hpp:55-58) and,
 * with alpha=1, beta=0, compute::matmul (compute_impl.hpp:52-72) and the
 * device branch of operator* (choreo-ir.hpp:53-71).
 * `workspace` must hold choreo_gemm_query(...).workspace_bytes bytes of device
 * memory (it is used when a stride or base address is not 16-byte aligned, so
 * the operand is first repacked). */
int choreo_gemm(const choreo_gemm_desc* d, void* workspace, size_t workspace_bytes,
                void* stream);

/* Size of the scratch array choreo_gemm_noalloc stages repacked operands and
 * K-split partial sums in (one per GPU that loads the library, held until
 * the process exits). */
#define CHOREO_GEMM_NOALLOC_SCRATCH_BYTES (32u * 1024u * 1024u)

/* choreo_gemm for callers that cannot allocate device memory: it takes no
 * workspace and allocates nothing. No counterpart in the reference (its
 * operator* allocates its output with cudaMalloc, tensor/tensor.hpp:671).
 * Callers such as plugins inside a runtime that owns all device buffers, or
 * loops that must not call cudaMalloc (it can synchronize the device and
 * break a pre-planned memory budget), pass only inputs and outputs. What
 * choreo_gemm would keep in its workspace lives in the library's built-in
 * scratch array of CHOREO_GEMM_NOALLOC_SCRATCH_BYTES instead: the repack of
 * an operand that is not 16-byte aligned (a request whose repack needs more
 * returns CHOREO_ERR_WORKSPACE) and, when they fit beside it, the fp32
 * partials of a K split (a long-K GEMM with few output tiles; when they do
 * not fit the GEMM runs unsplit). The first call on each device resolves the
 * array's address, whatever the request: make it before any stream capture;
 * a cudaDeviceReset after it is not supported. All calls on a device share
 * the array, aligned operands with a K split included: calls that overlap on
 * the GPU race, so keep them on one stream. */
int choreo_gemm_noalloc(const choreo_gemm_desc* d, void* stream);

/* Row-sharded GEMM over several GPUs of one process: descs[i] describes
 * device devices[i]'s slab (its own A rows, its replica of B and bias, its C
 * rows). One host thread per device launches on streams[i] (NULL = default
 * stream) and, if ms_out != NULL, synchronizes and stores that device's
 * kernel time in ms_out[i] (-1 where none was measured: the shard failed).
 * Returns the first failing shard's status, naming it by index and device
 * in choreo_last_error(). No data crosses between devices. The M-row
 * split of a large GEMM across the GPUs of one box, B replicated; the
 * reference has no multi-GPU code (core/device.hpp:136-156 only switches
 * devices). */
int choreo_gemm_rowsharded(const choreo_gemm_desc* descs, int ngpu, const int* devices,
                           void* const* streams, float* ms_out);

/* Rows [*row0, *row0 + *rows) of an M-row problem that shard `rank` of
 * `nshards` owns: contiguous slabs of whole 128-row tiles (only the last
 * slab may end in a partial tile), tile counts differing by at most one,
 * earlier shards taking the extra tiles. */
int choreo_shard_rows(int64_t m, int nshards, int rank, int64_t* row0, int64_t* rows);

/* ---- convolution ------------------------------------------------------- */

int choreo_conv2d_query(const choreo_conv_desc* d, choreo_launch_config* out);

/* Enqueues the implicit-GEMM convolution. Stands behind the conv2d() the
 * reference's benchmarks call (benchmark/performance/benchmark_suite.cpp:379)
 * with the semantics of benchmark/kernels/gemm_example.cu:208-253, in NHWC. */
int choreo_conv2d(const choreo_conv_desc* d, void* workspace, size_t workspace_bytes,
                  void* stream);

/* ---- host-buffer pipelines ----------------------------------------------
 * The reference moves data with Tensor::to_device()/to_host() (synchronous
 * cudaMemcpy, tensor/tensor.hpp:568-598, README.md:86-94) around a device
 * operator*. A host plan does the same job for inputs and outputs that live
 * in host memory, with the copies overlapped with the kernels: A (GEMM) or
 * the image batch (conv) is cut into parts; the host->device copy of part
 * i+1, the kernel of part i and the device->host copy of part i-1 run at
 * the same time on two library-owned copy streams and the caller's stream.
 * The plan owns its device buffers (allocated once, at create), its copy
 * streams and events; run() allocates nothing. Host memory that is pinned
 * (cudaHostAlloc / cudaHostRegister) gets the overlap; pageable memory works
 * but the driver stages its copies. A plan is used by one host thread at a
 * time; run() is asynchronous on `stream` like every other call: the host
 * buffers must stay valid and unchanged until the stream reaches the end of
 * the run. */
typedef struct choreo_host_plan choreo_host_plan;   /* opaque */

/* B and bias (GEMM), weight and bias (conv) are device memory of the plan's
 * device, read in place instead of copied from the host. */
#define CHOREO_HOST_OPERANDS_ON_DEVICE 1

/* C = act(alpha * A B + bias) for row-major contiguous A [m x k], B [k x n],
 * C [m x n] (leading dimensions k, n, n) and an optional n-vector bias. */
typedef struct choreo_host_gemm_desc {
  int64_t m, n, k;
  int32_t dtype_ab, dtype_c;   /* as choreo_gemm_desc */
  float alpha;
  int32_t has_bias, dtype_bias;
  int32_t relu;
  int32_t parts;               /* row slabs of A and C; 0 = library choice (every slab moving at least
                                  40 MiB over the host links, at most 16) */
  int32_t device;              /* CUDA device the plan runs on */
} choreo_host_gemm_desc;

typedef struct choreo_host_plan_info {
  int32_t parts;               /* row slabs (GEMM) or image runs (conv) */
  int32_t launches_per_run;    /* kernels one run enqueues */
  int64_t device_bytes;        /* device memory the plan holds */
  int64_t h2d_bytes;           /* bytes one run copies in (operands from the host) */
  int64_t d2h_bytes;           /* bytes one run copies out */
} choreo_host_plan_info;

/* Makes a GEMM plan: validates *d, allocates the device buffers, the copy
 * streams and events on d->device. */
int choreo_host_gemm_plan_create(const choreo_host_gemm_desc* d, choreo_host_plan** out);

/* Makes a conv plan for the shape in *d: its data pointers are not used,
 * except that a non-NULL d->bias makes a plan with a bias; alpha, bias type
 * and ReLU are taken from it. The batch is cut into `parts` runs of images
 * (0 = library choice: every run moving at least 40 MiB over the host links,
 * at most 16). */
int choreo_host_conv_plan_create(const choreo_conv_desc* d, int32_t parts, int32_t device,
                                 choreo_host_plan** out);

/* One GEMM through a GEMM plan: a and c in host memory; b and bias (NULL when
 * the plan has none) in host memory, or on the plan's device with
 * CHOREO_HOST_OPERANDS_ON_DEVICE in flags. */
int choreo_host_gemm_run(choreo_host_plan* p, const void* a, const void* b, const void* bias, void* c,
                         int32_t flags, void* stream);

/* One convolution through a conv plan (input NHWC and output in host memory;
 * weight KRSC and bias as b and bias above). */
int choreo_host_conv_run(choreo_host_plan* p, const void* input, const void* weight, const void* bias,
                         void* output, int32_t flags, void* stream);

int choreo_host_plan_info_get(const choreo_host_plan* p, choreo_host_plan_info* out);

/* Part i of the plan: first row (GEMM) or image (conv) and count. */
int choreo_host_plan_part(const choreo_host_plan* p, int32_t i, int64_t* first, int64_t* count);

/* Waits for the plan's work, frees its device buffers, streams and events. */
int choreo_host_plan_destroy(choreo_host_plan* p);

/* ---- elementwise (device kernels replacing host round trips) ---------- */

/* out[i] = max(in[i], 0). Replaces relu (choreo-ir.hpp:196-222). */
int choreo_relu(int32_t dtype, const void* in, void* out, int64_t numel, void* stream);

/* out[i] = a[i] + b[i]. Replaces operator+ (choreo-ir.hpp:150-191). */
int choreo_add(int32_t dtype, const void* a, const void* b, void* out, int64_t numel,
               void* stream);

/* dst[i] = value. Replaces the host-vector fill of Tensor::fill
 * (tensor/tensor.hpp:530-562). */
int choreo_fill(int32_t dtype, void* dst, double value, int64_t numel, void* stream);

/* dst = convert(src), element count numel (f16/bf16/f32 in any pairing).
 * Backs the mixed-precision operator* (choreo-ir.hpp:109-145) on the device. */
int choreo_convert(int32_t dtype_src, const void* src, int32_t dtype_dst, void* dst,
                   int64_t numel, void* stream);

/* ---- tile copies for user kernels -------------------------------------- */

/* Encodes a tiled TMA tensor map (a 128-byte CUtensorMap, 64-byte aligned) for
 * a strided 1- to 5-D f16/bf16/f32 tensor, so a user kernel can move tiles
 * between global and shared memory with cp.async.bulk.tensor
 * (include/choreo-ir/tensor/device_tile.hpp). Backs the TMA form of
 * TensorView::copy_to_shared / async_copy_to_shared and of the
 * `shared = global.tile(...)` assignment (tensor/tensor.hpp:164-254).
 * dims and box are innermost first; strides_bytes has rank - 1 entries (the
 * byte strides of dims 1..rank-1, each a multiple of 16); base is 16-byte
 * aligned; box[i] in 1..256 with box[0] * element size a multiple of 16;
 * swizzle_bytes is 0, 32, 64 or 128 (with a swizzle, box[0] * element size
 * must not exceed it). Elements past the tensor's edge read as zero. */
int choreo_tensor_map_encode(void* map, int32_t dtype, int32_t rank, const void* base,
                             const int64_t* dims, const int64_t* strides_bytes,
                             const uint32_t* box, int32_t swizzle_bytes);

#ifdef __cplusplus
}
#endif

#endif /* CHOREO_B200_H */
