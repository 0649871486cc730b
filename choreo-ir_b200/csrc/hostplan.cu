// hostplan.cu — host-buffer pipelines: GEMM and conv whose inputs and outputs
// live in host memory, with the PCIe copies overlapped with the kernels.
//
// The reference's flow is host tensor -> to_device() -> device operator* ->
// to_host() (tensor/tensor.hpp:568-598, README.md:86-94), three synchronous
// steps. A plan cuts the streamed operand (A's rows, or the image batch) into
// parts and runs three queues at once:
//   copy-in stream   B / bias (unless already on the device), then part 0, 1, ...
//   caller's stream  the kernel of part i once its inputs have landed
//   copy-out stream  part i of the output once its kernel has finished
// so the host->device copy of part i+1, the kernel of part i and the
// device->host copy of part i-1 overlap. Each copy is one cudaMemcpyAsync.
//
// Ordering across runs: the copy-in stream of run r+1 waits only for run r's
// kernels to be done reading the device buffers (event `kernels_done`), not
// for whatever the caller enqueued before run r+1 — so run r+1's copies can
// start while the caller's stream is still busy (for example with a
// collective that assembles B on the device). The caller's stream waits for
// the copy-out stream at the end of every run, which orders run r+1's kernels
// (they overwrite the device output) after run r's copies out.
#include <algorithm>
#include <new>
#include <vector>

#include "internal.h"

struct choreo_host_plan {
  int kind = 0;                 // 1 GEMM, 2 conv
  int device = 0;
  choreo_host_gemm_desc g{};    // GEMM shape
  choreo_conv_desc cv{};        // conv shape (pointers unused)
  int64_t conv_p = 0, conv_q = 0;
  // device buffers (owned)
  void* a = nullptr;            // A / input
  void* b = nullptr;            // B / weight
  void* bias = nullptr;
  void* c = nullptr;            // C / output
  void* ws = nullptr;           // GEMM workspace (K-split partials), shared by the parts
  size_t ws_bytes = 0;
  int64_t device_bytes = 0;
  std::vector<int64_t> first, count;
  int launches = 0;
  cudaStream_t s_in = nullptr, s_out = nullptr;
  std::vector<cudaEvent_t> ev_in, ev_kernel;
  cudaEvent_t kernels_done = nullptr, out_done = nullptr;
};

namespace choreo_impl {
namespace {

// Makes `dev` current for the scope and puts the caller's device back.
struct DeviceScope {
  int saved = -1;
  bool switched = false;
  cudaError_t err = cudaSuccess;
  explicit DeviceScope(int dev) {
    err = cudaGetDevice(&saved);
    if (err == cudaSuccess && saved != dev) {
      err = cudaSetDevice(dev);
      switched = err == cudaSuccess;
    }
  }
  ~DeviceScope() {
    if (switched) cudaSetDevice(saved);
  }
};

int64_t bytes_of(int dt) { return dtype_bytes(dt); }

void release(choreo_host_plan* p) {
  if (p == nullptr) return;
  for (void* q : {p->a, p->b, p->bias, p->c, p->ws})
    if (q) cudaFree(q);
  for (cudaEvent_t e : p->ev_in)
    if (e) cudaEventDestroy(e);
  for (cudaEvent_t e : p->ev_kernel)
    if (e) cudaEventDestroy(e);
  if (p->kernels_done) cudaEventDestroy(p->kernels_done);
  if (p->out_done) cudaEventDestroy(p->out_done);
  if (p->s_in) cudaStreamDestroy(p->s_in);
  if (p->s_out) cudaStreamDestroy(p->s_out);
  delete p;
}

int alloc(void** ptr, int64_t bytes, int64_t* total, const char* what) {
  if (bytes <= 0) return CHOREO_OK;
  cudaError_t e = cudaMalloc(ptr, static_cast<size_t>(bytes));
  if (e != cudaSuccess) {
    *ptr = nullptr;
    cudaGetLastError();
    return fail(CHOREO_ERR_CUDA, "host plan: cudaMalloc of %lld bytes for %s failed (%s)",
                static_cast<long long>(bytes), what, cudaGetErrorString(e));
  }
  *total += bytes;
  return CHOREO_OK;
}

// Streams and per-part events.
int make_queues(choreo_host_plan* p) {
  cudaError_t e;
  if ((e = cudaStreamCreateWithFlags(&p->s_in, cudaStreamNonBlocking)) != cudaSuccess ||
      (e = cudaStreamCreateWithFlags(&p->s_out, cudaStreamNonBlocking)) != cudaSuccess)
    return cuda_fail(e, "host plan: cudaStreamCreate");
  const size_t n = p->first.size();
  p->ev_in.assign(n, nullptr);
  p->ev_kernel.assign(n, nullptr);
  for (size_t i = 0; i < n; ++i) {
    if ((e = cudaEventCreateWithFlags(&p->ev_in[i], cudaEventDisableTiming)) != cudaSuccess ||
        (e = cudaEventCreateWithFlags(&p->ev_kernel[i], cudaEventDisableTiming)) != cudaSuccess)
      return cuda_fail(e, "host plan: cudaEventCreate");
  }
  if ((e = cudaEventCreateWithFlags(&p->kernels_done, cudaEventDisableTiming)) != cudaSuccess ||
      (e = cudaEventCreateWithFlags(&p->out_done, cudaEventDisableTiming)) != cudaSuccess)
    return cuda_fail(e, "host plan: cudaEventCreate");
  return CHOREO_OK;
}

// The library's part count: every part moves at least kMinPartBytes over the
// host links (in + out), at most 16 parts. More parts shorten the pipeline's
// ends (the first copy in and the last copy out run alone) but each adds a
// launch and cross-stream waits; on a B200 over PCIe 5 (55 GB/s in, 57 GB/s
// out) the 2.3 GB config-4 GEMM step was fastest at 16 parts (25.2 ms, from
// 25.3 at 8 and 25.7 at 32) and the 103 MB 32-image conv step at 2-3 runs
// (1.27 ms, from 1.42 at 8).
constexpr int64_t kMinPartBytes = 40ll << 20;
int64_t default_parts(int64_t bytes_moved, int64_t units) {
  return std::max<int64_t>(1, std::min<int64_t>({16, bytes_moved / kMinPartBytes, units}));
}

// Contiguous parts of `total` units: `parts` of them, each a multiple of
// `align` units (only the last may be shorter).
void split_parts(choreo_host_plan* p, int64_t total, int64_t parts, int64_t align) {
  int64_t per = (total + parts - 1) / parts;
  per = std::max<int64_t>(align, (per + align - 1) / align * align);
  for (int64_t f = 0; f < total; f += per) {
    p->first.push_back(f);
    p->count.push_back(std::min(per, total - f));
  }
}

// Host buffers must be host memory (pinned or pageable), device-resident
// operands device memory of the plan's device.
int check_host_ptr(const void* q, const char* name) {
  if (q == nullptr) return fail(CHOREO_ERR_INVALID_ARG, "host plan: %s is null", name);
  cudaPointerAttributes attr{};
  cudaError_t e = cudaPointerGetAttributes(&attr, q);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return CHOREO_OK;  // not known to CUDA: pageable host memory
  }
  if (attr.type == cudaMemoryTypeDevice)
    return fail(CHOREO_ERR_INVALID_ARG, "host plan: %s is device memory; host memory expected", name);
  return CHOREO_OK;
}

int check_dev_ptr(const void* q, int device, const char* name) {
  if (q == nullptr) return fail(CHOREO_ERR_INVALID_ARG, "host plan: %s is null", name);
  cudaPointerAttributes attr{};
  cudaError_t e = cudaPointerGetAttributes(&attr, q);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(CHOREO_ERR_INVALID_ARG, "host plan: %s is not device memory", name);
  }
  if (attr.type == cudaMemoryTypeManaged) return CHOREO_OK;
  if (attr.type != cudaMemoryTypeDevice || attr.device != device)
    return fail(CHOREO_ERR_INVALID_ARG, "host plan: %s must be device memory of device %d", name, device);
  if (reinterpret_cast<uintptr_t>(q) & 15u)
    return fail(CHOREO_ERR_INVALID_ARG, "host plan: %s must be 16-byte aligned", name);
  return CHOREO_OK;
}

int copy(void* dst, const void* src, int64_t bytes, cudaMemcpyKind kind, cudaStream_t s, const char* what) {
  if (bytes <= 0) return CHOREO_OK;
  cudaError_t e = cudaMemcpyAsync(dst, src, static_cast<size_t>(bytes), kind, s);
  return e == cudaSuccess ? CHOREO_OK : cuda_fail(e, what);
}

int record(cudaEvent_t ev, cudaStream_t s) {
  cudaError_t e = cudaEventRecord(ev, s);
  return e == cudaSuccess ? CHOREO_OK : cuda_fail(e, "host plan: cudaEventRecord");
}

int wait(cudaStream_t s, cudaEvent_t ev) {
  cudaError_t e = cudaStreamWaitEvent(s, ev, 0);
  return e == cudaSuccess ? CHOREO_OK : cuda_fail(e, "host plan: cudaStreamWaitEvent");
}

choreo_gemm_desc gemm_part(const choreo_host_plan* p, size_t i, const void* b, const void* bias) {
  const choreo_host_gemm_desc& g = p->g;
  const int64_t eab = bytes_of(g.dtype_ab), ec = bytes_of(g.dtype_c);
  choreo_gemm_desc d{};
  d.m = p->count[i];
  d.n = g.n;
  d.k = g.k;
  d.dtype_ab = g.dtype_ab;
  d.dtype_c = g.dtype_c;
  d.a = static_cast<const char*>(p->a) + p->first[i] * g.k * eab;
  d.lda = g.k;
  d.b = b;
  d.ldb = g.n;
  d.c = static_cast<char*>(p->c) + p->first[i] * g.n * ec;
  d.ldc = g.n;
  d.alpha = g.alpha;
  d.beta = 0.f;
  d.bias = bias;
  d.dtype_bias = g.dtype_bias;
  d.relu = g.relu;
  d.batch = 1;
  return d;
}

choreo_conv_desc conv_part(const choreo_host_plan* p, size_t i, const void* w, const void* bias) {
  const choreo_conv_desc& s = p->cv;
  choreo_conv_desc d = s;
  d.n = p->count[i];
  d.input = static_cast<const char*>(p->a) + p->first[i] * s.h * s.w * s.c * bytes_of(s.dtype);
  d.weight = w;
  d.output = static_cast<char*>(p->c) + p->first[i] * p->conv_p * p->conv_q * s.k * bytes_of(s.dtype_out);
  d.bias = bias;
  return d;
}

// The pipeline shared by both kinds. in_bytes/out_bytes per unit (row or
// image) of the streamed operand; `kernel(i)` enqueues part i's kernel on s.
template <typename Kernel>
int run_pipeline(choreo_host_plan* p, const void* host_in, int64_t in_unit, void* host_out, int64_t out_unit,
                 const void* b_src, int64_t b_bytes, const void* bias_src, int64_t bias_bytes, bool on_device,
                 cudaStream_t s, Kernel&& kernel) {
  int rc;
  // The previous run's kernels are done with the device buffers.
  if ((rc = wait(p->s_in, p->kernels_done))) return rc;
  if (!on_device) {
    if ((rc = copy(p->b, b_src, b_bytes, cudaMemcpyHostToDevice, p->s_in, "host plan: copy of B / weights"))) return rc;
    if (bias_src && (rc = copy(p->bias, bias_src, bias_bytes, cudaMemcpyHostToDevice, p->s_in, "host plan: bias")))
      return rc;
  }
  const size_t n = p->first.size();
  for (size_t i = 0; i < n; ++i) {
    if ((rc = copy(static_cast<char*>(p->a) + p->first[i] * in_unit,
                   static_cast<const char*>(host_in) + p->first[i] * in_unit, p->count[i] * in_unit,
                   cudaMemcpyHostToDevice, p->s_in, "host plan: copy in")))
      return rc;
    if ((rc = record(p->ev_in[i], p->s_in))) return rc;
  }
  for (size_t i = 0; i < n; ++i) {
    if ((rc = wait(s, p->ev_in[i]))) return rc;
    if ((rc = kernel(i))) return rc;
    if ((rc = record(p->ev_kernel[i], s))) return rc;
    if ((rc = wait(p->s_out, p->ev_kernel[i]))) return rc;
    if ((rc = copy(static_cast<char*>(host_out) + p->first[i] * out_unit,
                   static_cast<const char*>(p->c) + p->first[i] * out_unit, p->count[i] * out_unit,
                   cudaMemcpyDeviceToHost, p->s_out, "host plan: copy out")))
      return rc;
  }
  if ((rc = record(p->kernels_done, s))) return rc;
  if ((rc = record(p->out_done, p->s_out))) return rc;
  return wait(s, p->out_done);
}

}  // namespace
}  // namespace choreo_impl

using namespace choreo_impl;

extern "C" {

int choreo_host_gemm_plan_create(const choreo_host_gemm_desc* d, choreo_host_plan** out) {
  if (d == nullptr || out == nullptr) return fail(CHOREO_ERR_INVALID_ARG, "host GEMM plan: null argument");
  *out = nullptr;
  if (d->m <= 0 || d->n <= 0 || d->k <= 0)
    return fail(CHOREO_ERR_INVALID_ARG, "host GEMM plan: Invalid matrix dimensions: M=%lld, N=%lld, K=%lld",
                (long long)d->m, (long long)d->n, (long long)d->k);
  if (bytes_of(d->dtype_ab) == 0 || bytes_of(d->dtype_c) == 0 || (d->has_bias && bytes_of(d->dtype_bias) == 0))
    return fail(CHOREO_ERR_UNSUPPORTED, "host GEMM plan: unsupported dtype");
  if (d->parts < 0 || d->parts > 4096) return fail(CHOREO_ERR_INVALID_ARG, "host GEMM plan: parts %d", d->parts);
  if ((d->k * bytes_of(d->dtype_ab)) % 16 != 0 || (d->n * bytes_of(d->dtype_ab)) % 16 != 0)
    return fail(CHOREO_ERR_UNSUPPORTED,
                "host GEMM plan: rows of A and B must be a multiple of 16 bytes (K=%lld, N=%lld)", (long long)d->k,
                (long long)d->n);
  DeviceScope scope(d->device);
  if (scope.err != cudaSuccess) return cuda_fail(scope.err, "host GEMM plan: cudaSetDevice");
  auto* p = new (std::nothrow) choreo_host_plan();
  if (p == nullptr) return fail(CHOREO_ERR_CUDA, "host GEMM plan: out of host memory");
  p->kind = 1;
  p->device = d->device;
  p->g = *d;
  const int64_t eab = bytes_of(d->dtype_ab), ec = bytes_of(d->dtype_c);
  const int64_t moved = d->m * d->k * eab + d->k * d->n * eab + d->m * d->n * ec;
  const int64_t parts = d->parts > 0 ? d->parts : default_parts(moved, (d->m + 511) / 512);
  split_parts(p, d->m, parts, d->m >= 512 ? 512 : 1);  // whole wide-tile row blocks
  int rc;
  if ((rc = alloc(&p->a, d->m * d->k * eab, &p->device_bytes, "A")) ||
      (rc = alloc(&p->b, d->k * d->n * eab, &p->device_bytes, "B")) ||
      (rc = alloc(&p->c, d->m * d->n * ec, &p->device_bytes, "C")) ||
      (d->has_bias && (rc = alloc(&p->bias, d->n * bytes_of(d->dtype_bias), &p->device_bytes, "bias")))) {
    release(p);
    return rc;
  }
  // One workspace (K-split partials) serves every part: the parts' GEMMs run
  // in order on one stream.
  int64_t ws = 0;
  p->launches = 0;
  for (size_t i = 0; i < p->first.size(); ++i) {
    const choreo_gemm_desc gd = gemm_part(p, i, p->b, p->bias);
    choreo_launch_config q;
    if ((rc = choreo_gemm_query(&gd, &q))) {
      release(p);
      return rc;
    }
    ws = std::max<int64_t>(ws, q.workspace_bytes);
    p->launches += q.split_k > 1 ? 2 : 1;
  }
  if ((rc = alloc(&p->ws, ws, &p->device_bytes, "workspace")) || (rc = make_queues(p))) {
    release(p);
    return rc;
  }
  p->ws_bytes = static_cast<size_t>(ws);
  *out = p;
  return ok();
}

int choreo_host_conv_plan_create(const choreo_conv_desc* d, int32_t parts, int32_t device, choreo_host_plan** out) {
  if (d == nullptr || out == nullptr) return fail(CHOREO_ERR_INVALID_ARG, "host conv plan: null argument");
  *out = nullptr;
  if (d->n <= 0 || d->h <= 0 || d->w <= 0 || d->c <= 0 || d->k <= 0 || d->r <= 0 || d->s <= 0 ||
      d->stride_h < 1 || d->stride_w < 1 || d->dil_h < 1 || d->dil_w < 1 || d->pad_h < 0 || d->pad_w < 0)
    return fail(CHOREO_ERR_INVALID_ARG, "host conv plan: bad shape");
  if (bytes_of(d->dtype) != 2 || bytes_of(d->dtype_out) == 0 || (d->bias && bytes_of(d->dtype_bias) == 0))
    return fail(CHOREO_ERR_UNSUPPORTED, "host conv plan: unsupported dtype");
  if (parts < 0 || parts > 4096) return fail(CHOREO_ERR_INVALID_ARG, "host conv plan: parts %d", parts);
  const int64_t pp = (d->h + 2 * d->pad_h - d->dil_h * (d->r - 1) - 1) / d->stride_h + 1;
  const int64_t qq = (d->w + 2 * d->pad_w - d->dil_w * (d->s - 1) - 1) / d->stride_w + 1;
  if (pp <= 0 || qq <= 0) return fail(CHOREO_ERR_INVALID_ARG, "host conv plan: empty output");
  DeviceScope scope(device);
  if (scope.err != cudaSuccess) return cuda_fail(scope.err, "host conv plan: cudaSetDevice");
  auto* p = new (std::nothrow) choreo_host_plan();
  if (p == nullptr) return fail(CHOREO_ERR_CUDA, "host conv plan: out of host memory");
  p->kind = 2;
  p->device = device;
  p->cv = *d;
  p->conv_p = pp;
  p->conv_q = qq;
  const int64_t e = bytes_of(d->dtype);
  const int64_t moved = d->n * d->h * d->w * d->c * e + d->k * d->r * d->s * d->c * e +
                        d->n * pp * qq * d->k * bytes_of(d->dtype_out);
  const int64_t runs = parts > 0 ? parts : default_parts(moved, d->n);
  split_parts(p, d->n, runs, 1);
  int rc;
  if ((rc = alloc(&p->a, d->n * d->h * d->w * d->c * e, &p->device_bytes, "input")) ||
      (rc = alloc(&p->b, d->k * d->r * d->s * d->c * e, &p->device_bytes, "weight")) ||
      (rc = alloc(&p->c, d->n * pp * qq * d->k * bytes_of(d->dtype_out), &p->device_bytes, "output")) ||
      (d->bias && (rc = alloc(&p->bias, d->k * bytes_of(d->dtype_bias), &p->device_bytes, "bias")))) {
    release(p);
    return rc;
  }
  for (size_t i = 0; i < p->first.size(); ++i) {
    const choreo_conv_desc cd = conv_part(p, i, p->b, p->bias);
    choreo_launch_config q;
    if ((rc = choreo_conv2d_query(&cd, &q))) {
      release(p);
      return rc;
    }
    if (q.workspace_bytes != 0) {
      release(p);
      return fail(CHOREO_ERR_UNSUPPORTED, "host conv plan: the convolution needs a workspace");
    }
  }
  p->launches = static_cast<int>(p->first.size());
  if ((rc = make_queues(p))) {
    release(p);
    return rc;
  }
  *out = p;
  return ok();
}

int choreo_host_gemm_run(choreo_host_plan* p, const void* a, const void* b, const void* bias, void* c, int32_t flags,
                         void* stream) {
  if (p == nullptr || p->kind != 1) return fail(CHOREO_ERR_INVALID_ARG, "host GEMM run: not a GEMM plan");
  if ((flags & ~CHOREO_HOST_OPERANDS_ON_DEVICE) != 0)
    return fail(CHOREO_ERR_INVALID_ARG, "host GEMM run: unknown flags 0x%x", flags);
  if ((bias != nullptr) != (p->g.has_bias != 0))
    return fail(CHOREO_ERR_INVALID_ARG, "host GEMM run: the plan was made %s a bias", p->g.has_bias ? "with" : "without");
  const bool on_dev = (flags & CHOREO_HOST_OPERANDS_ON_DEVICE) != 0;
  DeviceScope scope(p->device);
  if (scope.err != cudaSuccess) return cuda_fail(scope.err, "host GEMM run: cudaSetDevice");
  int rc;
  if ((rc = check_host_ptr(a, "A")) || (rc = check_host_ptr(c, "C"))) return rc;
  if (on_dev) {
    if ((rc = check_dev_ptr(b, p->device, "B")) || (bias && (rc = check_dev_ptr(bias, p->device, "bias")))) return rc;
  } else if ((rc = check_host_ptr(b, "B")) || (bias && (rc = check_host_ptr(bias, "bias")))) {
    return rc;
  }
  const choreo_host_gemm_desc& g = p->g;
  const void* b_dev = on_dev ? b : p->b;
  const void* bias_dev = bias == nullptr ? nullptr : (on_dev ? bias : p->bias);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  rc = run_pipeline(p, a, g.k * bytes_of(g.dtype_ab), c, g.n * bytes_of(g.dtype_c), b, g.k * g.n * bytes_of(g.dtype_ab),
                    bias, g.n * bytes_of(g.dtype_bias), on_dev, s, [&](size_t i) {
                      const choreo_gemm_desc gd = gemm_part(p, i, b_dev, bias_dev);
                      return choreo_gemm(&gd, p->ws, p->ws_bytes, stream);
                    });
  return rc ? rc : ok();
}

int choreo_host_conv_run(choreo_host_plan* p, const void* input, const void* weight, const void* bias, void* output,
                         int32_t flags, void* stream) {
  if (p == nullptr || p->kind != 2) return fail(CHOREO_ERR_INVALID_ARG, "host conv run: not a conv plan");
  if ((flags & ~CHOREO_HOST_OPERANDS_ON_DEVICE) != 0)
    return fail(CHOREO_ERR_INVALID_ARG, "host conv run: unknown flags 0x%x", flags);
  if ((bias != nullptr) != (p->bias != nullptr))
    return fail(CHOREO_ERR_INVALID_ARG, "host conv run: the plan was made %s a bias", p->bias ? "with" : "without");
  const bool on_dev = (flags & CHOREO_HOST_OPERANDS_ON_DEVICE) != 0;
  DeviceScope scope(p->device);
  if (scope.err != cudaSuccess) return cuda_fail(scope.err, "host conv run: cudaSetDevice");
  int rc;
  if ((rc = check_host_ptr(input, "input")) || (rc = check_host_ptr(output, "output"))) return rc;
  if (on_dev) {
    if ((rc = check_dev_ptr(weight, p->device, "weight")) || (bias && (rc = check_dev_ptr(bias, p->device, "bias"))))
      return rc;
  } else if ((rc = check_host_ptr(weight, "weight")) || (bias && (rc = check_host_ptr(bias, "bias")))) {
    return rc;
  }
  const choreo_conv_desc& d = p->cv;
  const void* w_dev = on_dev ? weight : p->b;
  const void* bias_dev = bias == nullptr ? nullptr : (on_dev ? bias : p->bias);
  const int64_t e = bytes_of(d.dtype);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  rc = run_pipeline(p, input, d.h * d.w * d.c * e, output, p->conv_p * p->conv_q * d.k * bytes_of(d.dtype_out), weight,
                    d.k * d.r * d.s * d.c * e, bias, d.k * bytes_of(d.dtype_bias), on_dev, s, [&](size_t i) {
                      const choreo_conv_desc cd = conv_part(p, i, w_dev, bias_dev);
                      return choreo_conv2d(&cd, nullptr, 0, stream);
                    });
  return rc ? rc : ok();
}

int choreo_host_plan_info_get(const choreo_host_plan* p, choreo_host_plan_info* out) {
  if (p == nullptr || out == nullptr) return fail(CHOREO_ERR_INVALID_ARG, "host plan info: null argument");
  out->parts = static_cast<int32_t>(p->first.size());
  out->launches_per_run = p->launches;
  out->device_bytes = p->device_bytes;
  if (p->kind == 1) {
    const choreo_host_gemm_desc& g = p->g;
    out->h2d_bytes = (g.m * g.k + g.k * g.n) * bytes_of(g.dtype_ab) + (g.has_bias ? g.n * bytes_of(g.dtype_bias) : 0);
    out->d2h_bytes = g.m * g.n * bytes_of(g.dtype_c);
  } else {
    const choreo_conv_desc& d = p->cv;
    out->h2d_bytes = (d.n * d.h * d.w * d.c + d.k * d.r * d.s * d.c) * bytes_of(d.dtype) +
                     (p->bias ? d.k * bytes_of(d.dtype_bias) : 0);
    out->d2h_bytes = d.n * p->conv_p * p->conv_q * d.k * bytes_of(d.dtype_out);
  }
  return ok();
}

int choreo_host_plan_part(const choreo_host_plan* p, int32_t i, int64_t* first, int64_t* count) {
  if (p == nullptr || first == nullptr || count == nullptr || i < 0 || static_cast<size_t>(i) >= p->first.size())
    return fail(CHOREO_ERR_INVALID_ARG, "host plan part: bad arguments");
  *first = p->first[static_cast<size_t>(i)];
  *count = p->count[static_cast<size_t>(i)];
  return ok();
}

int choreo_host_plan_destroy(choreo_host_plan* p) {
  if (p == nullptr) return ok();
  DeviceScope scope(p->device);
  if (scope.err != cudaSuccess) return cuda_fail(scope.err, "host plan destroy: cudaSetDevice");
  // Work still queued on the plan's streams reads its buffers.
  if (p->s_in) cudaStreamSynchronize(p->s_in);
  if (p->s_out) cudaStreamSynchronize(p->s_out);
  if (p->kernels_done) cudaEventSynchronize(p->kernels_done);
  release(p);
  return ok();
}

}  // extern "C"
