// noalloc.cu — choreo_gemm_noalloc: the GEMM entry point for callers that
// cannot allocate device memory.
//
// Some callers may not call cudaMalloc at the point where they run a GEMM:
// a plugin inside a host runtime that owns every device buffer and hands the
// plugin's enqueue call only its inputs and outputs, or a latency-critical
// loop that must not allocate (cudaMalloc can synchronize the device and
// fragment a pre-planned memory budget). choreo_gemm uses a caller-provided
// workspace for two things: repacking an operand that is not 16-byte aligned
// (base, leading dimension or batch stride) before the TMA can read it, and
// the fp32 partial sums of a K split (a GEMM with few output tiles over a
// long K, cut into K ranges that run side by side and are summed by a second
// pass). This entry point stages both in a scratch array compiled into the
// library instead, so the caller passes inputs and outputs only.
//
// The scratch array is a file-scope __device__ array of
// CHOREO_GEMM_NOALLOC_SCRATCH_BYTES. Every GPU that loads the library holds
// it until the process exits. Requests whose repack alone needs more are
// rejected with CHOREO_ERR_WORKSPACE before anything is launched; a K split
// whose partials do not fit beside the repack runs unsplit instead.
//
// Set-up: every call first resolves the array's device address on the
// current device with cudaGetSymbolAddress (once per device, cached), even
// when the request needs no scratch, so the rule is simply that the first
// call on each device comes before any stream capture. Host code never
// passes the array's name to a kernel: in host code it names a host-side
// stand-in, not the device copy. The cached address assumes the device's
// context lives as long as the process: a cudaDeviceReset after the first
// call is not supported.
//
// Sharing: every call on a device uses the same array and leaves the last
// call's contents in it. Nothing in it has to start at zero (the repack
// writes every byte the GEMM then reads, padding included, and the first
// pass of a K split writes every partial the second pass reads). Calls that
// overlap on the GPU (different streams, or several host threads) race on
// the array, repacks and K-split partials alike: order them on one stream or
// serialize them.
#include <mutex>

#include "internal.h"

namespace {

__device__ __align__(256) unsigned char g_gemm_noalloc_scratch[CHOREO_GEMM_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device (set-up on first
// use per device). Returns nullptr after recording an error.
void* device_scratch() {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    choreo_impl::cuda_fail(e, "cudaGetDevice");
    return nullptr;
  }
  if (dev < 0 || dev >= kMaxDevices) {
    choreo_impl::fail(CHOREO_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_gemm_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      choreo_impl::cuda_fail(e, "cudaGetSymbolAddress(GEMM scratch)");
      return nullptr;
    }
    g_scratch_ptr[dev] = p;
  }
  return g_scratch_ptr[dev];
}

}  // namespace

extern "C" int choreo_gemm_noalloc(const choreo_gemm_desc* d, void* stream) {
  choreo_launch_config q;
  int rc = choreo_gemm_query(d, &q);
  if (rc) return rc;
  if (q.workspace_min_bytes > static_cast<int64_t>(CHOREO_GEMM_NOALLOC_SCRATCH_BYTES))
    return choreo_impl::fail(CHOREO_ERR_WORKSPACE,
                             "GEMM (no-alloc): repacking the unaligned operands needs %lld bytes of scratch; "
                             "the built-in scratch holds %u bytes. Align the operands (16-byte base and "
                             "leading dimension) or use choreo_gemm with a workspace.",
                             static_cast<long long>(q.workspace_min_bytes), CHOREO_GEMM_NOALLOC_SCRATCH_BYTES);
  // Resolved on every first call per device, needed or not (see set-up above).
  void* scratch = device_scratch();
  if (scratch == nullptr) return CHOREO_ERR_CUDA;
  if (q.workspace_bytes == 0) return choreo_gemm(d, nullptr, 0, stream);
  // Repacks first, then K-split partials if they fit in the rest.
  return choreo_gemm(d, scratch, CHOREO_GEMM_NOALLOC_SCRATCH_BYTES, stream);
}
