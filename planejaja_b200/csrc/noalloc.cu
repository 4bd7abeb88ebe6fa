// noalloc.cu -- decode GEMV for callers that cannot allocate device memory.
//
// nsq_gemv needs a workspace for the prepared activations when they do not
// fit on chip, and the caller must cudaMalloc it.  Some callers cannot: code
// that runs inside a tight memory budget where every allocation is accounted
// by another allocator (an engine whose arena already owns all of HBM), code
// called from a context that must not synchronise (cudaMalloc may), or thin
// FFI shims with nowhere to keep a device pointer between calls.
// nsq_gemv_noalloc serves them: the activation records live in a file-scope
// device array of fixed size that every GPU loading this library holds until
// the process exits, so the call itself allocates nothing.
//
// Limits and sharing:
//   * M * K <= NSQ_NOALLOC_MAX_ELEMS (the array holds M * K / 32 records of
//     80 bytes, 640 KiB); larger calls return NSQ_ERR_WORKSPACE.
//   * Every call on a device uses the same array and leaves the last call's
//     records in it.  Nothing in it has to start at zero: each call writes
//     all records it reads before reading them.  Calls that overlap on the
//     GPU (different streams, or host threads, without ordering between
//     them) race on the array and give wrong results; order them.
//   * The first call on a device looks the array's device address up
//     (cudaGetSymbolAddress, with that device current) and keeps it for the
//     life of the process.  Make that first call before capturing a stream
//     into a CUDA graph.  Do not use this entry point across a
//     cudaDeviceReset of the device: the kept address then belongs to the
//     destroyed context.
#include <mutex>

#include "nsq_common.cuh"

namespace nsq {

cudaError_t launch_prepare_x(const float* x, XGroup* xg, int64_t M, int64_t K, cudaStream_t st, int num_sms);
int run_gemv(const uint8_t* w, int type, int layout, const XGroup* xg, float* y, int64_t M, int64_t N, int64_t K,
             cudaStream_t st, int num_sms);
int check_weights(const void* w, int type, int layout, int64_t K);

constexpr size_t kNoAllocBytes = (size_t)(NSQ_NOALLOC_MAX_ELEMS / 32) * sizeof(XGroup);

// In host code this name is only a host-side stand-in for the array; its
// device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

struct NoAllocDev {
  void* scratch = nullptr;
  int num_sms = 0;
  int cc_major = 0;
};

// Per-device set-up, done once, with the device current.
static int noalloc_setup(NoAllocDev& out) {
  static std::mutex mu;
  static NoAllocDev cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return NSQ_ERR_CUDA;
  std::lock_guard<std::mutex> lk(mu);
  NoAllocDev& c = cache[dev];
  if (!c.scratch) {
    int sms = 0, major = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return NSQ_ERR_CUDA;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return NSQ_ERR_CUDA;
    if (major != 10) return NSQ_ERR_DEVICE;
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || !ptr) return NSQ_ERR_CUDA;
    c.num_sms = sms;
    c.cc_major = major;
    c.scratch = ptr;
  }
  out = c;
  return NSQ_OK;
}

}  // namespace nsq

using namespace nsq;

extern "C" int nsq_gemv_noalloc(const void* w, int ggml_type, int q6k_layout, const float* x, float* y, int64_t M,
                                int64_t N, int64_t K, void* stream) {
  // the weight checks of nsq_gemv (type, K-quant layout, pointer, K)
  int rc = check_weights(w, ggml_type, q6k_layout, K);
  if (rc) return rc;
  if (!x || !y) return NSQ_ERR_NULL;
  if ((reinterpret_cast<uintptr_t>(x) & 3) || (reinterpret_cast<uintptr_t>(y) & 3)) return NSQ_ERR_ALIGN;
  if (M < 1 || M > NSQ_GEMV_MAX_M || N < 1) return NSQ_ERR_SHAPE;
  if (M * K > NSQ_NOALLOC_MAX_ELEMS) return NSQ_ERR_WORKSPACE;  // beyond the built-in scratch
  NoAllocDev d;
  rc = noalloc_setup(d);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  XGroup* xg = static_cast<XGroup*>(d.scratch);
  if (launch_prepare_x(x, xg, M, K, st, d.num_sms) != cudaSuccess) return NSQ_ERR_CUDA;
  return run_gemv(static_cast<const uint8_t*>(w), ggml_type, q6k_layout, xg, y, M, N, K, st, d.num_sms);
}
