// api.cu -- the extern "C" entry points of libnsq (declared in include/nsq.h).
//
// Every entry point validates its arguments on the host (types, shapes,
// alignment, workspace size, device) and returns an NSQ_* status before
// launching anything; CUDA launch errors become NSQ_ERR_CUDA.  Nothing here
// allocates device memory.
#include <atomic>
#include <mutex>
#include <stdlib.h>

#include "nsq_common.cuh"

namespace nsq {
__device__ int g_device_status = 0;

cudaError_t launch_dequant(const uint8_t* w, int type, int layout, int out_dtype, void* out, int64_t n_elems,
                           cudaStream_t st, int num_sms);
cudaError_t launch_prepare_x(const float* x, XGroup* xg, int64_t M, int64_t K, cudaStream_t st, int num_sms);
int run_gemv(const uint8_t* w, int type, int layout, const XGroup* xg, float* y, int64_t M, int64_t N, int64_t K,
             cudaStream_t st, int num_sms);
int run_gemv_fused(const nsq_segment* segs, int nseg, const float* x, const XGroup* xg, int64_t M, int64_t K,
                   cudaStream_t st, int num_sms, const XchgDesc* xd = nullptr, int epi = 0,
                   const float* const* res = nullptr);
bool fused_covers(const nsq_segment* segs, int nseg, int64_t K);
bool fused_self_prepare_fits(int64_t M, int64_t K);
bool fused_self_prepare_preferred(int64_t M, int64_t K);
bool gemv_force_general();
int run_gemv_mma(const nsq_segment* segs, int nseg, const XGroup* xg, int64_t M, int64_t K, cudaStream_t st,
                 int num_sms, const XchgDesc* xd);
int gemv_mma_min_m();
bool gemv_mma_covers(const nsq_segment* segs, int nseg, int64_t M, int64_t K);
bool tc_covers(const nsq_segment* segs, int nseg, int64_t M, int64_t K);
int tc_min_m();
size_t tc_workspace_bytes(int64_t K);
int run_gemv_tc(const nsq_segment* segs, int nseg, const float* x, int64_t M, int64_t K, void* workspace,
                cudaStream_t st, int num_sms, const XchgDesc* xd = nullptr);
int run_gemm_bf16(const uint8_t* w, int type, int layout, const void* x, void* y, int64_t M, int64_t N, int64_t K,
                  cudaStream_t st, int num_sms);
cudaError_t launch_matmul_f32(const float* a, const float* b, float* c, int64_t M, int64_t K, int64_t N,
                              cudaStream_t st);
bool comm_desc(const nsq_comm* c, XchgDesc& d);
size_t comm_bytes(const nsq_comm* c);
cudaError_t comm_launch_wait(const nsq_comm* c, cudaStream_t st);

// ---- launch-planning switches (see TuneId)
static const char* const kTuneNames[kTuneCount] = {
    "NSQ_ROWS_R", "NSQ_ROWS_PPSM", "NSQ_ROWS_STAGES", "NSQ_ROWS_PRE", "NSQ_ROWS_L2HINT", "NSQ_ROWS_CPS",
    "NSQ_ROWS_C", "NSQ_ROWS_BAL", "NSQ_ROWS_CARVE", "NSQ_MMA_MIN_M", "NSQ_MMA_PPS", "NSQ_MMA_STAGES",
    "NSQ_GEMV_GENERAL", "NSQ_GEMM_SPLIT", "NSQ_GEMM_TOK", "NSQ_TC_MIN_M", "NSQ_TC_A"};
static std::atomic<int> g_tune_val[kTuneCount];
static std::atomic<bool> g_tune_set[kTuneCount];
static std::once_flag g_tune_once;

static void read_tuning() {
  for (int i = 0; i < kTuneCount; ++i) {
    const char* v = getenv(kTuneNames[i]);
    const bool set = v && v[0];
    g_tune_val[i].store(set ? atoi(v) : 0, std::memory_order_relaxed);
    g_tune_set[i].store(set, std::memory_order_release);
  }
}

std::atomic<uint64_t> g_launches{0};
void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

int tune(TuneId id, int dflt) {
  std::call_once(g_tune_once, read_tuning);
  return g_tune_set[id].load(std::memory_order_acquire) ? g_tune_val[id].load(std::memory_order_relaxed) : dflt;
}

struct DevInfo {
  int num_sms = 0;
  int cc_major = 0;
};

static DevInfo dev_info() {
  static std::mutex mu;
  static DevInfo cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return DevInfo{};
  std::lock_guard<std::mutex> lk(mu);
  if (cache[dev].num_sms == 0) {
    int sms = 0, major = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return DevInfo{};
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return DevInfo{};
    cache[dev].num_sms = sms;
    cache[dev].cc_major = major;
  }
  return cache[dev];
}

static bool type_ok(int t) {
  return t == NSQ_TYPE_Q4_0 || t == NSQ_TYPE_Q8_0 || t == NSQ_TYPE_Q4_K || t == NSQ_TYPE_Q5_K || t == NSQ_TYPE_Q6_K;
}

static int check_device(DevInfo& di) {
  di = dev_info();
  if (di.num_sms == 0) return NSQ_ERR_CUDA;
  if (di.cc_major != 10) return NSQ_ERR_DEVICE;
  return NSQ_OK;
}

// For the other translation units (nsz.cu): NSQ_OK and the SM count.
int device_check(int* num_sms) {
  DevInfo di;
  const int rc = check_device(di);
  *num_sms = di.num_sms;
  return rc;
}

// Also used by nsq_gemv_noalloc (noalloc.cu), so that both entry points
// accept and reject the same weight arguments.
int check_weights(const void* w, int type, int layout, int64_t K) {
  if (!type_ok(type)) return NSQ_ERR_TYPE;
  if ((type == NSQ_TYPE_Q6_K || type == NSQ_TYPE_Q5_K) && layout != NSQ_Q6K_GGML && layout != NSQ_Q6K_NODESTOR)
    return NSQ_ERR_TYPE;
  if (!w) return NSQ_ERR_NULL;
  if (reinterpret_cast<uintptr_t>(w) & 15) return NSQ_ERR_ALIGN;
  const int64_t qk = nsq_block_weights(type);
  if (K <= 0 || K % qk) return NSQ_ERR_SHAPE;
  return NSQ_OK;
}

}  // namespace nsq

using namespace nsq;

extern "C" {

int nsq_version(void) { return NSQ_VERSION; }

void nsq_reload_tuning(void) {
  std::call_once(g_tune_once, read_tuning);
  read_tuning();
}

uint64_t nsq_kernel_launches(void) { return nsq::g_launches.load(std::memory_order_relaxed); }

const char* nsq_strerror(int status) {
  switch (status) {
    case NSQ_OK: return "ok";
    case NSQ_ERR_TYPE: return "unsupported ggml type, Q6_K layout or output dtype";
    case NSQ_ERR_SHAPE: return "bad shape (K not a multiple of the block size, or M/N/K out of range)";
    case NSQ_ERR_ALIGN: return "pointer alignment violated";
    case NSQ_ERR_NULL: return "required pointer is NULL";
    case NSQ_ERR_CUDA: return "CUDA error";
    case NSQ_ERR_NCCL: return "NCCL error";
    case NSQ_ERR_TIMEOUT: return "device-side wait timed out";
    case NSQ_ERR_WORKSPACE: return "workspace missing or too small";
    case NSQ_ERR_DEVICE: return "current device is not sm_100";
    case NSQ_ERR_FORMAT: return "malformed NSZ tile stream";
    default: return "unknown status";
  }
}

int64_t nsq_block_bytes(int ggml_type) {
  switch (ggml_type) {
    case NSQ_TYPE_Q4_0: return 18;
    case NSQ_TYPE_Q8_0: return 34;
    case NSQ_TYPE_Q4_K: return 144;
    case NSQ_TYPE_Q5_K: return 176;
    case NSQ_TYPE_Q6_K: return 210;
    default: return 0;
  }
}

int64_t nsq_block_weights(int ggml_type) {
  switch (ggml_type) {
    case NSQ_TYPE_Q4_0:
    case NSQ_TYPE_Q8_0: return 32;
    case NSQ_TYPE_Q4_K:
    case NSQ_TYPE_Q5_K: return 256;
    case NSQ_TYPE_Q6_K: return 256;
    default: return 0;
  }
}

int nsq_device_status(int clear) {
  int v = 0;
  if (cudaDeviceSynchronize() != cudaSuccess) return NSQ_ERR_CUDA;
  if (cudaMemcpyFromSymbol(&v, g_device_status, sizeof(int)) != cudaSuccess) return NSQ_ERR_CUDA;
  if (clear) {
    const int z = 0;
    if (cudaMemcpyToSymbol(g_device_status, &z, sizeof(int)) != cudaSuccess) return NSQ_ERR_CUDA;
  }
  return v;
}

int nsq_dequant(const void* w, int ggml_type, int q6k_layout, int out_dtype, void* out, int64_t n_elems,
                void* stream) {
  if (out_dtype != NSQ_OUT_F32 && out_dtype != NSQ_OUT_BF16) return NSQ_ERR_TYPE;
  const int64_t qk = nsq_block_weights(ggml_type);
  int rc = check_weights(w, ggml_type, q6k_layout, qk ? qk : 1);
  if (rc) return rc;
  if (n_elems < 0 || n_elems % qk) return NSQ_ERR_SHAPE;
  if (n_elems == 0) return NSQ_OK;
  if (!out) return NSQ_ERR_NULL;
  if (reinterpret_cast<uintptr_t>(out) & (out_dtype == NSQ_OUT_F32 ? 3 : 1)) return NSQ_ERR_ALIGN;
  DevInfo di;
  if ((rc = check_device(di))) return rc;
  cudaError_t e = launch_dequant(static_cast<const uint8_t*>(w), ggml_type, q6k_layout, out_dtype, out, n_elems,
                                 static_cast<cudaStream_t>(stream), di.num_sms);
  return e == cudaSuccess ? NSQ_OK : NSQ_ERR_CUDA;
}

// Bytes of the prepared activation records alone (every path but the
// tensor-core one needs only these).
static size_t records_bytes(int64_t M, int64_t K) {
  if (M <= 0 || K <= 0 || K % 32) return 0;
  return (size_t)(M * (K / 32)) * sizeof(XGroup);
}

// The fused kernel prepares the activations on chip when they fit there and
// x is 16-byte aligned, unless the separate preparation kernel is the faster
// choice and the workspace can hold its records.
static bool use_self_prepare(int64_t M, int64_t K, const float* x, const void* ws, size_t ws_bytes) {
  if (!fused_self_prepare_fits(M, K) || (reinterpret_cast<uintptr_t>(x) & 15)) return false;
  if (fused_self_prepare_preferred(M, K)) return true;
  const bool ws_ok = ws && !(reinterpret_cast<uintptr_t>(ws) & 15) && ws_bytes >= records_bytes(M, K);
  return !ws_ok;
}

size_t nsq_gemv_workspace_size(int64_t M, int64_t K) {
  if (M <= 0 || K <= 0 || K % 32) return 0;
  const size_t rec = records_bytes(M, K);
  // 2..16 tokens over K-quants run on the tensor cores: fp16 activation
  // tiles, min-term tiles and split-tile partial sums
  if (M >= 2 && M <= NSQ_GEMV_MAX_M && K % 256 == 0) {
    const size_t tc = tc_workspace_bytes(K);
    return rec > tc ? rec : tc;
  }
  return rec;
}

int nsq_prepare_activations(const float* x, int64_t M, int64_t K, void* workspace, size_t workspace_bytes,
                            void* stream) {
  if (M < 1 || M > NSQ_GEMV_MAX_M || K <= 0 || K % 32) return NSQ_ERR_SHAPE;
  if (!x || !workspace) return x ? NSQ_ERR_WORKSPACE : NSQ_ERR_NULL;
  if (reinterpret_cast<uintptr_t>(x) & 3) return NSQ_ERR_ALIGN;
  if (reinterpret_cast<uintptr_t>(workspace) & 15) return NSQ_ERR_ALIGN;
  if (workspace_bytes < records_bytes(M, K)) return NSQ_ERR_WORKSPACE;
  DevInfo di;
  int rc = check_device(di);
  if (rc) return rc;
  cudaError_t e = launch_prepare_x(x, static_cast<XGroup*>(workspace), M, K, static_cast<cudaStream_t>(stream),
                                   di.num_sms);
  return e == cudaSuccess ? NSQ_OK : NSQ_ERR_CUDA;
}

int nsq_gemv_prepared(const void* w, int ggml_type, int q6k_layout, const void* workspace, float* y, int64_t M,
                      int64_t N, int64_t K, void* stream) {
  int rc = check_weights(w, ggml_type, q6k_layout, K);
  if (rc) return rc;
  if (M < 1 || M > NSQ_GEMV_MAX_M || N < 1) return NSQ_ERR_SHAPE;
  if (!workspace) return NSQ_ERR_WORKSPACE;
  if (!y) return NSQ_ERR_NULL;
  if ((reinterpret_cast<uintptr_t>(workspace) & 15) || (reinterpret_cast<uintptr_t>(y) & 3)) return NSQ_ERR_ALIGN;
  DevInfo di;
  if ((rc = check_device(di))) return rc;
  return run_gemv(static_cast<const uint8_t*>(w), ggml_type, q6k_layout, static_cast<const XGroup*>(workspace), y,
                  M, N, K, static_cast<cudaStream_t>(stream), di.num_sms);
}

int nsq_gemv(const void* w, int ggml_type, int q6k_layout, const float* x, float* y, int64_t M, int64_t N,
             int64_t K, void* workspace, size_t workspace_bytes, void* stream) {
  nsq_segment sg{w, ggml_type, q6k_layout, N, y};
  return nsq_gemv_multi(&sg, 1, x, M, K, workspace, workspace_bytes, stream);
}

int nsq_gemv_multi(const nsq_segment* segs, int nseg, const float* x, int64_t M, int64_t K, void* workspace,
                   size_t workspace_bytes, void* stream) {
  if (!segs) return NSQ_ERR_NULL;
  if (nseg < 1 || nseg > NSQ_MAX_SEGMENTS) return NSQ_ERR_SHAPE;
  int rc;
  for (int i = 0; i < nseg; ++i) {
    if ((rc = check_weights(segs[i].w, segs[i].ggml_type, segs[i].q6k_layout, K))) return rc;
    if (segs[i].N < 1) return NSQ_ERR_SHAPE;
    if (!segs[i].y) return NSQ_ERR_NULL;
    if (reinterpret_cast<uintptr_t>(segs[i].y) & 3) return NSQ_ERR_ALIGN;
  }
  if (M < 1 || M > NSQ_GEMV_MAX_M || K % 32) return NSQ_ERR_SHAPE;
  if (!x) return NSQ_ERR_NULL;
  if (reinterpret_cast<uintptr_t>(x) & 15) {
    // the on-chip path reads x with 16-byte loads; 4-byte aligned inputs go
    // through the workspace
    if (reinterpret_cast<uintptr_t>(x) & 3) return NSQ_ERR_ALIGN;
  }
  if (!gemv_force_general() && M >= tc_min_m() && tc_covers(segs, nseg, M, K) && workspace &&
      !(reinterpret_cast<uintptr_t>(workspace) & 15) && workspace_bytes >= tc_workspace_bytes(K)) {
    // 2..16 tokens over Q4_K / ggml Q6_K: tcgen05 tensor cores (gemv_tc.cu),
    // when the workspace holds its tiles (nsq_gemv_workspace_size sizes it so)
    DevInfo di;
    if ((rc = check_device(di))) return rc;
    rc = run_gemv_tc(segs, nseg, x, M, K, workspace, static_cast<cudaStream_t>(stream), di.num_sms);
    if (rc != -1) return rc;
  }
  const bool mma = !gemv_force_general() && M >= gemv_mma_min_m() && gemv_mma_covers(segs, nseg, M, K);
  const bool fused = !gemv_force_general() && fused_covers(segs, nseg, K);
  const bool self = !mma && fused && use_self_prepare(M, K, x, workspace, workspace_bytes);
  if (!self) {
    if (!workspace) return NSQ_ERR_WORKSPACE;
    if (reinterpret_cast<uintptr_t>(workspace) & 15) return NSQ_ERR_ALIGN;
    if (workspace_bytes < records_bytes(M, K)) return NSQ_ERR_WORKSPACE;
  }
  DevInfo di;
  if ((rc = check_device(di))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (self) {
    rc = run_gemv_fused(segs, nseg, x, nullptr, M, K, st, di.num_sms);
    if (rc != -1) return rc;
    // not covered on chip after all: go through the workspace
    if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & 15) ||
        workspace_bytes < records_bytes(M, K))
      return NSQ_ERR_WORKSPACE;
  }
  if (launch_prepare_x(x, static_cast<XGroup*>(workspace), M, K, st, di.num_sms) != cudaSuccess) return NSQ_ERR_CUDA;
  if (mma) {
    rc = run_gemv_mma(segs, nseg, static_cast<const XGroup*>(workspace), M, K, st, di.num_sms, nullptr);
    if (rc != -1) return rc;
  }
  if (fused) {
    rc = run_gemv_fused(segs, nseg, nullptr, static_cast<const XGroup*>(workspace), M, K, st, di.num_sms);
    if (rc != -1) return rc;
  }
  for (int i = 0; i < nseg; ++i) {
    rc = run_gemv(static_cast<const uint8_t*>(segs[i].w), segs[i].ggml_type, segs[i].q6k_layout,
                  static_cast<const XGroup*>(workspace), segs[i].y, M, segs[i].N, K, st, di.num_sms);
    if (rc) return rc;
  }
  return NSQ_OK;
}

// Shared body of the fused-epilogue entry points: fused kernel only.
static int gemv_epilogue(const nsq_segment* segs, int nseg, const float* x, int64_t M, int64_t K, void* workspace,
                         size_t workspace_bytes, void* stream, int epi, const float* const* res) {
  if (M < 1 || M > NSQ_GEMV_MAX_M || K % 256) return NSQ_ERR_SHAPE;
  if (!x) return NSQ_ERR_NULL;
  if (reinterpret_cast<uintptr_t>(x) & 3) return NSQ_ERR_ALIGN;
  if (!fused_covers(segs, nseg, K)) return NSQ_ERR_SHAPE;
  const bool self = use_self_prepare(M, K, x, workspace, workspace_bytes);
  if (!self) {
    if (!workspace) return NSQ_ERR_WORKSPACE;
    if (reinterpret_cast<uintptr_t>(workspace) & 15) return NSQ_ERR_ALIGN;
    if (workspace_bytes < records_bytes(M, K)) return NSQ_ERR_WORKSPACE;
  }
  DevInfo di;
  int rc;
  if ((rc = check_device(di))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (!self && launch_prepare_x(x, static_cast<XGroup*>(workspace), M, K, st, di.num_sms) != cudaSuccess)
    return NSQ_ERR_CUDA;
  rc = run_gemv_fused(segs, nseg, self ? x : nullptr, self ? nullptr : static_cast<const XGroup*>(workspace), M, K, st,
                      di.num_sms, nullptr, epi, res);
  return rc == -1 ? NSQ_ERR_SHAPE : rc;
}

int nsq_gemv_swiglu(const void* w_gate, const void* w_up, int ggml_type, int q6k_layout, const float* x, float* h,
                    int64_t M, int64_t N, int64_t K, void* workspace, size_t workspace_bytes, void* stream) {
  int rc;
  if ((rc = check_weights(w_gate, ggml_type, q6k_layout, K))) return rc;
  if ((rc = check_weights(w_up, ggml_type, q6k_layout, K))) return rc;
  if (N < 1) return NSQ_ERR_SHAPE;
  if (!h) return NSQ_ERR_NULL;
  if (reinterpret_cast<uintptr_t>(h) & 3) return NSQ_ERR_ALIGN;
  const nsq_segment segs[2] = {{w_gate, ggml_type, q6k_layout, N, h}, {w_up, ggml_type, q6k_layout, N, h}};
  return gemv_epilogue(segs, 2, x, M, K, workspace, workspace_bytes, stream, 2, nullptr);
}

int nsq_gemv_residual(const void* w, int ggml_type, int q6k_layout, const float* x, const float* residual, float* y,
                      int64_t M, int64_t N, int64_t K, void* workspace, size_t workspace_bytes, void* stream) {
  int rc;
  if ((rc = check_weights(w, ggml_type, q6k_layout, K))) return rc;
  if (N < 1) return NSQ_ERR_SHAPE;
  if (!y || !residual) return NSQ_ERR_NULL;
  if ((reinterpret_cast<uintptr_t>(y) & 3) || (reinterpret_cast<uintptr_t>(residual) & 3)) return NSQ_ERR_ALIGN;
  const nsq_segment seg{w, ggml_type, q6k_layout, N, y};
  const float* res[1] = {residual};
  return gemv_epilogue(&seg, 1, x, M, K, workspace, workspace_bytes, stream, 1, res);
}

int nsq_gemv_multi_xchg(const nsq_xsegment* segs, int nseg, const float* x, int64_t M, int64_t K, nsq_comm* comm,
                        void* workspace, size_t workspace_bytes, void* stream) {
  if (!segs || !comm) return NSQ_ERR_NULL;
  if (nseg < 1 || nseg > NSQ_MAX_SEGMENTS) return NSQ_ERR_SHAPE;
  if (M < 1 || M > NSQ_GEMV_MAX_M || K % 256) return NSQ_ERR_SHAPE;
  nsq::XchgDesc xd;
  if (!nsq::comm_desc(comm, xd)) return NSQ_ERR_SHAPE;
  const int64_t cap = (int64_t)nsq::comm_bytes(comm);
  nsq_segment sl[NSQ_MAX_SEGMENTS];
  int rc;
  for (int i = 0; i < nseg; ++i) {
    const nsq_xsegment& g = segs[i];
    if ((rc = check_weights(g.w, g.ggml_type, g.q6k_layout, K))) return rc;
    if (g.N < 1 || g.row0 < 0 || g.n_full < g.row0 + g.N) return NSQ_ERR_SHAPE;
    if (g.y_off < 0 || (g.y_off & 3)) return NSQ_ERR_ALIGN;
    if (g.y_off + M * g.n_full * 4 > cap) return NSQ_ERR_SHAPE;
    sl[i] = nsq_segment{g.w, g.ggml_type, g.q6k_layout, g.N, nullptr};
    xd.row0[i] = g.row0;
    xd.nfull[i] = g.n_full;
    xd.off[i] = g.y_off;
  }
  if (!x) return NSQ_ERR_NULL;
  if (reinterpret_cast<uintptr_t>(x) & 3) return NSQ_ERR_ALIGN;
  {
    // x must not lie in an output range this call writes: every rank stores
    // its rows into that range of every other rank's buffer, possibly while
    // that rank's own kernel is still reading its activations there.
    const uintptr_t xb = reinterpret_cast<uintptr_t>(x), xe = xb + (uintptr_t)(M * K * 4);
    const uintptr_t base = reinterpret_cast<uintptr_t>(nsq_comm_buffer(comm));
    for (int i = 0; i < nseg; ++i) {
      const uintptr_t yb = base + (uintptr_t)segs[i].y_off, ye = yb + (uintptr_t)(M * segs[i].n_full * 4);
      if (xb < ye && yb < xe) return NSQ_ERR_SHAPE;
    }
  }
  if (xd.P == 1) {
    // a one-rank group: the kernels' exchange epilogue is off (P == 1), so
    // the outputs go straight to this rank's buffer
    uint8_t* base = static_cast<uint8_t*>(nsq_comm_buffer(comm));
    for (int i = 0; i < nseg; ++i) {
      if (segs[i].row0 != 0 || segs[i].n_full != segs[i].N) return NSQ_ERR_SHAPE;  // one rank holds every row
      sl[i].y = reinterpret_cast<float*>(base + segs[i].y_off);
    }
  }
  if (!gemv_force_general() && M >= tc_min_m() && tc_covers(sl, nseg, M, K) && workspace &&
      !(reinterpret_cast<uintptr_t>(workspace) & 15) && workspace_bytes >= tc_workspace_bytes(K)) {
    // tcgen05 batched path with the exchange epilogue; every rank's previous
    // exchange lands here before its tile-preparation kernel reads x
    DevInfo di;
    if ((rc = check_device(di))) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (xd.P > 1 && comm_launch_wait(comm, st) != cudaSuccess) return NSQ_ERR_CUDA;
    xd.wait = false;
    rc = run_gemv_tc(sl, nseg, x, M, K, workspace, st, di.num_sms, &xd);
    if (rc != -1) return rc;
  }
  const bool mma = M >= gemv_mma_min_m() && gemv_mma_covers(sl, nseg, M, K);
  if (!mma && !fused_covers(sl, nseg, K)) return NSQ_ERR_SHAPE;
  const bool self = !mma && use_self_prepare(M, K, x, workspace, workspace_bytes);
  if (!self) {
    if (!workspace) return NSQ_ERR_WORKSPACE;
    if (reinterpret_cast<uintptr_t>(workspace) & 15) return NSQ_ERR_ALIGN;
    if (workspace_bytes < records_bytes(M, K)) return NSQ_ERR_WORKSPACE;
  }
  DevInfo di;
  if ((rc = check_device(di))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // every rank's previous exchange lands here before x is read: inside the
  // GEMV's prologue, or before the kernel that quantises x into the workspace
  if (!self) {
    xd.wait = false;
    if (comm_launch_wait(comm, st) != cudaSuccess ||
        launch_prepare_x(x, static_cast<XGroup*>(workspace), M, K, st, di.num_sms) != cudaSuccess)
      return NSQ_ERR_CUDA;
  }
  rc = mma ? run_gemv_mma(sl, nseg, static_cast<const XGroup*>(workspace), M, K, st, di.num_sms, &xd)
           : run_gemv_fused(sl, nseg, self ? x : nullptr, self ? nullptr : static_cast<const XGroup*>(workspace), M,
                            K, st, di.num_sms, &xd);
  return rc == -1 ? NSQ_ERR_SHAPE : rc;
}

int nsq_gemm_bf16(const void* w, int ggml_type, int q6k_layout, const void* x_bf16, void* y_bf16, int64_t M,
                  int64_t N, int64_t K, void* stream) {
  int rc = check_weights(w, ggml_type, q6k_layout, K);
  if (rc) return rc;
  if (M < 1 || N < 1 || K % 256) return NSQ_ERR_SHAPE;
  if (M > (int64_t)1 << 24 || N > (int64_t)1 << 24) return NSQ_ERR_SHAPE;
  if (!x_bf16 || !y_bf16) return NSQ_ERR_NULL;
  if ((reinterpret_cast<uintptr_t>(x_bf16) & 15) || (reinterpret_cast<uintptr_t>(y_bf16) & 15)) return NSQ_ERR_ALIGN;
  DevInfo di;
  if ((rc = check_device(di))) return rc;
  return run_gemm_bf16(static_cast<const uint8_t*>(w), ggml_type, q6k_layout, x_bf16, y_bf16, M, N, K,
                       static_cast<cudaStream_t>(stream), di.num_sms);
}

int nsq_matmul_f32(const float* a, const float* b, float* c, int64_t M, int64_t K, int64_t N, void* stream) {
  if (M < 1 || K < 1 || N < 1) return NSQ_ERR_SHAPE;
  if (!a || !b || !c) return NSQ_ERR_NULL;
  if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) | reinterpret_cast<uintptr_t>(c)) & 3)
    return NSQ_ERR_ALIGN;
  DevInfo di;
  int rc = check_device(di);
  if (rc) return rc;
  cudaError_t e = launch_matmul_f32(a, b, c, M, K, N, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? NSQ_OK : NSQ_ERR_CUDA;
}

}  // extern "C"
