// comm.cu -- exchange groups for the row-sharded GEMV (one process per GPU).
//
// Each rank owns one exchange buffer (cudaMalloc, zeroed): kXchgCtlBytes of
// control words (the peers' flag words, this rank's exchange count and CTA
// counter) followed by the outputs.  Peers map it through CUDA IPC handles,
// so an exchange kernel stores its rows into every rank's buffer with plain
// peer stores over NVLink (no bulk or tensor copies touch peer memory).
// The flag protocol is in gemv_rows.cu (publish at the end of a grid, bounded
// wait at the start of the next exchange) and in comm_wait_kernel below.
#include <string.h>

#include "nsq_common.cuh"

struct nsq_comm {
  int world = 1, rank = 0, dev = 0;
  size_t bytes = 0;  // outputs
  uint8_t* local = nullptr;
  uint8_t* peer[NSQ_MAX_RANKS] = {};
  bool connected = false;
};

namespace nsq {

bool comm_desc(const nsq_comm* c, XchgDesc& d) {
  if (!c || !c->connected) return false;
  d.P = c->world;
  d.rank = c->rank;
  for (int r = 0; r < c->world; ++r) d.buf[r] = c->peer[r];
  return true;
}

size_t comm_bytes(const nsq_comm* c) { return c ? c->bytes : 0; }

// One thread waits until every peer's flag word has reached this rank's own
// exchange count (bounded; NSQ_ERR_TIMEOUT after the limit).  Launched as a
// programmatic dependent of the previous exchange (its count is read after
// griddepcontrol.wait) and lets the next kernel launch early: that kernel's
// own griddepcontrol.wait then covers this wait.
__global__ void comm_wait_kernel(const uint32_t* ctl, int world, int rank) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (threadIdx.x != 0) return;
  const uint32_t want = ld_acquire_sys(ctl + kXchgSeq);
  for (int r = 0; r < world; ++r)
    if (r != rank && !wait_geq_bounded(ctl + r, want)) return;
}

// Enqueues comm_wait_kernel: at the end of a step, and before the kernel
// that quantises a workspace-mode exchange's activations.
cudaError_t comm_launch_wait(const nsq_comm* c, cudaStream_t st) {
  if (c->world == 1) return cudaSuccess;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(32);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  note_launch();
  return cudaLaunchKernelEx(&cfg, comm_wait_kernel, reinterpret_cast<const uint32_t*>(c->local), c->world, c->rank);
}

}  // namespace nsq

extern "C" {

size_t nsq_comm_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

int nsq_comm_create(int world, int rank, size_t bytes, nsq_comm** comm, void* handle_out) {
  if (!comm || !handle_out) return NSQ_ERR_NULL;
  *comm = nullptr;
  if (world < 1 || world > NSQ_MAX_RANKS || rank < 0 || rank >= world || bytes == 0) return NSQ_ERR_SHAPE;
  nsq_comm* c = new nsq_comm();
  c->world = world;
  c->rank = rank;
  c->bytes = (bytes + 255) & ~size_t(255);
  if (cudaGetDevice(&c->dev) != cudaSuccess) {
    delete c;
    return NSQ_ERR_CUDA;
  }
  void* p = nullptr;
  if (cudaMalloc(&p, nsq::kXchgCtlBytes + c->bytes) != cudaSuccess) {
    cudaGetLastError();
    delete c;
    return NSQ_ERR_CUDA;
  }
  c->local = static_cast<uint8_t*>(p);
  cudaIpcMemHandle_t h;
  if (cudaMemset(p, 0, nsq::kXchgCtlBytes + c->bytes) != cudaSuccess || cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaGetLastError();
    cudaFree(p);
    delete c;
    return NSQ_ERR_CUDA;
  }
  memcpy(handle_out, &h, sizeof(h));
  c->peer[rank] = c->local;
  if (world == 1) c->connected = true;
  *comm = c;
  return NSQ_OK;
}

int nsq_comm_connect(nsq_comm* comm, const void* handles) {
  if (!comm || !handles) return NSQ_ERR_NULL;
  if (comm->connected) return NSQ_OK;
  const uint8_t* hs = static_cast<const uint8_t*>(handles);
  for (int r = 0; r < comm->world; ++r) {
    if (r == comm->rank) continue;
    cudaIpcMemHandle_t h;
    memcpy(&h, hs + (size_t)r * sizeof(h), sizeof(h));
    void* p = nullptr;
    if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
      cudaGetLastError();
      for (int q = 0; q < r; ++q)
        if (q != comm->rank && comm->peer[q]) {
          cudaIpcCloseMemHandle(comm->peer[q]);
          comm->peer[q] = nullptr;
        }
      return NSQ_ERR_CUDA;
    }
    comm->peer[r] = static_cast<uint8_t*>(p);
  }
  comm->connected = true;
  return NSQ_OK;
}

void* nsq_comm_buffer(nsq_comm* comm) { return comm ? comm->local + nsq::kXchgCtlBytes : nullptr; }

int nsq_comm_wait(nsq_comm* comm, void* stream) {
  if (!comm) return NSQ_ERR_NULL;
  if (!comm->connected) return NSQ_ERR_SHAPE;
  return nsq::comm_launch_wait(comm, static_cast<cudaStream_t>(stream)) == cudaSuccess ? NSQ_OK : NSQ_ERR_CUDA;
}

int nsq_comm_destroy(nsq_comm* comm) {
  if (!comm) return NSQ_ERR_NULL;
  int rc = NSQ_OK;
  for (int r = 0; r < comm->world; ++r)
    if (r != comm->rank && comm->peer[r] && cudaIpcCloseMemHandle(comm->peer[r]) != cudaSuccess) rc = NSQ_ERR_CUDA;
  if (comm->local && cudaFree(comm->local) != cudaSuccess) rc = NSQ_ERR_CUDA;
  delete comm;
  return rc;
}

}  // extern "C"
