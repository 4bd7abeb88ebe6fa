/*
 * nsq.h -- C ABI of libnsq, the B200 (sm_100a) GGUF block-quantized
 * dequant + matmul library.
 *
 * It replaces the Vulkan dequant/matmul dispatch of NodeStor's engine
 * (nodestor/crates/nodestor-vulkan).  Paths below are relative to the
 * reference project root.
 *
 * Conventions
 *   - Weights W are GGUF-native: N rows of K weights, each row a run of
 *     quant blocks along K, exactly the bytes of a GGUF tensor (ggml ne0 = K).
 *     ggml_type is the GGUF/ggml type id: 2 = Q4_0, 8 = Q8_0, 12 = Q4_K,
 *     14 = Q6_K.  The weight pointer must be 16-byte aligned (GGUF tensor
 *     data is 32-byte aligned in the file; cudaMalloc gives 256).
 *   - q6k_layout selects the meaning of Q6_K and Q5_K bytes: NSQ_Q6K_GGML (what
 *     llama.cpp writes) or NSQ_Q6K_NODESTOR (the element mapping of the
 *     reference shader nodestor/crates/nodestor-vulkan/shaders/
 *     dequant_q6k.comp:50-99).  Ignored for the other types.
 *   - The matmul semantic is y[M x N] = x[M x K] . W^T (y[m,n] = sum_k
 *     x[m,k] W[n,k]); the reference's operator takes B = W^T as a [K x N]
 *     f32 matrix (crates/nodestor-vulkan/shaders/matmul.comp:10-16).
 *   - All pointers are device pointers owned by the caller.  Calls are
 *     asynchronous on `stream` (a cudaStream_t; NULL = legacy default
 *     stream) and allocate no device memory; scratch is passed explicitly.
 *   - Every entry point returns an NSQ_* status and never aborts.  Argument
 *     errors are detected on the host before any launch.
 */
#ifndef NSQ_H
#define NSQ_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NSQ_VERSION 10000 /* 1.0.0 */

/* status codes (mapped to NodeStorError variants by the host wrapper:
   crates/nodestor-core/src/error.rs:1-38) */
#define NSQ_OK 0
#define NSQ_ERR_TYPE 1      /* unsupported ggml_type, q6k_layout or out dtype */
#define NSQ_ERR_SHAPE 2     /* K not a multiple of the block, M/N/K out of range */
#define NSQ_ERR_ALIGN 3     /* pointer alignment violated */
#define NSQ_ERR_NULL 4      /* required pointer is NULL */
#define NSQ_ERR_CUDA 5      /* CUDA launch/runtime error */
#define NSQ_ERR_NCCL 6      /* NCCL error in a sharded call */
#define NSQ_ERR_TIMEOUT 7   /* a bounded device-side wait gave up */
#define NSQ_ERR_WORKSPACE 8 /* workspace missing or too small */
#define NSQ_ERR_DEVICE 9    /* current device is not sm_100 */
#define NSQ_ERR_FORMAT 10   /* malformed NSZ tile stream */

#define NSQ_TYPE_Q4_0 2
#define NSQ_TYPE_Q8_0 8
#define NSQ_TYPE_Q4_K 12
#define NSQ_TYPE_Q5_K 13
#define NSQ_TYPE_Q6_K 14

#define NSQ_Q6K_GGML 0
#define NSQ_Q6K_NODESTOR 1

#define NSQ_OUT_F32 0
#define NSQ_OUT_BF16 1

/* Largest M accepted by the decode GEMV (batch 1..16). */
#define NSQ_GEMV_MAX_M 16

/* Library version (NSQ_VERSION). */
int nsq_version(void);

/* Re-reads the NSQ_* launch-planning environment variables (kernel choice,
 * tile and pipeline sizes; all default to measured choices).  The library
 * reads them once, when it plans its first launch; call this after changing
 * them in the process environment (tests, tuning runs).  No counterpart in
 * the reference, which has no such switches. */
void nsq_reload_tuning(void);

/* Number of kernels this library has launched since it was loaded (a launch
 * captured into a CUDA graph counts once, at capture).  For benchmarks that
 * report how many kernels a step runs; no counterpart in the reference. */
uint64_t nsq_kernel_launches(void);

/* Text of a status code; static storage. */
const char *nsq_strerror(int status);

/* Bytes of one quant block and weights per block for a ggml type
 * (0 for unsupported types).  Replaces calculate_tensor_size /
 * QuantFormat::block_size_bytes (crates/nodestor-formats/src/gguf.rs:288-304,
 * crates/nodestor-inference/src/dequant/mod.rs:65-85), which have no Q4_K /
 * Q6_K entries and size Q8_0 at 36 B per 32 weights instead of 34. */
int64_t nsq_block_bytes(int ggml_type);
int64_t nsq_block_weights(int ggml_type);

/* Reads and optionally clears the device-side status word that bounded
 * waits inside kernels set (NSQ_ERR_TIMEOUT).  Synchronises the device. */
int nsq_device_status(int clear);

/*
 * Dequantize n_elems weights (a whole number of blocks) to f32 or bf16.
 * f32 results are bit-exact to the reference's dequant:
 *   Q8_0  crates/nodestor-inference/src/dequant/q8_0.rs:14-28
 *   Q4_K  crates/nodestor-inference/src/dequant/q4_k.rs:56-131
 *   Q4_0  crates/nodestor-vulkan/shaders/dequant_q4.comp:40-61
 *   Q6_K  crates/nodestor-vulkan/shaders/dequant_q6k.comp:50-99 (NODESTOR)
 * with IEEE fp16 scales (dequant/mod.rs:234-260).  bf16 is the f32 value
 * rounded to nearest-even.  Replaces DequantDispatcher::dequantize
 * (dequant/mod.rs:142-191) and the never-dispatched dequant pipelines
 * (crates/nodestor-vulkan/src/pipeline.rs:160-214, 1220-1252).
 */
int nsq_dequant(const void *w, int ggml_type, int q6k_layout, int out_dtype, void *out,
                int64_t n_elems, void *stream);

/*
 * Decode GEMV, batch M in 1..16: y[M x N] f32 = x[M x K] f32 . W^T,
 * fp32 output within 1e-3 relative error of the reference composition
 * cpu_matmul_f32(x, transpose(dequant(W))) (crates/nodestor-vulkan/src/
 * pipeline.rs:1256-1268).  Replaces VulkanEngine::matmul
 * (crates/nodestor-vulkan/src/lib.rs:117-122) on quantized weights and the
 * TensorOp::Matmul{quantized} dispatch (src/operator_registry.rs:246-259).
 *
 * Activations are split into per-32 scaled int16 limbs (on chip when x is
 * 16-byte aligned, M <= 4 and M * K / 32 * 80 <= 40 KB, else in `workspace`,
 * nsq_gemv_workspace_size bytes, 16-byte aligned, which may be NULL when
 * not needed); the GEMV accumulates exact integer dot products per 16 or 32
 * weights and combines them in fp32.
 *
 * For 5..16 tokens over every format and layout (K % 256 == 0) the GEMV runs
 * on the tcgen05 tensor cores: the 6-bit sub-scales folded into fp16 weight
 * operands held in tensor memory (exact products; Q4_0 / Q8_0 fold their
 * block scale, rounded once to fp16), x as fp16 hi + lo parts (22 bits), fp32
 * accumulation, one fp32 epilogue per 256 weights.  Its workspace (fp16
 * activation tiles and split-tile partial sums, about 21 KB per 256 of K
 * plus 4 MiB) is what nsq_gemv_workspace_size returns for M >= 2; with a
 * workspace of only the M * K / 32 * 80 bytes of prepared activations the
 * other kernels run instead.
 */
size_t nsq_gemv_workspace_size(int64_t M, int64_t K);
int nsq_gemv(const void *w, int ggml_type, int q6k_layout, const float *x, float *y, int64_t M,
             int64_t N, int64_t K, void *workspace, size_t workspace_bytes, void *stream);

/* The two halves of nsq_gemv, so that projections sharing one activation
 * (q|k|v, gate|up) prepare it once: */
int nsq_prepare_activations(const float *x, int64_t M, int64_t K, void *workspace,
                            size_t workspace_bytes, void *stream);
int nsq_gemv_prepared(const void *w, int ggml_type, int q6k_layout, const void *workspace,
                      float *y, int64_t M, int64_t N, int64_t K, void *stream);

/*
 * nsq_gemv for callers that cannot allocate device memory.  This entry point
 * has no counterpart in the reference.  It computes what nsq_gemv computes
 * (same kernels, same accuracy) but keeps the prepared activations in a
 * fixed scratch array inside the library (NSQ_NOALLOC_MAX_ELEMS / 32 records
 * of 80 bytes, 640 KiB, held by every GPU that loads the library until the
 * process exits), so the call allocates nothing and takes no workspace.
 * For engines whose memory is entirely owned by another allocator, or code
 * that may not call cudaMalloc (it can synchronise the device).
 *   - M * K must not exceed NSQ_NOALLOC_MAX_ELEMS; larger calls return
 *     NSQ_ERR_WORKSPACE.
 *   - All calls share the array: calls that overlap on the GPU (unordered
 *     streams or threads) race and give wrong results.
 *   - The first call on a device looks up the array's device address and
 *     keeps it until the process exits; make that call before capturing a
 *     stream into a CUDA graph, and do not call this entry point again
 *     after a cudaDeviceReset of that device.
 *   - Weight arguments are checked exactly as nsq_gemv checks them (type,
 *     Q5_K / Q6_K layout, 16-byte alignment, K).
 */
#define NSQ_NOALLOC_MAX_ELEMS 262144 /* M * K */
int nsq_gemv_noalloc(const void *w, int ggml_type, int q6k_layout, const float *x, float *y,
                     int64_t M, int64_t N, int64_t K, void *stream);

/*
 * Fused decode GEMV over several weight matrices that share one activation
 * (the q|k|v or gate|up projections of a transformer layer): for every
 * segment s, segs[s].y[M x N_s] = x[M x K] . W_s^T.  One launch streams all
 * segments; formats may differ between segments.  Same accuracy contract as
 * nsq_gemv.  `workspace` (nsq_gemv_workspace_size(M, K) bytes) is used only
 * when M * K is too large for the activations to be prepared on chip; it
 * may be NULL otherwise (the call then returns NSQ_ERR_WORKSPACE if it is
 * needed).  Replaces the per-projection engine.matmul calls of
 * Transformer::forward (crates/nodestor-vulkan/src/transformer.rs:241-315),
 * each of which is a separate submit + queue wait (src/pipeline.rs:486-487).
 */
typedef struct nsq_segment {
  const void *w;   /* GGUF blocks, N rows of K weights, 16-byte aligned */
  int ggml_type;
  int q6k_layout;
  int64_t N;
  float *y;        /* [M x N] f32 */
} nsq_segment;

#define NSQ_MAX_SEGMENTS 4

int nsq_gemv_multi(const nsq_segment *segs, int nseg, const float *x, int64_t M, int64_t K,
                   void *workspace, size_t workspace_bytes, void *stream);

/*
 * Fused FFN input projection: h[M x N] = silu(x . W_gate^T) * (x . W_up^T),
 * one launch that streams both matrices (same format and shape) and never
 * writes gate or up.  Replaces the reference's matmul(gate), matmul(up),
 * silu, mul sequence (crates/nodestor-vulkan/src/transformer.rs:311-314,
 * shaders/silu.comp:14-21, shaders/mul.comp), silu(g) = g * (1 / (1 +
 * exp(-g))).  Same workspace rule as nsq_gemv_multi; needs K % 256 == 0.
 */
int nsq_gemv_swiglu(const void *w_gate, const void *w_up, int ggml_type, int q6k_layout, const float *x,
                    float *h, int64_t M, int64_t N, int64_t K, void *workspace, size_t workspace_bytes,
                    void *stream);

/*
 * GEMV with the residual add fused: y[M x N] = residual + x . W^T (residual
 * may be y itself).  Replaces matmul followed by add
 * (crates/nodestor-vulkan/src/transformer.rs:314-319, shaders/add.comp).
 * Same workspace rule as nsq_gemv_multi; needs K % 256 == 0.
 */
int nsq_gemv_residual(const void *w, int ggml_type, int q6k_layout, const float *x, const float *residual,
                      float *y, int64_t M, int64_t N, int64_t K, void *workspace, size_t workspace_bytes,
                      void *stream);

/*
 * Prefill GEMM on tcgen05 tensor cores: y[M x N] bf16 = x[M x K] bf16 . W^T,
 * weights dequantized to bf16 in shared memory, fp32 accumulation in TMEM.
 * Within 2e-2 relative error of the reference composition on the same
 * (bf16-valued) inputs.  K % 256 == 0; x and y must be 16-byte aligned.  Same reference operator as nsq_gemv, for M > 16.
 */
int nsq_gemm_bf16(const void *w, int ggml_type, int q6k_layout, const void *x_bf16, void *y_bf16,
                  int64_t M, int64_t N, int64_t K, void *stream);

/*
 * Dense f32 matmul with the reference operator's own layout:
 * C[M x N] = A[M x K] . B[K x N], all row-major f32
 * (crates/nodestor-vulkan/shaders/matmul.comp:27-68,
 * crates/nodestor-vulkan/src/lib.rs:117-122).  For the unquantized (F32)
 * weights the reference engine also routes through `matmul`.
 */
int nsq_matmul_f32(const float *a, const float *b, float *c, int64_t M, int64_t K, int64_t N,
                   void *stream);


/*
 * Row-sharded decode GEMV with the all-gather fused into the kernel
 * (tensor parallelism over the GPUs of one node, one process per GPU).
 *
 * Each of `world` ranks holds a contiguous row slice of every weight matrix
 * (a row slice of a GGUF tensor is a contiguous byte range).  The GEMV
 * epilogue stores every output row straight into the exchange buffer of
 * every rank over NVLink (peer stores through CUDA IPC mappings); the last
 * CTA of the grid then publishes a sequence number to each rank's flag
 * word.  The next exchange call (or nsq_comm_wait) waits, with a bounded
 * spin, until every rank's previous exchange has landed before it reads
 * its activations, so the full y is in place on every rank without a
 * separate collective launch.  A wait that gives up after 2 s records
 * NSQ_ERR_TIMEOUT in nsq_device_status and lets the kernel finish.
 *
 * The reference has no collectives (its "fabric" crate simulates RDMA
 * in-process, crates/nodestor-fabric/src/rdma_sim.rs:6-17); this is the
 * build's multi-GPU form of Transformer::forward's matmul calls
 * (crates/nodestor-vulkan/src/transformer.rs:241-315).
 *
 * Setup, on every rank with its device current:
 *   nsq_comm_create(world, rank, bytes, &comm, handle)   -> this rank's handle
 *   (the host exchanges the world handles, e.g. an all-gather over sockets)
 *   nsq_comm_connect(comm, handles)                      -> maps the peers
 * Every rank must issue the same sequence of exchange calls.
 */
#define NSQ_MAX_RANKS 8

typedef struct nsq_comm nsq_comm;

size_t nsq_comm_handle_bytes(void);
/* Allocates this rank's exchange buffer (`bytes` of outputs, zeroed) and
 * writes its IPC handle (nsq_comm_handle_bytes() bytes) to handle_out. */
int nsq_comm_create(int world, int rank, size_t bytes, nsq_comm **comm, void *handle_out);
/* handles: world * nsq_comm_handle_bytes() bytes, rank order. */
int nsq_comm_connect(nsq_comm *comm, const void *handles);
/* Device pointer of this rank's outputs (exchange buffer offset 0). */
void *nsq_comm_buffer(nsq_comm *comm);
/* Enqueues a wait until every rank's latest exchange has landed here. */
int nsq_comm_wait(nsq_comm *comm, void *stream);
int nsq_comm_destroy(nsq_comm *comm);

typedef struct nsq_xsegment {
  const void *w;   /* this rank's rows of the GGUF tensor, 16-byte aligned */
  int ggml_type;
  int q6k_layout;
  int64_t N;       /* rows held by this rank */
  int64_t row0;    /* first row of this rank's slice in the full output */
  int64_t n_full;  /* rows of the full output */
  int64_t y_off;   /* byte offset of y [M x n_full] f32 in every exchange buffer */
} nsq_xsegment;

/* y[m, row0 + r] of every rank's buffer = x[m] . W_rank[r].  Same accuracy
 * contract and workspace rule as nsq_gemv_multi; needs K % 256 == 0.
 * x must not overlap any output range [y_off, y_off + M * n_full * 4) of
 * this call in this rank's buffer (NSQ_ERR_SHAPE): a peer that runs ahead
 * stores this call's rows there while this rank may still be reading x.
 * So an exchange whose input is the previous exchange's output writes a
 * different range (for a chain of exchanges, alternate two ranges). */
int nsq_gemv_multi_xchg(const nsq_xsegment *segs, int nseg, const float *x, int64_t M, int64_t K,
                        nsq_comm *comm, void *workspace, size_t workspace_bytes, void *stream);

/* ---- NSZ (NodeStor Zip) lossless tensors and ZipGEMM ----
 *
 * An NSZ tensor is the tile stream one index entry of an .nsz file points at
 * (crates/nodestor-formats/src/nsz_format.rs:13-44; written by
 * nsz_encoder.rs and nodestor-cli/src/bin/nsz_convert.rs): ceil(count/512)
 * tiles of 512 weights (the last may be shorter), each [header 8][match
 * bitmap][near bitmap][near deltas][residual exponents][mantissas][signs]
 * padded to 64 bytes.  Decoding is lossless: the original FP32 / FP16 / BF16
 * bits come back exactly as nsz_decoder.rs:19-196 restores them. */
#define NSQ_NSZ_FP32 0
#define NSQ_NSZ_FP16 1
#define NSQ_NSZ_BF16 2
#define NSQ_NSZ_TILE_WEIGHTS 512

/* Tiles of a tensor of num_weights weights; its offset table has one more entry. */
int64_t nsq_nsz_num_tiles(int64_t num_weights);

/* HOST function (no GPU): walks the tile headers of a tile stream in host
 * memory (e.g. the mmap of the .nsz file), checks each tile against its
 * bitmaps (dtype byte, near and residual counts, sizes, total length) and
 * writes num_tiles + 1 tile offsets in units of 64 bytes.  The table is what
 * the device entry points take (replaces the reference's fixed tile_stride /
 * tile_meta arguments, lib.rs:124-151, which cannot address variable-size
 * tiles).  NSQ_ERR_FORMAT on any inconsistency. */
int nsq_nsz_index(const void *tiles_host, int64_t nbytes, int64_t num_weights, int dtype, uint32_t *offsets_host);

/* Lossless decode of a whole tensor on the device: out receives num_weights
 * values in the original dtype (uint32 bits for FP32, uint16 for FP16/BF16);
 * bit-exact to nsz_decoder.rs.  tiles and out 16-byte aligned; offsets is the
 * device copy of the nsq_nsz_index table. */
int nsq_nsz_decode(const void *tiles, const uint32_t *offsets, int64_t num_weights, int dtype, void *out,
                   void *stream);

/* ZipGEMM (VulkanEngine::zipgemm, lib.rs:124-151; zipgemm.comp): fused
 * decompress + matmul, y[M x N] f32 = x[M x K] f32 . W^T with W [N x K] the
 * tensor's weights in stream order (GGUF ne0 = K contiguous).  The decoded
 * weights live only in registers.  fp32 accumulation; accuracy contract:
 * max_i |y_i - r_i| / max(|r_i|, rms(r)) <= 1e-3 against the sequential f32
 * oracle.  Any M >= 1 (tokens are processed 8 at a time); fastest with
 * K % 16 == 0 and x 16-byte aligned. */
int nsq_zipgemm(const void *tiles, const uint32_t *offsets, int dtype, const float *x, float *y, int64_t M,
                int64_t N, int64_t K, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* NSQ_H */
