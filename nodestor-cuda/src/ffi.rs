//! Raw declarations of libnsq's C ABI (include/nsq.h) and of the few CUDA
//! runtime calls the engine wrapper needs.  Every nsq_* function returns an
//! NSQ_* status (0 = ok) unless its return type says otherwise.

use std::os::raw::{c_char, c_int, c_void};

pub const NSQ_OK: c_int = 0;
pub const NSQ_ERR_TYPE: c_int = 1;
pub const NSQ_ERR_SHAPE: c_int = 2;
pub const NSQ_ERR_ALIGN: c_int = 3;
pub const NSQ_ERR_NULL: c_int = 4;
pub const NSQ_ERR_CUDA: c_int = 5;
pub const NSQ_ERR_NCCL: c_int = 6;
pub const NSQ_ERR_TIMEOUT: c_int = 7;
pub const NSQ_ERR_WORKSPACE: c_int = 8;
pub const NSQ_ERR_DEVICE: c_int = 9;
pub const NSQ_ERR_FORMAT: c_int = 10;

pub const NSQ_TYPE_Q4_0: c_int = 2;
pub const NSQ_TYPE_Q8_0: c_int = 8;
pub const NSQ_TYPE_Q4_K: c_int = 12;
pub const NSQ_TYPE_Q5_K: c_int = 13;
pub const NSQ_TYPE_Q6_K: c_int = 14;
pub const NSQ_Q6K_GGML: c_int = 0;
pub const NSQ_Q6K_NODESTOR: c_int = 1;
pub const NSQ_OUT_F32: c_int = 0;
pub const NSQ_OUT_BF16: c_int = 1;
pub const NSQ_GEMV_MAX_M: i64 = 16;
pub const NSQ_NOALLOC_MAX_ELEMS: i64 = 262144;
pub const NSQ_NSZ_FP32: c_int = 0;

#[repr(C)]
#[derive(Clone, Copy)]
pub struct NsqSegment {
    pub w: *const c_void,
    pub ggml_type: c_int,
    pub q6k_layout: c_int,
    pub n: i64,
    pub y: *mut f32,
}

#[repr(C)]
#[derive(Clone, Copy)]
pub struct NsqXSegment {
    pub w: *const c_void,
    pub ggml_type: c_int,
    pub q6k_layout: c_int,
    pub n: i64,
    pub row0: i64,
    pub n_full: i64,
    pub y_off: i64,
}

#[repr(C)]
pub struct NsqComm {
    _private: [u8; 0],
}

extern "C" {
    pub fn nsq_version() -> c_int;
    pub fn nsq_reload_tuning();
    pub fn nsq_kernel_launches() -> u64;
    pub fn nsq_strerror(status: c_int) -> *const c_char;
    pub fn nsq_block_bytes(ggml_type: c_int) -> i64;
    pub fn nsq_block_weights(ggml_type: c_int) -> i64;
    pub fn nsq_device_status(clear: c_int) -> c_int;
    pub fn nsq_dequant(w: *const c_void, ggml_type: c_int, q6k_layout: c_int, out_dtype: c_int, out: *mut c_void,
                       n_elems: i64, stream: *mut c_void) -> c_int;
    pub fn nsq_gemv_workspace_size(m: i64, k: i64) -> usize;
    pub fn nsq_gemv(w: *const c_void, ggml_type: c_int, q6k_layout: c_int, x: *const f32, y: *mut f32, m: i64,
                    n: i64, k: i64, workspace: *mut c_void, workspace_bytes: usize, stream: *mut c_void) -> c_int;
    pub fn nsq_prepare_activations(x: *const f32, m: i64, k: i64, workspace: *mut c_void, workspace_bytes: usize,
                                   stream: *mut c_void) -> c_int;
    pub fn nsq_gemv_prepared(w: *const c_void, ggml_type: c_int, q6k_layout: c_int, workspace: *const c_void,
                             y: *mut f32, m: i64, n: i64, k: i64, stream: *mut c_void) -> c_int;
    pub fn nsq_gemv_noalloc(w: *const c_void, ggml_type: c_int, q6k_layout: c_int, x: *const f32, y: *mut f32,
                            m: i64, n: i64, k: i64, stream: *mut c_void) -> c_int;
    pub fn nsq_gemv_multi(segs: *const NsqSegment, nseg: c_int, x: *const f32, m: i64, k: i64,
                          workspace: *mut c_void, workspace_bytes: usize, stream: *mut c_void) -> c_int;
    pub fn nsq_gemv_swiglu(w_gate: *const c_void, w_up: *const c_void, ggml_type: c_int, q6k_layout: c_int,
                           x: *const f32, h: *mut f32, m: i64, n: i64, k: i64, workspace: *mut c_void,
                           workspace_bytes: usize, stream: *mut c_void) -> c_int;
    pub fn nsq_gemv_residual(w: *const c_void, ggml_type: c_int, q6k_layout: c_int, x: *const f32,
                             residual: *const f32, y: *mut f32, m: i64, n: i64, k: i64, workspace: *mut c_void,
                             workspace_bytes: usize, stream: *mut c_void) -> c_int;
    pub fn nsq_gemm_bf16(w: *const c_void, ggml_type: c_int, q6k_layout: c_int, x_bf16: *const c_void,
                         y_bf16: *mut c_void, m: i64, n: i64, k: i64, stream: *mut c_void) -> c_int;
    pub fn nsq_matmul_f32(a: *const f32, b: *const f32, c: *mut f32, m: i64, k: i64, n: i64,
                          stream: *mut c_void) -> c_int;
    // row-sharded decode over the GPUs of a node (one process per GPU)
    pub fn nsq_comm_handle_bytes() -> usize;
    pub fn nsq_comm_create(world: c_int, rank: c_int, bytes: usize, comm: *mut *mut NsqComm,
                           handle_out: *mut c_void) -> c_int;
    pub fn nsq_comm_connect(comm: *mut NsqComm, handles: *const c_void) -> c_int;
    pub fn nsq_comm_buffer(comm: *mut NsqComm) -> *mut c_void;
    pub fn nsq_comm_wait(comm: *mut NsqComm, stream: *mut c_void) -> c_int;
    pub fn nsq_comm_destroy(comm: *mut NsqComm) -> c_int;
    pub fn nsq_gemv_multi_xchg(segs: *const NsqXSegment, nseg: c_int, x: *const f32, m: i64, k: i64,
                               comm: *mut NsqComm, workspace: *mut c_void, workspace_bytes: usize,
                               stream: *mut c_void) -> c_int;
    // NSZ (TCA-TBE) lossless tensors and ZipGEMM
    pub fn nsq_nsz_num_tiles(num_weights: i64) -> i64;
    pub fn nsq_nsz_index(tiles_host: *const c_void, nbytes: i64, num_weights: i64, dtype: c_int,
                         offsets_host: *mut u32) -> c_int;
    pub fn nsq_nsz_decode(tiles: *const c_void, offsets: *const u32, num_weights: i64, dtype: c_int,
                          out: *mut c_void, stream: *mut c_void) -> c_int;
    pub fn nsq_zipgemm(tiles: *const c_void, offsets: *const u32, dtype: c_int, x: *const f32, y: *mut f32,
                       m: i64, n: i64, k: i64, stream: *mut c_void) -> c_int;
}

/// The CUDA runtime calls the engine wrapper makes (libcudart).
pub mod cudart {
    use std::os::raw::{c_int, c_void};

    pub const MEMCPY_HOST_TO_DEVICE: c_int = 1;
    pub const MEMCPY_DEVICE_TO_HOST: c_int = 2;

    extern "C" {
        pub fn cudaSetDevice(device: c_int) -> c_int;
        pub fn cudaMalloc(ptr: *mut *mut c_void, bytes: usize) -> c_int;
        pub fn cudaFree(ptr: *mut c_void) -> c_int;
        pub fn cudaMemcpy(dst: *mut c_void, src: *const c_void, bytes: usize, kind: c_int) -> c_int;
        pub fn cudaStreamCreate(stream: *mut *mut c_void) -> c_int;
        pub fn cudaStreamSynchronize(stream: *mut c_void) -> c_int;
        pub fn cudaStreamDestroy(stream: *mut c_void) -> c_int;
    }
}
