//! NodeStor CUDA engine: the quantized dequant + matmul hot path on B200.
//!
//! `CudaEngine` keeps the shape of `VulkanEngine` (crates/nodestor-vulkan/
//! src/lib.rs): inputs are borrowed buffers, every operator returns a newly
//! allocated output buffer, errors come back as `NodeStorError`, and each
//! call blocks until its work is done, as the reference's submit-and-wait
//! dispatch does (crates/nodestor-vulkan/src/pipeline.rs:486-487).  The work
//! itself is libnsq's (include/nsq.h): GGUF-native weight bytes, the fused
//! decode GEMV for M <= 16, the tcgen05 prefill GEMM above that.
//!
//! Not compiled here: this environment has no cargo or rustc.

pub mod ffi;

use std::ffi::CStr;
use std::os::raw::{c_int, c_void};
use std::ptr;
use std::sync::Mutex;

use nodestor_core::NodeStorError;

use ffi::cudart;

/// Maps an NSQ_* status onto the reference's error type
/// (crates/nodestor-core/src/error.rs:1-38).  CUDA-side failures keep the
/// `VulkanError(String)` variant, so callers that match on it still work.
pub fn check(status: c_int, what: &str) -> Result<(), NodeStorError> {
    if status == ffi::NSQ_OK {
        return Ok(());
    }
    let text = unsafe { CStr::from_ptr(ffi::nsq_strerror(status)) }.to_string_lossy().into_owned();
    let msg = format!("{what}: {text}");
    Err(match status {
        ffi::NSQ_ERR_TYPE => NodeStorError::NotSupported(msg),
        ffi::NSQ_ERR_SHAPE | ffi::NSQ_ERR_ALIGN | ffi::NSQ_ERR_NULL | ffi::NSQ_ERR_WORKSPACE => {
            NodeStorError::ConfigError(msg)
        }
        ffi::NSQ_ERR_FORMAT => NodeStorError::InvalidModelFormat(msg),
        ffi::NSQ_ERR_TIMEOUT => NodeStorError::Timeout { ms: 2000 },
        _ => NodeStorError::VulkanError(msg),
    })
}

fn cuda(status: c_int, what: &str) -> Result<(), NodeStorError> {
    if status == 0 {
        Ok(())
    } else {
        Err(NodeStorError::VulkanError(format!("{what}: CUDA error {status}")))
    }
}

/// Device memory owned by the engine's caller; freed on drop (the
/// reference's GpuBuffer frees in Drop, buffer.rs:455-464).
pub struct CudaBuffer {
    ptr: *mut c_void,
    len: usize,
}

unsafe impl Send for CudaBuffer {}
unsafe impl Sync for CudaBuffer {}

impl CudaBuffer {
    pub fn alloc(len: usize) -> Result<Self, NodeStorError> {
        let mut p = ptr::null_mut();
        if len > 0 {
            cuda(unsafe { cudart::cudaMalloc(&mut p, len) }, "cudaMalloc")?;
        }
        Ok(Self { ptr: p, len })
    }

    /// Uploads host bytes (e.g. a GGUF tensor straight from the loader's
    /// mmap; the kernels read the file's block bytes unchanged).
    pub fn from_host(bytes: &[u8]) -> Result<Self, NodeStorError> {
        let b = Self::alloc(bytes.len())?;
        if !bytes.is_empty() {
            cuda(unsafe { cudart::cudaMemcpy(b.ptr, bytes.as_ptr() as *const c_void, bytes.len(),
                                             cudart::MEMCPY_HOST_TO_DEVICE) }, "cudaMemcpy")?;
        }
        Ok(b)
    }

    pub fn from_f32(v: &[f32]) -> Result<Self, NodeStorError> {
        let bytes = unsafe { std::slice::from_raw_parts(v.as_ptr() as *const u8, v.len() * 4) };
        Self::from_host(bytes)
    }

    pub fn to_f32_vec(&self) -> Result<Vec<f32>, NodeStorError> {
        let mut v = vec![0f32; self.len / 4];
        if !v.is_empty() {
            cuda(unsafe { cudart::cudaMemcpy(v.as_mut_ptr() as *mut c_void, self.ptr, v.len() * 4,
                                             cudart::MEMCPY_DEVICE_TO_HOST) }, "cudaMemcpy")?;
        }
        Ok(v)
    }

    pub fn len(&self) -> usize {
        self.len
    }

    pub fn is_empty(&self) -> bool {
        self.len == 0
    }

    pub fn as_ptr(&self) -> *const c_void {
        self.ptr
    }

    pub fn as_mut_ptr(&self) -> *mut c_void {
        self.ptr
    }
}

impl Drop for CudaBuffer {
    fn drop(&mut self) {
        if !self.ptr.is_null() {
            unsafe { cudart::cudaFree(self.ptr) };
        }
    }
}

/// Largest K the engine's workspace is sized for at M = 16.
pub const MAX_K: i64 = 65536;

pub struct CudaEngine {
    stream: *mut c_void,
    // prepared activations for nsq_gemv when they do not fit on chip; one
    // per engine, sized once, shared by calls under the lock
    workspace: Mutex<CudaBuffer>,
}

unsafe impl Send for CudaEngine {}
unsafe impl Sync for CudaEngine {}

impl CudaEngine {
    pub fn new(device: i32) -> Result<Self, NodeStorError> {
        cuda(unsafe { cudart::cudaSetDevice(device) }, "cudaSetDevice")?;
        let mut stream = ptr::null_mut();
        cuda(unsafe { cudart::cudaStreamCreate(&mut stream) }, "cudaStreamCreate")?;
        let ws = unsafe { ffi::nsq_gemv_workspace_size(ffi::NSQ_GEMV_MAX_M, MAX_K) };
        Ok(Self { stream, workspace: Mutex::new(CudaBuffer::alloc(ws)?) })
    }

    fn sync(&self) -> Result<(), NodeStorError> {
        cuda(unsafe { cudart::cudaStreamSynchronize(self.stream) }, "cudaStreamSynchronize")?;
        check(unsafe { ffi::nsq_device_status(1) }, "device status")
    }

    /// The reference operator (lib.rs:117-122): C[m x n] = A[m x k] . B[k x n],
    /// dense f32, row-major, B in the reference's [K x N] layout.
    pub fn matmul(&self, a: &CudaBuffer, b: &CudaBuffer, m: u32, k: u32, n: u32) -> Result<CudaBuffer, NodeStorError> {
        let out = CudaBuffer::alloc(m as usize * n as usize * 4)?;
        check(unsafe { ffi::nsq_matmul_f32(a.as_ptr() as *const f32, b.as_ptr() as *const f32,
                                           out.as_mut_ptr() as *mut f32, m as i64, k as i64, n as i64,
                                           self.stream) }, "matmul")?;
        self.sync()?;
        Ok(out)
    }

    /// y[m x n] = x[m x k] . W^T with W [n x k] GGUF blocks of `ggml_type`
    /// (the `quantized` form of TensorOp::Matmul, operator_registry.rs:43-49).
    /// m <= 16 runs the decode GEMV on f32 activations; above that the
    /// activations are rounded to bf16 on the host and the tcgen05 GEMM runs.
    pub fn matmul_quant(&self, x: &CudaBuffer, w: &CudaBuffer, ggml_type: i32, q6k_layout: i32, m: u32, k: u32,
                        n: u32) -> Result<CudaBuffer, NodeStorError> {
        let (m, k, n) = (m as i64, k as i64, n as i64);
        if m <= ffi::NSQ_GEMV_MAX_M {
            let out = CudaBuffer::alloc((m * n * 4) as usize)?;
            let ws = self.workspace.lock().map_err(|_| NodeStorError::ConfigError("workspace lock".into()))?;
            check(unsafe { ffi::nsq_gemv(w.as_ptr(), ggml_type, q6k_layout, x.as_ptr() as *const f32,
                                         out.as_mut_ptr() as *mut f32, m, n, k, ws.as_mut_ptr(), ws.len(),
                                         self.stream) }, "matmul_quant")?;
            self.sync()?;
            return Ok(out);
        }
        // prefill: bf16 operands, fp32 accumulation, bf16 out widened to f32
        let xf = x.to_f32_vec()?;
        let xb: Vec<u16> = xf.iter().map(|v| f32_to_bf16(*v)).collect();
        let xd = CudaBuffer::from_host(unsafe { std::slice::from_raw_parts(xb.as_ptr() as *const u8, xb.len() * 2) })?;
        let yb = CudaBuffer::alloc((m * n * 2) as usize)?;
        check(unsafe { ffi::nsq_gemm_bf16(w.as_ptr(), ggml_type, q6k_layout, xd.as_ptr(), yb.as_mut_ptr(), m, n, k,
                                          self.stream) }, "matmul_quant (prefill)")?;
        self.sync()?;
        let mut h = vec![0u16; (m * n) as usize];
        cuda(unsafe { cudart::cudaMemcpy(h.as_mut_ptr() as *mut c_void, yb.as_ptr(), h.len() * 2,
                                         cudart::MEMCPY_DEVICE_TO_HOST) }, "cudaMemcpy")?;
        let y: Vec<f32> = h.iter().map(|b| f32::from_bits((*b as u32) << 16)).collect();
        CudaBuffer::from_f32(&y)
    }

    /// One launch for several projections sharing x (q|k|v, gate|up of
    /// Transformer::forward, transformer.rs:241-315); one output per matrix.
    pub fn matmul_fused(&self, x: &CudaBuffer, mats: &[(&CudaBuffer, i32, i32, u32)], m: u32, k: u32)
                        -> Result<Vec<CudaBuffer>, NodeStorError> {
        let mut outs = Vec::with_capacity(mats.len());
        let mut segs = Vec::with_capacity(mats.len());
        for (w, t, lay, n) in mats {
            let y = CudaBuffer::alloc(m as usize * *n as usize * 4)?;
            segs.push(ffi::NsqSegment { w: w.as_ptr(), ggml_type: *t, q6k_layout: *lay, n: *n as i64,
                                        y: y.as_mut_ptr() as *mut f32 });
            outs.push(y);
        }
        let ws = self.workspace.lock().map_err(|_| NodeStorError::ConfigError("workspace lock".into()))?;
        check(unsafe { ffi::nsq_gemv_multi(segs.as_ptr(), segs.len() as c_int, x.as_ptr() as *const f32, m as i64,
                                           k as i64, ws.as_mut_ptr(), ws.len(), self.stream) }, "matmul_fused")?;
        self.sync()?;
        Ok(outs)
    }

    /// h = silu(x . W_gate^T) * (x . W_up^T) in one launch: the gate, up,
    /// silu and mul calls of transformer.rs:311-314.
    pub fn ffn_in(&self, x: &CudaBuffer, w_gate: &CudaBuffer, w_up: &CudaBuffer, ggml_type: i32, q6k_layout: i32,
                  m: u32, k: u32, n: u32) -> Result<CudaBuffer, NodeStorError> {
        let h = CudaBuffer::alloc(m as usize * n as usize * 4)?;
        let ws = self.workspace.lock().map_err(|_| NodeStorError::ConfigError("workspace lock".into()))?;
        check(unsafe { ffi::nsq_gemv_swiglu(w_gate.as_ptr(), w_up.as_ptr(), ggml_type, q6k_layout,
                                            x.as_ptr() as *const f32, h.as_mut_ptr() as *mut f32, m as i64,
                                            n as i64, k as i64, ws.as_mut_ptr(), ws.len(), self.stream) },
              "ffn_in")?;
        self.sync()?;
        Ok(h)
    }

    /// y = residual + x . W^T (the down projection and its residual add,
    /// transformer.rs:314-319).
    pub fn matmul_add(&self, x: &CudaBuffer, w: &CudaBuffer, residual: &CudaBuffer, ggml_type: i32,
                      q6k_layout: i32, m: u32, k: u32, n: u32) -> Result<CudaBuffer, NodeStorError> {
        let y = CudaBuffer::alloc(m as usize * n as usize * 4)?;
        let ws = self.workspace.lock().map_err(|_| NodeStorError::ConfigError("workspace lock".into()))?;
        check(unsafe { ffi::nsq_gemv_residual(w.as_ptr(), ggml_type, q6k_layout, x.as_ptr() as *const f32,
                                              residual.as_ptr() as *const f32, y.as_mut_ptr() as *mut f32,
                                              m as i64, n as i64, k as i64, ws.as_mut_ptr(), ws.len(),
                                              self.stream) }, "matmul_add")?;
        self.sync()?;
        Ok(y)
    }

    /// Dequantizes n_elems weights to f32 (bit-exact to the reference's
    /// dequant kernels and DequantDispatcher).
    pub fn dequant(&self, w: &CudaBuffer, ggml_type: i32, q6k_layout: i32, n_elems: u64)
                   -> Result<CudaBuffer, NodeStorError> {
        let out = CudaBuffer::alloc(n_elems as usize * 4)?;
        check(unsafe { ffi::nsq_dequant(w.as_ptr(), ggml_type, q6k_layout, ffi::NSQ_OUT_F32, out.as_mut_ptr(),
                                        n_elems as i64, self.stream) }, "dequant")?;
        self.sync()?;
        Ok(out)
    }

    /// ZipGEMM over an NSZ tensor (VulkanEngine::zipgemm, lib.rs:124-151).
    /// The reference's tile_meta / tile_stride / num_k_tiles /
    /// weights_per_tile arguments become the tile offset table built once
    /// by `nsz_offsets` (NSZ tiles vary in size).
    pub fn zipgemm(&self, tiles: &CudaBuffer, offsets: &CudaBuffer, activations: &CudaBuffer, m: u32, k: u32,
                   n: u32) -> Result<CudaBuffer, NodeStorError> {
        let out = CudaBuffer::alloc(m as usize * n as usize * 4)?;
        check(unsafe { ffi::nsq_zipgemm(tiles.as_ptr(), offsets.as_ptr() as *const u32, ffi::NSQ_NSZ_FP32,
                                        activations.as_ptr() as *const f32, out.as_mut_ptr() as *mut f32, m as i64,
                                        n as i64, k as i64, self.stream) }, "zipgemm")?;
        self.sync()?;
        Ok(out)
    }

    /// Host side of ZipGEMM's set-up: the tile offset table of an NSZ tile
    /// stream held in host memory (the .nsz mmap), checked tile by tile.
    pub fn nsz_offsets(tiles_host: &[u8], num_weights: u64) -> Result<CudaBuffer, NodeStorError> {
        let nt = unsafe { ffi::nsq_nsz_num_tiles(num_weights as i64) } as usize;
        let mut off = vec![0u32; nt + 1];
        check(unsafe { ffi::nsq_nsz_index(tiles_host.as_ptr() as *const c_void, tiles_host.len() as i64,
                                          num_weights as i64, ffi::NSQ_NSZ_FP32, off.as_mut_ptr()) },
              "nsz_index")?;
        CudaBuffer::from_host(unsafe { std::slice::from_raw_parts(off.as_ptr() as *const u8, off.len() * 4) })
    }
}

impl Drop for CudaEngine {
    fn drop(&mut self) {
        unsafe {
            cudart::cudaStreamSynchronize(self.stream);
            cudart::cudaStreamDestroy(self.stream);
        }
    }
}

/// Round to nearest even, as the GEMM's bf16 operands are defined (NaN kept quiet).
fn f32_to_bf16(v: f32) -> u16 {
    let b = v.to_bits();
    if v.is_nan() {
        return ((b >> 16) | 0x40) as u16;
    }
    let round = 0x7FFF + ((b >> 16) & 1);
    (b.wrapping_add(round) >> 16) as u16
}
