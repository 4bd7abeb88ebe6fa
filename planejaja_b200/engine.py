"""Host-side mirror of the reference engine's matmul / dequant operators.

`CudaEngine` keeps the shape of NodeStor's `VulkanEngine`
(nodestor/crates/nodestor-vulkan/src/lib.rs:38-271) for the hot path:

  upload(bytes)                 -> device buffer       (lib.rs:221-224)
  download_f32(buf)             -> host f32 array      (lib.rs:236-239)
  matmul(a, b, m, k, n)         -> C = A[m,k] . B[k,n] (lib.rs:117-122, dense f32)
  matmul_quant(x, w, t, m, k, n)-> y = x . W^T over GGUF blocks (the quantized
                                   branch of TensorOp::Matmul,
                                   src/operator_registry.rs:43-49, 246-259)
  dequant(w, t, n)              -> f32 / bf16 weights (DequantDispatcher::dequantize,
                                   crates/nodestor-inference/src/dequant/mod.rs:142-191)
  zipgemm(w, x, m, k, n)        -> y = x . W^T from an NSZ (TCA-TBE) tensor,
                                   decompressed in registers (lib.rs:124-151)
  nsz_decode(w)                 -> the NSZ tensor's original weights, bit-exact
                                   (nsz_decoder.rs:19-196)

Device memory, streams and the output buffers come from PyTorch; every
computation is a call into libnsq.so.  Like the reference, calls are
synchronous by default (the reference waits for queue idle after every
dispatch, src/pipeline.rs:486-487); pass `sync=False` to stay asynchronous on
the current CUDA stream.  Errors raise NsqError (the reference returns
NodeStorError, crates/nodestor-core/src/error.rs:1-38).

Kernel choice for matmul_quant: M <= 16 uses the decode GEMV (fp32
activations and output); larger M uses the tcgen05 prefill GEMM (bf16
operands, fp32 accumulate, bf16 output widened back to f32).  The
environment variable NSQ_MATMUL_PATH=gemv|gemm forces one of them.
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional

import numpy as np
import torch

from . import _lib
from .formats import FORMATS, Q6K_GGML, fmt
from ._lib import NsqError, check


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


class CudaEngine:
    """Engine facade over libnsq for one CUDA device."""

    def __init__(self, device: int | str | torch.device = 0):
        if not torch.cuda.is_available():
            raise NsqError(_lib.ERR_DEVICE, "no CUDA device")
        self.device = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
        self.lib = _lib.load()
        self._ws: Optional[torch.Tensor] = None

    # ---- buffers ---------------------------------------------------------
    def upload(self, data) -> torch.Tensor:
        """Copy host bytes (bytes / numpy array) to a new device uint8 buffer."""
        arr = np.frombuffer(data, np.uint8) if isinstance(data, (bytes, bytearray, memoryview)) else \
            np.ascontiguousarray(data).view(np.uint8).reshape(-1)
        return torch.from_numpy(arr.copy()).to(self.device)

    def upload_f32(self, data) -> torch.Tensor:
        return torch.as_tensor(np.ascontiguousarray(data, np.float32)).to(self.device)

    def download_f32(self, buf: torch.Tensor) -> np.ndarray:
        return buf.detach().float().cpu().numpy()

    def workspace(self, nbytes: int) -> torch.Tensor:
        """Scratch for prepared activations; grown outside the hot calls."""
        if self._ws is None or self._ws.numel() < nbytes:
            self._ws = torch.empty(max(nbytes, 1 << 16), dtype=torch.uint8, device=self.device)
        return self._ws

    def _stream(self) -> int:
        return _stream_handle(self.device)

    def _sync(self, sync: bool):
        if sync:
            torch.cuda.synchronize(self.device)

    # ---- operators ---------------------------------------------------------
    def dequant(self, w: torch.Tensor, ggml_type: int, n_elems: int, out_dtype: str = "f32",
                q6k_layout: int = Q6K_GGML, out: Optional[torch.Tensor] = None, sync: bool = True) -> torch.Tensor:
        od = _lib.OUT_F32 if out_dtype == "f32" else _lib.OUT_BF16
        if out is None:
            out = torch.empty(n_elems, dtype=torch.float32 if od == _lib.OUT_F32 else torch.bfloat16,
                              device=self.device)
        check(self.lib.nsq_dequant(_ptr(w), ggml_type, q6k_layout, od, _ptr(out), n_elems, self._stream()),
              "nsq_dequant")
        self._sync(sync)
        return out

    def gemv(self, w: torch.Tensor, ggml_type: int, x: torch.Tensor, n: int, k: int,
             q6k_layout: int = Q6K_GGML, y: Optional[torch.Tensor] = None, sync: bool = True) -> torch.Tensor:
        m = x.numel() // k
        if y is None:
            y = torch.empty((m, n), dtype=torch.float32, device=self.device)
        wsb = self.lib.nsq_gemv_workspace_size(m, k)
        ws = self.workspace(wsb)
        check(self.lib.nsq_gemv(_ptr(w), ggml_type, q6k_layout, _ptr(x), _ptr(y), m, n, k, _ptr(ws), ws.numel(),
                                self._stream()), "nsq_gemv")
        self._sync(sync)
        return y

    def gemv_multi(self, segments, x: torch.Tensor, k: int, sync: bool = True):
        """Fused GEMV over matrices sharing `x` (q|k|v, gate|up).

        segments: list of (w, ggml_type, n) or (w, ggml_type, n, q6k_layout);
        returns the list of outputs [m, n_s] (f32)."""
        m = x.numel() // k
        segs = (_lib.Segment * len(segments))()
        outs = []
        for i, sg in enumerate(segments):
            w, t, n = sg[0], sg[1], sg[2]
            layout = sg[3] if len(sg) > 3 else Q6K_GGML
            y = torch.empty((m, n), dtype=torch.float32, device=self.device)
            outs.append(y)
            segs[i] = _lib.Segment(_ptr(w), t, layout, n, _ptr(y))
        wsb = self.lib.nsq_gemv_workspace_size(m, k)
        ws = self.workspace(wsb)
        check(self.lib.nsq_gemv_multi(ctypes.cast(segs, ctypes.c_void_p), len(segments), _ptr(x), m, k, _ptr(ws),
                                      ws.numel(), self._stream()), "nsq_gemv_multi")
        self._sync(sync)
        return outs

    def gemv_swiglu(self, w_gate: torch.Tensor, w_up: torch.Tensor, ggml_type: int, x: torch.Tensor, n: int, k: int,
                    q6k_layout: int = Q6K_GGML, out: Optional[torch.Tensor] = None, sync: bool = True) -> torch.Tensor:
        """h[m, n] = silu(x . Wg^T) * (x . Wu^T) in one launch (the FFN input
        projection with the reference's silu + mul fused in)."""
        m = x.numel() // k
        h = out if out is not None else torch.empty(m, n, dtype=torch.float32, device=self.device)
        x = x.contiguous().float()
        ws = self.workspace(self.lib.nsq_gemv_workspace_size(m, k))
        check(self.lib.nsq_gemv_swiglu(_ptr(w_gate), _ptr(w_up), ggml_type, q6k_layout, _ptr(x), _ptr(h), m, n, k,
                                       _ptr(ws), ws.numel(), self._stream()), "nsq_gemv_swiglu")
        self._sync(sync)
        return h

    def gemv_residual(self, w: torch.Tensor, ggml_type: int, x: torch.Tensor, residual: torch.Tensor, n: int, k: int,
                      q6k_layout: int = Q6K_GGML, out: Optional[torch.Tensor] = None, sync: bool = True) -> torch.Tensor:
        """y = residual + x . W^T in one launch; `out` may be `residual` (in place)."""
        m = x.numel() // k
        y = out if out is not None else torch.empty(m, n, dtype=torch.float32, device=self.device)
        x = x.contiguous().float()
        residual = residual.contiguous().float()
        ws = self.workspace(self.lib.nsq_gemv_workspace_size(m, k))
        check(self.lib.nsq_gemv_residual(_ptr(w), ggml_type, q6k_layout, _ptr(x), _ptr(residual), _ptr(y), m, n, k,
                                         _ptr(ws), ws.numel(), self._stream()), "nsq_gemv_residual")
        self._sync(sync)
        return y

    def prepare(self, x: torch.Tensor, k: int, ws: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Prepare activations once for several GEMVs (q|k|v, gate|up)."""
        m = x.numel() // k
        nbytes = self.lib.nsq_gemv_workspace_size(m, k)
        if ws is None:
            ws = torch.empty(nbytes, dtype=torch.uint8, device=self.device)
        check(self.lib.nsq_prepare_activations(_ptr(x), m, k, _ptr(ws), ws.numel(), self._stream()),
              "nsq_prepare_activations")
        return ws

    def gemv_prepared(self, w: torch.Tensor, ggml_type: int, ws: torch.Tensor, m: int, n: int, k: int,
                      q6k_layout: int = Q6K_GGML, y: Optional[torch.Tensor] = None) -> torch.Tensor:
        if y is None:
            y = torch.empty((m, n), dtype=torch.float32, device=self.device)
        check(self.lib.nsq_gemv_prepared(_ptr(w), ggml_type, q6k_layout, _ptr(ws), _ptr(y), m, n, k,
                                         self._stream()), "nsq_gemv_prepared")
        return y

    def gemm_bf16(self, w: torch.Tensor, ggml_type: int, x: torch.Tensor, n: int, k: int,
                  q6k_layout: int = Q6K_GGML, y: Optional[torch.Tensor] = None, sync: bool = True) -> torch.Tensor:
        if x.dtype != torch.bfloat16:
            raise NsqError(_lib.ERR_TYPE, "gemm_bf16 expects bf16 activations")
        m = x.numel() // k
        if y is None:
            y = torch.empty((m, n), dtype=torch.bfloat16, device=self.device)
        check(self.lib.nsq_gemm_bf16(_ptr(w), ggml_type, q6k_layout, _ptr(x), _ptr(y), m, n, k, self._stream()),
              "nsq_gemm_bf16")
        self._sync(sync)
        return y

    def matmul(self, a: torch.Tensor, b: torch.Tensor, m: int, k: int, n: int, sync: bool = True) -> torch.Tensor:
        """Dense f32 C[m, n] = A[m, k] . B[k, n] (the reference operator's layout)."""
        c = torch.empty((m, n), dtype=torch.float32, device=self.device)
        check(self.lib.nsq_matmul_f32(_ptr(a), _ptr(b), _ptr(c), m, k, n, self._stream()), "nsq_matmul_f32")
        self._sync(sync)
        return c

    def matmul_quant(self, x: torch.Tensor, w: torch.Tensor, ggml_type: int, m: int, k: int, n: int,
                     q6k_layout: int = Q6K_GGML, sync: bool = True) -> torch.Tensor:
        """y[m, n] f32 = x[m, k] . W^T with W[n, k] in GGUF blocks of `ggml_type`."""
        if ggml_type not in FORMATS:
            raise NsqError(_lib.ERR_TYPE, f"matmul_quant: ggml type {ggml_type}")
        if w.numel() < fmt(ggml_type).tensor_bytes(n, k):
            raise NsqError(_lib.ERR_SHAPE, "matmul_quant: weight buffer smaller than N*row_bytes")
        path = os.environ.get("NSQ_MATMUL_PATH", "")
        if path == "gemv" or (path != "gemm" and m <= _lib.GEMV_MAX_M):
            return self.gemv(w, ggml_type, x.reshape(m, k).float().contiguous(), n, k, q6k_layout, sync=sync)
        xb = x.reshape(m, k).to(torch.bfloat16).contiguous()
        return self.gemm_bf16(w, ggml_type, xb, n, k, q6k_layout, sync=sync).float()

    # ---- NSZ (TCA-TBE) tensors and ZipGEMM --------------------------------
    def nsz_upload(self, stream, num_weights: int, dtype: int = _lib.NSZ_FP32, shape=()) -> "NszTensor":
        """One-time upload of an NSZ tile stream and its validated offset table."""
        from .nsz import NszTensor, index
        stream = np.ascontiguousarray(stream, np.uint8).reshape(-1)
        off = index(stream, num_weights, dtype)
        tiles = torch.from_numpy(stream.copy()).to(self.device) if stream.size else \
            torch.empty(16, dtype=torch.uint8, device=self.device)
        offsets = torch.from_numpy(off.view(np.int32)).to(self.device)
        return NszTensor(tiles, offsets, int(num_weights), int(dtype), tuple(shape))

    def nsz_decode(self, t, out: Optional[torch.Tensor] = None, sync: bool = True) -> torch.Tensor:
        """Lossless decode: float32 / float16 / bfloat16 weights, bit-exact."""
        dt = {_lib.NSZ_FP32: torch.float32, _lib.NSZ_FP16: torch.float16, _lib.NSZ_BF16: torch.bfloat16}[t.dtype]
        if out is None:
            out = torch.empty(max(t.count, 1), dtype=dt, device=self.device)[:t.count]
        check(self.lib.nsq_nsz_decode(_ptr(t.tiles), _ptr(t.offsets), t.count, t.dtype, _ptr(out),
                                      self._stream()), "nsq_nsz_decode")
        self._sync(sync)
        return out

    def zipgemm(self, w, x: torch.Tensor, m: int, k: int, n: int, out: Optional[torch.Tensor] = None,
                sync: bool = True) -> torch.Tensor:
        """ZipGEMM (VulkanEngine::zipgemm, lib.rs:124-151): y[m, n] f32 =
        x[m, k] . W^T, W [n x k] decompressed on the fly from an NszTensor."""
        if w.count != n * k:
            raise NsqError(_lib.ERR_SHAPE, f"zipgemm: tensor holds {w.count} weights, not {n} x {k}")
        x = x.reshape(m, k)
        if x.dtype != torch.float32 or not x.is_contiguous():
            x = x.float().contiguous()
        if out is None:
            out = torch.empty((m, n), dtype=torch.float32, device=self.device)
        check(self.lib.nsq_zipgemm(_ptr(w.tiles), _ptr(w.offsets), w.dtype, _ptr(x), _ptr(out), m, n, k,
                                   self._stream()), "nsq_zipgemm")
        self._sync(sync)
        return out

    def device_status(self, clear: bool = True) -> int:
        """NSQ_ERR_TIMEOUT if a bounded device-side wait gave up, else 0."""
        return self.lib.nsq_device_status(1 if clear else 0)
