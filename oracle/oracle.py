"""ctypes binding of the CPU oracle (liboracle.so, built from nsq_oracle.c).

TEST INFRASTRUCTURE ONLY: the checker for libnsq.  Imported by tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline / reference legs, never by
the product package.  Function-by-function reference citations are in
nsq_oracle.c.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

_u8p = ctypes.POINTER(ctypes.c_uint8)
_f32p = ctypes.POINTER(ctypes.c_float)
_f64p = ctypes.POINTER(ctypes.c_double)
_i64 = ctypes.c_int64


def build(force: bool = False) -> str:
    srcs = [os.path.join(_HERE, f) for f in ("nsq_oracle.c", "nsz_oracle.c")]
    if force or not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < max(map(os.path.getmtime, srcs)):
        subprocess.run(["make", "-s", "-C", _HERE, "liboracle.so"], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        L.orc_half_to_f32.restype = ctypes.c_float
        L.orc_half_to_f32.argtypes = [ctypes.c_uint16]
        L.orc_half_to_f32_shader.restype = ctypes.c_float
        L.orc_half_to_f32_shader.argtypes = [ctypes.c_uint16]
        L.orc_get_scale_min_k4.restype = ctypes.c_uint32
        L.orc_get_scale_min_k4.argtypes = [ctypes.c_int, _u8p]
        L.orc_dequant.restype = ctypes.c_int
        L.orc_dequant.argtypes = [_u8p, ctypes.c_int, ctypes.c_int, _i64, _f32p, ctypes.c_int]
        L.orc_dequant_q4_k_avx2.restype = None
        L.orc_dequant_q4_k_avx2.argtypes = [_u8p, _i64, _f32p]
        L.orc_matmul_f32.restype = None
        L.orc_matmul_f32.argtypes = [_f32p, _f32p, _f32p, _i64, _i64, _i64]
        L.orc_matmul_f64.restype = None
        L.orc_matmul_f64.argtypes = [_f32p, _f32p, _f64p, _i64, _i64, _i64]
        L.orc_quant_matmul.restype = ctypes.c_int
        L.orc_quant_matmul.argtypes = [_u8p, ctypes.c_int, ctypes.c_int, _f32p, _f32p, _i64, _i64, _i64]
        L.orc_quant_matmul_mt.restype = ctypes.c_int
        L.orc_quant_matmul_mt.argtypes = [_u8p, ctypes.c_int, ctypes.c_int, _f32p, _f32p, _i64, _i64, _i64,
                                          ctypes.c_int]
        L.orc_num_threads.restype = ctypes.c_int
        L.orc_block_weights.restype = _i64
        L.orc_block_weights.argtypes = [ctypes.c_int]
        L.orc_block_bytes.restype = _i64
        L.orc_block_bytes.argtypes = [ctypes.c_int]
        L.orc_nsz_max_tile_bytes.restype = _i64
        L.orc_nsz_max_tile_bytes.argtypes = [ctypes.c_int]
        L.orc_nsz_encode_tile.restype = _i64
        L.orc_nsz_encode_tile.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, _u8p]
        L.orc_nsz_decode_tile.restype = _i64
        L.orc_nsz_decode_tile.argtypes = [_u8p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
        L.orc_nsz_encode.restype = _i64
        L.orc_nsz_encode.argtypes = [ctypes.c_void_p, _i64, ctypes.c_int, ctypes.c_int, _u8p, _i64]
        L.orc_nsz_offsets.restype = ctypes.c_int
        L.orc_nsz_offsets.argtypes = [_u8p, _i64, _i64, ctypes.c_int, ctypes.POINTER(_i64)]
        L.orc_nsz_decode.restype = ctypes.c_int
        L.orc_nsz_decode.argtypes = [_u8p, _i64, _i64, ctypes.c_int, ctypes.c_void_p]
        L.orc_nsz_matmul.restype = ctypes.c_int
        L.orc_nsz_matmul.argtypes = [_u8p, _i64, _f32p, _f32p, _i64, _i64, _i64]
        _lib = L
    return _lib


def _p(a: np.ndarray, t):
    return a.ctypes.data_as(t)


def half_to_f32(bits: int) -> float:
    return lib().orc_half_to_f32(bits)


def half_to_f32_shader(bits: int) -> float:
    return lib().orc_half_to_f32_shader(bits)


def get_scale_min_k4(j: int, scales) -> tuple[int, int]:
    s = np.ascontiguousarray(np.asarray(scales, np.uint8))
    v = lib().orc_get_scale_min_k4(j, _p(s, _u8p))
    return v & 0xFF, (v >> 8) & 0xFF


def dequant(raw: np.ndarray, type_id: int, q6k_layout: int = 0, fp16_mode: int = 0) -> np.ndarray:
    """Dequantize whole blocks of `raw` (uint8) to float32."""
    raw = np.ascontiguousarray(raw, np.uint8)
    L = lib()
    bw, bb = L.orc_block_weights(type_id), L.orc_block_bytes(type_id)
    if bw == 0 or raw.size % bb:
        raise ValueError(f"bad type {type_id} or size {raw.size}")
    nb = raw.size // bb
    out = np.empty(nb * bw, np.float32)
    if L.orc_dequant(_p(raw, _u8p), type_id, q6k_layout, nb, _p(out, _f32p), fp16_mode):
        raise ValueError("orc_dequant failed")
    return out


def dequant_q4_k_avx2(raw: np.ndarray) -> np.ndarray:
    raw = np.ascontiguousarray(raw, np.uint8)
    nb = raw.size // 144
    out = np.empty(nb * 256, np.float32)
    lib().orc_dequant_q4_k_avx2(_p(raw, _u8p), nb, _p(out, _f32p))
    return out


def matmul_f32(a: np.ndarray, b: np.ndarray, m: int, k: int, n: int) -> np.ndarray:
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    c = np.empty(m * n, np.float32)
    lib().orc_matmul_f32(_p(a, _f32p), _p(b, _f32p), _p(c, _f32p), m, k, n)
    return c.reshape(m, n)


def matmul_f64(a: np.ndarray, b: np.ndarray, m: int, k: int, n: int) -> np.ndarray:
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    c = np.empty(m * n, np.float64)
    lib().orc_matmul_f64(_p(a, _f32p), _p(b, _f32p), _p(c, _f64p), m, k, n)
    return c.reshape(m, n)


def quant_matmul(w: np.ndarray, type_id: int, x: np.ndarray, n: int, k: int,
                 q6k_layout: int = 0, threads: int = 1) -> np.ndarray:
    """y[M, N] = cpu_matmul_f32(x[M, K], transpose(dequant(W[N, K])))."""
    w = np.ascontiguousarray(w, np.uint8)
    x = np.ascontiguousarray(x, np.float32).reshape(-1, k)
    m = x.shape[0]
    y = np.empty((m, n), np.float32)
    L = lib()
    if threads == 1:
        rc = L.orc_quant_matmul(_p(w, _u8p), type_id, q6k_layout, _p(x, _f32p), _p(y, _f32p), m, n, k)
    else:
        rc = L.orc_quant_matmul_mt(_p(w, _u8p), type_id, q6k_layout, _p(x, _f32p), _p(y, _f32p), m, n, k,
                                   threads)
    if rc:
        raise ValueError(f"orc_quant_matmul failed rc={rc}")
    return y


def num_threads() -> int:
    return lib().orc_num_threads()


# ---------------------------------------------------------------- NSZ (TCA-TBE)
NSZ_FP32, NSZ_FP16, NSZ_BF16 = 0, 1, 2
NSZ_TILE = 512


def _nsz_words(w: np.ndarray, dtype: int) -> np.ndarray:
    """FP32 weights as uint32 bits, FP16 / BF16 as uint16 bits."""
    w = np.ascontiguousarray(w)
    if dtype == NSZ_FP32:
        return w.view(np.uint32) if w.dtype != np.uint32 else w
    return w.view(np.uint16) if w.dtype != np.uint16 else w


def nsz_encode_tile(w: np.ndarray, dtype: int = NSZ_FP32, reference_quirks: bool = True) -> bytes:
    b = _nsz_words(w, dtype).reshape(-1)
    assert 1 <= b.size <= NSZ_TILE
    out = np.zeros(lib().orc_nsz_max_tile_bytes(dtype), np.uint8)
    size = lib().orc_nsz_encode_tile(b.ctypes.data, b.size, dtype, int(reference_quirks), _p(out, _u8p))
    return out[:size].tobytes()


def nsz_encode(w: np.ndarray, dtype: int = NSZ_FP32, reference_quirks: bool = True) -> np.ndarray:
    """The tensor's tile stream (uint8), as the reference's encoder writes it."""
    b = _nsz_words(w, dtype).reshape(-1)
    L = lib()
    cap = max(1, -(-b.size // NSZ_TILE)) * L.orc_nsz_max_tile_bytes(dtype)
    out = np.zeros(cap, np.uint8)
    size = L.orc_nsz_encode(b.ctypes.data, b.size, dtype, int(reference_quirks), _p(out, _u8p), cap)
    if size < 0:
        raise ValueError("orc_nsz_encode failed")
    return out[:size].copy()


def nsz_offsets(data: np.ndarray, count: int, dtype: int = NSZ_FP32) -> np.ndarray:
    data = np.ascontiguousarray(data, np.uint8)
    off = np.zeros(-(-count // NSZ_TILE) + 1, np.int64)
    if lib().orc_nsz_offsets(_p(data, _u8p), data.size, count, dtype, off.ctypes.data_as(ctypes.POINTER(_i64))):
        raise ValueError("NSZ stream does not hold the given weight count")
    return off


def nsz_decode(data: np.ndarray, count: int, dtype: int = NSZ_FP32) -> np.ndarray:
    """Decoded weights: float32 for FP32, raw uint16 bits for FP16 / BF16."""
    data = np.ascontiguousarray(data, np.uint8)
    out = np.zeros(count, np.uint32 if dtype == NSZ_FP32 else np.uint16)
    if lib().orc_nsz_decode(_p(data, _u8p), data.size, count, dtype, out.ctypes.data):
        raise ValueError("orc_nsz_decode failed")
    return out.view(np.float32) if dtype == NSZ_FP32 else out


def nsz_matmul(data: np.ndarray, x: np.ndarray, n: int, k: int) -> np.ndarray:
    """y[M, N] = cpu_matmul_f32(x[M, K], transpose(decode(W[N, K]))), FP32 weights."""
    data = np.ascontiguousarray(data, np.uint8)
    x = np.ascontiguousarray(x, np.float32).reshape(-1, k)
    y = np.empty((x.shape[0], n), np.float32)
    if lib().orc_nsz_matmul(_p(data, _u8p), data.size, _p(x, _f32p), _p(y, _f32p), x.shape[0], n, k):
        raise ValueError("orc_nsz_matmul failed")
    return y
