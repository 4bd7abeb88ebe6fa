"""ctypes binding of libnsq.so (the C ABI in include/nsq.h).

The library is built in-tree (planejaja_b200/libnsq.so) by
`python -m planejaja_b200.build` or `make -C planejaja_b200/csrc`.  There is
no fallback: if the shared library is missing or fails to load, every
compute call raises NsqError.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libnsq.so")

OK = 0
ERR_TYPE = 1
ERR_SHAPE = 2
ERR_ALIGN = 3
ERR_NULL = 4
ERR_CUDA = 5
ERR_NCCL = 6
ERR_TIMEOUT = 7
ERR_WORKSPACE = 8
ERR_DEVICE = 9
ERR_FORMAT = 10

NSZ_FP32, NSZ_FP16, NSZ_BF16 = 0, 1, 2
NSZ_TILE_WEIGHTS = 512

OUT_F32 = 0
OUT_BF16 = 1
GEMV_MAX_M = 16

# (name, restype, argtypes) for every symbol declared in include/nsq.h
_vp, _i64, _int, _sz = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_size_t
SIGNATURES = [
    ("nsq_version", _int, []),
    ("nsq_reload_tuning", None, []),
    ("nsq_kernel_launches", ctypes.c_uint64, []),
    ("nsq_strerror", ctypes.c_char_p, [_int]),
    ("nsq_block_bytes", _i64, [_int]),
    ("nsq_block_weights", _i64, [_int]),
    ("nsq_device_status", _int, [_int]),
    ("nsq_dequant", _int, [_vp, _int, _int, _int, _vp, _i64, _vp]),
    ("nsq_gemv_workspace_size", _sz, [_i64, _i64]),
    ("nsq_gemv", _int, [_vp, _int, _int, _vp, _vp, _i64, _i64, _i64, _vp, _sz, _vp]),
    ("nsq_prepare_activations", _int, [_vp, _i64, _i64, _vp, _sz, _vp]),
    ("nsq_gemv_prepared", _int, [_vp, _int, _int, _vp, _vp, _i64, _i64, _i64, _vp]),
    ("nsq_gemv_multi", _int, [ctypes.c_void_p, _int, _vp, _i64, _i64, _vp, _sz, _vp]),
    ("nsq_gemv_noalloc", _int, [_vp, _int, _int, _vp, _vp, _i64, _i64, _i64, _vp]),
    ("nsq_gemm_bf16", _int, [_vp, _int, _int, _vp, _vp, _i64, _i64, _i64, _vp]),
    ("nsq_matmul_f32", _int, [_vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    ("nsq_gemv_swiglu", _int, [_vp, _vp, _int, _int, _vp, _vp, _i64, _i64, _i64, _vp, _sz, _vp]),
    ("nsq_gemv_residual", _int, [_vp, _int, _int, _vp, _vp, _vp, _i64, _i64, _i64, _vp, _sz, _vp]),
    ("nsq_comm_handle_bytes", _sz, []),
    ("nsq_comm_create", _int, [_int, _int, _sz, ctypes.POINTER(ctypes.c_void_p), _vp]),
    ("nsq_comm_connect", _int, [_vp, _vp]),
    ("nsq_comm_buffer", _vp, [_vp]),
    ("nsq_comm_wait", _int, [_vp, _vp]),
    ("nsq_comm_destroy", _int, [_vp]),
    ("nsq_gemv_multi_xchg", _int, [ctypes.c_void_p, _int, _vp, _i64, _i64, _vp, _vp, _sz, _vp]),
    ("nsq_nsz_num_tiles", _i64, [_i64]),
    ("nsq_nsz_index", _int, [_vp, _i64, _i64, _int, _vp]),
    ("nsq_nsz_decode", _int, [_vp, _vp, _i64, _int, _vp, _vp]),
    ("nsq_zipgemm", _int, [_vp, _vp, _int, _vp, _vp, _i64, _i64, _i64, _vp]),
]


class Segment(ctypes.Structure):
    """struct nsq_segment (include/nsq.h)."""
    _fields_ = [("w", ctypes.c_void_p), ("ggml_type", ctypes.c_int), ("q6k_layout", ctypes.c_int),
                ("N", ctypes.c_int64), ("y", ctypes.c_void_p)]


class XSegment(ctypes.Structure):
    """struct nsq_xsegment (include/nsq.h): one rank's rows of a row-sharded matrix."""
    _fields_ = [("w", ctypes.c_void_p), ("ggml_type", ctypes.c_int), ("q6k_layout", ctypes.c_int),
                ("N", ctypes.c_int64), ("row0", ctypes.c_int64), ("n_full", ctypes.c_int64),
                ("y_off", ctypes.c_int64)]


MAX_SEGMENTS = 4
MAX_RANKS = 8
NOALLOC_MAX_ELEMS = 262144  # NSQ_NOALLOC_MAX_ELEMS: largest M * K of nsq_gemv_noalloc


class NsqError(RuntimeError):
    def __init__(self, status: int, what: str = ""):
        self.status = status
        msg = strerror(status) if _lib_or_none() is not None else f"status {status}"
        super().__init__(f"{what}: {msg} (status {status})" if what else f"{msg} (status {status})")


_lib = None
_load_error = None


def _lib_or_none():
    return _lib


def load():
    """Load libnsq.so once; raises NsqError-like RuntimeError if absent."""
    global _lib, _load_error
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"libnsq.so not built (expected at {LIB_PATH}); run `python -m planejaja_b200.build`")
    L = ctypes.CDLL(LIB_PATH)
    for name, res, args in SIGNATURES:
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def strerror(status: int) -> str:
    return load().nsq_strerror(status).decode()


def check(status: int, what: str = "") -> None:
    if status != OK:
        raise NsqError(status, what)
