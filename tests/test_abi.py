"""CPU tests of the C ABI: libnsq.so loads, exports every symbol declared in
include/nsq.h, and rejects bad arguments on the host before any launch.
No call here reaches a kernel (there is no GPU in this environment)."""
import ctypes
import os
import re

import pytest

from planejaja_b200 import _lib
from planejaja_b200.formats import FORMATS

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    src = open(os.path.join(ROOT, "include", "nsq.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(nsq_[a-z0-9_]+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(_lib.LIB_PATH):
        from planejaja_b200.build import build
        build()
    return _lib.load()


def test_every_declared_symbol_is_exported(lib):
    syms = header_symbols()
    assert len(syms) >= 11
    for s in syms:
        assert hasattr(lib, s), s
    bound = {name for name, _, _ in _lib.SIGNATURES}
    assert set(syms) == bound


def test_version_and_strerror(lib):
    assert lib.nsq_version() == 10000
    for code in range(0, 10):
        assert lib.nsq_strerror(code)
    assert b"unknown" in lib.nsq_strerror(99)


def test_block_table_matches_formats(lib):
    for tid, f in FORMATS.items():
        assert lib.nsq_block_bytes(tid) == f.block_bytes
        assert lib.nsq_block_weights(tid) == f.block_weights
    # ids the reference maps wrongly / not at all (gguf.rs:268-304)
    assert lib.nsq_block_bytes(9) == 0 and lib.nsq_block_bytes(0) == 0
    assert lib.nsq_block_bytes(8) == 34


def test_workspace_size(lib):
    assert lib.nsq_gemv_workspace_size(1, 4096) == 128 * 80
    # 2..16 tokens with K % 256 == 0 may run on the tensor cores: fp16
    # activation tiles (16 KB per 256 of K), min-term tiles (5 KB per 256),
    # 1 KB of counters and 512 partial-sum slots of 8 KB
    tc = 1024 + 56 * 16384 + 56 * 5120 + 512 * 8192
    assert lib.nsq_gemv_workspace_size(16, 14336) == max(16 * 448 * 80, tc)
    assert lib.nsq_gemv_workspace_size(2, 4096) == 1024 + 16 * 16384 + 16 * 5120 + 512 * 8192
    assert lib.nsq_gemv_workspace_size(2, 4096 + 32) == 2 * 129 * 80
    assert lib.nsq_gemv_workspace_size(1, 33) == 0


def test_host_side_argument_errors(lib):
    al = ctypes.c_void_p(0x10000)  # never dereferenced: every call below fails validation first
    assert lib.nsq_dequant(al, 3, 0, 0, al, 32, None) == _lib.ERR_TYPE
    assert lib.nsq_dequant(al, 12, 0, 7, al, 256, None) == _lib.ERR_TYPE
    assert lib.nsq_dequant(al, 14, 5, 0, al, 256, None) == _lib.ERR_TYPE
    assert lib.nsq_dequant(None, 12, 0, 0, al, 256, None) == _lib.ERR_NULL
    assert lib.nsq_dequant(ctypes.c_void_p(0x10008), 12, 0, 0, al, 256, None) == _lib.ERR_ALIGN
    assert lib.nsq_dequant(al, 12, 0, 0, al, 100, None) == _lib.ERR_SHAPE
    assert lib.nsq_gemv(al, 12, 0, al, al, 1, 16, 300, al, 1 << 20, None) == _lib.ERR_SHAPE
    assert lib.nsq_gemv(al, 12, 0, al, al, 17, 16, 256, al, 1 << 20, None) == _lib.ERR_SHAPE
    assert lib.nsq_gemv(al, 12, 0, al, al, 0, 16, 256, al, 1 << 20, None) == _lib.ERR_SHAPE
    x4 = ctypes.c_void_p(0x10004)  # only 4-byte aligned: needs the workspace path
    assert lib.nsq_gemv(al, 12, 0, x4, al, 1, 16, 256, al, 10, None) == _lib.ERR_WORKSPACE
    assert lib.nsq_gemv(al, 12, 0, x4, al, 1, 16, 256, None, 1 << 20, None) == _lib.ERR_WORKSPACE
    assert lib.nsq_gemv(al, 12, 0, ctypes.c_void_p(0x10002), al, 1, 16, 256, al, 1 << 20, None) == _lib.ERR_ALIGN
    assert lib.nsq_gemv(al, 12, 0, None, al, 1, 16, 256, al, 1 << 20, None) == _lib.ERR_NULL
    assert lib.nsq_gemm_bf16(al, 8, 0, al, al, 128, 128, 96, None) == _lib.ERR_SHAPE
    assert lib.nsq_gemm_bf16(al, 12, 0, ctypes.c_void_p(0x10004), al, 128, 128, 256, None) == _lib.ERR_ALIGN
    segs = (_lib.Segment * 2)(_lib.Segment(0x10000, 12, 0, 16, 0x10000), _lib.Segment(0x10000, 3, 0, 16, 0x10000))
    assert lib.nsq_gemv_multi(ctypes.cast(segs, ctypes.c_void_p), 2, al, 1, 256, None, 0, None) == _lib.ERR_TYPE
    assert lib.nsq_gemv_multi(ctypes.cast(segs, ctypes.c_void_p), 5, al, 1, 256, None, 0, None) == _lib.ERR_SHAPE
    assert lib.nsq_gemv_multi(None, 1, al, 1, 256, None, 0, None) == _lib.ERR_NULL
    # the allocation-free GEMV checks its weight arguments as nsq_gemv does
    for t in (13, 14):  # Q5_K, Q6_K: the layout must be GGML or NODESTOR
        assert lib.nsq_gemv_noalloc(al, t, 5, al, al, 1, 16, 256, None) == _lib.ERR_TYPE
        assert lib.nsq_gemv(al, t, 5, al, al, 1, 16, 256, al, 1 << 20, None) == _lib.ERR_TYPE
    assert lib.nsq_gemv_noalloc(al, 3, 0, al, al, 1, 16, 256, None) == _lib.ERR_TYPE
    assert lib.nsq_gemv_noalloc(ctypes.c_void_p(0x10008), 12, 0, al, al, 1, 16, 256, None) == _lib.ERR_ALIGN
    assert lib.nsq_gemv_noalloc(al, 12, 0, al, al, 1, 16, 300, None) == _lib.ERR_SHAPE
    assert lib.nsq_gemv_noalloc(al, 12, 0, None, al, 1, 16, 256, None) == _lib.ERR_NULL
    assert lib.nsq_gemv_noalloc(al, 12, 0, al, al, 2, 16, 131072 + 256, None) == _lib.ERR_WORKSPACE
    assert lib.nsq_matmul_f32(None, al, al, 2, 2, 2, None) == _lib.ERR_NULL
    assert lib.nsq_matmul_f32(al, al, al, 0, 2, 2, None) == _lib.ERR_SHAPE


def test_exchange_argument_errors(lib):
    assert lib.nsq_comm_handle_bytes() == 64
    comm = ctypes.c_void_p()
    h = ctypes.create_string_buffer(64)
    assert lib.nsq_comm_create(0, 0, 1024, ctypes.byref(comm), h) == _lib.ERR_SHAPE
    assert lib.nsq_comm_create(9, 0, 1024, ctypes.byref(comm), h) == _lib.ERR_SHAPE
    assert lib.nsq_comm_create(2, 2, 1024, ctypes.byref(comm), h) == _lib.ERR_SHAPE
    assert lib.nsq_comm_create(2, 0, 0, ctypes.byref(comm), h) == _lib.ERR_SHAPE
    assert lib.nsq_comm_create(2, 0, 1024, None, h) == _lib.ERR_NULL
    assert lib.nsq_comm_create(2, 0, 1024, ctypes.byref(comm), None) == _lib.ERR_NULL
    assert lib.nsq_comm_connect(None, h) == _lib.ERR_NULL
    assert lib.nsq_comm_wait(None, None) == _lib.ERR_NULL
    assert lib.nsq_comm_destroy(None) == _lib.ERR_NULL
    assert not lib.nsq_comm_buffer(None)
    xs = (_lib.XSegment * 1)(_lib.XSegment(0x10000, 12, 0, 16, 0, 32, 0))
    assert lib.nsq_gemv_multi_xchg(ctypes.cast(xs, ctypes.c_void_p), 1, ctypes.c_void_p(0x10000), 1, 256, None,
                                   None, 0, None) == _lib.ERR_NULL
    assert lib.nsq_gemv_multi_xchg(None, 1, ctypes.c_void_p(0x10000), 1, 256, None, None, 0, None) == _lib.ERR_NULL


def test_engine_fails_loudly_without_gpu():
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    from planejaja_b200.engine import CudaEngine
    with pytest.raises(_lib.NsqError):
        CudaEngine(0)
