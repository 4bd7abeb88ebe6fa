"""NSZ (NodeStor Zip) files: TCA-TBE lossless tensors for ZipGEMM.

Replaces the reference's NSZ format, encoder and converter
(nodestor/crates/nodestor-formats/src/nsz_format.rs, nsz_encoder.rs,
nodestor-cli/src/bin/nsz_convert.rs) on the host side of the ZipGEMM path.

File layout (nsz_format.rs:115-245, nsz_convert.rs:205-262), little-endian:
  header 28 bytes   magic "NSZ1", version u16 (1), flags u16, num_tensors u32,
                    original_total_bytes u64, compressed_total_bytes u64
  index             num_tensors entries of 128 bytes: name[64] zero padded,
                    dtype u8 (0 FP32, 1 FP16, 2 BF16), original_size u64,
                    compressed_offset u64 (absolute), compressed_size u64,
                    num_tiles u32, num_weights u64, shape u32[4] (GGUF order,
                    ne0 first), zero padding
  data              from the next multiple of 64: each tensor's tile stream

A tile stream is ceil(num_weights / 512) tiles (nsz_format.rs:13-44):
[modal u8][num_residuals u16][dtype u8][num_near u16][reserved 2] | match
bitmap | near bitmap | near deltas | residual exponents | mantissas | signs,
padded to 64 bytes.  `encode` writes exactly the reference encoder's bytes
(tests compare it with the oracle's restatement), with one deliberate change:
when a tile's modal exponent is 255 the reference encoder files exponent 0 as
"near" (nsz_encoder.rs:111, wrapping_add) and its decoder restores 254; here
that exponent is a residual, so every stream this module writes is lossless.

The device side (decode and ZipGEMM) takes a tile stream plus the offset
table that `index` builds (libnsq's nsq_nsz_index, a host function that also
validates every tile header against its bitmaps).
"""
from __future__ import annotations

import ctypes
import mmap
import struct
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

from . import _lib

MAGIC = b"NSZ1"
VERSION = 1
TILE = _lib.NSZ_TILE_WEIGHTS
ALIGN = 64
FP32, FP16, BF16 = _lib.NSZ_FP32, _lib.NSZ_FP16, _lib.NSZ_BF16
HEADER_SIZE = 28
ENTRY_SIZE = 128
_MB = {FP32: 3, FP16: 2, BF16: 1}
_ELEM = {FP32: 4, FP16: 2, BF16: 2}


class NSZError(ValueError):
    pass


def num_tiles(num_weights: int) -> int:
    return -(-num_weights // TILE) if num_weights > 0 else 0


def max_tile_bytes(dtype: int) -> int:
    raw = 8 + 3 * 64 + 512 + TILE * _MB[dtype] + 64
    return -(-raw // ALIGN) * ALIGN


# ---------------------------------------------------------------- encoder
def _words(w: np.ndarray, dtype: int) -> np.ndarray:
    w = np.ascontiguousarray(w).reshape(-1)
    if dtype == FP32:
        if w.dtype not in (np.float32, np.uint32, np.int32):
            raise NSZError(f"FP32 stream from {w.dtype}")
        return w.view(np.uint32)
    if w.dtype not in (np.float16, np.uint16, np.int16):
        raise NSZError(f"16-bit stream from {w.dtype} (pass float16 or the raw bf16 bits as uint16)")
    return w.view(np.uint16)


def _split(b: np.ndarray, dtype: int):
    b = b.astype(np.uint32)
    if dtype == FP32:
        return (b >> 23) & 0xFF, b & 0x7FFFFF, (b >> 31) & 1
    if dtype == FP16:
        return (b >> 10) & 0x1F, b & 0x3FF, (b >> 15) & 1
    return (b >> 7) & 0xFF, b & 0x7F, (b >> 15) & 1


def _encode_tiles(bits: np.ndarray, dtype: int) -> np.ndarray:
    """Tiles of bits [C, n] (n <= 512 weights each) -> their concatenated bytes."""
    C, n = bits.shape
    e, m, s = _split(bits, dtype)
    rows = np.arange(C)[:, None]
    hist = np.bincount((rows * 256 + e).ravel(), minlength=C * 256).reshape(C, 256)
    modal = hist.argmax(axis=1).astype(np.int64)  # first exponent with the highest count
    mc = modal[:, None]
    match = e == mc
    near = ~match & (((mc < 255) & (e == mc + 1)) | ((mc > 0) & (e == mc - 1)))
    res = ~(match | near)
    delta = near & (e > mc)
    nn, nr = near.sum(axis=1), res.sum(axis=1)
    B = (n + 7) // 8
    mb = _MB[dtype]
    dl = (nn + 7) // 8
    sizes = -(-(8 + 3 * B + dl + nr + n * mb) // ALIGN) * ALIGN
    offs = np.concatenate([[0], np.cumsum(sizes)])
    out = np.zeros(int(offs[-1]), np.uint8)
    o = offs[:-1, None]

    def put(col0, data):
        data = np.asarray(data, np.uint8)
        out[o + col0 + np.arange(data.shape[1])[None, :]] = data

    put(0, np.stack([modal, nr & 0xFF, nr >> 8, np.full(C, dtype), nn & 0xFF, nn >> 8,
                     np.zeros(C, np.int64), np.zeros(C, np.int64)], axis=1))
    put(8, np.packbits(match, axis=1, bitorder="little"))
    put(8 + B, np.packbits(near, axis=1, bitorder="little"))
    # compacted streams: the k-th near delta / residual exponent at rank k
    order_n = np.argsort(~near, axis=1, kind="stable")
    put(8 + 2 * B, np.packbits(np.take_along_axis(delta, order_n, 1), axis=1, bitorder="little"))
    order_r = np.argsort(~res, axis=1, kind="stable")
    rex = np.take_along_axis(e, order_r, 1)
    rex = np.where(np.arange(n)[None, :] < nr[:, None], rex, 0)
    out[o + (8 + 2 * B) + dl[:, None] + np.arange(n)[None, :]] = rex.astype(np.uint8)
    mo = (8 + 2 * B) + dl[:, None] + nr[:, None]
    if dtype == FP32:
        mant = np.stack([m & 0xFF, (m >> 8) & 0xFF, (m >> 16) & 0x7F], axis=2).reshape(C, 3 * n)
    elif dtype == FP16:
        mant = np.stack([m & 0xFF, (m >> 8) & 0x03], axis=2).reshape(C, 2 * n)
    else:
        mant = m
    out[o + mo + np.arange(n * mb)[None, :]] = mant.astype(np.uint8)
    out[o + mo + n * mb + np.arange(B)[None, :]] = np.packbits(s.astype(bool), axis=1, bitorder="little")
    # the zero padding was never written; the bytes past each section that
    # the wide writes above touched were all overwritten by a later section
    return out


def encode(w: np.ndarray, dtype: int = FP32, chunk_tiles: int = 4096) -> np.ndarray:
    """The tile stream (uint8) of tensor w: float32 for FP32, float16 for FP16,
    raw bf16 bits (uint16) for BF16."""
    b = _words(w, dtype)
    count = b.size
    full = count // TILE
    parts: List[np.ndarray] = []
    for t0 in range(0, full, chunk_tiles):
        t1 = min(full, t0 + chunk_tiles)
        parts.append(_encode_tiles(b[t0 * TILE:t1 * TILE].reshape(t1 - t0, TILE), dtype))
    if count % TILE:
        parts.append(_encode_tiles(b[full * TILE:].reshape(1, -1), dtype))
    return np.concatenate(parts) if parts else np.zeros(0, np.uint8)


# ---------------------------------------------------------------- index
def index(stream: np.ndarray, num_weights: int, dtype: int = FP32) -> np.ndarray:
    """Tile offsets (uint32, units of 64 bytes, num_tiles + 1 entries) of a
    tile stream, every tile validated (libnsq nsq_nsz_index; host only)."""
    stream = np.ascontiguousarray(stream, np.uint8).reshape(-1)
    off = np.zeros(num_tiles(num_weights) + 1, np.uint32)
    lib = _lib.load()
    rc = lib.nsq_nsz_index(stream.ctypes.data if stream.size else None, stream.size, num_weights, dtype,
                           off.ctypes.data)
    if rc == _lib.ERR_FORMAT:
        raise NSZError("malformed NSZ tile stream")
    _lib.check(rc, "nsq_nsz_index")
    return off


# ---------------------------------------------------------------- files
@dataclass(frozen=True)
class Entry:
    name: str
    dtype: int
    original_size: int
    compressed_offset: int
    compressed_size: int
    num_tiles: int
    num_weights: int
    shape: Tuple[int, int, int, int]

    def matrix(self) -> Tuple[int, int]:
        """(N rows, K weights per row): GGUF order, ne0 = K contiguous."""
        dims = [d for d in self.shape if d]
        if len(dims) == 1:
            return 1, dims[0]
        if len(dims) != 2:
            raise NSZError(f"{self.name}: {len(dims)}-D tensor is not a matrix")
        return dims[1], dims[0]

    def to_bytes(self) -> bytes:
        nb = self.name.encode("utf-8")[:64]
        b = nb + b"\0" * (64 - len(nb)) + struct.pack("<B", self.dtype)
        b += struct.pack("<QQQIQ", self.original_size, self.compressed_offset, self.compressed_size,
                         self.num_tiles, self.num_weights)
        b += struct.pack("<4I", *self.shape)
        return b + b"\0" * (ENTRY_SIZE - len(b))

    @staticmethod
    def from_bytes(b: bytes) -> "Entry":
        name = b[:64].split(b"\0")[0].decode("utf-8", "replace")
        if b[64] not in _MB:
            raise NSZError(f"{name}: dtype {b[64]}")
        osz, coff, csz, nt, nw = struct.unpack("<QQQIQ", b[65:101])
        return Entry(name, b[64], osz, coff, csz, nt, nw, struct.unpack("<4I", b[101:117]))


class NSZFile:
    """A parsed .nsz file; tile streams are views of a read-only memory map."""

    def __init__(self, path: str):
        self.path = path
        self._f = open(path, "rb")
        try:
            self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
        except ValueError as e:
            self._f.close()
            raise NSZError(f"{path}: {e}") from e
        try:
            self._parse()
        except Exception:
            self.close()
            raise

    def _parse(self) -> None:
        mm = self._mm
        if len(mm) < HEADER_SIZE or mm[:4] != MAGIC:
            raise NSZError(f"{self.path}: not an NSZ file")
        self.version, self.flags, n, self.original_total_bytes, self.compressed_total_bytes = \
            struct.unpack("<HHIQQ", mm[4:HEADER_SIZE])
        if self.version != VERSION:
            raise NSZError(f"{self.path}: NSZ version {self.version}")
        if HEADER_SIZE + n * ENTRY_SIZE > len(mm):
            raise NSZError(f"{self.path}: index runs past the end of the file")
        self.entries: Dict[str, Entry] = {}
        for i in range(n):
            e = Entry.from_bytes(mm[HEADER_SIZE + i * ENTRY_SIZE:HEADER_SIZE + (i + 1) * ENTRY_SIZE])
            if e.compressed_offset + e.compressed_size > len(mm):
                raise NSZError(f"{e.name}: tiles run past the end of the file")
            if e.num_tiles != num_tiles(e.num_weights):
                raise NSZError(f"{e.name}: {e.num_tiles} tiles for {e.num_weights} weights")
            if e.original_size != e.num_weights * _ELEM[e.dtype]:
                raise NSZError(f"{e.name}: original size {e.original_size} for {e.num_weights} weights")
            if e.name in self.entries:
                raise NSZError(f"{e.name}: appears twice")
            self.entries[e.name] = e

    def stream(self, name: str) -> np.ndarray:
        e = self.entries[name]
        return np.frombuffer(self._mm, np.uint8, count=e.compressed_size, offset=e.compressed_offset)

    def index(self, name: str) -> np.ndarray:
        e = self.entries[name]
        return index(self.stream(name), e.num_weights, e.dtype)

    def to_device(self, engine, name: str):
        e = self.entries[name]
        return engine.nsz_upload(self.stream(name), e.num_weights, e.dtype, shape=e.shape)

    def close(self) -> None:
        mm, f = getattr(self, "_mm", None), getattr(self, "_f", None)
        self._mm = None
        if mm is not None:
            try:
                mm.close()
            except BufferError:
                pass
        if f is not None:
            f.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def open_nsz(path: str) -> NSZFile:
    return NSZFile(path)


def write(path: str, tensors: Sequence[Tuple[str, np.ndarray, Optional[Sequence[int]]]], dtype: int = FP32,
          flags: int = 0) -> None:
    """Writes an .nsz file the way nsz_convert.rs:205-262 lays it out, from
    (name, weights, GGUF shape or None) records."""
    entries, blobs = [], []
    data_start = -(-(HEADER_SIZE + ENTRY_SIZE * len(tensors)) // ALIGN) * ALIGN
    pos = data_start
    for name, w, shape in tensors:
        w = np.asarray(w)
        blob = encode(w, dtype)
        count = w.size
        shp = tuple(shape) if shape is not None else tuple(reversed(w.shape))
        shp = (tuple(int(d) for d in shp) + (0, 0, 0, 0))[:4]
        entries.append(Entry(name, dtype, count * _ELEM[dtype], pos, blob.size, num_tiles(count), count, shp))
        blobs.append(blob)
        pos += blob.size
    head = MAGIC + struct.pack("<HHIQQ", VERSION, flags, len(entries), sum(e.original_size for e in entries),
                               sum(b.size for b in blobs))
    with open(path, "wb") as f:
        f.write(head)
        for e in entries:
            f.write(e.to_bytes())
        f.write(b"\0" * (data_start - HEADER_SIZE - ENTRY_SIZE * len(entries)))
        for b in blobs:
            f.write(b.tobytes())


@dataclass
class NszTensor:
    """An NSZ tensor resident on the device: its tile stream, the offset
    table, the weight count and the original dtype."""
    tiles: "object"    # torch uint8
    offsets: "object"  # torch int32 (uint32 values)
    count: int
    dtype: int
    shape: Tuple[int, ...] = ()

    @property
    def nbytes(self) -> int:
        return int(self.tiles.numel())
