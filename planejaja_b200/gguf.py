"""GGUF reader for the dequant + matmul path: tensors as GGUF-native bytes.

Replaces the reference loader's tensor sizing and type mapping
(nodestor/crates/nodestor-formats/src/gguf.rs).  What it keeps: the layout
of the file (magic "GGUF", versions 2 and 3, little-endian counts, the
13 metadata value types, tensor-info records of name / dims / ggml type /
offset; gguf.rs:58-160, 184-266).  What it fixes:

* ggml type ids 12 (Q4_K), 13 (Q5_K) and 14 (Q6_K) are mapped and sized
  (144 / 176 / 210 bytes per 256 weights); the reference has no entry for
  them and sizes any unknown id as F32 (gguf.rs:268-304);
* Q8_0 is 34 bytes per 32 weights, not 36 (gguf.rs:297);
* id 9 is Q8_1 (36 bytes per 32), not Q8_0 (gguf.rs:277);
* an unknown type id is an error, not a silent F32;
* the data section starts at the file's `general.alignment` (default 32),
  not always at 32 (gguf.rs:127-130), and every tensor offset is checked
  against it and against the file size;
* metadata arrays are read whole (the reference keeps the first 1000
  elements, gguf.rs:208-217).

Tensors come back as read-only numpy views of a memory map: a GGUF matrix
is ne[1] rows of ne[0] weights (`shape` is in ggml order, ne[0] first), and
its bytes are exactly what the libnsq kernels consume.  `to_device` uploads
one tensor's bytes (16-byte aligned) for `CudaEngine`.
"""
from __future__ import annotations

import mmap
import struct
from dataclasses import dataclass
from typing import Any, Dict, List, Optional, Tuple

import numpy as np

from .formats import FORMATS

GGUF_MAGIC = b"GGUF"
DEFAULT_ALIGNMENT = 32

# ggml type id -> (name, weights per block, bytes per block).  The block
# formats of the matmul path come from formats.FORMATS; the rest are
# sized so that files holding them parse correctly, and marked unsupported
# for compute.
_EXTRA_TYPES = {
    0: ("F32", 1, 4), 1: ("F16", 1, 2), 30: ("BF16", 1, 2),
    3: ("Q4_1", 32, 20), 6: ("Q5_0", 32, 22), 7: ("Q5_1", 32, 24), 9: ("Q8_1", 32, 36),
    10: ("Q2_K", 256, 84), 11: ("Q3_K", 256, 110), 15: ("Q8_K", 256, 292),
    24: ("I8", 1, 1), 25: ("I16", 1, 2), 26: ("I32", 1, 4), 27: ("I64", 1, 8), 28: ("F64", 1, 8),
}
TYPES: Dict[int, Tuple[str, int, int]] = dict(_EXTRA_TYPES)
for _tid, _f in FORMATS.items():
    TYPES[_tid] = (_f.name, _f.block_weights, _f.block_bytes)

# metadata value types (GGUF spec; gguf.rs:185-187)
_SCALARS = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q", 12: "<d"}
_STRING, _ARRAY = 8, 9


class GGUFError(ValueError):
    pass


@dataclass(frozen=True)
class Tensor:
    name: str
    shape: Tuple[int, ...]  # ggml order: ne[0] (contiguous) first
    type_id: int
    offset: int             # absolute byte offset in the file
    nbytes: int

    @property
    def type_name(self) -> str:
        return TYPES[self.type_id][0]

    @property
    def n_elements(self) -> int:
        n = 1
        for d in self.shape:
            n *= d
        return n

    @property
    def matmul_supported(self) -> bool:
        """True if libnsq's dequant / GEMV / GEMM take this tensor's bytes."""
        return self.type_id in FORMATS

    def matrix(self) -> Tuple[int, int]:
        """(N rows, K weights per row) of a 1-D or 2-D tensor."""
        if len(self.shape) == 1:
            return 1, self.shape[0]
        if len(self.shape) != 2:
            raise GGUFError(f"{self.name}: {len(self.shape)}-D tensor is not a matrix")
        return self.shape[1], self.shape[0]


def tensor_nbytes(shape, type_id: int) -> int:
    if type_id not in TYPES:
        raise GGUFError(f"unknown ggml type id {type_id}")
    name, bw, bb = TYPES[type_id]
    if not shape:
        raise GGUFError("tensor without dimensions")
    if shape[0] % bw:
        raise GGUFError(f"{name}: ne[0]={shape[0]} is not a multiple of the block size {bw}")
    n = 1
    for d in shape:
        n *= d
    return n // bw * bb


class _Cursor:
    def __init__(self, buf, pos: int = 0):
        self.buf, self.pos = buf, pos

    def take(self, n: int) -> bytes:
        if self.pos + n > len(self.buf):
            raise GGUFError("file ends inside the header")
        b = self.buf[self.pos:self.pos + n]
        self.pos += n
        return bytes(b)

    def unpack(self, fmt: str):
        return struct.unpack(fmt, self.take(struct.calcsize(fmt)))[0]

    def string(self) -> str:
        n = self.unpack("<Q")
        if n > (1 << 30):
            raise GGUFError(f"string of {n} bytes")
        return self.take(n).decode("utf-8")

    def value(self, vtype: int) -> Any:
        if vtype in _SCALARS:
            return self.unpack(_SCALARS[vtype])
        if vtype == _STRING:
            return self.string()
        if vtype == _ARRAY:
            etype = self.unpack("<I")
            count = self.unpack("<Q")
            if etype in _SCALARS and etype != 7:
                fmt = _SCALARS[etype]
                size = struct.calcsize(fmt)
                raw = self.take(size * count)
                return np.frombuffer(raw, dtype=np.dtype(fmt)).tolist()
            return [self.value(etype) for _ in range(count)]
        raise GGUFError(f"unknown metadata value type {vtype}")


class GGUFFile:
    """A parsed GGUF file; tensors are views of a read-only memory map."""

    def __init__(self, path: str):
        self.path = path
        self._f = open(path, "rb")
        try:
            self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
        except ValueError as e:  # empty file
            self._f.close()
            raise GGUFError(f"{path}: {e}") from e
        try:
            self._parse()
        except Exception:
            self.close()
            raise

    def _parse(self) -> None:
        c = _Cursor(self._mm)
        if c.take(4) != GGUF_MAGIC:
            raise GGUFError(f"{self.path}: bad magic (not a GGUF file)")
        self.version = c.unpack("<I")
        if self.version not in (2, 3):
            raise GGUFError(f"{self.path}: GGUF version {self.version} not supported (2 or 3)")
        n_tensors = c.unpack("<Q")
        n_kv = c.unpack("<Q")
        self.metadata: Dict[str, Any] = {}
        for _ in range(n_kv):
            key = c.string()
            self.metadata[key] = c.value(c.unpack("<I"))
        self.alignment = int(self.metadata.get("general.alignment", DEFAULT_ALIGNMENT))
        if self.alignment <= 0 or self.alignment & (self.alignment - 1):
            raise GGUFError(f"{self.path}: general.alignment {self.alignment} is not a power of two")
        infos: List[Tuple[str, Tuple[int, ...], int, int]] = []
        for i in range(n_tensors):
            name = c.string()
            n_dims = c.unpack("<I")
            if n_dims < 1 or n_dims > 8:
                raise GGUFError(f"tensor {i} ({name}): {n_dims} dimensions")
            shape = tuple(c.unpack("<Q") for _ in range(n_dims))
            type_id = c.unpack("<I")
            off = c.unpack("<Q")
            infos.append((name, shape, type_id, off))
        self.data_offset = (c.pos + self.alignment - 1) // self.alignment * self.alignment
        size = len(self._mm)
        self.tensors: Dict[str, Tensor] = {}
        for name, shape, type_id, off in infos:
            if name in self.tensors:
                raise GGUFError(f"tensor {name!r} appears twice")
            if off % self.alignment:
                raise GGUFError(f"{name}: offset {off} is not aligned to {self.alignment}")
            nb = tensor_nbytes(shape, type_id)
            start = self.data_offset + off
            if start + nb > size:
                raise GGUFError(f"{name}: bytes [{start}, {start + nb}) run past the end of the file ({size})")
            self.tensors[name] = Tensor(name, shape, type_id, start, nb)

    # ---- access
    def data(self, name: str) -> np.ndarray:
        """The tensor's bytes (read-only uint8 view of the memory map)."""
        t = self.tensors[name]
        return np.frombuffer(self._mm, dtype=np.uint8, count=t.nbytes, offset=t.offset)

    def to_device(self, engine, name: str):
        """Upload one tensor's GGUF bytes for the libnsq kernels."""
        t = self.tensors[name]
        if not t.matmul_supported:
            raise GGUFError(f"{name}: {t.type_name} is not a libnsq matmul format")
        return engine.upload(self.data(name))

    def close(self) -> None:
        mm, f = getattr(self, "_mm", None), getattr(self, "_f", None)
        self._mm = None
        if mm is not None:
            try:
                mm.close()
            except BufferError:  # views still alive; the map closes with them
                pass
        if f is not None:
            f.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __repr__(self) -> str:
        return f"GGUFFile({self.path!r}, v{self.version}, {len(self.tensors)} tensors, alignment {self.alignment})"


def open_gguf(path: str) -> GGUFFile:
    return GGUFFile(path)


def write_minimal(path: str, tensors, metadata: Optional[Dict[str, Any]] = None, alignment: int = DEFAULT_ALIGNMENT,
                  version: int = 3) -> None:
    """Writes a GGUF file from (name, shape in ggml order, type_id, bytes)
    records and string / int / float metadata.  For tests and fixtures of the
    reader; it is not on the compute path."""
    def s(x: str) -> bytes:
        b = x.encode("utf-8")
        return struct.pack("<Q", len(b)) + b

    meta = dict(metadata or {})
    if alignment != DEFAULT_ALIGNMENT:
        meta["general.alignment"] = alignment
    kv = b""
    for k, v in meta.items():
        kv += s(k)
        if isinstance(v, bool):
            kv += struct.pack("<I", 7) + struct.pack("<?", v)
        elif isinstance(v, int):
            kv += struct.pack("<I", 4 if 0 <= v < (1 << 32) else 11) + struct.pack("<I" if 0 <= v < (1 << 32) else "<q", v)
        elif isinstance(v, float):
            kv += struct.pack("<I", 6) + struct.pack("<f", v)
        else:
            kv += struct.pack("<I", 8) + s(str(v))
    info, blobs, off = b"", [], 0
    for name, shape, type_id, data in tensors:
        data = bytes(data)
        if len(data) != tensor_nbytes(shape, type_id):
            raise GGUFError(f"{name}: {len(data)} bytes for shape {shape} of type {type_id}")
        off = (off + alignment - 1) // alignment * alignment
        info += s(name) + struct.pack("<I", len(shape)) + b"".join(struct.pack("<Q", d) for d in shape)
        info += struct.pack("<I", type_id) + struct.pack("<Q", off)
        blobs.append((off, data))
        off += len(data)
    head = GGUF_MAGIC + struct.pack("<I", version) + struct.pack("<Q", len(tensors)) + struct.pack("<Q", len(meta))
    head += kv + info
    start = (len(head) + alignment - 1) // alignment * alignment
    out = bytearray(head + b"\0" * (start - len(head)))
    for o, data in blobs:
        out += b"\0" * (start + o - len(out))
        out += data
    with open(path, "wb") as f:
        f.write(out)
