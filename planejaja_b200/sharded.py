"""Row-sharded decode GEMV across GPUs (one process per GPU, NCCL).

A weight matrix W [N x K] in GGUF blocks is split by rows into `world`
contiguous slices; a row slice of a GGUF tensor is a contiguous byte range,
so each rank uploads only its bytes.  Every rank holds the whole activation
x [M x K] (in a transformer it arrives replicated from the previous
all-gather), computes y_p = x . W_p^T for its rows with libnsq, and an
all-gather over NVLink assembles y [M x N].  This is the tensor-parallel
decode the reference does not have (it has no collectives at all; its
"fabric" crate simulates RDMA in-process, nodestor/crates/nodestor-fabric/
src/rdma_sim.rs:6-17).

`shard_bounds` / `shard_bytes` / `assemble` are pure host logic; the compute
callable is injectable so the exchange can be tested on CPU ranks (gloo).

Two exchanges:
  * `ShardedGemv`: libnsq GEMV then torch.distributed all_gather (NCCL).
  * `Exchange` + `ShardedGemvP2P`: the all-gather fused into the GEMV
    kernel.  Every rank maps every other rank's exchange buffer (CUDA IPC);
    the kernel's epilogue stores its rows into all of them over NVLink and
    publishes a sequence number; the next exchange waits (bounded) for all
    ranks before reading its activations (nsq_gemv_multi_xchg, nsq.h).
"""
from __future__ import annotations

import ctypes
from typing import Callable, Optional

import numpy as np
import torch
import torch.distributed as dist

from . import _lib
from .formats import fmt


def shard_bounds(n: int, world: int, rank: int) -> tuple[int, int]:
    """Rows [r0, r1) of rank `rank`; equal slices (n must divide by world)."""
    if n % world:
        raise ValueError(f"N={n} does not split evenly over {world} ranks")
    rows = n // world
    return rank * rows, (rank + 1) * rows


def shard_bytes(w: np.ndarray, type_id: int, n: int, k: int, world: int, rank: int) -> np.ndarray:
    """The GGUF bytes of this rank's rows (a contiguous sub-range of `w`)."""
    rb = fmt(type_id).row_bytes(k)
    r0, r1 = shard_bounds(n, world, rank)
    return w[r0 * rb:r1 * rb]


def assemble(gathered: torch.Tensor, world: int, m: int, rows: int) -> torch.Tensor:
    """[world * M * rows] (all-gather of per-rank [M x rows]) -> [M x world*rows]."""
    return gathered.view(world, m, rows).permute(1, 0, 2).reshape(m, world * rows)


class ShardedGemv:
    """One rank's part of a row-sharded GEMV followed by an all-gather."""

    def __init__(self, w_rank: torch.Tensor, type_id: int, n: int, k: int,
                 group: Optional[dist.ProcessGroup] = None,
                 compute: Optional[Callable[[torch.Tensor, torch.Tensor, int, int], torch.Tensor]] = None,
                 engine=None):
        self.world = dist.get_world_size(group)
        self.group = group
        self.n, self.k, self.type_id = n, k, type_id
        self.rows = n // self.world
        self.w = w_rank
        if compute is None:
            if engine is None:
                from .engine import CudaEngine
                engine = CudaEngine(w_rank.device)
            compute = lambda w, x, rows, k: engine.gemv(w, type_id, x, rows, k, sync=False)  # noqa: E731
        self.compute = compute

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        m = x.numel() // self.k
        y_local = self.compute(self.w, x, self.rows, self.k).reshape(m, self.rows).contiguous()
        out = torch.empty(self.world * m * self.rows, dtype=y_local.dtype, device=y_local.device)
        dist.all_gather_into_tensor(out, y_local.reshape(-1), group=self.group)
        return assemble(out, self.world, m, self.rows)


class _DeviceArray:
    """A raw device pointer seen by torch through __cuda_array_interface__."""

    def __init__(self, ptr: int, shape, typestr: str = "<f4"):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


class Exchange:
    """One exchange group: this rank's buffer, mapped by every other rank.

    `nbytes` of outputs; callers lay out their full outputs [M x n_full] f32
    at byte offsets of their choosing (`view`).  The IPC handles travel over
    the process group (all_gather_object).  `lib` may be replaced by a fake
    with the same functions for host-only tests.
    """

    def __init__(self, nbytes: int, group: Optional[dist.ProcessGroup] = None, lib=None):
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.nbytes = int(nbytes)
        self.lib = lib if lib is not None else _lib.load()
        hsize = int(self.lib.nsq_comm_handle_bytes())
        handle = ctypes.create_string_buffer(hsize)
        comm = ctypes.c_void_p()
        _lib.check(self.lib.nsq_comm_create(self.world, self.rank, self.nbytes, ctypes.byref(comm), handle),
                   "nsq_comm_create")
        self.comm = comm
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle.raw), group=group)
        if any(h is None or len(h) != hsize for h in handles):
            raise ValueError("exchange handles missing or of the wrong size")
        self._blob = ctypes.create_string_buffer(b"".join(handles), hsize * self.world)
        _lib.check(self.lib.nsq_comm_connect(self.comm, self._blob), "nsq_comm_connect")
        self.base = int(self.lib.nsq_comm_buffer(self.comm) or 0)

    def view(self, offset: int, shape) -> torch.Tensor:
        """f32 tensor over this rank's buffer at byte `offset` (no copy)."""
        n = int(np.prod(shape)) * 4
        if offset < 0 or offset % 4 or offset + n > self.nbytes:
            raise ValueError(f"view [{offset}, {offset + n}) outside the {self.nbytes}-byte exchange buffer")
        return torch.as_tensor(_DeviceArray(self.base + offset, shape), device="cuda")

    def wait(self, stream: int) -> None:
        """Enqueue a wait until every rank's latest exchange has landed here."""
        _lib.check(self.lib.nsq_comm_wait(self.comm, stream), "nsq_comm_wait")

    def close(self) -> None:
        if self.comm is not None and self.comm.value:
            _lib.check(self.lib.nsq_comm_destroy(self.comm), "nsq_comm_destroy")
        self.comm = None


class OutputLayout:
    """Byte offsets of full outputs [M x n_full] f32 in an exchange buffer."""

    def __init__(self):
        self.offsets: dict = {}
        self.nbytes = 0

    def add(self, name, m: int, n_full: int) -> int:
        if name in self.offsets:
            raise KeyError(f"output {name!r} laid out twice")
        off = self.nbytes
        self.offsets[name] = (off, m, n_full)
        self.nbytes += (m * n_full * 4 + 255) // 256 * 256
        return off


def xchg_parts(metas, world: int, rank: int, layout: OutputLayout, names, m: int, q6k_layout: int = 0):
    """nsq_xsegment fields for this rank: metas are (w_ptr, ggml_type, n_full)."""
    parts = []
    for (w, t, n_full), name in zip(metas, names):
        r0, r1 = shard_bounds(n_full, world, rank)
        off, mm, nf = layout.offsets[name]
        if mm != m or nf != n_full:
            raise ValueError(f"layout of {name!r} is [{mm} x {nf}], not [{m} x {n_full}]")
        parts.append((w, t, q6k_layout, r1 - r0, r0, n_full, off))
    return parts


def xsegments(parts) -> "ctypes.Array":
    """ctypes nsq_xsegment array from (w_ptr, ggml_type, q6k_layout, N, row0, n_full, y_off) tuples."""
    arr = (_lib.XSegment * len(parts))()
    for i, (w, t, lay, n, row0, n_full, off) in enumerate(parts):
        arr[i] = _lib.XSegment(w, t, lay, n, row0, n_full, off)
    return arr


class ShardedGemvP2P:
    """Row-sharded GEMV of one or more matrices sharing x, all-gather fused.

    `mats`: list of (w_rank uint8 device tensor, ggml_type, n_full) for this
    rank; each matrix's rows split evenly over the ranks.  Outputs land in
    `exchange` at the offsets of `layout` under `names`.
    """

    def __init__(self, exchange: Exchange, mats, k: int, m: int, layout: OutputLayout, names,
                 q6k_layout: int = 0):
        self.ex, self.k, self.m = exchange, k, m
        parts = xchg_parts([(w.data_ptr(), t, n_full) for w, t, n_full in mats], exchange.world, exchange.rank,
                           layout, names, m, q6k_layout)
        self.keep = [w for w, _, _ in mats]
        self.segs = xsegments(parts)
        self.nseg = len(parts)
        self.outputs = [exchange.view(layout.offsets[nm][0], (m, n_full)) for (_, _, n_full), nm in zip(mats, names)]

    def __call__(self, x: torch.Tensor, ws: Optional[torch.Tensor] = None, stream: Optional[int] = None):
        lib = self.ex.lib
        st = torch.cuda.current_stream().cuda_stream if stream is None else stream
        ws_ptr, ws_n = (ws.data_ptr(), ws.numel()) if ws is not None else (None, 0)
        _lib.check(lib.nsq_gemv_multi_xchg(ctypes.cast(self.segs, ctypes.c_void_p), self.nseg, x.data_ptr(),
                                           self.m, self.k, self.ex.comm, ws_ptr, ws_n, st),
                   "nsq_gemv_multi_xchg")
        return self.outputs
