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
"""
from __future__ import annotations

from typing import Callable, Optional

import numpy as np
import torch
import torch.distributed as dist

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
