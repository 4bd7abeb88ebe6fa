"""CPU tests of the row-sharded GEMV exchange: world size 2, gloo backend.

Each rank takes its contiguous byte range of a GGUF tensor, computes its
rows with the CPU oracle (standing in for libnsq on a GPU rank), and the
all-gather + assemble must give exactly the unsharded result.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from planejaja_b200 import quantize as Q
from planejaja_b200.formats import Q4_K, Q6_K
from planejaja_b200.sharded import ShardedGemv, assemble, shard_bounds, shard_bytes


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_shard_bounds_and_assemble():
    assert shard_bounds(16, 4, 0) == (0, 4) and shard_bounds(16, 4, 3) == (12, 16)
    with pytest.raises(ValueError):
        shard_bounds(10, 4, 0)
    g = torch.arange(2 * 3 * 4, dtype=torch.float32)  # world=2, M=3, rows=4
    y = assemble(g, 2, 3, 4)
    assert y.shape == (3, 8)
    assert y[1].tolist() == [4, 5, 6, 7, 16, 17, 18, 19]


def _worker(rank, world, port, tid, n, k, m, out_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import oracle as O
        w = Q.synthetic_weights(n, k, tid, seed=5)
        x = Q.synthetic_activations(m, k, seed=6)

        def compute(w_rank, xt, rows, kk):
            return torch.from_numpy(O.quant_matmul(w_rank.numpy(), tid, xt.numpy(), rows, kk))

        sg = ShardedGemv(torch.from_numpy(shard_bytes(w, tid, n, k, world, rank).copy()), tid, n, k, compute=compute)
        y = sg(torch.from_numpy(x)).numpy()
        if rank == 0:
            np.save(out_path, y)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("tid,m", [(Q4_K, 1), (Q6_K, 3)])
def test_sharded_gemv_gloo_world2(tmp_path, oracle, tid, m):
    n, k, world = 64, 512, 2
    out = str(tmp_path / "y.npy")
    mp.start_processes(_worker, args=(world, _free_port(), tid, n, k, m, out), nprocs=world, start_method="spawn")
    y = np.load(out)
    w = Q.synthetic_weights(n, k, tid, seed=5)
    x = Q.synthetic_activations(m, k, seed=6)
    ref = oracle.quant_matmul(w, tid, x, n, k)
    assert np.array_equal(y.view(np.uint32), ref.view(np.uint32))


# ---- fused exchange (nsq_comm_* / nsq_gemv_multi_xchg): host logic ------------

class _FakeCommLib:
    """Stands in for libnsq's exchange calls on CPU ranks: records what the
    host passes (handle bytes, connect blob) without touching a device."""

    HSIZE = 64

    def __init__(self):
        self.connected_blob = None
        self.destroyed = False

    def nsq_comm_handle_bytes(self):
        return self.HSIZE

    def nsq_comm_create(self, world, rank, nbytes, comm_ref, handle):
        import ctypes
        ctypes.memmove(handle, bytes([rank + 1]) * self.HSIZE, self.HSIZE)
        comm_ref._obj.value = 0x1000 + rank
        self.nbytes = nbytes
        return 0

    def nsq_comm_connect(self, comm, blob):
        self.connected_blob = bytes(blob.raw)
        return 0

    def nsq_comm_buffer(self, comm):
        return 0x10000

    def nsq_comm_destroy(self, comm):
        self.destroyed = True
        return 0


def _xchg_worker(rank, world, port, out_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from planejaja_b200.sharded import Exchange, OutputLayout, xchg_parts
        lay = OutputLayout()
        lay.add("gate", 1, 64)
        lay.add("up", 1, 64)
        lib = _FakeCommLib()
        ex = Exchange(lay.nbytes, lib=lib)
        parts = xchg_parts([(111, Q4_K, 64), (222, Q4_K, 64)], world, rank, lay, ["gate", "up"], 1)
        ex.close()
        np.save(out_path + f".{rank}.npy", np.array([list(lib.connected_blob), [lib.nbytes] * 64 * world,
                                                      [int(lib.destroyed)] * 64 * world], dtype=np.int64))
        with open(out_path + f".{rank}.parts", "w") as f:
            f.write(repr(parts))
    finally:
        dist.destroy_process_group()


def test_exchange_handles_and_parts_gloo_world2(tmp_path):
    """Every rank connects with all ranks' handles in rank order; each rank's
    segments cover its own rows and point at the same output offsets."""
    world = 2
    out = str(tmp_path / "x")
    mp.start_processes(_xchg_worker, args=(world, _free_port(), out), nprocs=world, start_method="spawn")
    for rank in range(world):
        blob, nbytes, destroyed = np.load(out + f".{rank}.npy")
        assert list(blob) == [1] * 64 + [2] * 64
        assert nbytes[0] == 2 * 256 and destroyed[0] == 1
        parts = eval(open(out + f".{rank}.parts").read())
        assert parts == [(111, Q4_K, 0, 32, 32 * rank, 64, 0), (222, Q4_K, 0, 32, 32 * rank, 64, 256)]


def test_output_layout():
    from planejaja_b200.sharded import OutputLayout
    lay = OutputLayout()
    assert lay.add("a", 1, 10) == 0
    assert lay.add("b", 4, 100) == 256
    assert lay.nbytes == 256 + 1792
    with pytest.raises(KeyError):
        lay.add("a", 1, 10)
