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
