"""Row-sharded GEMV with the all-gather fused into the kernel, on 2 GPUs.

Each rank (one process per GPU) holds a row slice of every matrix; the
exchange kernel stores its rows into both ranks' buffers over NVLink and the
flag protocol orders consecutive exchanges (the fused dp4a kernel for 1..2
tokens, the tcgen05 kernel for 6..16).  Both ranks must end with the
same full outputs, within the GEMV tolerance of the oracle on the full
matrices.  A second test lets one rank skip an exchange: the other rank's
bounded wait must give up and report NSQ_ERR_TIMEOUT (no fault, no hang).
Skipped when fewer than two GPUs are visible.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from planejaja_b200 import quantize as Q
from planejaja_b200.formats import Q4_0, Q4_K, Q6_K

pytestmark = pytest.mark.gpu

GEMV_TOL = 1e-3
WORLD = 2

# (name, n_full, K, type, M); names sharing a group id run as one launch
CASES = [
    ("gate", 1024, 4096, Q4_K, 1, "gu"), ("up", 1024, 4096, Q4_K, 1, "gu"),
    ("down", 512, 14336, Q6_K, 1, "down"),
    ("down_m2", 512, 14336, Q6_K, 2, "down_m2"),
    ("q40_m6", 512, 2048, Q4_0, 6, "q40_m6"),
    ("gate_m16", 512, 4096, Q4_K, 16, "gu_m16"), ("up_m16", 512, 4096, Q4_K, 16, "gu_m16"),
    ("down_m8", 384, 8192, Q6_K, 8, "down_m8"),
    ("q", 512, 2048, Q4_K, 1, "qkv"), ("k", 128, 2048, Q4_K, 1, "qkv"), ("v", 128, 2048, Q6_K, 1, "qkv"),
]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _weights(name, n, k, t):
    return Q.synthetic_weights(n, k, t, seed=sum(map(ord, name)))


def _acts(group, m, k):
    return Q.synthetic_activations(m, k, seed=len(group) * 7 + k % 97)


def _worker(rank, world, port, out_dir, skip_one):
    import torch.distributed as dist

    from planejaja_b200.engine import CudaEngine
    from planejaja_b200.sharded import Exchange, OutputLayout, ShardedGemvP2P, shard_bytes

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        eng = CudaEngine(rank)
        lay = OutputLayout()
        for name, n, k, t, m, g in CASES:
            lay.add(name, m, n)
        ex = Exchange(lay.nbytes)
        groups = {}
        for name, n, k, t, m, g in CASES:
            w = eng.upload(shard_bytes(_weights(name, n, k, t), t, n, k, world, rank))
            groups.setdefault(g, {"k": k, "m": m, "mats": [], "names": []})
            groups[g]["mats"].append((w, t, n))
            groups[g]["names"].append(name)
        # room for the tcgen05 tiles, so the 5..16-token cases take that kernel
        ws = eng.workspace(eng.lib.nsq_gemv_workspace_size(16, 14336))
        st = torch.cuda.current_stream().cuda_stream
        runs = []
        for g, d in groups.items():
            op = ShardedGemvP2P(ex, d["mats"], d["k"], d["m"], lay, d["names"])
            x = torch.from_numpy(_acts(g, d["m"], d["k"])).cuda()
            runs.append((op, x))
        for _ in range(2):  # twice: the second round waits on the first's flags
            for op, x in runs:
                op(x, ws, st)
        if skip_one:
            # rank 0 runs one more exchange than rank 1, then waits for it
            if rank == 0:
                op, x = runs[0]
                op(x, ws, st)
                ex.wait(st)
                torch.cuda.synchronize()
                np.save(os.path.join(out_dir, "status.npy"), np.array([eng.device_status()]))
            dist.barrier()  # rank 1 keeps its buffer mapped until rank 0 is done
        else:
            ex.wait(st)
            torch.cuda.synchronize()
            status = eng.device_status()
            for (op, x), g in zip(runs, groups):
                for name, y in zip(groups[g]["names"], op.outputs):
                    np.save(os.path.join(out_dir, f"{name}.{rank}.npy"), y.cpu().numpy())
            np.save(os.path.join(out_dir, f"status.{rank}.npy"), np.array([status]))
            dist.barrier()
        torch.cuda.synchronize()
        ex.close()
    finally:
        dist.destroy_process_group()


def _need_gpus():
    if torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs")


def test_fused_exchange_matches_oracle(tmp_path, oracle):
    _need_gpus()
    mp.start_processes(_worker, args=(WORLD, _free_port(), str(tmp_path), False), nprocs=WORLD, start_method="spawn")
    for r in range(WORLD):
        assert int(np.load(tmp_path / f"status.{r}.npy")[0]) == 0
    for name, n, k, t, m, g in CASES:
        ys = [np.load(tmp_path / f"{name}.{r}.npy") for r in range(WORLD)]
        for y in ys[1:]:
            assert np.array_equal(y.view(np.uint32), ys[0].view(np.uint32)), name
        ref = oracle.quant_matmul(_weights(name, n, k, t), t, _acts(g, m, k), n, k, threads=8)
        y = ys[0].astype(np.float64)
        rms = np.sqrt(np.mean(ref.astype(np.float64) ** 2))
        err = np.max(np.abs(y - ref) / np.maximum(np.abs(ref), max(rms, 1e-30)))
        assert err <= GEMV_TOL, (name, err)


def test_fused_exchange_wait_times_out_without_peer(tmp_path):
    _need_gpus()
    mp.start_processes(_worker, args=(WORLD, _free_port(), str(tmp_path), True), nprocs=WORLD, start_method="spawn")
    from planejaja_b200 import _lib
    assert int(np.load(tmp_path / "status.npy")[0]) == _lib.ERR_TIMEOUT


def test_exchange_rejects_input_inside_its_output():
    """One GPU, a one-rank exchange group: x inside an output range of the
    same call is refused before any launch (a peer that ran ahead would
    store this call's rows there while this rank still reads x); x in the
    other half of the buffer (the previous exchange's output) is accepted."""
    import ctypes

    from planejaja_b200 import _lib
    lib = _lib.load()
    k, n, m = 256, 256, 1
    half = m * max(n, k) * 4
    comm, h = ctypes.c_void_p(), ctypes.create_string_buffer(int(lib.nsq_comm_handle_bytes()))
    assert lib.nsq_comm_create(1, 0, 2 * half, ctypes.byref(comm), h) == 0
    try:
        assert lib.nsq_comm_connect(comm, h) == 0
        base = int(lib.nsq_comm_buffer(comm))
        w = torch.from_numpy(Q.synthetic_weights(n, k, Q4_K, seed=3)).cuda()
        st = torch.cuda.current_stream().cuda_stream
        ws = torch.empty(1 << 16, dtype=torch.uint8, device="cuda")

        def call(x_ptr, y_off):
            xs = (_lib.XSegment * 1)(_lib.XSegment(w.data_ptr(), Q4_K, 0, n, 0, n, y_off))
            return lib.nsq_gemv_multi_xchg(ctypes.cast(xs, ctypes.c_void_p), 1, ctypes.c_void_p(x_ptr), m, k, comm,
                                           ws.data_ptr(), ws.numel(), st)

        assert call(base, 0) == _lib.ERR_SHAPE              # x is the slot written
        assert call(base + 512, 0) == _lib.ERR_SHAPE        # x starts inside it
        assert call(base + half, half) == _lib.ERR_SHAPE    # same, second slot
        torch.cuda.current_stream().synchronize()
        assert call(base + half, 0) == 0                    # x in the other slot
        assert call(base, half) == 0                        # and back
        torch.cuda.synchronize()
    finally:
        assert lib.nsq_comm_destroy(comm) == 0
