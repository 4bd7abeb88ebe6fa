"""nsq_gemv_noalloc: the decode GEMV for callers that cannot allocate device memory.

Some callers cannot call cudaMalloc: an engine whose device memory is all
owned by its own arena allocator, or code that must not synchronise the
device.  nsq_gemv_noalloc keeps the prepared activations in a fixed scratch
array inside libnsq instead of a caller workspace.  This file checks it,
through the C ABI, against nsq_gemv on two calls in a row (the array keeps
the previous call's contents, so the second call must not depend on them),
and checks that sizes beyond the array are rejected.  It is named so that
pytest collects it last.
"""
import ctypes

import numpy as np
import pytest
import torch

from planejaja_b200 import _lib
from planejaja_b200 import quantize as Q
from planejaja_b200.formats import Q4_K, Q5_K, Q6_K, Q8_0, Q6K_GGML, Q6K_NODESTOR

pytestmark = pytest.mark.gpu

GEMV_TOL = 1e-3


def rel_err(y, r):
    y = np.asarray(y, np.float64).reshape(-1)
    r = np.asarray(r, np.float64).reshape(-1)
    rms = np.sqrt(np.mean(r * r))
    return float(np.max(np.abs(y - r) / np.maximum(np.abs(r), max(rms, 1e-30))))


def _gemv_reference(lib, w, t, lay, x, n, k):
    """Output of the existing entry point nsq_gemv (caller workspace)."""
    m = x.shape[0]
    y = torch.empty((m, n), dtype=torch.float32, device="cuda")
    ws = torch.empty(lib.nsq_gemv_workspace_size(m, k), dtype=torch.uint8, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    assert lib.nsq_gemv(w.data_ptr(), t, lay, x.data_ptr(), y.data_ptr(), m, n, k, ws.data_ptr(), ws.numel(),
                        st) == 0
    return y


def test_noalloc_matches_gemv_two_calls_in_a_row():
    lib = _lib.load()
    st = torch.cuda.current_stream().cuda_stream
    cases = [(Q4_K, 0, 1, 512, 4096, 11), (Q6_K, 0, 4, 300, 14336, 12), (Q8_0, 0, 16, 200, 1024, 13),
             (Q5_K, Q6K_NODESTOR, 3, 256, 8192, 14), (Q5_K, Q6K_GGML, 2, 96, 2048, 15)]
    for t, lay, m, n, k, seed in cases:
        w = torch.from_numpy(Q.synthetic_weights(n, k, t, seed=seed, q6k_layout=lay)).cuda()
        outs = []
        for call in range(2):  # two calls in a row, different activations
            x = torch.from_numpy(Q.synthetic_activations(m, k, seed=100 * seed + call)).cuda()
            y = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
            rc = lib.nsq_gemv_noalloc(w.data_ptr(), t, lay, x.data_ptr(), y.data_ptr(), m, n, k, st)
            assert rc == 0, _lib.strerror(rc)
            ref = _gemv_reference(lib, w, t, lay, x, n, k)
            torch.cuda.synchronize()
            assert torch.isfinite(y).all()
            assert rel_err(y.cpu().numpy(), ref.cpu().numpy()) <= GEMV_TOL
            outs.append(y.cpu().numpy())
        assert not np.array_equal(outs[0], outs[1])
    assert lib.nsq_device_status(1) == 0


def test_noalloc_rejects_sizes_beyond_its_scratch():
    lib = _lib.load()
    st = torch.cuda.current_stream().cuda_stream
    k = 32768
    m = _lib.NOALLOC_MAX_ELEMS // k + 1  # M * K just over the limit
    w = torch.zeros(144 * (k // 256) * 2, dtype=torch.uint8, device="cuda")
    x = torch.zeros(m, k, device="cuda")
    y = torch.zeros(m, 2, device="cuda")
    rc = lib.nsq_gemv_noalloc(w.data_ptr(), Q4_K, 0, x.data_ptr(), y.data_ptr(), m, 2, k, st)
    assert rc == _lib.ERR_WORKSPACE
    assert "workspace" in _lib.strerror(rc)
