"""GPU parity at the full benchmark shapes, through size-independent checks.

The oracle cannot run full matrices in seconds, so each check compares a
seeded random sample of rows (and tokens) of a full-size result with the
oracle on exactly those rows: rows of a GGUF tensor are contiguous byte
ranges, so the oracle sees the same bytes the kernel read.

Shapes: Llama-3-8B Q4_K_M (gate/up [14336 x 4096] Q4_K, down [4096 x 14336]
Q6_K), Llama-2-7B Q4_0 (gate [11008 x 4096], down [4096 x 11008]),
Llama-2-70B FFN ([28672 x 8192], [8192 x 28672] Q4_K), and the prefill GEMM
at M = 512 / 2048.
"""
import numpy as np
import pytest
import torch

from planejaja_b200 import quantize as Q
from planejaja_b200.formats import Q4_0, Q4_K, Q6_K, fmt

pytestmark = pytest.mark.gpu

GEMV_TOL = 1e-3
GEMM_TOL = 2e-2


@pytest.fixture(scope="module")
def eng():
    from planejaja_b200.engine import CudaEngine
    e = CudaEngine(0)
    yield e
    assert e.device_status() == 0


def rel_err(y, r):
    y = np.asarray(y, np.float64).reshape(-1)
    r = np.asarray(r, np.float64).reshape(-1)
    rms = np.sqrt(np.mean(r * r))
    return float(np.max(np.abs(y - r) / np.maximum(np.abs(r), max(rms, 1e-30))))


def sample_rows(w, tid, n, k, rows):
    rb = fmt(tid).row_bytes(k)
    return np.concatenate([w[r * rb:(r + 1) * rb] for r in rows])


@pytest.mark.parametrize("name,n,k,tid,m", [
    ("l3_gate", 14336, 4096, Q4_K, 1), ("l3_down", 4096, 14336, Q6_K, 1), ("l3_gate_b16", 14336, 4096, Q4_K, 16),
    ("l2_gate_q40", 11008, 4096, Q4_0, 1), ("l2_down_q40", 4096, 11008, Q4_0, 4),
    ("l70_gate", 28672, 8192, Q4_K, 1), ("l70_down", 8192, 28672, Q4_K, 16)])
def test_gemv_full_size_sampled_rows(eng, oracle, name, n, k, tid, m):
    w = Q.synthetic_weights(n, k, tid, seed=sum(map(ord, name)))
    x = Q.synthetic_activations(m, k, seed=7)
    y = eng.gemv(eng.upload(w), tid, torch.from_numpy(x).to(eng.device), n, k).cpu().numpy()
    rows = np.sort(np.random.default_rng(1).choice(n, 48, replace=False))
    ref = oracle.quant_matmul(sample_rows(w, tid, n, k, rows), tid, x, len(rows), k, threads=8)
    assert rel_err(y[:, rows], ref) <= GEMV_TOL


def test_gemv_full_size_linearity(eng):
    """y(a*x1 + x2) = a*y(x1) + y(x2) on the full gate matrix (each side within tolerance)."""
    n, k = 14336, 4096
    wd = eng.upload(Q.synthetic_weights(n, k, Q4_K, seed=3))
    x1 = torch.randn(1, k, device=eng.device)
    x2 = torch.randn(1, k, device=eng.device)
    y1 = eng.gemv(wd, Q4_K, x1, n, k)
    y2 = eng.gemv(wd, Q4_K, x2, n, k)
    y12 = eng.gemv(wd, Q4_K, 0.5 * x1 + x2, n, k)
    assert rel_err(y12.cpu().numpy(), (0.5 * y1 + y2).cpu().numpy()) <= 3 * GEMV_TOL


@pytest.mark.parametrize("name,n,k,tid,m", [("gate_m512", 14336, 4096, Q4_K, 512),
                                            ("down_m2048", 4096, 14336, Q6_K, 2048)])
def test_gemm_full_size_sampled(eng, oracle, name, n, k, tid, m):
    w = Q.synthetic_weights(n, k, tid, seed=11)
    xb = torch.randn(m, k, device=eng.device).to(torch.bfloat16)
    y = eng.gemm_bf16(eng.upload(w), tid, xb, n, k).float().cpu().numpy()
    rng = np.random.default_rng(2)
    rows = np.sort(rng.choice(n, 32, replace=False))
    toks = np.sort(rng.choice(m, 16, replace=False))
    xs = xb.float().cpu().numpy()[toks]
    ref = oracle.quant_matmul(sample_rows(w, tid, n, k, rows), tid, xs, len(rows), k, threads=8)
    assert rel_err(y[np.ix_(toks, rows)], ref) <= GEMM_TOL


def test_dequant_full_size_bit_exact_sample(eng, oracle):
    n, k = 14336, 4096
    w = Q.synthetic_weights(n, k, Q4_K, seed=13)
    out = eng.dequant(eng.upload(w), Q4_K, n * k).cpu().numpy().reshape(n, k)
    rows = np.sort(np.random.default_rng(3).choice(n, 64, replace=False))
    ref = oracle.dequant(sample_rows(w, Q4_K, n, k, rows), Q4_K).reshape(len(rows), k)
    assert np.array_equal(out[rows].view(np.uint32), ref.view(np.uint32))
