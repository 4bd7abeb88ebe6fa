"""The tcgen05 batched decode GEMV (2..16 tokens, every format and layout).

Covered beside the parity suites (which run it as their "tc" kernel):
  * stream-K: shapes whose 128-row tiles are split over many CTAs, so most
    outputs are sums of partials from several CTAs, against the oracle;
  * determinism: the partials are summed in CTA order, so repeated calls give
    the same bits;
  * Q6_K scales whose products sc * (q - 32) exceed 2048 (fp16 then rounds
    them to even integers): still within the GEMV tolerance of the oracle;
  * mixed q|k|v segments (Q4_K, Q4_K, Q6_K) in one launch;
  * every format and layout with the fp16 weight operand in tensor memory (the
    default) and in shared memory (NSQ_TC_A=0).
"""
import numpy as np
import pytest
import torch

from planejaja_b200 import quantize as Q
from planejaja_b200.formats import Q4_K, Q6_K

pytestmark = pytest.mark.gpu

GEMV_TOL = 1e-3


@pytest.fixture(scope="module")
def eng():
    from planejaja_b200.engine import CudaEngine
    e = CudaEngine(0)
    yield e
    assert e.device_status() == 0


@pytest.fixture(autouse=True)
def tc_on(tuning):
    tuning.set("NSQ_TC_MIN_M", "2")


def rel_err(y, r):
    y = np.asarray(y, np.float64).reshape(-1)
    r = np.asarray(r, np.float64).reshape(-1)
    rms = np.sqrt(np.mean(r * r))
    return float(np.max(np.abs(y - r) / np.maximum(np.abs(r), max(rms, 1e-30))))


@pytest.mark.parametrize("tid", [Q4_K, Q6_K])
@pytest.mark.parametrize("n,k,m", [(128, 256, 2), (129, 512, 16), (300, 2048, 5), (1000, 4096, 16),
                                   (64, 14336, 3), (40, 28672, 16), (4096, 256, 8)])
def test_tc_stream_k_shapes(eng, oracle, tid, n, k, m):
    w = Q.synthetic_weights(n, k, tid, seed=n + k)
    x = Q.synthetic_activations(m, k, seed=m)
    y = eng.gemv(eng.upload(w), tid, torch.from_numpy(x).to(eng.device), n, k).cpu().numpy()
    assert rel_err(y, oracle.quant_matmul(w, tid, x, n, k, threads=8)) <= GEMV_TOL


@pytest.mark.parametrize("tid", [Q4_K, Q6_K])
def test_tc_repeatable_bits(eng, tid):
    n, k, m = 700, 4096, 16
    wd = eng.upload(Q.synthetic_weights(n, k, tid, seed=3))
    x = torch.from_numpy(Q.synthetic_activations(m, k, seed=4)).to(eng.device)
    ys = [eng.gemv(wd, tid, x, n, k).cpu().numpy() for _ in range(3)]
    for y in ys[1:]:
        assert np.array_equal(y.view(np.uint32), ys[0].view(np.uint32))


def test_tc_q6k_large_scale_products(eng, oracle):
    """Q6_K blocks with int8 scales of magnitude 100..127 and random 6-bit
    values: many sc * (q - 32) exceed 2048 in magnitude."""
    n, k, m = 256, 2048, 4
    rng = np.random.default_rng(7)
    w = rng.integers(0, 256, size=(n * k // 256, 210), dtype=np.uint8)
    sc = rng.integers(100, 128, size=(n * k // 256, 16)) * rng.choice([-1, 1], size=(n * k // 256, 16))
    w[:, 192:208] = sc.astype(np.int8).view(np.uint8)
    w[:, 208:210] = np.full((n * k // 256, 1), 0.0005, np.float16).view(np.uint8)
    w = w.reshape(-1)
    x = Q.synthetic_activations(m, k, seed=8)
    y = eng.gemv(eng.upload(w), Q6_K, torch.from_numpy(x).to(eng.device), n, k).cpu().numpy()
    assert rel_err(y, oracle.quant_matmul(w, Q6_K, x, n, k, threads=8)) <= GEMV_TOL


@pytest.mark.parametrize("m", [2, 16])
def test_tc_mixed_segments(eng, oracle, m):
    k = 4096
    specs = [(Q4_K, 4096), (Q4_K, 1024), (Q6_K, 1024)]
    ws = [Q.synthetic_weights(n, k, t, seed=30 + i) for i, (t, n) in enumerate(specs)]
    x = Q.synthetic_activations(m, k, seed=31)
    outs = eng.gemv_multi([(eng.upload(w), t, n) for w, (t, n) in zip(ws, specs)],
                          torch.from_numpy(x).to(eng.device), k)
    for w, (t, n), y in zip(ws, specs, outs):
        rows = np.sort(np.random.default_rng(n).choice(n, 64, replace=False))
        from planejaja_b200.formats import fmt
        rb = fmt(t).row_bytes(k)
        ref = oracle.quant_matmul(np.concatenate([w[r * rb:(r + 1) * rb] for r in rows]), t, x, len(rows), k,
                                  threads=8)
        assert rel_err(y.cpu().numpy()[:, rows], ref) <= GEMV_TOL


@pytest.mark.parametrize("m", [5, 16])
def test_tc_every_format_in_one_launch(eng, oracle, m):
    """Q4_0, Q8_0, NodeStor Q5_K and NodeStor Q6_K segments in one launch: the
    mixed-format kernel with the widest raw column (Q8_0's 272 bytes)."""
    from planejaja_b200.formats import Q4_0, Q8_0, Q5_K, Q6K_NODESTOR
    k = 2048
    specs = [(Q4_0, 0, 200), (Q8_0, 0, 72), (Q5_K, Q6K_NODESTOR, 64), (Q6_K, Q6K_NODESTOR, 40)]
    ws = [Q.synthetic_weights(n, k, t, seed=40 + i, q6k_layout=l) for i, (t, l, n) in enumerate(specs)]
    x = Q.synthetic_activations(m, k, seed=41)
    outs = eng.gemv_multi([(eng.upload(w), t, n, l) for w, (t, l, n) in zip(ws, specs)],
                          torch.from_numpy(x).to(eng.device), k)
    for w, (t, l, n), y in zip(ws, specs, outs):
        assert rel_err(y.cpu().numpy(), oracle.quant_matmul(w, t, x, n, k, l, threads=8)) <= GEMV_TOL


@pytest.mark.parametrize("a_in", ["1", "0"])
@pytest.mark.parametrize("tid,layout", [("Q4_K", 0), ("Q6_K", 0), ("Q6_K", 1), ("Q5_K", 0), ("Q5_K", 1),
                                        ("Q4_0", 0), ("Q8_0", 0)])
def test_tc_a_operand_in_tmem_and_smem(eng, oracle, tuning, a_in, tid, layout):
    """Both homes of the fp16 weight operand (NSQ_TC_A=1: tensor memory, written
    by tcgen05.st and read by the MMA's A-from-TMEM form; 0: 128B-swizzled
    shared-memory tiles), every format and layout, against the oracle on a
    stream-K shape (tiles split over CTAs) at 16 and 7 tokens."""
    from planejaja_b200 import formats as F
    t = getattr(F, tid)
    tuning.set("NSQ_TC_A", a_in)
    n, k = 1100, 4096
    w = Q.synthetic_weights(n, k, t, seed=50 + layout, q6k_layout=layout)
    wd = eng.upload(w)
    for m in (16, 7):
        x = Q.synthetic_activations(m, k, seed=51 + m)
        y = eng.gemv(wd, t, torch.from_numpy(x).to(eng.device), n, k, q6k_layout=layout).cpu().numpy()
        assert rel_err(y, oracle.quant_matmul(w, t, x, n, k, layout, threads=8)) <= GEMV_TOL
