"""GPU parity on LLM-like activations: outlier channels and lopsided groups.

Every decode GEMV kernel turns each run of 32 fp32 activations into int16
values with one fp32 scale (amax / 32767) before the integer dot products, so
its error grows with each group's largest magnitude.  Real activations carry
a few channels 100-1000x the rms of the rest.  These tests draw such vectors
and compare every kernel (one lane per row, integer tensor cores, general)
with the oracle (the reference's dequant composed with its cpu_matmul_f32,
pipeline.rs:1256-1268), for every weight format and both K-quant layouts.

The bar is the GEMV bar, checked per token:
    max_i |y_i - r_i| / max(|r_i|, rms(r over that token)) <= 1e-3
so a token of small magnitude next to a large one is held to its own scale.
"""
import numpy as np
import pytest
import torch

from planejaja_b200 import quantize as Q
from planejaja_b200.formats import Q4_0, Q4_K, Q5_K, Q6_K, Q8_0, Q6K_GGML, Q6K_NODESTOR, fmt

pytestmark = pytest.mark.gpu

GEMV_TOL = 1e-3
ALL = [(Q4_0, 0), (Q8_0, 0), (Q4_K, 0), (Q5_K, Q6K_GGML), (Q5_K, Q6K_NODESTOR), (Q6_K, Q6K_GGML),
       (Q6_K, Q6K_NODESTOR)]
IDS = ["Q4_0", "Q8_0", "Q4_K", "Q5_K", "Q5_K_nodestor", "Q6_K", "Q6_K_nodestor"]


@pytest.fixture(scope="module")
def eng():
    from planejaja_b200.engine import CudaEngine
    e = CudaEngine(0)
    yield e
    assert e.device_status() == 0


@pytest.fixture(params=["rows", "mma", "general", "tc"])
def gemv_kernel(request, tuning):
    tuning.unset("NSQ_GEMV_GENERAL")
    tuning.set("NSQ_TC_MIN_M", "17")
    if request.param == "general":
        tuning.set("NSQ_GEMV_GENERAL", "1")
    elif request.param == "mma":
        tuning.set("NSQ_MMA_MIN_M", "1")
    elif request.param == "tc":
        # tcgen05 path for M >= 2 over Q4_K / ggml Q6_K; the other formats
        # (and M = 1) take the one-lane-per-row kernel
        tuning.set("NSQ_TC_MIN_M", "2")
        tuning.set("NSQ_MMA_MIN_M", "17")
    else:
        tuning.set("NSQ_MMA_MIN_M", "17")
    return request.param


def llm_activations(m: int, k: int, seed: int) -> np.ndarray:
    """N(0, 1) activations with outlier channels at 100x, 300x and 1000x the
    rms (two channels each, the same channels in every token), one group
    holding a single value of 3000 beside values of 1e-3, and tokens whose
    overall magnitude differs by up to 1000x."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((m, k)).astype(np.float32)
    ch = rng.choice(k, 6, replace=False)
    for c, f in zip(ch, [100, 100, 300, 300, 1000, 1000]):
        x[:, c] *= np.float32(f)
    g = int(rng.integers(0, k // 32))
    x[:, 32 * g:32 * g + 32] = rng.standard_normal((m, 32)).astype(np.float32) * np.float32(1e-3)
    x[:, 32 * g + int(rng.integers(0, 32))] = 3000.0
    tok_scale = np.float32(10.0) ** rng.integers(-1, 3, size=(m, 1)).astype(np.float32)
    return (x * tok_scale).astype(np.float32)


def per_token_err(y, r):
    y = np.asarray(y, np.float64).reshape(r.shape)
    r = np.asarray(r, np.float64)
    worst = 0.0
    for t in range(r.shape[0]):
        rms = max(float(np.sqrt(np.mean(r[t] * r[t]))), 1e-30)
        worst = max(worst, float(np.max(np.abs(y[t] - r[t]) / np.maximum(np.abs(r[t]), rms))))
    return worst


@pytest.mark.parametrize("tid,layout", ALL, ids=IDS)
@pytest.mark.parametrize("m", [1, 4, 16])
def test_gemv_outlier_activations(eng, oracle, gemv_kernel, tid, layout, m):
    n, k = 300, 2048
    w = Q.synthetic_weights(n, k, tid, seed=500 + tid, q6k_layout=layout)
    x = llm_activations(m, k, seed=600 + m)
    ref = oracle.quant_matmul(w, tid, x, n, k, layout, threads=8).reshape(m, n)
    y = eng.gemv(eng.upload(w), tid, torch.from_numpy(x).to(eng.device), n, k, layout).cpu().numpy()
    assert per_token_err(y, ref) <= GEMV_TOL


@pytest.mark.parametrize("m", [1, 3, 16])
def test_gemv_multi_outlier_activations(eng, oracle, m):
    """q|k|v-style fused launch (two Q4_K segments and a Q6_K one) on outlier activations."""
    k = 4096
    specs = [(Q4_K, 0, 256), (Q4_K, 0, 64), (Q6_K, Q6K_NODESTOR, 64)]
    ws = [Q.synthetic_weights(n, k, t, seed=90 + i, q6k_layout=l) for i, (t, l, n) in enumerate(specs)]
    x = llm_activations(m, k, seed=91)
    outs = eng.gemv_multi([(eng.upload(w), t, n, l) for w, (t, l, n) in zip(ws, specs)],
                          torch.from_numpy(x).to(eng.device), k)
    for w, (t, l, n), y in zip(ws, specs, outs):
        ref = oracle.quant_matmul(w, t, x, n, k, l, threads=8).reshape(m, n)
        assert per_token_err(y.cpu().numpy(), ref) <= GEMV_TOL


@pytest.mark.parametrize("name,n,k,tid,layout,m", [
    ("l3_gate", 14336, 4096, Q4_K, 0, 1), ("l3_gate_b16", 14336, 4096, Q4_K, 0, 16),
    ("l3_down", 4096, 14336, Q6_K, Q6K_GGML, 1), ("l3_down_nodestor", 4096, 14336, Q6_K, Q6K_NODESTOR, 4)])
def test_gemv_outlier_full_size_sampled_rows(eng, oracle, name, n, k, tid, layout, m):
    """Full Llama-3-8B FFN shapes; the oracle checks a seeded sample of 48 rows."""
    w = Q.synthetic_weights(n, k, tid, seed=sum(map(ord, name)), q6k_layout=layout)
    x = llm_activations(m, k, seed=13)
    y = eng.gemv(eng.upload(w), tid, torch.from_numpy(x).to(eng.device), n, k, layout).cpu().numpy()
    rows = np.sort(np.random.default_rng(4).choice(n, 48, replace=False))
    rb = fmt(tid).row_bytes(k)
    ws = np.concatenate([w[r * rb:(r + 1) * rb] for r in rows])
    ref = oracle.quant_matmul(ws, tid, x, len(rows), k, layout, threads=8).reshape(m, len(rows))
    assert per_token_err(y.reshape(m, n)[:, rows], ref) <= GEMV_TOL
