"""GPU parity tests: libnsq (through its C ABI) against the CPU oracle.

Bars:
  dequant  -- bit-exact f32 (and bf16 = round-to-nearest-even of the f32 value)
  GEMV     -- max_i |y_i - r_i| / max(|r_i|, rms(r)) <= 1e-3   (r: oracle f32)
  GEMM     -- the same metric <= 2e-2 (bf16 operands, fp32 accumulate)
"""
import numpy as np
import pytest
import torch

from planejaja_b200 import quantize as Q
from planejaja_b200 import _lib
from planejaja_b200.formats import FORMATS, Q4_0, Q4_K, Q5_K, Q6_K, Q8_0, Q6K_GGML, Q6K_NODESTOR

pytestmark = pytest.mark.gpu

GEMV_TOL = 1e-3
GEMM_TOL = 2e-2
ALL = [(Q4_0, 0), (Q8_0, 0), (Q4_K, 0), (Q5_K, Q6K_GGML), (Q5_K, Q6K_NODESTOR), (Q6_K, Q6K_GGML),
       (Q6_K, Q6K_NODESTOR)]
IDS = ["Q4_0", "Q8_0", "Q4_K", "Q5_K", "Q5_K_nodestor", "Q6_K", "Q6_K_nodestor"]


@pytest.fixture(scope="module")
def eng():
    from planejaja_b200.engine import CudaEngine
    e = CudaEngine(0)
    yield e
    assert e.device_status() == 0


def rel_err(y, r):
    y = np.asarray(y, np.float64).reshape(-1)
    r = np.asarray(r, np.float64).reshape(-1)
    rms = np.sqrt(np.mean(r * r)) if r.size else 0.0
    den = np.maximum(np.abs(r), max(rms, 1e-30))
    return float(np.max(np.abs(y - r) / den)) if r.size else 0.0


def bf16_round(a: np.ndarray) -> np.ndarray:
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(torch.bfloat16).float().numpy()


# ---------------------------------------------------------------- dequant
@pytest.mark.parametrize("tid,layout", ALL, ids=IDS)
def test_dequant_bit_exact_random(eng, oracle, tid, layout):
    raw = Q.synthetic_weights(96, 1024, tid, seed=11, q6k_layout=layout)
    ref = oracle.dequant(raw, tid, layout)
    w = eng.upload(raw)
    out = eng.dequant(w, tid, ref.size, "f32", layout).cpu().numpy()
    assert np.array_equal(out.view(np.uint32), ref.view(np.uint32))
    outb = eng.dequant(w, tid, ref.size, "bf16", layout).float().cpu().numpy()
    assert np.array_equal(outb.view(np.uint32), bf16_round(ref).view(np.uint32))


@pytest.mark.parametrize("name,tid,layout", [("Q4_0", Q4_0, 0), ("Q8_0", Q8_0, 0), ("Q4_K", Q4_K, 0),
                                             ("Q5_K", Q5_K, 0), ("Q5_K_NODESTOR", Q5_K, 1),
                                             ("Q6_K", Q6_K, 0), ("Q6_K_NODESTOR", Q6_K, 1)])
def test_dequant_golden_and_fuzz(eng, golden, name, tid, layout):
    raw, ref = golden[f"{name}_raw"], golden[f"{name}_f32"]
    out = eng.dequant(eng.upload(raw), tid, ref.size, "f32", layout).cpu().numpy()
    assert np.array_equal(out.view(np.uint32), ref.view(np.uint32))


def test_dequant_reference_known_answers(eng, golden):
    out = eng.dequant(eng.upload(golden["kat_q4k_uniform_raw"]), Q4_K, 256).cpu().numpy()
    assert np.all(out[:128] == 28.0)
    out = eng.dequant(eng.upload(golden["kat_q8_raw"]), Q8_0, 96).cpu().numpy().reshape(3, 32)
    assert np.all(out[0] == 0) and np.all(out[1] == 5.0) and out[2, 0] == -1.0
    out = eng.dequant(eng.upload(golden["kat_q5k_high_raw"]), Q5_K, 256, "f32", Q6K_NODESTOR).cpu().numpy()
    assert np.all(out >= 0) and np.all(out[:128] == 31.0)


def test_dequant_subnormal_scale_follows_rust_conversion(eng, oracle):
    blk = np.zeros(34, np.uint8)
    blk[0:2] = np.array([0x0200], np.uint16).view(np.uint8)  # d = 2^-15 (subnormal fp16)
    blk[2:] = np.arange(32, dtype=np.int8).view(np.uint8)
    out = eng.dequant(eng.upload(blk), Q8_0, 32).cpu().numpy()
    assert np.array_equal(out, oracle.dequant(blk, Q8_0, 0, fp16_mode=0))
    assert out[1] == 2.0 ** -15


def test_dequant_empty(eng):
    w = eng.upload(np.zeros(144, np.uint8))
    out = torch.empty(0, device=eng.device)
    eng.dequant(w, Q4_K, 0, out=out)


# ---------------------------------------------------------------- GEMV
@pytest.fixture(params=["rows", "mma", "general", "tc"])
def gemv_kernel(request, tuning):
    """Runs a test with each GEMV kernel: one lane per row (dp4a, every M),
    integer tensor cores (mma.sync, every M), the general kernel, and the
    tcgen05 kernel (M >= 2, every format)."""
    tuning.unset("NSQ_GEMV_GENERAL")
    tuning.set("NSQ_TC_MIN_M", "17")
    if request.param == "general":
        tuning.set("NSQ_GEMV_GENERAL", "1")
    elif request.param == "mma":
        tuning.set("NSQ_MMA_MIN_M", "1")
    elif request.param == "tc":
        # tcgen05 path for M >= 2; M = 1 takes the one-lane-per-row kernel
        tuning.set("NSQ_TC_MIN_M", "2")
        tuning.set("NSQ_MMA_MIN_M", "17")
    else:
        tuning.set("NSQ_MMA_MIN_M", "17")
    return request.param


@pytest.mark.parametrize("tid,layout", ALL, ids=IDS)
@pytest.mark.parametrize("m", [1, 2, 3, 4, 5, 8, 16])
def test_gemv_parity(eng, oracle, gemv_kernel, tid, layout, m):
    n, k = 300, 2048
    w = Q.synthetic_weights(n, k, tid, seed=100 + tid, q6k_layout=layout)
    x = Q.synthetic_activations(m, k, seed=200 + m)
    ref = oracle.quant_matmul(w, tid, x, n, k, layout, threads=8)
    y = eng.gemv(eng.upload(w), tid, torch.from_numpy(x).to(eng.device), n, k, layout).cpu().numpy()
    assert rel_err(y, ref) <= GEMV_TOL


@pytest.mark.parametrize("tid,layout", ALL, ids=IDS)
@pytest.mark.parametrize("n,k", [(1, 256), (7, 512), (129, 768), (1000, 256), (64, 14336), (33, 28672),
                                 (4096, 4096), (300, 2304)])
def test_gemv_shapes(eng, oracle, gemv_kernel, tid, layout, n, k):
    w = Q.synthetic_weights(n, k, tid, seed=7, q6k_layout=layout)
    x = Q.synthetic_activations(1, k, seed=8)
    ref = oracle.quant_matmul(w, tid, x, n, k, layout, threads=8)
    y = eng.gemv(eng.upload(w), tid, torch.from_numpy(x).to(eng.device), n, k, layout).cpu().numpy()
    assert rel_err(y, ref) <= GEMV_TOL


@pytest.mark.parametrize("tid", [Q4_0, Q8_0])
@pytest.mark.parametrize("n,k", [(5, 32), (40, 96), (130, 1120)])
def test_gemv_small_blocks(eng, oracle, tid, n, k):
    """K not a multiple of 256: only the general kernel covers it."""
    w = Q.synthetic_weights(n, k, tid, seed=17)
    x = Q.synthetic_activations(2, k, seed=18)
    y = eng.gemv(eng.upload(w), tid, torch.from_numpy(x).to(eng.device), n, k).cpu().numpy()
    assert rel_err(y, oracle.quant_matmul(w, tid, x, n, k)) <= GEMV_TOL


def test_gemv_micro_config(eng, oracle):
    """Micro-model Q8_0 matvec W[1536 x 512], x[1 x 512] (seeded N(0,0.02) / N(0,1))."""
    n, k = 1536, 512
    w = Q.synthetic_weights(n, k, Q8_0, seed=1000)
    x = Q.synthetic_activations(1, k, seed=2000)
    ref = oracle.quant_matmul(w, Q8_0, x, n, k)
    y = eng.matmul_quant(torch.from_numpy(x).to(eng.device), eng.upload(w), Q8_0, 1, k, n).cpu().numpy()
    assert rel_err(y, ref) <= GEMV_TOL


@pytest.mark.parametrize("m", [1, 2, 4, 5])
def test_gemv_multi_mixed_segments(eng, oracle, m):
    """Fused q|k|v-style launch: two Q4_K segments and a Q6_K one sharing x."""
    k = 2048
    specs = [(Q4_K, 0, 200), (Q4_K, 0, 64), (Q6_K, Q6K_GGML, 72)]
    ws = [Q.synthetic_weights(n, k, t, seed=50 + i, q6k_layout=l) for i, (t, l, n) in enumerate(specs)]
    x = Q.synthetic_activations(m, k, seed=51)
    outs = eng.gemv_multi([(eng.upload(w), t, n, l) for w, (t, l, n) in zip(ws, specs)],
                          torch.from_numpy(x).to(eng.device), k)
    for w, (t, l, n), y in zip(ws, specs, outs):
        assert rel_err(y.cpu().numpy(), oracle.quant_matmul(w, t, x, n, k, l)) <= GEMV_TOL


@pytest.mark.parametrize("layout", [Q6K_GGML, Q6K_NODESTOR])
@pytest.mark.parametrize("m", [1, 3, 12])
def test_gemv_multi_q5k_mix(eng, oracle, gemv_kernel, layout, m):
    """Q5_K_M-style q|k|v: two Q5_K segments and a Q6_K one, one launch."""
    k = 2048
    specs = [(Q5_K, layout, 136), (Q5_K, layout, 40), (Q6_K, layout, 40)]
    ws = [Q.synthetic_weights(n, k, t, seed=80 + i, q6k_layout=l) for i, (t, l, n) in enumerate(specs)]
    x = Q.synthetic_activations(m, k, seed=81)
    outs = eng.gemv_multi([(eng.upload(w), t, n, l) for w, (t, l, n) in zip(ws, specs)],
                          torch.from_numpy(x).to(eng.device), k)
    for w, (t, l, n), y in zip(ws, specs, outs):
        assert rel_err(y.cpu().numpy(), oracle.quant_matmul(w, t, x, n, k, l, threads=8)) <= GEMV_TOL


def test_gemv_multi_workspace_mode(eng, oracle):
    """M * K too large for on-chip preparation: activations go through the workspace."""
    m, k = 4, 14336
    specs = [(Q4_K, 0, 40), (Q6_K, Q6K_NODESTOR, 24)]
    ws = [Q.synthetic_weights(n, k, t, seed=60 + i, q6k_layout=l) for i, (t, l, n) in enumerate(specs)]
    x = Q.synthetic_activations(m, k, seed=61)
    outs = eng.gemv_multi([(eng.upload(w), t, n, l) for w, (t, l, n) in zip(ws, specs)],
                          torch.from_numpy(x).to(eng.device), k)
    for w, (t, l, n), y in zip(ws, specs, outs):
        assert rel_err(y.cpu().numpy(), oracle.quant_matmul(w, t, x, n, k, l, threads=8)) <= GEMV_TOL


@pytest.mark.parametrize("tid,layout,k", [(Q4_K, 0, 14336), (Q6_K, Q6K_GGML, 14336), (Q6_K, Q6K_NODESTOR, 14336),
                                          (Q4_0, 0, 11008), (Q5_K, Q6K_GGML, 8448)])
def test_gemv_long_rows_with_and_without_workspace(eng, oracle, tuning, tid, layout, k):
    """One token with long rows: given a workspace, the separate preparation
    kernel writes the records; without one, the fused kernel quantises them on
    chip (CTA pairs for K >= 8192).  Both against the oracle."""
    tuning.set("NSQ_TC_MIN_M", "17")
    lib = eng.lib
    n = 200
    w = Q.synthetic_weights(n, k, tid, seed=k + tid, q6k_layout=layout)
    x = Q.synthetic_activations(1, k, seed=k)
    ref = oracle.quant_matmul(w, tid, x, n, k, layout, threads=8)
    wd, xd = eng.upload(w), torch.from_numpy(x).to(eng.device)
    st = torch.cuda.current_stream().cuda_stream
    wsb = lib.nsq_gemv_workspace_size(1, k)
    ws = torch.empty(wsb, dtype=torch.uint8, device=eng.device)
    for ptr, size in [(ws.data_ptr(), wsb), (None, 0)]:
        y = torch.full((1, n), float("nan"), device=eng.device)
        rc = lib.nsq_gemv(wd.data_ptr(), tid, layout, xd.data_ptr(), y.data_ptr(), 1, n, k, ptr, size, st)
        assert rc == 0, _lib.strerror(rc)
        torch.cuda.synchronize()
        assert rel_err(y.cpu().numpy(), ref) <= GEMV_TOL


def test_gemv_unaligned_activations(eng, oracle):
    """x only 4-byte aligned: taken through the workspace path."""
    n, k = 96, 1024
    w = Q.synthetic_weights(n, k, Q4_K, seed=70)
    x = Q.synthetic_activations(1, k, seed=71)
    buf = torch.empty(k + 1, device=eng.device)
    buf[1:] = torch.from_numpy(x[0]).to(eng.device)
    y = eng.gemv(eng.upload(w), Q4_K, buf[1:], n, k).cpu().numpy()
    assert rel_err(y, oracle.quant_matmul(w, Q4_K, x, n, k)) <= GEMV_TOL


def _adversarial_activations(m, k, seed):
    """Groups of 32 that stress the activation quantisation: Gaussian, a NaN
    inside a group, exact rounding ties (amax 32767, so x * 32767 / amax lands
    on .5), amax too small for 32767 / amax (the fallback conversion), an
    infinite value, all zeros."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((m, k)).astype(np.float32)
    g = x.reshape(m, k // 32, 32)
    g[:, 1, 5] = np.nan
    g[:, 2, :] = np.arange(-16, 16, dtype=np.float32) + 0.5
    g[:, 2, 0] = 32767.0
    g[:, 3, :] = rng.standard_normal(32).astype(np.float32) * np.float32(1e-38)
    g[:, 4, 7] = np.inf
    g[:, 5, :] = 0.0
    g[:, 6, :] = -2.5
    return x


@pytest.mark.parametrize("m", [1, 3])
def test_gemv_on_chip_quantiser_matches_prepare_kernel(eng, tuning, m):
    """The fused kernel quantises activations on chip (x 16-byte aligned);
    with x only 4-byte aligned the standalone preparation kernel writes the
    records and the same fused kernel reads them.  Both plans are identical
    at this shape, so equal outputs, bit for bit, mean equal records."""
    tuning.set("NSQ_TC_MIN_M", "17")  # the fused kernel for M = 3 too
    n, k = 256, 1024
    w = eng.upload(Q.synthetic_weights(n, k, Q4_K, seed=12))
    x = torch.from_numpy(_adversarial_activations(m, k, seed=13)).to(eng.device)
    buf = torch.empty(m * k + 1, device=eng.device)
    buf[1:] = x.reshape(-1)
    y_chip = eng.gemv(w, Q4_K, x, n, k).cpu().numpy()
    y_prep = eng.gemv(w, Q4_K, buf[1:], n, k).cpu().numpy()
    assert np.array_equal(np.isnan(y_chip), np.isnan(y_prep))
    ok = ~np.isnan(y_chip)
    assert np.array_equal(y_chip[ok].view(np.uint32), y_prep[ok].view(np.uint32))


def test_gemv_prepared_shares_activations(eng, oracle):
    k = 1024
    x = Q.synthetic_activations(2, k, seed=9)
    xd = torch.from_numpy(x).to(eng.device)
    ws = eng.prepare(xd, k)
    for tid, n in [(Q4_K, 256), (Q6_K, 96), (Q8_0, 40)]:
        w = Q.synthetic_weights(n, k, tid, seed=n)
        y = eng.gemv_prepared(eng.upload(w), tid, ws, 2, n, k)
        torch.cuda.synchronize()
        assert rel_err(y.cpu().numpy(), oracle.quant_matmul(w, tid, x, n, k)) <= GEMV_TOL


def test_gemv_zero_and_constant_activations(eng, oracle):
    n, k = 64, 512
    w = Q.synthetic_weights(n, k, Q4_K, seed=3)
    wd = eng.upload(w)
    y = eng.gemv(wd, Q4_K, torch.zeros(1, k, device=eng.device), n, k).cpu().numpy()
    assert np.all(y == 0)
    x = np.full((1, k), 0.5, np.float32)
    y = eng.gemv(wd, Q4_K, torch.from_numpy(x).to(eng.device), n, k).cpu().numpy()
    assert rel_err(y, oracle.quant_matmul(w, Q4_K, x, n, k)) <= GEMV_TOL


def test_gemv_offset_weight_pointer(eng, oracle):
    """A weight tensor at a 16-byte offset inside a larger buffer (GGUF data section)."""
    n, k = 50, 512
    w = Q.synthetic_weights(n, k, Q6_K, seed=4)
    buf = eng.upload(np.concatenate([np.zeros(48, np.uint8), w, np.zeros(5, np.uint8)]))
    x = Q.synthetic_activations(1, k, seed=5)
    y = eng.gemv(buf[48:48 + w.size], Q6_K, torch.from_numpy(x).to(eng.device), n, k).cpu().numpy()
    assert rel_err(y, oracle.quant_matmul(w, Q6_K, x, n, k)) <= GEMV_TOL


def test_gemv_errors_on_gpu(eng):
    w = eng.upload(np.zeros(144 * 4, np.uint8))
    x = torch.zeros(1, 256, device=eng.device)
    with pytest.raises(_lib.NsqError) as e:
        eng.gemv(w[1:], Q4_K, x, 2, 256)
    assert e.value.status == _lib.ERR_ALIGN
    with pytest.raises(_lib.NsqError) as e:
        eng.gemv(w, 3, x, 2, 256)
    assert e.value.status == _lib.ERR_TYPE


# ---------------------------------------------------------------- GEMM
@pytest.fixture(params=["tok_auto", "tok128", "tok512", "nosplit"])
def gemm_tok(request, tuning):
    """Runs a GEMM test with the default token tile (and the default split-K,
    which small grids get), 128-token tiles, 512-token tiles (two N = 256
    MMAs per K step; Q8_0 falls back to 256), and split-K switched off."""
    tuning.unset("NSQ_GEMM_TOK")
    tuning.unset("NSQ_GEMM_SPLIT")
    if request.param == "tok128":
        tuning.set("NSQ_GEMM_TOK", "128")
    elif request.param == "tok512":
        tuning.set("NSQ_GEMM_TOK", "512")
    elif request.param == "nosplit":
        tuning.set("NSQ_GEMM_SPLIT", "1")
    return request.param


@pytest.mark.parametrize("tid,layout", ALL, ids=IDS)
@pytest.mark.parametrize("m,n,k", [(128, 256, 512), (17, 200, 1024), (129, 130, 256), (300, 384, 2048)])
def test_gemm_parity(eng, oracle, gemm_tok, tid, layout, m, n, k):
    w = Q.synthetic_weights(n, k, tid, seed=300 + n, q6k_layout=layout)
    x = bf16_round(Q.synthetic_activations(m, k, seed=400 + m))
    ref = oracle.quant_matmul(w, tid, x, n, k, layout, threads=8)
    xd = torch.from_numpy(x).to(eng.device).to(torch.bfloat16)
    y = eng.gemm_bf16(eng.upload(w), tid, xd, n, k, layout).float().cpu().numpy()
    assert rel_err(y, ref) <= GEMM_TOL


def test_gemm_matches_dequant_plus_torch(eng):
    """bf16 GEMM equals (dequant -> bf16) @ x in fp32 closely (same bf16 operands)."""
    n, k, m = 512, 4096, 256
    w = Q.synthetic_weights(n, k, Q4_K, seed=21)
    wd = eng.upload(w)
    x = torch.randn(m, k, device=eng.device).to(torch.bfloat16)
    wb = eng.dequant(wd, Q4_K, n * k, "bf16").reshape(n, k)
    ref = (x.float() @ wb.float().T)
    y = eng.gemm_bf16(wd, Q4_K, x, n, k).float()
    assert rel_err(y.cpu().numpy(), ref.cpu().numpy()) <= 1e-2


# ---------------------------------------------------------------- dense f32 matmul
def test_matmul_f32(eng, oracle):
    rng = np.random.default_rng(0)
    m, k, n = 33, 70, 45
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = rng.standard_normal((k, n)).astype(np.float32)
    c = eng.matmul(torch.from_numpy(a).to(eng.device), torch.from_numpy(b).to(eng.device), m, k, n)
    assert rel_err(c.cpu().numpy(), oracle.matmul_f32(a, b, m, k, n)) <= 1e-5
    c = eng.matmul(torch.tensor([[1., 2.], [3., 4.]], device=eng.device),
                   torch.tensor([[5., 6.], [7., 8.]], device=eng.device), 2, 2, 2)
    assert c.cpu().tolist() == [[19.0, 22.0], [43.0, 50.0]]


# ---------------------------------------------------------------- fused epilogues
def _silu(v):
    return v * (1.0 / (1.0 + np.exp(-v)))


@pytest.mark.parametrize("tid,layout", ALL, ids=IDS)
@pytest.mark.parametrize("m", [1, 3, 6])
def test_gemv_swiglu_parity(eng, oracle, tid, layout, m):
    """h = silu(x Wg^T) * (x Wu^T) in one launch, against the oracle GEMVs
    composed with the reference's silu and mul (in f64)."""
    n, k = 300, 2048
    wg = Q.synthetic_weights(n, k, tid, seed=500 + tid, q6k_layout=layout)
    wu = Q.synthetic_weights(n, k, tid, seed=600 + tid, q6k_layout=layout)
    x = Q.synthetic_activations(m, k, seed=700 + m)
    g = oracle.quant_matmul(wg, tid, x, n, k, layout, threads=8).astype(np.float64)
    u = oracle.quant_matmul(wu, tid, x, n, k, layout, threads=8).astype(np.float64)
    ref = _silu(g) * u
    h = eng.gemv_swiglu(eng.upload(wg), eng.upload(wu), tid, torch.from_numpy(x).to(eng.device), n, k, layout)
    assert rel_err(h.cpu().numpy(), ref) <= 2 * GEMV_TOL


@pytest.mark.parametrize("tid,layout", ALL, ids=IDS)
@pytest.mark.parametrize("m", [1, 5])
def test_gemv_residual_parity(eng, oracle, tid, layout, m):
    n, k = 257, 4096
    w = Q.synthetic_weights(n, k, tid, seed=800 + tid, q6k_layout=layout)
    x = Q.synthetic_activations(m, k, seed=801)
    res = np.random.default_rng(9).standard_normal((m, n)).astype(np.float32)
    ref = oracle.quant_matmul(w, tid, x, n, k, layout, threads=8).astype(np.float64) + res
    wd = eng.upload(w)
    xd = torch.from_numpy(x).to(eng.device)
    y = eng.gemv_residual(wd, tid, xd, torch.from_numpy(res).to(eng.device), n, k, layout)
    assert rel_err(y.cpu().numpy(), ref) <= GEMV_TOL
    # in place: the residual buffer receives the sum
    buf = torch.from_numpy(res).to(eng.device)
    eng.gemv_residual(wd, tid, xd, buf, n, k, layout, out=buf)
    assert rel_err(buf.cpu().numpy(), ref) <= GEMV_TOL


def test_gemv_swiglu_rejects_mismatched_pairs(eng):
    wg = eng.upload(Q.synthetic_weights(64, 512, Q4_K, seed=1))
    wu = eng.upload(Q.synthetic_weights(64, 512, Q4_K, seed=2))
    x = torch.zeros(1, 300, device=eng.device)
    with pytest.raises(_lib.NsqError):  # K % 256
        eng.gemv_swiglu(wg, wu, Q4_K, x, 64, 300)


def test_kernel_launch_counter(eng, tuning):
    """nsq_kernel_launches counts the library's kernels: one fused launch for a
    one-token GEMV prepared on chip, two (preparation + fused) when the
    activations go through the workspace, two (tile preparation + tcgen05) for
    16 tokens."""
    tuning.set("NSQ_TC_MIN_M", "5")
    lib = eng.lib
    n = 256
    for k, m, kernels in [(4096, 1, 1), (14336, 1, 2), (4096, 16, 2)]:
        w = eng.upload(Q.synthetic_weights(n, k, Q4_K, seed=k))
        x = torch.from_numpy(Q.synthetic_activations(m, k, seed=m)).to(eng.device)
        before = lib.nsq_kernel_launches()
        eng.gemv(w, Q4_K, x, n, k)
        assert lib.nsq_kernel_launches() - before == kernels, (k, m)
