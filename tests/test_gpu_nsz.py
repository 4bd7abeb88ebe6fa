"""NSZ decode and ZipGEMM on the GPU through libnsq's C ABI, against the
oracle: decode bit-exact; ZipGEMM within the GEMV bar
max_i |y_i - r_i| / max(|r_i|, rms(r)) <= 1e-3 (r: sequential f32 oracle)."""
import numpy as np
import pytest
import torch

from planejaja_b200 import _lib
from planejaja_b200 import nsz as Z

pytestmark = pytest.mark.gpu

TOL = 1e-3
FIXTURE = {"output_norm.weight": (1, 64), "blk.0.attn_q.weight": (64, 64), "token_embd.weight": (128, 64),
           "blk.0.ffn_down.weight": (64, 172)}


@pytest.fixture(scope="module")
def eng():
    from planejaja_b200.engine import CudaEngine
    e = CudaEngine(0)
    yield e
    assert e.device_status() == 0


@pytest.fixture(scope="module")
def nszg():
    import os
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    return dict(np.load(os.path.join(root, "tests", "golden", "nsz_golden.npz")))


def rel_err(y, r):
    y = np.asarray(y, np.float64).reshape(-1)
    r = np.asarray(r, np.float64).reshape(-1)
    rms = np.sqrt(np.mean(r * r))
    return float(np.max(np.abs(y - r) / np.maximum(np.abs(r), max(rms, 1e-30))))


def _weights(rng, dt, n, std=0.02):
    if dt == Z.FP32:
        return (rng.standard_normal(n) * std).astype(np.float32)
    if dt == Z.FP16:
        return (rng.standard_normal(n) * std).astype(np.float16)
    return ((rng.standard_normal(n) * std).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)


def _as_f32(bits, dt):
    """Decoded weights (oracle.nsz_decode: f32, or raw uint16 bits) as float32."""
    if dt == Z.FP32:
        return bits.astype(np.float32)
    if dt == Z.FP16:
        return bits.view(np.float16).astype(np.float32)
    return (bits.astype(np.uint32) << 16).view(np.float32)


# ---------------------------------------------------------------- decode
@pytest.mark.parametrize("dt", [Z.FP32, Z.FP16, Z.BF16])
@pytest.mark.parametrize("n", [1, 37, 512, 1500, 4096, 11008, 300000])
def test_decode_bit_exact(eng, oracle, dt, n):
    w = _weights(np.random.default_rng(n + dt), dt, n)
    s = Z.encode(w, dt)
    out = eng.nsz_decode(eng.nsz_upload(s, n, dt)).cpu()
    got = out.view(torch.int32).numpy().view(np.uint32) if dt == Z.FP32 else out.view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(got, oracle.nsz_decode(s, n, dt).view(got.dtype))


def test_decode_fuzz_and_special_values(eng, oracle):
    rng = np.random.default_rng(7)
    w = rng.integers(0, 2 ** 32, 20000, dtype=np.uint64).astype(np.uint32)
    w[:8] = np.array([np.inf, -np.inf, -0.0, 1e-45, 3e38, -3e38, np.nan, 0.0], np.float32).view(np.uint32)
    s = Z.encode(w.view(np.float32))
    got = eng.nsz_decode(eng.nsz_upload(s, w.size)).cpu().view(torch.int32).numpy().view(np.uint32)
    assert np.array_equal(got, w)
    for dt in (Z.FP16, Z.BF16):
        h = rng.integers(0, 2 ** 16, 7000, dtype=np.uint32).astype(np.uint16)
        s = Z.encode(h if dt == Z.BF16 else h.view(np.float16), dt)
        got = eng.nsz_decode(eng.nsz_upload(s, h.size, dt)).cpu().view(torch.int16).numpy().view(np.uint16)
        assert np.array_equal(got, h)


def test_decode_reference_streams(eng, oracle, nszg):
    for name, (n, k) in FIXTURE.items():
        s = nszg["stream_" + name.replace(".", "_")]
        got = eng.nsz_decode(eng.nsz_upload(s, n * k)).cpu().numpy()
        assert np.array_equal(got.view(np.uint32), oracle.nsz_decode(s, n * k).view(np.uint32)), name


def test_decode_modal_255_tiles_from_the_reference_encoder(eng, oracle):
    """Bytes written by the reference encoder's near rule at modal 255 decode
    exactly as its decoder does (exponent 0 comes back as 254)."""
    w = np.full(1024, np.inf, np.float32)
    w[[3, 700]] = 1e-40
    s = oracle.nsz_encode(w, reference_quirks=True)
    got = eng.nsz_decode(eng.nsz_upload(s, w.size)).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), oracle.nsz_decode(s, w.size).view(np.uint32))


# ---------------------------------------------------------------- ZipGEMM
@pytest.mark.parametrize("m", [1, 2, 3, 5, 8, 9, 16])
@pytest.mark.parametrize("n,k", [(300, 2048), (1000, 512), (129, 4096), (64, 64), (172, 64), (7, 1536)])
def test_zipgemm_parity(eng, oracle, m, n, k):
    rng = np.random.default_rng(n * 7 + k + m)
    w = _weights(rng, Z.FP32, n * k)
    x = rng.standard_normal((m, k)).astype(np.float32)
    t = eng.nsz_upload(Z.encode(w), n * k)
    y = eng.zipgemm(t, torch.from_numpy(x).to(eng.device), m, k, n).cpu().numpy()
    assert rel_err(y, oracle.nsz_matmul(Z.encode(w), x, n, k)) <= TOL


@pytest.mark.parametrize("n,k", [(64, 172), (33, 100), (5, 7), (40, 520)])
@pytest.mark.parametrize("m", [1, 4])
def test_zipgemm_ragged_k(eng, oracle, n, k, m):
    """K % 16 != 0: rows start inside a lane's 16 weights (general path)."""
    rng = np.random.default_rng(n + k)
    w = _weights(rng, Z.FP32, n * k)
    x = rng.standard_normal((m, k)).astype(np.float32)
    s = Z.encode(w)
    y = eng.zipgemm(eng.nsz_upload(s, n * k), torch.from_numpy(x).to(eng.device), m, k, n).cpu().numpy()
    assert rel_err(y, oracle.nsz_matmul(s, x, n, k)) <= TOL


def test_zipgemm_unaligned_activations(eng, oracle):
    n, k = 96, 1024
    rng = np.random.default_rng(4)
    w = _weights(rng, Z.FP32, n * k)
    x = rng.standard_normal((2, k)).astype(np.float32)
    buf = torch.empty(2 * k + 1, device=eng.device)
    buf[1:] = torch.from_numpy(x.reshape(-1)).to(eng.device)
    s = Z.encode(w)
    y = eng.zipgemm(eng.nsz_upload(s, n * k), buf[1:], 2, k, n).cpu().numpy()
    assert rel_err(y, oracle.nsz_matmul(s, x, n, k)) <= TOL


@pytest.mark.parametrize("dt", [Z.FP16, Z.BF16])
@pytest.mark.parametrize("m", [1, 3])
def test_zipgemm_half_dtypes(eng, oracle, dt, m):
    n, k = 200, 1024
    rng = np.random.default_rng(dt + m)
    w = _weights(rng, dt, n * k, std=0.05)
    x = rng.standard_normal((m, k)).astype(np.float32)
    s = Z.encode(w, dt)
    wf = _as_f32(oracle.nsz_decode(s, n * k, dt), dt).reshape(n, k)
    ref = oracle.matmul_f32(x, np.ascontiguousarray(wf.T), m, k, n)
    y = eng.zipgemm(eng.nsz_upload(s, n * k, dt), torch.from_numpy(x).to(eng.device), m, k, n).cpu().numpy()
    assert rel_err(y, ref) <= TOL


def test_zipgemm_reference_streams(eng, oracle, nszg):
    """The micro model's q and ffn_down projections straight from the
    reference's .nsz bytes (y = x . W^T, W [N x K] in stream order)."""
    rng = np.random.default_rng(11)
    for name, (n, k) in FIXTURE.items():
        s = nszg["stream_" + name.replace(".", "_")]
        x = rng.standard_normal((1, k)).astype(np.float32)
        y = eng.zipgemm(eng.nsz_upload(s, n * k), torch.from_numpy(x).to(eng.device), 1, k, n).cpu().numpy()
        assert rel_err(y, oracle.nsz_matmul(s, x, n, k)) <= TOL, name


def test_zipgemm_large_rows(eng, oracle):
    """Rows split over every CTA, several waves of tiles per warp; checked
    against the oracle on a sample of rows (whole-matrix oracle too slow)."""
    n, k = 14336, 4096
    rng = np.random.default_rng(12)
    w = _weights(rng, Z.FP32, n * k)
    x = rng.standard_normal((1, k)).astype(np.float32)
    t = eng.nsz_upload(Z.encode(w), n * k)
    y = eng.zipgemm(t, torch.from_numpy(x).to(eng.device), 1, k, n).cpu().numpy()
    rows = np.unique(np.concatenate([np.arange(0, n, 997), [n - 1]]))
    sub = w.reshape(n, k)[rows]
    ref = oracle.nsz_matmul(Z.encode(sub), x, rows.size, k)
    assert rel_err(y[:, rows], ref) <= TOL
    # decode of the same tensor is bit-exact
    d = eng.nsz_decode(t).cpu().numpy()
    assert np.array_equal(d.view(np.uint32), w.view(np.uint32))


def test_zipgemm_argument_errors(eng):
    w = _weights(np.random.default_rng(0), Z.FP32, 64 * 64)
    t = eng.nsz_upload(Z.encode(w), 64 * 64)
    x = torch.zeros(1, 64, device=eng.device)
    with pytest.raises(_lib.NsqError):
        eng.zipgemm(t, x, 1, 64, 32)  # holds 64 x 64 weights
    lib = eng.lib
    y = torch.empty(64, device=eng.device)
    st = torch.cuda.current_stream().cuda_stream
    assert lib.nsq_zipgemm(t.tiles.data_ptr(), t.offsets.data_ptr(), 7, x.data_ptr(), y.data_ptr(), 1, 64, 64,
                           st) == _lib.ERR_TYPE
    assert lib.nsq_zipgemm(t.tiles.data_ptr() + 8, t.offsets.data_ptr(), 0, x.data_ptr(), y.data_ptr(), 1, 64, 64,
                           st) == _lib.ERR_ALIGN
    assert lib.nsq_zipgemm(None, t.offsets.data_ptr(), 0, x.data_ptr(), y.data_ptr(), 1, 64, 64,
                           st) == _lib.ERR_NULL
