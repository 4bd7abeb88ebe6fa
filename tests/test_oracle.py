"""CPU tests: the oracle against golden vectors and the reference's own known answers.

These pin the oracle (oracle/nsq_oracle.c) before it is used as the checker
for the CUDA library.  Reference test citations are relative to the
reference project root (nodestor/...).
"""
import numpy as np
import pytest

from planejaja_b200 import quantize as Q
from planejaja_b200.formats import Q4_0, Q4_K, Q5_K, Q6_K, Q8_0, Q6K_GGML, Q6K_NODESTOR


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


# ---- half_to_f32: crates/nodestor-inference/src/dequant/mod.rs:266-283 ----
def test_half_to_f32_known_answers(oracle):
    assert oracle.half_to_f32(0x0000) == 0.0
    assert oracle.half_to_f32(0x3C00) == 1.0
    assert oracle.half_to_f32(0xC000) == -2.0


def test_half_to_f32_exhaustive_matches_ieee(oracle):
    h = np.arange(1 << 16, dtype=np.uint16)
    ours = np.array([oracle.half_to_f32(int(v)) for v in h], np.float32)
    ref = h.view(np.float16).astype(np.float32)
    nan = np.isnan(ref)
    assert np.array_equal(np.isnan(ours), nan)
    assert np.array_equal(bits(ours)[~nan], bits(ref)[~nan])


def test_shader_fp16_matches_on_normals_and_diverges_on_subnormals(oracle):
    """The shaders' f16_to_f32 (dequant_q4.comp:27-38) equals IEEE on normal
    numbers but scales subnormals by an extra 2^-10; the library follows the
    Rust conversion (mod.rs:234-260) everywhere."""
    for h in (0x3C00, 0xC000, 0x0400, 0x7BFF, 0x1234, 0x9A5F):
        assert oracle.half_to_f32_shader(h) == oracle.half_to_f32(h)
    sub = 0x0200  # 2^-15
    assert oracle.half_to_f32(sub) == 2.0 ** -15
    assert oracle.half_to_f32_shader(sub) == 2.0 ** -25


# ---- Q4_K: q4_k.rs:166-234 ----
def test_q4k_reference_known_answers(oracle, golden):
    out = oracle.dequant(golden["kat_q4k_zero_raw"], Q4_K)
    assert out.shape == (256,) and np.all(out == 0.0)
    out = oracle.dequant(golden["kat_q4k_uniform_raw"], Q4_K)
    assert np.all(out[:128] == 28.0) and np.all(np.isfinite(out))
    out = oracle.dequant(golden["kat_q4k_range_raw"], Q4_K)
    assert np.all(np.isfinite(out))
    two = np.concatenate([golden["kat_q4k_uniform_raw"]] * 2)
    assert oracle.dequant(two, Q4_K).shape == (512,)


def test_get_scale_min_k4_reference(oracle, golden):
    d, m = oracle.get_scale_min_k4(0, golden["kat_q4k_scales"])
    assert (d, m) == (0x15 & 0x3F, 0x01 & 0x3F)


def test_q4k_avx2_equals_scalar(oracle, golden):
    """simd_x86.rs:235-256: AVX2 path equals the scalar path."""
    raw = golden["Q4_K_raw"]
    assert np.array_equal(bits(oracle.dequant_q4_k_avx2(raw)), bits(oracle.dequant(raw, Q4_K)))


# ---- Q8_0: q8_0.rs:36-61 ----
def test_q8_reference_known_answers(oracle, golden):
    out = oracle.dequant(golden["kat_q8_raw"], Q8_0).reshape(3, 32)
    assert np.all(out[0] == 0.0)
    assert np.all(out[1] == 5.0)
    assert out[2, 0] == -1.0


# ---- every format against the golden vectors ----
@pytest.mark.parametrize("name,tid,layout", [
    ("Q4_0", Q4_0, 0), ("Q8_0", Q8_0, 0), ("Q4_K", Q4_K, 0), ("Q5_K", Q5_K, Q6K_GGML),
    ("Q5_K_NODESTOR", Q5_K, Q6K_NODESTOR), ("Q6_K", Q6_K, Q6K_GGML), ("Q6_K_NODESTOR", Q6_K, Q6K_NODESTOR)])
def test_oracle_bit_exact_vs_golden(oracle, golden, name, tid, layout):
    raw, ref = golden[f"{name}_raw"], golden[f"{name}_f32"]
    out = oracle.dequant(raw, tid, layout)
    assert np.array_equal(bits(out), bits(ref))


def test_q5k_reference_known_answers(oracle, golden):
    """q5_k.rs unit tests: zero weights; nibble 15 + high bit = 31 with
    dmin = 0 gives only non-negative weights (scale 1 on sub-blocks 0..3)."""
    out = oracle.dequant(golden["kat_q5k_zero_raw"], Q5_K, Q6K_NODESTOR)
    assert out.size == 256 and np.all(np.isfinite(out)) and np.all(np.abs(out) < 1e-4)
    out = oracle.dequant(golden["kat_q5k_high_raw"], Q5_K, Q6K_NODESTOR)
    assert np.all(out >= 0) and np.all(out[:128] == 31.0)


def test_q5k_layouts_differ(oracle, golden):
    raw = golden["Q5_K_raw"]
    assert not np.array_equal(oracle.dequant(raw, Q5_K, Q6K_GGML), oracle.dequant(raw, Q5_K, Q6K_NODESTOR))


def test_q6k_layouts_differ(oracle, golden):
    raw = golden["Q6_K_raw"]
    assert not np.array_equal(oracle.dequant(raw, Q6_K, Q6K_GGML), oracle.dequant(raw, Q6_K, Q6K_NODESTOR))


# ---- cpu_matmul_f32: crates/nodestor-vulkan/src/pipeline.rs:1323-1350 ----
def test_matmul_identity_and_known_values(oracle):
    a = np.array([1, 2, 3, 4], np.float32)
    assert np.array_equal(oracle.matmul_f32(a, np.array([1, 0, 0, 1], np.float32), 2, 2, 2).reshape(-1), a)
    c = oracle.matmul_f32(a, np.array([5, 6, 7, 8], np.float32), 2, 2, 2)
    assert c.tolist() == [[19.0, 22.0], [43.0, 50.0]]


def test_fase4_02_shape_no_nan(oracle):
    """mega_test.rs:389-431: 1x896x896 with sin/cos inputs gives no NaN."""
    i = np.arange(896 * 896, dtype=np.float32)
    a = np.sin(0.001 * np.arange(896, dtype=np.float32))
    b = np.cos(0.001 * i).astype(np.float32)
    c = oracle.matmul_f32(a, b, 1, 896, 896)
    assert not np.isnan(c).any()


@pytest.mark.parametrize("tid,layout", [(Q4_0, 0), (Q8_0, 0), (Q4_K, 0), (Q6_K, 0), (Q6_K, 1)])
def test_quant_matmul_is_composition(oracle, tid, layout):
    """orc_quant_matmul == cpu_matmul_f32(x, transpose(dequant(W))) bit for bit."""
    n, k, m = 24, 512, 3
    w = Q.synthetic_weights(n, k, tid, seed=5, q6k_layout=layout)
    x = Q.synthetic_activations(m, k, seed=6)
    y = oracle.quant_matmul(w, tid, x, n, k, layout)
    wt = oracle.dequant(w, tid, layout).reshape(n, k).T.copy()
    ref = oracle.matmul_f32(x, wt, m, k, n)
    assert np.array_equal(bits(y), bits(ref))
    y_mt = oracle.quant_matmul(w, tid, x, n, k, layout, threads=4)
    assert np.array_equal(bits(y_mt), bits(y))


def test_quantizers_round_trip_small_error(oracle):
    rng = np.random.default_rng(1)
    w = (rng.standard_normal((8, 512)) * 0.02).astype(np.float32)
    for tid, layout, tol in [(Q8_0, 0, 2e-3), (Q4_0, 0, 2e-2), (Q4_K, 0, 2e-2), (Q6_K, 0, 5e-3), (Q6_K, 1, 5e-3)]:
        out = oracle.dequant(Q.quantize(w, tid, layout), tid, layout).reshape(w.shape)
        assert np.abs(out - w).max() < tol, (tid, layout)


def test_synthetic_scales_are_normal_fp16():
    """Synthetic quantizers keep every fp16 scale in the normal range."""
    w = Q.synthetic_weights(64, 1024, Q4_K, seed=3).reshape(-1, 144)
    d = w[:, 0:2].copy().view(np.float16).astype(np.float32)
    dm = w[:, 2:4].copy().view(np.float16).astype(np.float32)
    assert (d >= 2.0 ** -14).all() and (dm >= 2.0 ** -14).all()
