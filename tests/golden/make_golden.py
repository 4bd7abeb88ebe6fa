"""Generate the golden dequant vectors under tests/golden/.

Run from the repository root:  python tests/golden/make_golden.py

Sources of truth (nothing here uses the oracle, so the fixtures check it):
  * gguf-py 0.19.0 (`gguf.quants.dequantize`), ggml's published block
    formats, for Q4_0, Q8_0, Q4_K, Q5_K and Q6_K (GGML layout);
  * an independent numpy restatement of the reference shader
    nodestor/crates/nodestor-vulkan/shaders/dequant_q6k.comp:50-99 for the
    NODESTOR Q6_K layout (the reference has no test for it);
  * an independent numpy restatement of the reference's Q5_K
    (nodestor/crates/nodestor-inference/src/dequant/q5_k.rs:33-88) for its
    NODESTOR high-bit mapping;
  * the reference's own unit-test blocks (known answers), re-expressed:
    q4_k.rs:166-222, q8_0.rs:36-61, q5_k.rs:101-160.

Blocks: seeded N(0, 0.02) weights quantized by planejaja_b200.quantize, plus
"fuzz" blocks of random bytes whose fp16 scale fields are overwritten with
random normal-range values (so every bit pattern of the quant fields appears).
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from planejaja_b200 import quantize as Q  # noqa: E402
from planejaja_b200.formats import FORMATS, Q4_0, Q4_K, Q5_K, Q6_K, Q8_0, Q6K_GGML, Q6K_NODESTOR  # noqa: E402


def _rand_normal_f16(rng, n):
    """Random fp16 bit patterns with exponent in the normal range, both signs."""
    e = rng.integers(5, 20, n)       # 2^-10 .. 2^4
    m = rng.integers(0, 1024, n)
    s = rng.integers(0, 2, n)
    return ((s << 15) | (e << 10) | m).astype(np.uint16)


def _fuzz_blocks(rng, type_id, nblocks):
    f = FORMATS[type_id]
    raw = rng.integers(0, 256, (nblocks, f.block_bytes), dtype=np.uint8)
    if type_id in (Q4_0, Q8_0):
        raw[:, 0:2] = _rand_normal_f16(rng, nblocks).view(np.uint8).reshape(-1, 2)
    elif type_id in (Q4_K, Q5_K):
        raw[:, 0:2] = _rand_normal_f16(rng, nblocks).view(np.uint8).reshape(-1, 2)
        raw[:, 2:4] = _rand_normal_f16(rng, nblocks).view(np.uint8).reshape(-1, 2)
    elif type_id == Q6_K:
        raw[:, 208:210] = _rand_normal_f16(rng, nblocks).view(np.uint8).reshape(-1, 2)
    return raw.reshape(-1)


def shader_q6k_numpy(raw: np.ndarray) -> np.ndarray:
    """dequant_q6k.comp:50-99, vectorised (independent of the C oracle)."""
    b = raw.reshape(-1, 210)
    i = np.arange(256)
    qlb = b[:, i >> 1].astype(np.uint32)
    lo = np.where((i & 1) == 0, qlb & 0xF, (qlb >> 4) & 0xF)
    hi = (b[:, 128 + (i >> 2)].astype(np.uint32) >> ((i & 3) * 2)) & 3
    q = (lo | (hi << 4)).astype(np.int32) - 32
    scale = (b[:, 192 + (i >> 4)].astype(np.int32) - 128).astype(np.float32) / np.float32(64.0)
    d = b[:, 208:210].copy().view(np.float16).astype(np.float32)  # [nb, 1]
    return ((d * scale) * q.astype(np.float32)).astype(np.float32).reshape(-1)


def q5k_nodestor_numpy(raw: np.ndarray) -> np.ndarray:
    """q5_k.rs:33-88 (NODESTOR high bits), vectorised (independent of the C oracle)."""
    b = raw.reshape(-1, 176)
    nb = b.shape[0]
    d = b[:, 0:2].copy().view(np.float16).astype(np.float32)       # [nb, 1]
    dmin = b[:, 2:4].copy().view(np.float16).astype(np.float32)
    s = b[:, 4:16].astype(np.uint32)
    sc = np.empty((nb, 8), np.float32)
    mn = np.empty((nb, 8), np.float32)
    for j in range(8):  # get_scale_min_k4 (q5_k.rs:93-101)
        if j < 4:
            sc[:, j], mn[:, j] = s[:, j] & 63, s[:, j + 4] & 63
        else:
            sc[:, j] = (s[:, j + 4] & 15) | ((s[:, j - 4] >> 6) << 4)
            mn[:, j] = (s[:, j + 4] >> 4) | ((s[:, j] >> 6) << 4)
    qh, qs = b[:, 16:48].astype(np.uint32), b[:, 48:176].astype(np.uint32)
    out = np.empty((nb, 256), np.float32)
    l = np.arange(32)
    for c in range(4):
        for h in range(2):
            j = 2 * c + h
            nib = (qs[:, 32 * c + l] >> (4 * h)) & 15
            hb = (qh[:, 8 * c + 4 * h + l // 8] >> (l % 8)) & 1
            q = (nib | (hb << 4)).astype(np.float32)
            d1 = d * sc[:, j:j + 1]
            m1 = dmin * mn[:, j:j + 1]
            out[:, 64 * c + 32 * h + l] = (d1 * q).astype(np.float32) - m1
    return out.reshape(-1)


def gguf_dequant(raw: np.ndarray, type_id: int) -> np.ndarray:
    from gguf import GGMLQuantizationType as T
    from gguf import quants
    gt = {Q4_0: T.Q4_0, Q8_0: T.Q8_0, Q4_K: T.Q4_K, Q5_K: T.Q5_K, Q6_K: T.Q6_K}[type_id]
    f = FORMATS[type_id]
    return quants.dequantize(raw.reshape(-1, f.block_bytes), gt).reshape(-1).astype(np.float32)


def main():
    import gguf
    rng = np.random.default_rng(20240601)
    out = {"gguf_version": np.array(getattr(gguf, "__version__", "0.19.0"))}
    for tid in (Q4_0, Q8_0, Q4_K, Q6_K):
        f = FORMATS[tid]
        w = rng.standard_normal((4, 512)).astype(np.float32) * np.float32(0.02)
        raw = np.concatenate([Q.quantize(w, tid), _fuzz_blocks(rng, tid, 24 if f.block_weights == 256 else 96)])
        out[f"{f.name}_raw"] = raw
        out[f"{f.name}_f32"] = gguf_dequant(raw, tid)
    # NODESTOR Q6_K layout: shader restatement only
    w = rng.standard_normal((4, 512)).astype(np.float32) * np.float32(0.02)
    raw = np.concatenate([Q.quantize(w, Q6_K, Q6K_NODESTOR), _fuzz_blocks(rng, Q6_K, 24)])
    out["Q6_K_NODESTOR_raw"] = raw
    out["Q6_K_NODESTOR_f32"] = shader_q6k_numpy(raw)

    # Reference unit-test blocks (known answers).
    def q4k_block(d16, dmin16, scale, qn):  # q4_k.rs:138-163
        blk = np.zeros(144, np.uint8)
        blk[0], blk[1] = d16 & 0xFF, d16 >> 8
        blk[2], blk[3] = dmin16 & 0xFF, dmin16 >> 8
        blk[4:8] = scale & 0x3F
        blk[8:12] = 0
        blk[16:144] = (qn & 0xF) | ((qn & 0xF) << 4)
        return blk
    out["kat_q4k_zero_raw"] = q4k_block(0x3C00, 0x0000, 1, 0)          # q4_k.rs:166-175 -> all 0
    out["kat_q4k_uniform_raw"] = q4k_block(0x3C00, 0x0000, 4, 7)       # q4_k.rs:178-197 -> [:128] = 28
    out["kat_q4k_range_raw"] = q4k_block(0x3C00, 0x3C00, 15, 15)       # q4_k.rs:225-234 -> finite
    out["kat_q4k_scales"] = np.array([0x15, 0x20, 0x3F, 0x0A, 0x01, 0x02, 0x08, 0x10, 0, 0, 0, 0], np.uint8)
    q8 = np.zeros((3, 34), np.uint8)                                    # q8_0.rs:36-61
    q8[:, 0], q8[:, 1] = 0x00, 0x3C
    q8[1, 2:] = 5
    q8[2, 2] = 0xFF
    out["kat_q8_raw"] = q8.reshape(-1)
    # Q5_K (added later; its own generator so the entries above keep their values)
    rng5 = np.random.default_rng(20241201)
    w = rng5.standard_normal((4, 512)).astype(np.float32) * np.float32(0.02)
    raw = np.concatenate([Q.quantize(w, Q5_K, Q6K_GGML), _fuzz_blocks(rng5, Q5_K, 24)])
    out["Q5_K_raw"] = raw
    out["Q5_K_f32"] = gguf_dequant(raw, Q5_K)
    w = rng5.standard_normal((4, 512)).astype(np.float32) * np.float32(0.02)
    raw = np.concatenate([Q.quantize(w, Q5_K, Q6K_NODESTOR), _fuzz_blocks(rng5, Q5_K, 24)])
    out["Q5_K_NODESTOR_raw"] = raw
    out["Q5_K_NODESTOR_f32"] = q5k_nodestor_numpy(raw)

    def q5k_block(d16, dmin16, scale, qn, high):  # q5_k.rs:101-123
        blk = np.zeros(176, np.uint8)
        blk[0], blk[1] = d16 & 0xFF, d16 >> 8
        blk[2], blk[3] = dmin16 & 0xFF, dmin16 >> 8
        blk[4:8] = scale & 0x3F
        blk[16:48] = 0xFF if high else 0
        blk[48:176] = (qn & 0xF) | ((qn & 0xF) << 4)
        return blk
    out["kat_q5k_zero_raw"] = q5k_block(0x3C00, 0x0000, 1, 0, 0)     # q5_k.rs test_q5k_zero_weights -> ~0
    out["kat_q5k_high_raw"] = q5k_block(0x3C00, 0x0000, 1, 15, 1)    # q5_k.rs test_q5k_higher_range -> >= 0
    np.savez_compressed(os.path.join(HERE, "dequant_golden.npz"), **out)
    print("wrote", os.path.join(HERE, "dequant_golden.npz"), sorted(out))


if __name__ == "__main__":
    main()
