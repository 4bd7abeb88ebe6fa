"""Generate the golden dequant vectors under tests/golden/.

Run from the repository root:  python tests/golden/make_golden.py

Sources of truth (nothing here uses the oracle, so the fixtures check it):
  * gguf-py 0.19.0 (`gguf.quants.dequantize`), ggml's published block
    formats, for Q4_0, Q8_0, Q4_K and Q6_K (GGML layout);
  * an independent numpy restatement of the reference shader
    nodestor/crates/nodestor-vulkan/shaders/dequant_q6k.comp:50-99 for the
    NODESTOR Q6_K layout (the reference has no test for it);
  * the reference's own unit-test blocks (known answers), re-expressed:
    q4_k.rs:166-222, q8_0.rs:36-61.

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
from planejaja_b200.formats import FORMATS, Q4_0, Q4_K, Q6_K, Q8_0, Q6K_GGML, Q6K_NODESTOR  # noqa: E402


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
    elif type_id == Q4_K:
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


def gguf_dequant(raw: np.ndarray, type_id: int) -> np.ndarray:
    from gguf import GGMLQuantizationType as T
    from gguf import quants
    gt = {Q4_0: T.Q4_0, Q8_0: T.Q8_0, Q4_K: T.Q4_K, Q6_K: T.Q6_K}[type_id]
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
    np.savez_compressed(os.path.join(HERE, "dequant_golden.npz"), **out)
    print("wrote", os.path.join(HERE, "dequant_golden.npz"), sorted(out))


if __name__ == "__main__":
    main()
