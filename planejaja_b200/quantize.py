"""Seeded synthetic GGUF weights: fp32 -> Q4_0 / Q8_0 / Q4_K / Q6_K block bytes.

These quantizers make the benchmark and test inputs (the weight matrices the
reference's configs describe as "N(0, 0.02) quantized to ...").  They are
simple absmax/min-max rounders written for this library, not ggml's
iterative searches; the dequant path only needs well-formed blocks whose fp16
scales stay in the normal range.  Every routine is vectorised over blocks.

Block byte layouts (little-endian, ggml's):
  Q8_0  34 B / 32 w : d f16 | qs int8[32]                      y = d*q
  Q4_0  18 B / 32 w : d f16 | qs u8[16] (lo nibble = w[i], hi = w[i+16])
                                                               y = (q-8)*d
  Q4_K 144 B / 256 w: d f16 | dmin f16 | scales u8[12] | qs u8[128]
  Q5_K 176 B / 256 w: d f16 | dmin f16 | scales u8[12] | qh u8[32] | qs u8[128]
                      8 sub-blocks of 32, 6-bit scale/min each  y = d*sc*q - dmin*m
  Q6_K 210 B / 256 w: ql u8[128] | qh u8[64] | scales [16] | d f16
                      GGML layout: int8 scales per 16 weights   y = d*sc*(q-32)
                      NODESTOR layout: scale byte b -> (b-128)/64, linear
                      element order (dequant_q6k.comp:50-99)
"""
from __future__ import annotations

import numpy as np

from .formats import Q4_0, Q4_K, Q5_K, Q6_K, Q8_0, Q6K_GGML, Q6K_NODESTOR, fmt

F16_MIN_NORMAL = np.float32(2.0 ** -14)


def _f16_normal(v: np.ndarray) -> np.ndarray:
    """Round positive scales to fp16, never below the smallest normal."""
    v = np.maximum(np.asarray(v, np.float32), F16_MIN_NORMAL)
    return v.astype(np.float16)


def _f16_bytes(h: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(h.astype(np.float16)).view(np.uint8).reshape(*h.shape, 2)


def quantize_q8_0(w: np.ndarray) -> np.ndarray:
    b = w.reshape(-1, 32).astype(np.float32)
    amax = np.abs(b).max(axis=1)
    d = _f16_normal(amax / 127.0)
    df = d.astype(np.float32)[:, None]
    q = np.clip(np.rint(b / df), -127, 127).astype(np.int8)
    out = np.empty((b.shape[0], 34), np.uint8)
    out[:, 0:2] = _f16_bytes(d)
    out[:, 2:] = q.view(np.uint8)
    return out.reshape(-1)


def quantize_q4_0(w: np.ndarray) -> np.ndarray:
    b = w.reshape(-1, 32).astype(np.float32)
    idx = np.abs(b).argmax(axis=1)
    smax = b[np.arange(b.shape[0]), idx]  # signed value of largest magnitude
    dv = smax / -8.0
    sign = np.where(dv < 0, -1.0, 1.0).astype(np.float32)
    d = (sign * _f16_normal(np.abs(dv)).astype(np.float32)).astype(np.float16)
    df = d.astype(np.float32)[:, None]
    q = np.clip(np.rint(b / df) + 8, 0, 15).astype(np.uint8)
    out = np.empty((b.shape[0], 18), np.uint8)
    out[:, 0:2] = _f16_bytes(d)
    out[:, 2:] = q[:, :16] | (q[:, 16:] << 4)
    return out.reshape(-1)


def _pack_q4k_scales(sc: np.ndarray, mn: np.ndarray) -> np.ndarray:
    """Inverse of get_scale_min_k4 (q4_k.rs:120-131) for 8 (scale, min) pairs."""
    s = np.zeros((sc.shape[0], 12), np.uint8)
    s[:, 0:4] = (sc[:, 0:4] & 63) | ((sc[:, 4:8] >> 4) << 6)
    s[:, 4:8] = (mn[:, 0:4] & 63) | ((mn[:, 4:8] >> 4) << 6)
    s[:, 8:12] = (sc[:, 4:8] & 15) | ((mn[:, 4:8] & 15) << 4)
    return s


def quantize_q4_k(w: np.ndarray) -> np.ndarray:
    b = w.reshape(-1, 8, 32).astype(np.float32)
    nb = b.shape[0]
    lo = np.minimum(b.min(axis=2), 0.0)
    hi = b.max(axis=2)
    scale = (hi - lo) / 15.0           # per sub-block step
    mins = -lo                         # per sub-block offset (>= 0)
    d = _f16_normal(scale.max(axis=1) / 63.0)
    dmin = _f16_normal(mins.max(axis=1) / 63.0)
    df, dmf = d.astype(np.float32)[:, None], dmin.astype(np.float32)[:, None]
    sc = np.clip(np.rint(scale / df), 0, 63).astype(np.uint8)
    mn = np.clip(np.rint(mins / dmf), 0, 63).astype(np.uint8)
    d1 = (df * sc.astype(np.float32))[:, :, None]
    m1 = (dmf * mn.astype(np.float32))[:, :, None]
    safe = np.where(d1 > 0, d1, 1.0)
    q = np.where(d1 > 0, np.clip(np.rint((b + m1) / safe), 0, 15), 0).astype(np.uint8)
    # qs[32c + l]: lo nibble = sub-block 2c element l, hi nibble = sub-block 2c+1
    qs = q[:, 0::2, :] | (q[:, 1::2, :] << 4)  # [nb, 4, 32]
    out = np.empty((nb, 144), np.uint8)
    out[:, 0:2] = _f16_bytes(d)
    out[:, 2:4] = _f16_bytes(dmin)
    out[:, 4:16] = _pack_q4k_scales(sc, mn)
    out[:, 16:] = qs.reshape(nb, 128)
    return out.reshape(-1)


def quantize_q5_k(w: np.ndarray, layout: int = Q6K_GGML) -> np.ndarray:
    """Q5_K: Q4_K's scheme with 5-bit values; qs holds the low nibbles as in
    Q4_K, qh the high bits in the ggml or the NodeStor mapping."""
    b = w.reshape(-1, 8, 32).astype(np.float32)
    nb = b.shape[0]
    lo = np.minimum(b.min(axis=2), 0.0)
    hi = b.max(axis=2)
    scale = (hi - lo) / 31.0
    mins = -lo
    d = _f16_normal(scale.max(axis=1) / 63.0)
    dmin = _f16_normal(mins.max(axis=1) / 63.0)
    df, dmf = d.astype(np.float32)[:, None], dmin.astype(np.float32)[:, None]
    sc = np.clip(np.rint(scale / df), 0, 63).astype(np.uint8)
    mn = np.clip(np.rint(mins / dmf), 0, 63).astype(np.uint8)
    d1 = (df * sc.astype(np.float32))[:, :, None]
    m1 = (dmf * mn.astype(np.float32))[:, :, None]
    safe = np.where(d1 > 0, d1, 1.0)
    q = np.where(d1 > 0, np.clip(np.rint((b + m1) / safe), 0, 31), 0).astype(np.uint8)  # [nb, 8 sub-blocks, 32]
    low = q & 15
    qs = low[:, 0::2, :] | (low[:, 1::2, :] << 4)  # [nb, 4 chunks, 32]
    hbit = (q >> 4) & 1                               # sub-block 2c+h, element l
    if layout == Q6K_GGML:
        # qh[l] bit (2c + h) = high bit of sub-block 2c + h, element l
        qh = np.zeros((nb, 32), np.uint8)
        for s8 in range(8):
            qh |= (hbit[:, s8, :] << s8).astype(np.uint8)
    elif layout == Q6K_NODESTOR:
        # qh[8c + 4h + l/8] bit (l % 8)
        bits = hbit.reshape(nb, 4, 2, 4, 8)  # [nb, c, h, l/8, l%8]
        qh = np.zeros((nb, 4, 2, 4), np.uint8)
        for t in range(8):
            qh |= (bits[..., t] << t).astype(np.uint8)
        qh = qh.reshape(nb, 32)
    else:
        raise ValueError(f"unknown Q5_K layout {layout}")
    out = np.empty((nb, 176), np.uint8)
    out[:, 0:2] = _f16_bytes(d)
    out[:, 2:4] = _f16_bytes(dmin)
    out[:, 4:16] = _pack_q4k_scales(sc, mn)
    out[:, 16:48] = qh
    out[:, 48:] = qs.reshape(nb, 128)
    return out.reshape(-1)


def _q6k_pack_ggml(q: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """q: [nb, 256] uint8 in 0..63 in element order -> (ql[nb,128], qh[nb,64])."""
    nb = q.shape[0]
    q4 = q.reshape(nb, 2, 4, 32)  # [half n, j, l]
    ql = np.empty((nb, 2, 2, 32), np.uint8)  # [n, j&1, l]
    ql[:, :, 0, :] = (q4[:, :, 0, :] & 15) | ((q4[:, :, 2, :] & 15) << 4)
    ql[:, :, 1, :] = (q4[:, :, 1, :] & 15) | ((q4[:, :, 3, :] & 15) << 4)
    hb = q4 >> 4  # [n, j, l] 2-bit
    qh = hb[:, :, 0, :] | (hb[:, :, 1, :] << 2) | (hb[:, :, 2, :] << 4) | (hb[:, :, 3, :] << 6)
    return ql.reshape(nb, 128), qh.reshape(nb, 64).astype(np.uint8)


def _q6k_pack_nodestor(q: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    nb = q.shape[0]
    ql = (q[:, 0::2] & 15) | ((q[:, 1::2] & 15) << 4)
    h = (q >> 4).reshape(nb, 64, 4)
    qh = h[:, :, 0] | (h[:, :, 1] << 2) | (h[:, :, 2] << 4) | (h[:, :, 3] << 6)
    return ql.astype(np.uint8), qh.astype(np.uint8)


def quantize_q6_k(w: np.ndarray, layout: int = Q6K_GGML) -> np.ndarray:
    b = w.reshape(-1, 16, 16).astype(np.float32)  # [nb, sub-block, 16]
    nb = b.shape[0]
    amax = np.abs(b).max(axis=2)                    # [nb, 16]
    out = np.empty((nb, 210), np.uint8)
    if layout == Q6K_GGML:
        step = amax / 31.0                          # value of one q unit
        d = _f16_normal(step.max(axis=1) / 127.0)
        df = d.astype(np.float32)[:, None]
        sc = np.clip(np.rint(step / df), 0, 127).astype(np.int8)
        eff = (df * sc.astype(np.float32))[:, :, None]
        scale_bytes = sc.view(np.uint8)
    elif layout == Q6K_NODESTOR:
        smax = 127.0 / 64.0
        d = _f16_normal(amax.max(axis=1) / (31.0 * smax))
        df = d.astype(np.float32)[:, None]
        s = amax / (31.0 * df)
        sb = np.clip(np.rint(64.0 * s) + 128, 128, 255).astype(np.uint8)
        eff = (df * ((sb.astype(np.float32) - 128.0) / 64.0))[:, :, None]
        scale_bytes = sb
    else:
        raise ValueError(f"unknown Q6_K layout {layout}")
    safe = np.where(eff > 0, eff, 1.0)
    q = np.where(eff > 0, np.clip(np.rint(b / safe), -32, 31), 0).astype(np.int16) + 32
    q = q.reshape(nb, 256).astype(np.uint8)
    ql, qh = (_q6k_pack_ggml if layout == Q6K_GGML else _q6k_pack_nodestor)(q)
    out[:, 0:128] = ql
    out[:, 128:192] = qh
    out[:, 192:208] = scale_bytes
    out[:, 208:210] = _f16_bytes(d)
    return out.reshape(-1)


def quantize(w: np.ndarray, type_id: int, q6k_layout: int = Q6K_GGML) -> np.ndarray:
    """Quantize an [N, K] float matrix row by row; returns N*row_bytes uint8."""
    f = fmt(type_id)
    if w.ndim != 2 or w.shape[1] % f.block_weights:
        raise ValueError(f"{f.name}: need [N, K] with K % {f.block_weights} == 0, got {w.shape}")
    if type_id == Q8_0:
        return quantize_q8_0(w)
    if type_id == Q4_0:
        return quantize_q4_0(w)
    if type_id == Q4_K:
        return quantize_q4_k(w)
    if type_id == Q5_K:
        return quantize_q5_k(w, q6k_layout)
    if type_id == Q6_K:
        return quantize_q6_k(w, q6k_layout)
    raise ValueError(f"unsupported type {type_id}")


def synthetic_weights(n: int, k: int, type_id: int, seed: int, std: float = 0.02,
                      q6k_layout: int = Q6K_GGML, chunk_rows: int = 2048, rows=None) -> np.ndarray:
    """W[n, k] ~ N(0, std) drawn with `seed`, quantized; returns GGUF bytes.

    Rows are drawn and quantized in chunks so that large matrices (e.g. the
    28672 x 8192 FFN weights) never hold the full fp32 matrix at once.
    rows=(r0, r1) returns only the bytes of rows [r0, r1) (a row shard): the
    rows before r0 are drawn but not quantized, so the bytes equal that slice
    of the whole matrix's bytes.
    """
    f = fmt(type_id)
    r_lo, r_hi = (0, n) if rows is None else (int(rows[0]), int(rows[1]))
    if not 0 <= r_lo <= r_hi <= n:
        raise ValueError(f"rows {rows} outside [0, {n}]")
    rng = np.random.default_rng(seed)
    rb = f.row_bytes(k)
    out = np.empty((r_hi - r_lo) * rb, np.uint8)
    for c0 in range(0, r_hi, chunk_rows):
        c1 = min(n, c0 + chunk_rows)
        w = rng.standard_normal((c1 - c0, k), dtype=np.float32) * np.float32(std)
        a, b = max(c0, r_lo), min(c1, r_hi)
        if a < b:
            out[(a - r_lo) * rb:(b - r_lo) * rb] = quantize(w[a - c0:b - c0], type_id, q6k_layout)
    return out


def synthetic_activations(m: int, k: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return rng.standard_normal((m, k), dtype=np.float32)
