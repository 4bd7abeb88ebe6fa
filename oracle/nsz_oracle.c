/*
 * nsz_oracle.c -- CPU restatement of NodeStor's NSZ / TCA-TBE tile codec and
 * of the ZipGEMM operator's arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  The checker for libnsq's NSZ decoder and fused
 * decompress-GEMV: only tests/, __graft_entry__.smoke() and bench.py's CPU
 * legs may load it.  The product never calls it.
 *
 * Reference routines restated (paths relative to nodestor/):
 *
 *   orc_nsz_encode_tile   crates/nodestor-formats/src/nsz_encoder.rs:79-275
 *                         (encode_tile_fp32 / _fp16 / _bf16), find_modal_exp
 *                         :300-314, pack_bits :317-326, serialization
 *                         NszTile::to_bytes nsz_format.rs:291-307
 *   orc_nsz_decode_tile   crates/nodestor-formats/src/nsz_decoder.rs:19-196
 *                         (decode_tile_fp32 / _fp16 / _bf16), sections laid
 *                         out as NszTile::to_bytes writes them
 *   orc_nsz_matmul        the ZipGEMM operator (VulkanEngine::zipgemm,
 *                         crates/nodestor-vulkan/src/lib.rs:124-151) as its
 *                         decoder + cpu_matmul_f32 composition:
 *                         y = cpu_matmul_f32(x, transpose(decode(W))), W the
 *                         tensor's [N x K] weights in stream order.
 *
 * Tile bytes (nsz_format.rs:13-44, NszTile::to_bytes): header 8 bytes
 * [modal u8][num_residuals u16][dtype u8][num_near u16][reserved 2], match
 * bitmap ceil(n/8), near bitmap ceil(n/8), near deltas ceil(num_near/8),
 * residual exponents num_residuals, mantissas n * {3, 2, 1} bytes (FP32,
 * FP16, BF16), signs ceil(n/8), zero padding to a multiple of 64.  n is 512
 * except in a tensor's last tile; it is not stored in the tile.
 *
 * Two behaviours of the reference kept as they are:
 *  - the encoder's near test `exp == modal.wrapping_add(1) || (modal > 0 &&
 *    exp == modal - 1)` (nsz_encoder.rs:111, :180, :243) takes exponent 0 as "near" when
 *    the modal exponent is 255, with delta 0, which the decoder reads back as
 *    254: such a tile is not lossless (orc_nsz_encode_tile with
 *    reference_quirks = 1 reproduces it; 0 stores that exponent as a residual);
 *  - the decoder's out-of-range reads return 0 (nsz_decoder.rs:41-45, 54-58).
 *
 * Pin: the reference's own converter output micro_modelo_ignition.nsz
 * (nsz_convert.rs) decodes and re-encodes to the same bytes
 * (tests/golden/make_nsz_golden.py, tests/test_nsz.py).
 */
#include <stdint.h>
#include <string.h>
#include <stdlib.h>

#define NSZ_TILE 512
#define NSZ_ALIGN 64
#define NSZ_FP32 0
#define NSZ_FP16 1
#define NSZ_BF16 2

static int mant_bytes(int dtype) { return dtype == NSZ_FP32 ? 3 : dtype == NSZ_FP16 ? 2 : 1; }

int64_t orc_nsz_max_tile_bytes(int dtype) {
  int64_t raw = 8 + 64 + 64 + 64 + 512 + (int64_t)NSZ_TILE * mant_bytes(dtype) + 64;
  return (raw + NSZ_ALIGN - 1) / NSZ_ALIGN * NSZ_ALIGN;
}

/* Serialized size of a tile of n weights from its header fields. */
static int64_t tile_bytes(int n, int num_near, int num_res, int dtype) {
  int64_t bm = (n + 7) / 8;
  int64_t raw = 8 + 2 * bm + (num_near + 7) / 8 + num_res + (int64_t)n * mant_bytes(dtype) + bm;
  return (raw + NSZ_ALIGN - 1) / NSZ_ALIGN * NSZ_ALIGN;
}

/* Exponent, mantissa and sign of element i (nsz_encoder.rs:86-93, 161-165, 224-228). */
static void split(const void *w, int64_t i, int dtype, uint8_t *e, uint32_t *m, uint8_t *s) {
  if (dtype == NSZ_FP32) {
    uint32_t b = ((const uint32_t *)w)[i];
    *s = (b >> 31) & 1;
    *e = (b >> 23) & 0xFF;
    *m = b & 0x7FFFFF;
  } else {
    uint16_t b = ((const uint16_t *)w)[i];
    *s = (b >> 15) & 1;
    if (dtype == NSZ_FP16) {
      *e = (b >> 10) & 0x1F;
      *m = b & 0x3FF;
    } else {
      *e = (b >> 7) & 0xFF;
      *m = b & 0x7F;
    }
  }
}

/* Encodes n (1..512) weights (FP32 bits as uint32, FP16/BF16 as uint16) into
 * out; returns the serialized size (padded to 64). */
int64_t orc_nsz_encode_tile(const void *w, int n, int dtype, int reference_quirks, uint8_t *out) {
  uint8_t e[NSZ_TILE], s[NSZ_TILE];
  uint32_t m[NSZ_TILE];
  uint32_t hist[256] = {0};
  for (int i = 0; i < n; ++i) {
    split(w, i, dtype, &e[i], &m[i], &s[i]);
    hist[e[i]]++;
  }
  /* find_modal_exp: first exponent with the highest count */
  uint8_t modal = 0;
  uint32_t best = 0;
  for (int i = 0; i < 256; ++i)
    if (hist[i] > best) {
      best = hist[i];
      modal = (uint8_t)i;
    }
  const int bm = (n + 7) / 8;
  uint8_t match[64] = {0}, nearb[64] = {0}, deltas[64] = {0}, resid[NSZ_TILE];
  int num_near = 0, num_res = 0;
  for (int i = 0; i < n; ++i) {
    const uint8_t up = (uint8_t)(modal + 1);
    const int is_near = reference_quirks ? (e[i] == up || (modal > 0 && e[i] == modal - 1))
                                         : ((modal < 255 && e[i] == up) || (modal > 0 && e[i] == modal - 1));
    if (e[i] == modal) {
      match[i / 8] |= (uint8_t)(1u << (i % 8));
    } else if (is_near) {
      nearb[i / 8] |= (uint8_t)(1u << (i % 8));
      if (e[i] > modal) deltas[num_near / 8] |= (uint8_t)(1u << (num_near % 8));
      num_near++;
    } else {
      resid[num_res++] = e[i];
    }
  }
  uint8_t *p = out;
  p[0] = modal;
  p[1] = (uint8_t)(num_res & 0xFF);
  p[2] = (uint8_t)(num_res >> 8);
  p[3] = (uint8_t)dtype;
  p[4] = (uint8_t)(num_near & 0xFF);
  p[5] = (uint8_t)(num_near >> 8);
  p[6] = p[7] = 0;
  p += 8;
  memcpy(p, match, bm);
  p += bm;
  memcpy(p, nearb, bm);
  p += bm;
  memcpy(p, deltas, (num_near + 7) / 8);
  p += (num_near + 7) / 8;
  memcpy(p, resid, num_res);
  p += num_res;
  for (int i = 0; i < n; ++i) {
    if (dtype == NSZ_FP32) {
      *p++ = m[i] & 0xFF;
      *p++ = (m[i] >> 8) & 0xFF;
      *p++ = (m[i] >> 16) & 0x7F;
    } else if (dtype == NSZ_FP16) {
      *p++ = m[i] & 0xFF;
      *p++ = (m[i] >> 8) & 0x03;
    } else {
      *p++ = (uint8_t)m[i];
    }
  }
  uint8_t sg[64] = {0};
  for (int i = 0; i < n; ++i)
    if (s[i]) sg[i / 8] |= (uint8_t)(1u << (i % 8));
  memcpy(p, sg, bm);
  p += bm;
  int64_t len = p - out, padded = tile_bytes(n, num_near, num_res, dtype);
  memset(p, 0, padded - len);
  return padded;
}

/* Decodes one tile of n weights; the section lengths come from its header
 * (as NszTile's vectors would hold them).  Returns the serialized size. */
int64_t orc_nsz_decode_tile(const uint8_t *t, int n, int dtype, void *out) {
  const uint8_t modal = t[0];
  const int num_res = t[1] | (t[2] << 8), num_near = t[4] | (t[5] << 8);
  const int bm = (n + 7) / 8, nd = (num_near + 7) / 8, mb = mant_bytes(dtype);
  const uint8_t *match = t + 8, *nearb = match + bm, *deltas = nearb + bm, *resid = deltas + nd;
  const uint8_t *mant = resid + num_res, *sg = mant + (int64_t)n * mb;
  int near_idx = 0, res_idx = 0;
  for (int i = 0; i < n; ++i) {
    const int is_match = (match[i / 8] >> (i % 8)) & 1, is_near = (nearb[i / 8] >> (i % 8)) & 1;
    uint8_t ex;
    if (is_match) {
      ex = modal;
    } else if (is_near) {
      const int db = near_idx / 8;
      const int d = db < nd ? (deltas[db] >> (near_idx % 8)) & 1 : 0;
      near_idx++;
      ex = d ? (uint8_t)(modal + 1) : (uint8_t)(modal - 1);
    } else {
      ex = res_idx < num_res ? resid[res_idx] : 0;
      res_idx++;
    }
    const uint32_t sign = (sg[i / 8] >> (i % 8)) & 1;
    if (dtype == NSZ_FP32) {
      const uint32_t mm = mant[3 * i] | ((uint32_t)mant[3 * i + 1] << 8) | ((uint32_t)(mant[3 * i + 2] & 0x7F) << 16);
      ((uint32_t *)out)[i] = (sign << 31) | ((uint32_t)ex << 23) | mm;
    } else if (dtype == NSZ_FP16) {
      const uint32_t mm = mant[2 * i] | ((uint32_t)(mant[2 * i + 1] & 0x03) << 8);
      ((uint16_t *)out)[i] = (uint16_t)((sign << 15) | ((uint32_t)(ex & 0x1F) << 10) | mm);
    } else {
      ((uint16_t *)out)[i] = (uint16_t)((sign << 15) | ((uint32_t)ex << 7) | (mant[i] & 0x7F));
    }
  }
  return tile_bytes(n, num_near, num_res, dtype);
}

/* Whole tensor: count weights in ceil(count/512) tiles.  Returns the bytes
 * written, or -1 if cap is too small. */
int64_t orc_nsz_encode(const void *w, int64_t count, int dtype, int reference_quirks, uint8_t *out, int64_t cap) {
  const int es = dtype == NSZ_FP32 ? 4 : 2;
  int64_t pos = 0;
  for (int64_t t0 = 0; t0 < count; t0 += NSZ_TILE) {
    const int n = (int)(count - t0 < NSZ_TILE ? count - t0 : NSZ_TILE);
    if (pos + orc_nsz_max_tile_bytes(dtype) > cap) return -1;
    pos += orc_nsz_encode_tile((const uint8_t *)w + t0 * es, n, dtype, reference_quirks, out + pos);
  }
  return pos;
}

/* Walks the tile headers: writes the byte offset of each tile (num_tiles + 1
 * entries) and checks that the stream holds exactly count weights.  Returns 0
 * or -1 (stream too short / too long). */
int orc_nsz_offsets(const uint8_t *data, int64_t nbytes, int64_t count, int dtype, int64_t *offsets) {
  int64_t pos = 0, t = 0;
  for (int64_t t0 = 0; t0 < count; t0 += NSZ_TILE, ++t) {
    const int n = (int)(count - t0 < NSZ_TILE ? count - t0 : NSZ_TILE);
    if (pos + 8 > nbytes) return -1;
    const uint8_t *h = data + pos;
    offsets[t] = pos;
    pos += tile_bytes(n, h[4] | (h[5] << 8), h[1] | (h[2] << 8), dtype);
    if (pos > nbytes) return -1;
  }
  offsets[t] = pos;
  return pos == nbytes ? 0 : -1;
}

int orc_nsz_decode(const uint8_t *data, int64_t nbytes, int64_t count, int dtype, void *out) {
  const int es = dtype == NSZ_FP32 ? 4 : 2;
  int64_t pos = 0;
  for (int64_t t0 = 0; t0 < count; t0 += NSZ_TILE) {
    const int n = (int)(count - t0 < NSZ_TILE ? count - t0 : NSZ_TILE);
    if (pos + 8 > nbytes) return -1;
    const uint8_t *h = data + pos;
    if (pos + tile_bytes(n, h[4] | (h[5] << 8), h[1] | (h[2] << 8), dtype) > nbytes) return -1;
    pos += orc_nsz_decode_tile(data + pos, n, dtype, (uint8_t *)out + t0 * es);
  }
  return pos == nbytes ? 0 : -1;
}

void orc_matmul_f32(const float *a, const float *b, float *c, int64_t m, int64_t k, int64_t n);

/* y[M x N] = cpu_matmul_f32(x[M x K], transpose(decode(W[N x K]))), FP32 weights. */
int orc_nsz_matmul(const uint8_t *data, int64_t nbytes, const float *x, float *y, int64_t m, int64_t n, int64_t k) {
  float *w = (float *)malloc(sizeof(float) * (size_t)(n * k > 0 ? n * k : 1));
  float *wt = (float *)malloc(sizeof(float) * (size_t)(n * k > 0 ? n * k : 1));
  if (!w || !wt) {
    free(w);
    free(wt);
    return -2;
  }
  int rc = orc_nsz_decode(data, nbytes, n * k, NSZ_FP32, w);
  if (!rc) {
    for (int64_t r = 0; r < n; ++r)
      for (int64_t c = 0; c < k; ++c) wt[c * n + r] = w[r * k + c];
    orc_matmul_f32(x, wt, y, m, k, n);
  }
  free(w);
  free(wt);
  return rc;
}
