// gemv_rows.cuh -- decode GEMV, "one lane per weight row" layout (M = 1..4).
//
// The kernel template and its launcher.  Host-side planning is in
// gemv_rows.cu; the instantiations are spread over gemv_rows_<format>.cu so
// that they compile in parallel.
//
//   y[m, n] = sum_k x[m, k] * W[n, k]
//
// A CTA owns R consecutive rows of W (R = 32, 16, 8 or 4).  Lane l of each
// consumer warp works on row l % R; the 32 / R lane groups of a warp and the
// 4 consumer warps split K.  K is walked in chunks: the producer warp copies,
// per chunk, every row's byte run with one 1-D bulk copy (TMA) into a shared
// row of padded pitch (so 16-byte reads of 32 rows hit distinct banks) and
// the prepared activation records of the chunk after them.  Consumers then
// work on "pieces" of 256 weights: one Q4_K / Q6_K super-block or 8 Q4_0 /
// Q8_0 blocks, all scale fields at compile-time positions.  Activation
// records are read as warp-wide broadcasts.  Each lane accumulates its row in
// registers; partials of the lane groups and warps are reduced once per CTA.
//
// Integer dot products (dp4a) of the 4/6/8-bit weights against the two
// activation bytes are exact; each 16 or 32 weights are scaled once in fp32.
// High nibbles are masked in place (value * 16) and the 1/16 is folded into
// the fp32 scale.  Error analysis as for the prepared activations (see
// gemv.cu): about 3e-5 relative.
//
// Programmatic dependent launch: the weight copies of the first stages are
// issued before griddepcontrol.wait, so they overlap the tail of the kernel
// that produces the activation records.
//
// Self-prepared activations: every CTA needs all K/32 activation records.
// With thread-block clusters of C CTAs, each CTA quantises 1/C of the groups
// and stores the records into the shared memory of every CTA of its cluster
// (distributed shared memory), so the L2 serves each activation line to 1/C
// as many CTAs; one cluster barrier publishes the records.
#pragma once

#include "nsq_common.cuh"

namespace nsq {

constexpr int kRowsConsumers = 4;
constexpr int kRowsThreads = 32 * (1 + kRowsConsumers);
// Self-prepared activations sit in shared memory as runs of 8 records (80 B
// each) per 256-weight piece, every run padded by 16 bytes.  The lane groups
// of a warp read the records of consecutive pieces at once; unpadded (640 B
// apart) those reads fall in the same banks and the 16-byte loads replay 2-4
// times, padded they fall in disjoint banks.
constexpr int kXPieceSelf = 8 * 80 + 16;


__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Activation group (broadcast read from shared memory).
struct XG {
  uint4 hi0, hi1, lo0, lo1;
  float sx;
  int t0, t1;
};
__device__ __forceinline__ void lds_xg(const uint8_t* p, XG& x) {
  const uint4* q = reinterpret_cast<const uint4*>(p);
  x.hi0 = q[0]; x.hi1 = q[1]; x.lo0 = q[2]; x.lo1 = q[3];
  const uint4 e = q[4];
  x.sx = __uint_as_float(e.x);
  x.t0 = (int)e.y;
  x.t1 = (int)e.z;
}

// Integer dot of 8 weight words (32 weights, unsigned or signed bytes)
// against a group's two activation bytes; returns the two 16-weight halves
// S_h = 256 * (q . hi) + (q . lo).
template <bool SIGNED>
__device__ __forceinline__ void dot8(const uint32_t (&q)[8], const XG& x, int& s0, int& s1) {
  const uint32_t hi[8] = {x.hi0.x, x.hi0.y, x.hi0.z, x.hi0.w, x.hi1.x, x.hi1.y, x.hi1.z, x.hi1.w};
  const uint32_t lo[8] = {x.lo0.x, x.lo0.y, x.lo0.z, x.lo0.w, x.lo1.x, x.lo1.y, x.lo1.z, x.lo1.w};
  int h0 = 0, l0 = 0, h1 = 0, l1 = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if constexpr (SIGNED) {
      h0 = dp4a_ss(q[i], hi[i], h0);
      l0 = dp4a_su(q[i], lo[i], l0);
      h1 = dp4a_ss(q[i + 4], hi[i + 4], h1);
      l1 = dp4a_su(q[i + 4], lo[i + 4], l1);
    } else {
      h0 = dp4a_us(q[i], hi[i], h0);
      l0 = dp4a_uu(q[i], lo[i], l0);
      h1 = dp4a_us(q[i + 4], hi[i + 4], h1);
      l1 = dp4a_uu(q[i + 4], lo[i + 4], l1);
    }
  }
  s0 = (h0 << 8) + l0;
  s1 = (h1 << 8) + l1;
}

// ---------------------------------------------------------------------------
// Pieces.  `pc` points at the piece of this lane's row in shared memory,
// `xp` at the activation records of the piece's 8 groups for token 0 (token
// m at xp + m * xstride).
template <int TYPE, int LAYOUT, int M>
struct Piece;

// Q4_K super-block [d][dmin][scales 12][qs 128] (q4_k.rs:75-131).  Chunk
// pair c: qs[32c .. 32c+32) low nibbles = group 2c, high nibbles = 2c+1.
template <int LAYOUT, int M>
struct Piece<NSQ_TYPE_Q4_K, LAYOUT, M> {
  __device__ static void run(const uint8_t* pc, const uint8_t* xp, int xstride, float (&acc)[M]) {
    const uint4 hdr = *reinterpret_cast<const uint4*>(pc);
    const float d = h2f((uint16_t)(hdr.x & 0xFFFF)), dmin = h2f((uint16_t)(hdr.x >> 16));
    const uint32_t S0 = hdr.y, S1 = hdr.z, S2 = hdr.w;
    // the 8 6-bit scales and mins of get_scale_min_k4 (q4_k.rs:120-131),
    // four per word: bytes j of sclo/mnlo are sub-blocks 0..3, of schi/mnhi 4..7
    const uint32_t sclo = S0 & 0x3F3F3F3Fu, mnlo = S1 & 0x3F3F3F3Fu;
    const uint32_t schi = (S2 & 0x0F0F0F0Fu) | ((S0 >> 2) & 0x30303030u);
    const uint32_t mnhi = ((S2 >> 4) & 0x0F0F0F0Fu) | ((S1 >> 2) & 0x30303030u);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const uint32_t scw = c < 2 ? sclo : schi, mnw = c < 2 ? mnlo : mnhi;
      const int sh0 = 16 * (c & 1), sh1 = sh0 + 8;
      const float a0 = d * (float)((scw >> sh0) & 0xFF), b0 = dmin * (float)((mnw >> sh0) & 0xFF);
      const float a1 = d * (float)((scw >> sh1) & 0xFF) * 0.0625f, b1 = dmin * (float)((mnw >> sh1) & 0xFF);
      const uint4 qa = *reinterpret_cast<const uint4*>(pc + 16 + 32 * c);
      const uint4 qb = *reinterpret_cast<const uint4*>(pc + 32 + 32 * c);
      const uint32_t qw[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
      uint32_t ql[8], qh[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        ql[i] = qw[i] & 0x0F0F0F0Fu;
        qh[i] = qw[i] & 0xF0F0F0F0u;  // 16 * high nibble
      }
#pragma unroll
      for (int m = 0; m < M; ++m) {
        XG x0, x1;
        lds_xg(xp + m * xstride + (2 * c) * 80, x0);
        lds_xg(xp + m * xstride + (2 * c + 1) * 80, x1);
        int s00, s01, s10, s11;
        dot8<false>(ql, x0, s00, s01);
        dot8<false>(qh, x1, s10, s11);
        float r = x0.sx * fmaf(a0, (float)(s00 + s01), -b0 * (float)(x0.t0 + x0.t1));
        r = fmaf(x1.sx, fmaf(a1, (float)(s10 + s11), -b1 * (float)(x1.t0 + x1.t1)), r);
        acc[m] += r;
      }
    }
  }
};

// Q5_K super-block [d][dmin][scales 12][qh 32][qs 128]: Q4_K's nibbles (at
// byte 48) plus the fifth bit of each weight: ggml: bit j of qh[l];
// NODESTOR (q5_k.rs:57-70): bit l%8 of qh[8(j>>1) + 4(j&1) + l/8].
template <int LAYOUT, int M>
struct Piece<NSQ_TYPE_Q5_K, LAYOUT, M> {
  __device__ static void run(const uint8_t* pc, const uint8_t* xp, int xstride, float (&acc)[M]) {
    const uint4 hdr = *reinterpret_cast<const uint4*>(pc);
    const float d = h2f((uint16_t)(hdr.x & 0xFFFF)), dmin = h2f((uint16_t)(hdr.x >> 16));
    const uint32_t S0 = hdr.y, S1 = hdr.z, S2 = hdr.w;
    const uint32_t sclo = S0 & 0x3F3F3F3Fu, mnlo = S1 & 0x3F3F3F3Fu;
    const uint32_t schi = (S2 & 0x0F0F0F0Fu) | ((S0 >> 2) & 0x30303030u);
    const uint32_t mnhi = ((S2 >> 4) & 0x0F0F0F0Fu) | ((S1 >> 2) & 0x30303030u);
    uint32_t hw[8];
    if constexpr (LAYOUT != NSQ_Q6K_NODESTOR) {
      const uint4 ha = *reinterpret_cast<const uint4*>(pc + 16), hb = *reinterpret_cast<const uint4*>(pc + 32);
      hw[0] = ha.x; hw[1] = ha.y; hw[2] = ha.z; hw[3] = ha.w;
      hw[4] = hb.x; hw[5] = hb.y; hw[6] = hb.z; hw[7] = hb.w;
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const uint32_t scw = c < 2 ? sclo : schi, mnw = c < 2 ? mnlo : mnhi;
      const int sh0 = 16 * (c & 1), sh1 = sh0 + 8;
      const float a0 = d * (float)((scw >> sh0) & 0xFF), b0 = dmin * (float)((mnw >> sh0) & 0xFF);
      const float a1 = d * (float)((scw >> sh1) & 0xFF), b1 = dmin * (float)((mnw >> sh1) & 0xFF);
      const uint4 qa = *reinterpret_cast<const uint4*>(pc + 48 + 32 * c);
      const uint4 qb = *reinterpret_cast<const uint4*>(pc + 64 + 32 * c);
      const uint32_t qw[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
      uint32_t ql[8], qh[8];
      if constexpr (LAYOUT == NSQ_Q6K_NODESTOR) {
        const uint2 h = *reinterpret_cast<const uint2*>(pc + 16 + 8 * c);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          ql[i] = (qw[i] & 0x0F0F0F0Fu) | (spread4(((h.x >> (8 * (i >> 1))) >> (4 * (i & 1))) & 0xF) << 4);
          qh[i] = ((qw[i] >> 4) & 0x0F0F0F0Fu) | (spread4(((h.y >> (8 * (i >> 1))) >> (4 * (i & 1))) & 0xF) << 4);
        }
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          ql[i] = (qw[i] & 0x0F0F0F0Fu) | (((hw[i] >> (2 * c)) & 0x01010101u) << 4);
          qh[i] = ((qw[i] >> 4) & 0x0F0F0F0Fu) | (((hw[i] >> (2 * c + 1)) & 0x01010101u) << 4);
        }
      }
#pragma unroll
      for (int m = 0; m < M; ++m) {
        XG x0, x1;
        lds_xg(xp + m * xstride + (2 * c) * 80, x0);
        lds_xg(xp + m * xstride + (2 * c + 1) * 80, x1);
        int s00, s01, s10, s11;
        dot8<false>(ql, x0, s00, s01);
        dot8<false>(qh, x1, s10, s11);
        float r = x0.sx * fmaf(a0, (float)(s00 + s01), -b0 * (float)(x0.t0 + x0.t1));
        r = fmaf(x1.sx, fmaf(a1, (float)(s10 + s11), -b1 * (float)(x1.t0 + x1.t1)), r);
        acc[m] += r;
      }
    }
  }
};

// Q6_K, ggml layout: half n, group j (0..3), element l: ql[64n + 32(j&1) + l]
// nibble (j>>1), qh[32n + l] bits 2j, int8 scale sc[8n + 2j + l/16].
template <int M>
struct Piece<NSQ_TYPE_Q6_K, NSQ_Q6K_GGML, M> {
  __device__ static void run(const uint8_t* pc, const uint8_t* xp, int xstride, float (&acc)[M]) {
    const float d = h2f(ld_u16(pc + 208));
    uint32_t scw[4];
    ld_words_unaligned<4>(pc + 192, scw);
#pragma unroll
    for (int n = 0; n < 2; ++n) {
      uint32_t ql[16], qh[8];
      ld_words_unaligned<16>(pc + 64 * n, ql);
      ld_words_unaligned<8>(pc + 128 + 32 * n, qh);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint32_t q[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint32_t lw = (j >> 1) ? (ql[8 * (j & 1) + i] >> 4) : ql[8 * (j & 1) + i];
          q[i] = (lw & 0x0F0F0F0Fu) | (((qh[i] >> (2 * j)) & 0x03030303u) << 4);
        }
        const int si = 8 * n + 2 * j;  // scale bytes si, si+1
        const uint32_t sw = scw[si >> 2] >> (8 * (si & 3));
        const float a0 = d * (float)(int8_t)(sw & 0xFF), a1 = d * (float)(int8_t)((sw >> 8) & 0xFF);
#pragma unroll
        for (int m = 0; m < M; ++m) {
          XG x;
          lds_xg(xp + m * xstride + (4 * n + j) * 80, x);
          int s0, s1;
          dot8<false>(q, x, s0, s1);
          acc[m] = fmaf(x.sx, fmaf(a0, (float)(s0 - 32 * x.t0), a1 * (float)(s1 - 32 * x.t1)), acc[m]);
        }
      }
    }
  }
};

// Q6_K, NodeStor layout (dequant_q6k.comp:50-99): element i: ql[i>>1] nibble
// (i&1), qh[i>>2] bits 2(i&3), scale (b[192 + i>>4] - 128) / 64.
template <int M>
struct Piece<NSQ_TYPE_Q6_K, NSQ_Q6K_NODESTOR, M> {
  __device__ static void run(const uint8_t* pc, const uint8_t* xp, int xstride, float (&acc)[M]) {
    const float d = h2f(ld_u16(pc + 208));
    uint32_t scw[4];
    ld_words_unaligned<4>(pc + 192, scw);
#pragma unroll
    for (int g = 0; g < 8; ++g) {
      uint32_t ql[4], qh[2];
      ld_words_unaligned<4>(pc + 16 * g, ql);
      ld_words_unaligned<2>(pc + 128 + 8 * g, qh);
      uint32_t q[8];
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        const uint32_t v = (ql[t >> 1] >> (16 * (t & 1))) & 0xFFFFu;
        const uint32_t tt = __byte_perm(v, 0, 0x1100);
        const uint32_t lo4 = (tt & 0x000F000Fu) | ((tt >> 4) & 0x0F000F00u);
        const uint32_t h = (qh[t >> 2] >> (8 * (t & 3))) & 0xFFu;
        q[t] = lo4 | (((h | (h << 6) | (h << 12) | (h << 18)) & 0x03030303u) << 4);
      }
      const uint32_t sw = scw[g >> 1] >> (16 * (g & 1));
      const float a0 = d * ((float)((int)(sw & 0xFF) - 128) * 0.015625f);
      const float a1 = d * ((float)((int)((sw >> 8) & 0xFF) - 128) * 0.015625f);
#pragma unroll
      for (int m = 0; m < M; ++m) {
        XG x;
        lds_xg(xp + m * xstride + g * 80, x);
        int s0, s1;
        dot8<false>(q, x, s0, s1);
        acc[m] = fmaf(x.sx, fmaf(a0, (float)(s0 - 32 * x.t0), a1 * (float)(s1 - 32 * x.t1)), acc[m]);
      }
    }
  }
};

// Q4_0: 8 blocks [d][qs 16]: low nibbles = weights 0..15, high = 16..31
// (dequant_q4.comp:40-61).
// A piece (144 bytes) starts 16-byte aligned, so it is read as 16-byte words
// in two halves (words 0..19 and 16..35) and every block field sits at a
// compile-time position: even blocks start word-aligned (scale in the low
// half-word, quants shifted by 2 bytes), odd blocks 2 bytes into a word
// (scale in the high half-word, quants word-aligned).
template <int LAYOUT, int M>
struct Piece<NSQ_TYPE_Q4_0, LAYOUT, M> {
  __device__ static void run(const uint8_t* pc, const uint8_t* xp, int xstride, float (&acc)[M]) {
    const uint4* pv = reinterpret_cast<const uint4*>(pc);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint32_t w[20];  // words 16h .. 16h + 19 of the piece
#pragma unroll
      for (int i = 0; i < 5; ++i) {
        const uint4 t = pv[4 * h + i];
        w[4 * i] = t.x; w[4 * i + 1] = t.y; w[4 * i + 2] = t.z; w[4 * i + 3] = t.w;
      }
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const int g = 4 * h + b;
        const int byte0 = 18 * g - 64 * h;  // block start, relative to word 16h
        const int wi = byte0 >> 2;
        float d;
        uint32_t q[8];
        if ((byte0 & 3) == 0) {
          d = h2f((uint16_t)(w[wi] & 0xFFFF));
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint32_t qs = __funnelshift_r(w[wi + i], w[wi + i + 1], 16);  // block bytes 2+4i .. 5+4i
            q[i] = qs & 0x0F0F0F0Fu;
            q[i + 4] = qs & 0xF0F0F0F0u;  // 16 * high nibble
          }
        } else {
          d = h2f((uint16_t)(w[wi] >> 16));
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint32_t qs = w[wi + 1 + i];
            q[i] = qs & 0x0F0F0F0Fu;
            q[i + 4] = qs & 0xF0F0F0F0u;
          }
        }
#pragma unroll
        for (int m = 0; m < M; ++m) {
          XG x;
          lds_xg(xp + m * xstride + g * 80, x);
          int s0, s1;
          dot8<false>(q, x, s0, s1);
          acc[m] = fmaf(x.sx * d, (float)(s0 - 8 * x.t0) + 0.0625f * (float)(s1 - 128 * x.t1), acc[m]);
        }
      }
    }
  }
};

// Q8_0: 8 blocks [d][qs int8 32] (q8_0.rs:14-28).  A piece (272 bytes)
// starts 16-byte aligned; the block pair k (bytes 68k .. 68k+67) is read as
// the 16-byte words 4k .. 4k+4 (bytes 64k .. 64k+79), where it starts at
// word k: block 2k word-aligned (scale in the low half-word, quants shifted
// by 2 bytes), block 2k+1 at word k+8 plus 2 bytes (scale in the high
// half-word, quants word-aligned from word k+9).
template <int LAYOUT, int M>
struct Piece<NSQ_TYPE_Q8_0, LAYOUT, M> {
  __device__ static void run(const uint8_t* pc, const uint8_t* xp, int xstride, float (&acc)[M]) {
    const uint4* pv = reinterpret_cast<const uint4*>(pc);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      uint32_t w[20];
#pragma unroll
      for (int i = 0; i < 5; ++i) {
        const uint4 t = pv[4 * k + i];
        w[4 * i] = t.x; w[4 * i + 1] = t.y; w[4 * i + 2] = t.z; w[4 * i + 3] = t.w;
      }
#pragma unroll
      for (int b = 0; b < 2; ++b) {
        const int g = 2 * k + b;
        float d;
        uint32_t q[8];
        if (b == 0) {
          d = h2f((uint16_t)(w[k] & 0xFFFF));
#pragma unroll
          for (int i = 0; i < 8; ++i) q[i] = __funnelshift_r(w[k + i], w[k + i + 1], 16);
        } else {
          d = h2f((uint16_t)(w[k + 8] >> 16));
#pragma unroll
          for (int i = 0; i < 8; ++i) q[i] = w[k + 9 + i];
        }
#pragma unroll
        for (int m = 0; m < M; ++m) {
          XG x;
          lds_xg(xp + m * xstride + g * 80, x);
          int s0, s1;
          dot8<true>(q, x, s0, s1);
          acc[m] = fmaf(x.sx * d, (float)(s0 + s1), acc[m]);
        }
      }
    }
  }
};

// ---------------------------------------------------------------------------
// ---------------------------------------------------------------------------
// Fused kernel: several segments (weight matrices sharing the activation),
// rows concatenated, walked by persistent CTAs in row blocks x K chunks.
enum : int { kQ4K = 0, kQ6KG = 1, kQ6KN = 2, kQ40 = 3, kQ80 = 4, kQ5KG = 5, kQ5KN = 6 };

struct FSeg {
  const uint8_t* w;
  float* y;
  int64_t N, RB, row0;  // rows, row bytes, first row in the concatenated row space
  int code, piece_bytes, chunk_bytes, pitch;
};

struct FusedParams {
  FSeg seg[NSQ_MAX_SEGMENTS];
  int nseg;
  int64_t T;            // total rows
  const float* x;       // activations (self-prepared mode)
  const XGroup* xg;     // prepared activations (workspace mode)
  int64_t K, GX;        // GX = K / 32
  int R, KS, PPS, npieces, nchunks;
  int xstride;          // bytes per token of per-stage activation records (workspace mode)
  int stage_bytes, nstages, max_pitch;
  int npre;             // stages whose weights are copied before the dependency wait (<= nstages)
  int l2hint;           // 1: weight copies evict_first in the L2; 2: also activation reads evict_last
  int Rblk;             // rows per block walked by the cursor: R, or R / 2 with the SwiGLU epilogue
  const float* res[NSQ_MAX_SEGMENTS];  // residual-add epilogue: y = res + x . W^T (may alias y)
  int C;                // self-prepared mode: CTAs per cluster sharing the activation quantisation
  int64_t nrb;          // row blocks of R rows in the concatenated row space
  // Row-sharded exchange (P > 1): every output row is stored into the
  // exchange buffer of each of the P ranks.  Segment s writes y[M x xnfull]
  // f32 at byte offset kXchgCtlBytes + xoff[s] of every buffer, this rank's
  // rows starting at xrow0[s].  xwait: first wait until every rank's
  // previous exchange has landed here.
  int P, rank, xwait;
  uint8_t* xbuf[NSQ_MAX_RANKS];
  int64_t xrow0[NSQ_MAX_SEGMENTS], xnfull[NSQ_MAX_SEGMENTS], xoff[NSQ_MAX_SEGMENTS];
};

// CODE >= 0: every segment has that format (one decoder compiled in);
// CODE == kMixed: dispatch on the segment's format.
constexpr int kMixed = -1;
template <int M, int CODE>
__device__ __forceinline__ void run_piece(int code, const uint8_t* pc, const uint8_t* xp, int xstride, float (&acc)[M]) {
  if constexpr (CODE == kQ4K) { Piece<NSQ_TYPE_Q4_K, 0, M>::run(pc, xp, xstride, acc); return; }
  if constexpr (CODE == kQ6KG) { Piece<NSQ_TYPE_Q6_K, NSQ_Q6K_GGML, M>::run(pc, xp, xstride, acc); return; }
  if constexpr (CODE == kQ6KN) { Piece<NSQ_TYPE_Q6_K, NSQ_Q6K_NODESTOR, M>::run(pc, xp, xstride, acc); return; }
  if constexpr (CODE == kQ40) { Piece<NSQ_TYPE_Q4_0, 0, M>::run(pc, xp, xstride, acc); return; }
  if constexpr (CODE == kQ80) { Piece<NSQ_TYPE_Q8_0, 0, M>::run(pc, xp, xstride, acc); return; }
  if constexpr (CODE == kQ5KG) { Piece<NSQ_TYPE_Q5_K, NSQ_Q6K_GGML, M>::run(pc, xp, xstride, acc); return; }
  if constexpr (CODE == kQ5KN) { Piece<NSQ_TYPE_Q5_K, NSQ_Q6K_NODESTOR, M>::run(pc, xp, xstride, acc); return; }
  switch (code) {
    case kQ4K: Piece<NSQ_TYPE_Q4_K, 0, M>::run(pc, xp, xstride, acc); break;
    case kQ6KG: Piece<NSQ_TYPE_Q6_K, NSQ_Q6K_GGML, M>::run(pc, xp, xstride, acc); break;
    case kQ6KN: Piece<NSQ_TYPE_Q6_K, NSQ_Q6K_NODESTOR, M>::run(pc, xp, xstride, acc); break;
    case kQ40: Piece<NSQ_TYPE_Q4_0, 0, M>::run(pc, xp, xstride, acc); break;
    case kQ5KG: Piece<NSQ_TYPE_Q5_K, NSQ_Q6K_GGML, M>::run(pc, xp, xstride, acc); break;
    case kQ5KN: Piece<NSQ_TYPE_Q5_K, NSQ_Q6K_NODESTOR, M>::run(pc, xp, xstride, acc); break;
    default: Piece<NSQ_TYPE_Q8_0, 0, M>::run(pc, xp, xstride, acc); break;
  }
}

// Loads one group of 32 activations (8 x 16 bytes); with `hint`, at L2
// priority evict_last.
__device__ __forceinline__ void load_group(const float* __restrict__ xs, float4 (&f)[8], bool hint, uint64_t pol) {
  const float4* q = reinterpret_cast<const float4*>(xs);
  if (hint) {
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = ldg_f4_hint(q + i, pol);
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = __ldg(q + i);
  }
}

// Quantize one group of 32 activations into an 80-byte record (same math as
// prepare_x_kernel in gemv.cu, one thread per group), returned as 5 words of
// 16 bytes.
__device__ __forceinline__ void quantize_group(const float4 (&f)[8], uint4 (&o)[5]) {
  float v[32];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    v[4 * i] = f[i].x; v[4 * i + 1] = f[i].y; v[4 * i + 2] = f[i].z; v[4 * i + 3] = f[i].w;
  }
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
  const float inv = amax > 0.f ? 32767.0f / amax : 0.f;
  uint32_t hw[8], lw[8];
  int s0 = 0, s1 = 0;
  if (inv < 3.0e38f) {
    // |v| <= amax, so X = rn(v * inv) lies in [-32767, 32767] and needs no
    // clamp.  Adding 1.5 * 2^23 rounds the product into the low mantissa
    // bits: the sum's bits are 0x4B400000 + X, whose two low bytes are X's
    // (a NaN product counts as 0, as cvt.rni gives).  One byte permute per
    // value packs the high and low bytes; the sums are sums of the bits.
    uint32_t b[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      float y = __fmul_rn(v[i], inv);
      y = (y == y) ? y : 0.f;
      b[i] = __float_as_uint(__fadd_rn(y, 12582912.0f));
    }
    uint32_t t0 = 0, t1 = 0;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      const uint32_t p01 = __byte_perm(b[4 * w], b[4 * w + 1], 0x5140);  // X0.b0 X1.b0 X0.b1 X1.b1
      const uint32_t p23 = __byte_perm(b[4 * w + 2], b[4 * w + 3], 0x5140);
      lw[w] = __byte_perm(p01, p23, 0x5410);
      hw[w] = __byte_perm(p01, p23, 0x7632);
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      t0 += b[i];
      t1 += b[16 + i];
    }
    s0 = (int)(t0 - 16u * 0x4B400000u);
    s1 = (int)(t1 - 16u * 0x4B400000u);
  } else {
    // 32767 / amax overflowed (amax below ~1e-34): convert and clamp
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      uint32_t h = 0, l = 0;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        int X = __float2int_rn(v[4 * w + b] * inv);
        X = max(-32767, min(32767, X));
        if (w < 4) s0 += X; else s1 += X;
        h |= ((uint32_t)(X >> 8) & 0xFF) << (8 * b);
        l |= ((uint32_t)X & 0xFF) << (8 * b);
      }
      hw[w] = h;
      lw[w] = l;
    }
  }
  o[0] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
  o[1] = make_uint4(hw[4], hw[5], hw[6], hw[7]);
  o[2] = make_uint4(lw[0], lw[1], lw[2], lw[3]);
  o[3] = make_uint4(lw[4], lw[5], lw[6], lw[7]);
  o[4] = make_uint4(__float_as_uint(amax / 32767.0f), (uint32_t)s0, (uint32_t)s1, 0u);
}

// Thread-block cluster helpers (distributed shared memory).
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_arrive_relaxed() { asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_arrive_release() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait_acquire() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
__device__ __forceinline__ uint32_t cluster_map(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ void st_cluster_v4(uint32_t addr, const uint4& v) {
  asm volatile("st.shared::cluster.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// Walk of one CTA's work: items (segment, row block, chunk) in order.
struct ItemCursor {
  int seg;
  int64_t row0, rows;  // segment-local first row and row count of the block
  int c;               // chunk
  __device__ void first(const FusedParams& p, int64_t r_begin, int64_t r_end) {
    seg = 0;
    while (seg < p.nseg - 1 && r_begin >= p.seg[seg].row0 + p.seg[seg].N) ++seg;
    row0 = r_begin - p.seg[seg].row0;
    const int64_t seg_end = min(r_end, p.seg[seg].row0 + p.seg[seg].N) - p.seg[seg].row0;
    rows = min((int64_t)p.Rblk, seg_end - row0);
    c = 0;
  }
  // advance; returns false when the CTA's rows are done
  __device__ bool next(const FusedParams& p, int64_t r_end) {
    if (++c < p.nchunks) return true;
    c = 0;
    row0 += rows;
    const int64_t seg_end_g = min(r_end, p.seg[seg].row0 + p.seg[seg].N);
    if (p.seg[seg].row0 + row0 >= seg_end_g) {
      if (seg_end_g >= r_end || seg + 1 >= p.nseg) return false;
      ++seg;
      row0 = 0;
    }
    const int64_t seg_end = min(r_end, p.seg[seg].row0 + p.seg[seg].N) - p.seg[seg].row0;
    rows = min((int64_t)p.Rblk, seg_end - row0);
    return rows > 0;
  }
};

// EPI: 0 = y, 1 = y = residual + x . W^T, 2 = SwiGLU pair: segments 0 (gate)
// and 1 (up) have the same rows; a block holds Rblk = R/2 rows of each (gate
// in shared rows [0, R/2), up in [R/2, R)) and the output is
// h = silu(gate) * up into segment 0's y.
template <int M, bool XSELF, int CODE, int EPI>
__global__ void __launch_bounds__(kRowsThreads, 4) gemv_fused_kernel(const __grid_constant__ FusedParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* stages = smem;
  uint8_t* xsm = smem + (size_t)p.stage_bytes * p.nstages;  // self-prepared activations [M][pieces] padded record runs
  const size_t xsm_bytes = XSELF ? (size_t)M * p.npieces * kXPieceSelf : 0;
  float* red = reinterpret_cast<float*>(xsm + xsm_bytes);  // [2][4][32][M]
  uint64_t* full = reinterpret_cast<uint64_t*>(red + 2 * kRowsConsumers * 32 * M);
  uint64_t* empty = full + p.nstages;
  __shared__ int s_fail;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // rows per CTA: whole row blocks (nrb > 0; the counts differ by at most
  // one) or an even split of the rows
  const int64_t r_begin = p.nrb > 0 ? min(p.T, p.Rblk * (p.nrb * blockIdx.x / gridDim.x)) : p.T * blockIdx.x / gridDim.x;
  const int64_t r_end = p.nrb > 0 ? min(p.T, p.Rblk * (p.nrb * (blockIdx.x + 1) / gridDim.x))
                                  : p.T * (blockIdx.x + 1) / gridDim.x;
  const bool clustered = XSELF && p.C > 1;

  if (tid == 0) {
    s_fail = 0;
    for (int s = 0; s < p.nstages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kRowsConsumers);
    }
    fence_mbar_init();
  }
  __syncthreads();
  // cluster phase 1: every CTA of the cluster has started before any writes
  // into its shared memory
  if (clustered) cluster_arrive_relaxed();

  if (warp == 0) {
    // producer warp: lane r issues row r's bulk copy, lane 0 the barrier
    // bookkeeping and the activation copies
    if (r_begin < r_end) {
      const uint64_t wpol = l2_policy_evict_first(), xpol = l2_policy_evict_last();
      // weight row runs are read once: evict them first (l2hint)
      auto copy_w = [&](void* dst, const void* src, int bytes, uint64_t* bar) {
        if (p.l2hint) bulk_g2s_hint(dst, src, (uint32_t)bytes, bar, wpol);
        else bulk_g2s(dst, src, (uint32_t)bytes, bar);
      };
      auto issue = [&](const ItemCursor& it, int s, bool with_w, bool with_x) {
        const FSeg& sg = p.seg[it.seg];
        const int64_t off = (int64_t)it.c * sg.chunk_bytes;
        const int rbytes = (int)min((int64_t)sg.chunk_bytes, sg.RB - off);
        const int ng = (int)(min((int64_t)p.PPS, (int64_t)p.npieces - (int64_t)it.c * p.PPS)) * 8;
        uint8_t* slot = stages + (size_t)s * p.stage_bytes;
        if (with_w) {
          if (lane == 0)
            mbar_arrive_expect_tx(&full[s],
                                  (uint32_t)((EPI == 2 ? 2 : 1) * it.rows * rbytes + (XSELF ? 0 : M * ng * 80)));
          __syncwarp();
          if constexpr (EPI == 2) {
            // the block's gate rows and the same rows of up
            const FSeg& su = p.seg[1];
            for (int r = lane; r < 2 * (int)it.rows; r += 32) {
              const bool up = r >= (int)it.rows;
              const int rr = up ? r - (int)it.rows : r;
              copy_w(slot + (up ? rr + p.Rblk : rr) * sg.pitch, (up ? su.w : sg.w) + (it.row0 + rr) * sg.RB + off,
                     rbytes, &full[s]);
            }
          } else {
            for (int r = lane; r < (int)it.rows; r += 32)
              copy_w(slot + r * sg.pitch, sg.w + (it.row0 + r) * sg.RB + off, rbytes, &full[s]);
          }
        }
        if (!XSELF && with_x && lane == 0) {
          uint8_t* xs = slot + p.R * p.max_pitch;
          for (int m = 0; m < M; ++m) {
            const void* src = p.xg + m * p.GX + (int64_t)it.c * p.PPS * 8;
            if (p.l2hint >= 2) bulk_g2s_hint(xs + m * p.xstride, src, (uint32_t)(ng * 80), &full[s], xpol);
            else bulk_g2s(xs + m * p.xstride, src, (uint32_t)(ng * 80), &full[s]);
          }
        }
      };
      // weights of the first stages do not depend on the previous kernel
      ItemCursor it;
      it.first(p, r_begin, r_end);
      ItemCursor pre[8];
      int npre = 0;
      bool more = true;
      while (more && npre < p.npre) {
        pre[npre] = it;
        issue(it, npre, true, false);
        ++npre;
        more = it.next(p, r_end);
      }
      __syncwarp();
      grid_dep_wait();
      grid_dep_launch();
      if (clustered) {
        cluster_wait_acquire();
        cluster_arrive_relaxed();
        cluster_wait_acquire();
      }
      for (int t = 0; t < npre; ++t) issue(pre[t], t, false, true);
      // stage t = npre, npre + 1, ...: slot t % nstages, waiting for the
      // consumers' release of its previous use (parity (t / nstages - 1) & 1),
      // counted incrementally
      int s = npre == p.nstages ? 0 : npre;
      uint32_t epar = npre == p.nstages ? 0u : 1u;
      while (more) {
        if (!mbar_wait_bounded(&empty[s], epar)) {
          s_fail = 1;
          break;
        }
        fence_proxy_async_smem();
        issue(it, s, true, true);
        more = it.next(p, r_end);
        if (++s == p.nstages) {
          s = 0;
          epar ^= 1u;
        }
      }
    } else {
      grid_dep_wait();
      grid_dep_launch();
      if (clustered) {
        cluster_wait_acquire();
        cluster_arrive_relaxed();
        cluster_wait_acquire();
      }
    }
  } else {
    const int cw = warp - 1, ct = tid - 32;
    grid_dep_wait();
    grid_dep_launch();
    if (p.P > 1 && p.xwait) {
      // every rank's previous exchange has landed here before the
      // activations (in a transformer, that exchange's output) are read
      if (ct == 0) {
        const uint32_t* ctl = reinterpret_cast<const uint32_t*>(p.xbuf[p.rank]);
        const uint32_t want = ld_acquire_sys(ctl + kXchgSeq);
        for (int r = 0; r < p.P; ++r)
          if (r != p.rank && !wait_geq_bounded(ctl + r, want)) {
            s_fail = 1;
            break;
          }
      }
      asm volatile("bar.sync 1, %0;" ::"r"(kRowsConsumers * 32) : "memory");
    }
    if constexpr (XSELF) {
      // the cluster's CTAs quantise disjoint ranges of the groups and write
      // every record into each CTA of the cluster (the L2 serves each
      // activation line to 1/C as many CTAs)
      const int64_t ng = (int64_t)M * p.GX;
      const int q = clustered ? (int)cluster_rank() : 0, C = clustered ? p.C : 1;
      if (clustered) cluster_wait_acquire();
      const bool xh = p.l2hint >= 2;
      const uint64_t xpol = l2_policy_evict_last();
      const int64_t g_end = ng * (q + 1) / C;
      auto put = [&](int64_t gi, const float4 (&f)[8]) {
        const int64_t m = gi / p.GX, g = gi - m * p.GX;
        uint8_t* rec = xsm + m * ((int64_t)p.npieces * kXPieceSelf) + (g >> 3) * kXPieceSelf + (g & 7) * 80;
        uint4 o[5];
        quantize_group(f, o);
        if (clustered) {
          for (int qq = 0; qq < C; ++qq) {
            const uint32_t ra = cluster_map(rec, (uint32_t)qq);
#pragma unroll
            for (int i = 0; i < 5; ++i) st_cluster_v4(ra + 16 * i, o[i]);
          }
        } else {
          uint4* d = reinterpret_cast<uint4*>(rec);
#pragma unroll
          for (int i = 0; i < 5; ++i) d[i] = o[i];
        }
      };
      auto src = [&](int64_t gi) {
        const int64_t m = gi / p.GX, g = gi - m * p.GX;
        return p.x + m * p.K + 32 * g;
      };
      constexpr int kStride = kRowsConsumers * 32;
      for (int64_t gi = ng * q / C + ct; gi < g_end; gi += kStride) {
        float4 fa[8];
        load_group(src(gi), fa, xh, xpol);
        put(gi, fa);
      }
      if (clustered) {
        // cluster phase 2: all records of the cluster have landed
        cluster_arrive_release();
        cluster_wait_acquire();
      } else {
        asm volatile("bar.sync 1, %0;" ::"r"(kRowsConsumers * 32) : "memory");
      }
    }
    const int r = lane % p.R, ks = lane / p.R;
    const int lanes_per_piece = kRowsConsumers * p.KS;
    const int xstride = XSELF ? p.npieces * kXPieceSelf : p.xstride;
    const int xpiece = XSELF ? kXPieceSelf : 8 * 80;  // bytes between the record runs of consecutive pieces
    float acc[M];
#pragma unroll
    for (int m = 0; m < M; ++m) acc[m] = 0.f;
    bool ok = true;
    int par = 0;
    if (r_begin < r_end) {
      ItemCursor it;
      it.first(p, r_begin, r_end);
      bool more = true;
      // stage t: slot t % nstages, parity (t / nstages) & 1, counted incrementally
      int s = 0;
      uint32_t fpar = 0u;
      for (; more; s = (s + 1 == p.nstages) ? 0 : s + 1, fpar ^= (s == 0) ? 1u : 0u) {
        const FSeg& sg = p.seg[it.seg];
        if (ok) ok = mbar_wait_bounded(&full[s], fpar);
        if (ok) {
          const int np = (int)min((int64_t)p.PPS, (int64_t)p.npieces - (int64_t)it.c * p.PPS);
          const uint8_t* slot = stages + (size_t)s * p.stage_bytes;
          const uint8_t* xbase = XSELF ? xsm + (int64_t)it.c * p.PPS * kXPieceSelf : slot + p.R * p.max_pitch;
          if ((EPI == 2 ? (r & (p.Rblk - 1)) : r) < it.rows) {
            for (int j = cw * p.KS + ks; j < np; j += lanes_per_piece)
              run_piece<M, CODE>(sg.code, slot + r * sg.pitch + j * sg.piece_bytes, xbase + j * xpiece, xstride, acc);
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[s]);
        } else {
          s_fail = 1;
        }
        if (it.c == p.nchunks - 1) {
          float* rd = red + (size_t)par * kRowsConsumers * 32 * M;
#pragma unroll
          for (int m = 0; m < M; ++m) {
            float v = acc[m];
            for (int o = p.R; o < 32; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            rd[(cw * 32 + lane) * M + m] = v;
            acc[m] = 0.f;
          }
          asm volatile("bar.sync 1, %0;" ::"r"(kRowsConsumers * 32) : "memory");
          if (ct < it.rows * M && s_fail == 0) {
            const int rr = ct / M, m = ct - rr * M;
            float v = 0.f;
#pragma unroll
            for (int w = 0; w < kRowsConsumers; ++w) v += rd[(w * 32 + rr) * M + m];
            if constexpr (EPI == 1) v += p.res[it.seg][(int64_t)m * sg.N + it.row0 + rr];
            if constexpr (EPI == 2) {
              float u = 0.f;
#pragma unroll
              for (int w = 0; w < kRowsConsumers; ++w) u += rd[(w * 32 + rr + p.Rblk) * M + m];
              // silu.comp:18-20 then mul.comp: (g * sigmoid(g)) * up
              const float sig = 1.0f / (1.0f + expf(-v));
              v = v * sig * u;
            }
            if (p.P > 1) {
              const int64_t idx = (int64_t)m * p.xnfull[it.seg] + p.xrow0[it.seg] + it.row0 + rr;
              for (int pr = 0; pr < p.P; ++pr)
                reinterpret_cast<float*>(p.xbuf[pr] + kXchgCtlBytes + p.xoff[it.seg])[idx] = v;
            } else {
              sg.y[(int64_t)m * sg.N + it.row0 + rr] = v;
            }
          }
          par ^= 1;
        }
        more = it.next(p, r_end);
      }
    }
  }
  __syncthreads();
  if (p.P > 1 && tid == 0) {
    // Publish: the fence orders this CTA's peer stores before its count;
    // the grid's last CTA advances the exchange count and writes it to this
    // rank's flag word in every buffer with release stores at system scope.
    fence_acq_rel_gpu();
    uint32_t* ctl = reinterpret_cast<uint32_t*>(p.xbuf[p.rank]);
    if (atomicAdd(ctl + kXchgDone, 1u) == gridDim.x - 1) {
      fence_acq_rel_gpu();  // acquire side: every CTA's stores precede the flags
      ctl[kXchgDone] = 0;
      const uint32_t seq = ctl[kXchgSeq] + 1;
      ctl[kXchgSeq] = seq;
      for (int pr = 0; pr < p.P; ++pr) st_release_sys(reinterpret_cast<uint32_t*>(p.xbuf[pr]) + p.rank, seq);
    }
  }
}

// ---------------------------------------------------------------------------
// Launcher
constexpr int kNoRoom = -2;  // launch_fused: the clusters do not all fit at once

template <int M, bool XSELF, int CODE, int EPI>
static cudaError_t launch_fused(const FusedParams& p, int blocks, size_t smem, cudaStream_t st, int* max_clusters) {
  auto kern = gemv_fused_kernel<M, XSELF, CODE, EPI>;
  static size_t configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || smem > configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    // every instantiation asks for the same (largest) shared-memory carveout,
    // so the CTAs of consecutive launches with different shared-memory sizes
    // can share an SM (programmatic dependent launch) without the SM first
    // draining to switch its L1 / shared split
    if (tune(kTuneRowsCarve, 1)) {
      e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
      if (e != cudaSuccess) return e;
    }
    if (dev >= 0 && dev < 64) configured[dev] = smem;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)blocks);
  cfg.blockDim = dim3(kRowsThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = (unsigned)(XSELF ? p.C : 1);
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  const int C = XSELF ? p.C : 1;
  cfg.numAttrs = C > 1 ? 2 : 1;
  if (C > 1) {
    // all clusters must be resident at once: a second wave would double the
    // time.  The answer is cached per device, cluster size and smem size.
    struct Fit { int dev, S; size_t smem; int n; };
    static Fit cache[32];
    static int ncache = 0;
    int n = -1;
    for (int i = 0; i < ncache; ++i)
      if (cache[i].dev == dev && cache[i].S == C && cache[i].smem == smem) n = cache[i].n;
    if (n < 0) {
      cudaLaunchConfig_t q = cfg;
      q.numAttrs = 1;
      q.attrs = attr + 1;
      if (cudaOccupancyMaxActiveClusters(&n, kern, &q) != cudaSuccess || n < 1) {
        cudaGetLastError();
        n = 0;
      }
      if (ncache < 32) cache[ncache++] = Fit{dev, C, smem, n};
    }
    if (n < 1) return cudaErrorInvalidConfiguration;
    if (blocks > n * C) {
      *max_clusters = n;
      return static_cast<cudaError_t>(kNoRoom);
    }
  }
  note_launch();
  return cudaLaunchKernelEx(&cfg, kern, p);
}

template <bool XSELF, int CODE, int EPI>
static cudaError_t launch_fused_mc(int M, const FusedParams& p, int blocks, size_t smem, cudaStream_t st, int* mc) {
  switch (M) {
    case 1: return launch_fused<1, XSELF, CODE, EPI>(p, blocks, smem, st, mc);
    case 2: return launch_fused<2, XSELF, CODE, EPI>(p, blocks, smem, st, mc);
    case 3: return launch_fused<3, XSELF, CODE, EPI>(p, blocks, smem, st, mc);
    default: return launch_fused<4, XSELF, CODE, EPI>(p, blocks, smem, st, mc);
  }
}

// Every (XSELF, EPI, M) launcher of one format; the epilogue forms take one
// format, so the mixed-format code has only the plain epilogue.
template <int CODE>
cudaError_t launch_fused_code(bool xself, int epi, int M, const FusedParams& p, int blocks, size_t smem,
                              cudaStream_t st, int* mc) {
  if constexpr (CODE == kMixed) {
    if (epi != 0) return cudaErrorInvalidValue;
    return xself ? launch_fused_mc<true, CODE, 0>(M, p, blocks, smem, st, mc)
                 : launch_fused_mc<false, CODE, 0>(M, p, blocks, smem, st, mc);
  } else {
    switch (epi) {
      case 1: return xself ? launch_fused_mc<true, CODE, 1>(M, p, blocks, smem, st, mc)
                           : launch_fused_mc<false, CODE, 1>(M, p, blocks, smem, st, mc);
      case 2: return xself ? launch_fused_mc<true, CODE, 2>(M, p, blocks, smem, st, mc)
                           : launch_fused_mc<false, CODE, 2>(M, p, blocks, smem, st, mc);
      default: return xself ? launch_fused_mc<true, CODE, 0>(M, p, blocks, smem, st, mc)
                            : launch_fused_mc<false, CODE, 0>(M, p, blocks, smem, st, mc);
    }
  }
}

#define NSQ_FUSED_CODES(X) X(kQ4K) X(kQ6KG) X(kQ6KN) X(kQ40) X(kQ80) X(kQ5KG) X(kQ5KN) X(kMixed)
#define NSQ_FUSED_EXTERN(C)                                                                             \
  extern template cudaError_t launch_fused_code<C>(bool, int, int, const FusedParams&, int, size_t, \
                                                   cudaStream_t, int*);
NSQ_FUSED_CODES(NSQ_FUSED_EXTERN)
#undef NSQ_FUSED_EXTERN

}  // namespace nsq
