// gemv_mma.cu -- decode GEMV for M = 9..16 tokens on the integer tensor cores.
//
//   y[m, n] = sum_k x[m, k] * W[n, k]
//
// With more than a few tokens the per-lane dp4a kernel (gemv_rows.cu) turns
// compute bound: every weight is multiplied M times on the CUDA cores.  Here
// the products run on mma.sync integer tensor cores straight from the GGUF
// bytes: the A operand is a 16-row x 32 (or 16) weight tile as unsigned 4/6-
// bit values (signed bytes for Q8_0) extracted with a few logic ops, the B
// operand the activations' high and low bytes (x ~ sx * (256 * hi + lo), the
// prepared records of prepare_x_kernel, gemv.cu) for 8 tokens; the int32
// sums of one 32- or 16-weight scale group are exact and get the group's
// weight scale, the activation scale and the min/offset term in fp32.
//
// Walk: K in chunks of PPS pieces (256 weights), outer; the CTA's rows in
// blocks of 64, inner.  One chunk of activation records (all M tokens) is
// copied to shared memory once and serves every row block of the CTA, and the
// weights are still streamed exactly once.  Consumer warp w owns rows
// [16w, 16w + 16) of every block and keeps its partial sums for each block in
// shared memory between chunks.  One producer warp issues the bulk copies
// (TMA, 1-D, one per weight row and chunk, one per token and chunk of
// activation records) against full/empty mbarriers; all waits are bounded.
//
// Row-sharded exchange (P > 1): the epilogue stores into every rank's
// exchange buffer and the grid's last CTA publishes, as in gemv_rows.cu.
#include <stdlib.h>

#include "nsq_common.cuh"

namespace nsq {

constexpr int kMmaConsumers = 4;
constexpr int kMmaThreads = 32 * (1 + kMmaConsumers);
constexpr int kMmaRows = 16 * kMmaConsumers;  // rows per block

enum : int { kMQ4K = 0, kMQ6KG = 1, kMQ6KN = 2, kMQ40 = 3, kMQ80 = 4, kMQ5KG = 5, kMQ5KN = 6, kMMixed = -1 };

struct MSeg {
  const uint8_t* w;
  float* y;
  int64_t N, RB, row0;  // rows, row bytes, first row in the concatenated row space
  int code, pb, pitch;
};

struct MmaParams {
  MSeg seg[NSQ_MAX_SEGMENTS];
  int nseg;
  int64_t T;          // total rows
  const XGroup* xg;   // prepared activations [M][GX]
  int M;
  int64_t K, GX;
  int npieces, PPS, nchunks;
  int stage_bytes, nstages;
  int xstride;        // bytes per token in a chunk buffer (records + 16 bytes of bank offset)
  int xbuf_bytes;
  int max_items;      // partial-sum slots per CTA
  int64_t nrb;        // row blocks of kMmaRows rows
  int P, rank;        // row-sharded exchange, see gemv_rows.cu
  uint8_t* xbuf[NSQ_MAX_RANKS];
  int64_t xrow0[NSQ_MAX_SEGMENTS], xnfull[NSQ_MAX_SEGMENTS], xoff[NSQ_MAX_SEGMENTS];
};

__device__ __forceinline__ void grid_dep_wait_m() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch_m() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------------------
// Integer MMA, D = A . B (C = 0).  Fragments (g = lane / 4, t = lane % 4):
// k32: a0 = A[g][4t..4t+3], a1 = A[g+8][4t..], a2 = A[g][16+4t..], a3 =
// A[g+8][16+4t..]; b0 = B[4t..4t+3][g], b1 = B[16+4t..][g]; k16: a0, a1, b0.
// d0 = D[g][2t], d1 = D[g][2t+1], d2 = D[g+8][2t], d3 = D[g+8][2t+1].
#define NSQ_MMA_K32(ATY, BTY)                                                                                       \
  __device__ __forceinline__ void mma_k32_##ATY##BTY(int (&d)[4], const uint32_t (&a)[4], uint32_t b0,            \
                                                     uint32_t b1) {                                               \
    asm volatile("mma.sync.aligned.m16n8k32.row.col.s32." #ATY "." #BTY                                           \
                 ".s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"                                 \
                 : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])                                                 \
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0));                         \
  }
NSQ_MMA_K32(u8, s8)
NSQ_MMA_K32(u8, u8)
NSQ_MMA_K32(s8, s8)
NSQ_MMA_K32(s8, u8)
#undef NSQ_MMA_K32

__device__ __forceinline__ void mma_k16_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
  asm volatile("mma.sync.aligned.m16n8k16.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%7,%7,%7};"
               : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
               : "r"(a0), "r"(a1), "r"(b0), "r"(0));
}
__device__ __forceinline__ void mma_k16_u8u8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
  asm volatile("mma.sync.aligned.m16n8k16.row.col.s32.u8.u8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%7,%7,%7};"
               : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
               : "r"(a0), "r"(a1), "r"(b0), "r"(0));
}

__device__ __forceinline__ uint32_t lds32(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }
// 4 bytes at a 2-byte aligned shared address
__device__ __forceinline__ uint32_t lds32_a2(const uint8_t* p) {
  uint32_t w[1];
  ld_words_unaligned<1>(p, w);
  return w[0];
}

// Per-token activation data of one 32-group for the epilogue: scale and
// the integer sums of the two 16-element halves.
struct TokG {
  float sx;
  int t0, t1;
};
__device__ __forceinline__ TokG tok_group(const uint8_t* rec, bool valid) {
  TokG r{0.f, 0, 0};
  if (valid) {
    const uint4 e = *reinterpret_cast<const uint4*>(rec + 64);
    r.sx = __uint_as_float(e.x);
    r.t0 = (int)e.y;
    r.t1 = (int)e.z;
  }
  return r;
}

// The B fragments (high and low activation bytes) of token column g of one
// octet for a 32-group, k32 layout, or for one 16-element half, k16 layout.
__device__ __forceinline__ void b_k32(const uint8_t* rec, bool valid, int t, uint32_t& h0, uint32_t& h1,
                                      uint32_t& l0, uint32_t& l1) {
  h0 = h1 = l0 = l1 = 0u;
  if (valid) {
    h0 = lds32(rec + 4 * t);
    h1 = lds32(rec + 16 + 4 * t);
    l0 = lds32(rec + 32 + 4 * t);
    l1 = lds32(rec + 48 + 4 * t);
  }
}

// Accumulates acc[o][i] += sx * (a_row * S - b_row * T) for the fragment's
// 2 rows x 2 tokens of one octet.  S = 256 * Dhi + Dlo (exact int32).
__device__ __forceinline__ void epi(float (&acc)[4], const int (&dh)[4], const int (&dl)[4], float a0, float b0,
                                    float a1, float b1, const TokG& e0, const TokG& e1, int T0, int T1) {
  const float S0 = (float)((dh[0] << 8) + dl[0]), S1 = (float)((dh[1] << 8) + dl[1]);
  const float S2 = (float)((dh[2] << 8) + dl[2]), S3 = (float)((dh[3] << 8) + dl[3]);
  acc[0] = fmaf(e0.sx, fmaf(a0, S0, -b0 * (float)T0), acc[0]);
  acc[1] = fmaf(e1.sx, fmaf(a0, S1, -b0 * (float)T1), acc[1]);
  acc[2] = fmaf(e0.sx, fmaf(a1, S2, -b1 * (float)T0), acc[2]);
  acc[3] = fmaf(e1.sx, fmaf(a1, S3, -b1 * (float)T1), acc[3]);
}

// ---------------------------------------------------------------------------
// One piece (256 weights of rows g and g+8 of the warp's tile, at p0 / p1)
// against the chunk's activation records (xp: the piece's 8 groups of token
// 0; token m at xp + m * xstride).
template <int NOCT>
struct MmaPieces {
  // Q4_K [d][dmin][scales 12][qs 128] (q4_k.rs:75-131)
  __device__ static void q4k(const uint8_t* p0, const uint8_t* p1, const uint8_t* xp, int xstride, int M, int g,
                             int t, float (&acc)[NOCT][4]) {
    const uint4 h0 = *reinterpret_cast<const uint4*>(p0), h1 = *reinterpret_cast<const uint4*>(p1);
    const float d0 = h2f((uint16_t)(h0.x & 0xFFFF)), m0 = h2f((uint16_t)(h0.x >> 16));
    const float d1 = h2f((uint16_t)(h1.x & 0xFFFF)), m1 = h2f((uint16_t)(h1.x >> 16));
    // get_scale_min_k4 (q4_k.rs:120-131), four per word: sub-blocks 0..3 / 4..7
    const uint32_t sl0 = h0.y & 0x3F3F3F3Fu, ml0 = h0.z & 0x3F3F3F3Fu;
    const uint32_t sh0 = (h0.w & 0x0F0F0F0Fu) | ((h0.y >> 2) & 0x30303030u);
    const uint32_t mh0 = ((h0.w >> 4) & 0x0F0F0F0Fu) | ((h0.z >> 2) & 0x30303030u);
    const uint32_t sl1 = h1.y & 0x3F3F3F3Fu, ml1 = h1.z & 0x3F3F3F3Fu;
    const uint32_t sh1 = (h1.w & 0x0F0F0F0Fu) | ((h1.y >> 2) & 0x30303030u);
    const uint32_t mh1 = ((h1.w >> 4) & 0x0F0F0F0Fu) | ((h1.z >> 2) & 0x30303030u);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const uint32_t w00 = lds32(p0 + 16 + 32 * c + 4 * t), w01 = lds32(p1 + 16 + 32 * c + 4 * t);
      const uint32_t w10 = lds32(p0 + 32 + 32 * c + 4 * t), w11 = lds32(p1 + 32 + 32 * c + 4 * t);
#pragma unroll
      for (int nib = 0; nib < 2; ++nib) {
        const int sb = 2 * c + nib;
        const int sh = 4 * nib;
        const uint32_t a[4] = {(w00 >> sh) & 0x0F0F0F0Fu, (w01 >> sh) & 0x0F0F0F0Fu, (w10 >> sh) & 0x0F0F0F0Fu,
                               (w11 >> sh) & 0x0F0F0F0Fu};
        const int bs = 8 * (sb & 3);
        const uint32_t s0w = sb < 4 ? sl0 : sh0, m0w = sb < 4 ? ml0 : mh0;
        const uint32_t s1w = sb < 4 ? sl1 : sh1, m1w = sb < 4 ? ml1 : mh1;
        const float a0 = d0 * (float)((s0w >> bs) & 0xFF), b0 = m0 * (float)((m0w >> bs) & 0xFF);
        const float a1 = d1 * (float)((s1w >> bs) & 0xFF), b1 = m1 * (float)((m1w >> bs) & 0xFF);
#pragma unroll
        for (int o = 0; o < NOCT; ++o) {
          const int tb = 8 * o + g, te = 8 * o + 2 * t;
          uint32_t bh0, bh1, bl0, bl1;
          b_k32(xp + (size_t)tb * xstride + sb * 80, tb < M, t, bh0, bh1, bl0, bl1);
          int dh[4], dl[4];
          mma_k32_u8s8(dh, a, bh0, bh1);
          mma_k32_u8u8(dl, a, bl0, bl1);
          const TokG e0 = tok_group(xp + (size_t)te * xstride + sb * 80, te < M);
          const TokG e1 = tok_group(xp + (size_t)(te + 1) * xstride + sb * 80, te + 1 < M);
          epi(acc[o], dh, dl, a0, b0, a1, b1, e0, e1, e0.t0 + e0.t1, e1.t0 + e1.t1);
        }
      }
    }
  }

  // Q5_K [d][dmin][scales 12][qh 32][qs 128]: Q4_K's nibbles at byte 48 and
  // a fifth bit per weight, element l of sub-block j: ggml bit j of qh[l];
  // NodeStor (q5_k.rs:57-70) bit l%8 of qh[8(j>>1) + 4(j&1) + l/8].
  template <int LAYOUT>
  __device__ static void q5k(const uint8_t* p0, const uint8_t* p1, const uint8_t* xp, int xstride, int M, int g,
                             int t, float (&acc)[NOCT][4]) {
    const uint4 h0 = *reinterpret_cast<const uint4*>(p0), h1 = *reinterpret_cast<const uint4*>(p1);
    const float d0 = h2f((uint16_t)(h0.x & 0xFFFF)), m0 = h2f((uint16_t)(h0.x >> 16));
    const float d1 = h2f((uint16_t)(h1.x & 0xFFFF)), m1 = h2f((uint16_t)(h1.x >> 16));
    const uint32_t sl0 = h0.y & 0x3F3F3F3Fu, ml0 = h0.z & 0x3F3F3F3Fu;
    const uint32_t sh0 = (h0.w & 0x0F0F0F0Fu) | ((h0.y >> 2) & 0x30303030u);
    const uint32_t mh0 = ((h0.w >> 4) & 0x0F0F0F0Fu) | ((h0.z >> 2) & 0x30303030u);
    const uint32_t sl1 = h1.y & 0x3F3F3F3Fu, ml1 = h1.z & 0x3F3F3F3Fu;
    const uint32_t sh1 = (h1.w & 0x0F0F0F0Fu) | ((h1.y >> 2) & 0x30303030u);
    const uint32_t mh1 = ((h1.w >> 4) & 0x0F0F0F0Fu) | ((h1.z >> 2) & 0x30303030u);
    // ggml: the qh words of elements 4t.. and 16+4t.., shared by all sub-blocks
    uint32_t q00 = 0, q01 = 0, q10 = 0, q11 = 0;
    if constexpr (LAYOUT != NSQ_Q6K_NODESTOR) {
      q00 = lds32(p0 + 16 + 4 * t); q01 = lds32(p1 + 16 + 4 * t);
      q10 = lds32(p0 + 32 + 4 * t); q11 = lds32(p1 + 32 + 4 * t);
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const uint32_t w00 = lds32(p0 + 48 + 32 * c + 4 * t), w01 = lds32(p1 + 48 + 32 * c + 4 * t);
      const uint32_t w10 = lds32(p0 + 64 + 32 * c + 4 * t), w11 = lds32(p1 + 64 + 32 * c + 4 * t);
#pragma unroll
      for (int nib = 0; nib < 2; ++nib) {
        const int sb = 2 * c + nib;
        const int sh = 4 * nib;
        uint32_t hb[4];
        if constexpr (LAYOUT == NSQ_Q6K_NODESTOR) {
          const int hb0 = 16 + 8 * c + 4 * nib + (t >> 1), ns = 4 * (t & 1);
          hb[0] = spread4(((uint32_t)p0[hb0] >> ns) & 0xF);
          hb[1] = spread4(((uint32_t)p1[hb0] >> ns) & 0xF);
          hb[2] = spread4(((uint32_t)p0[hb0 + 2] >> ns) & 0xF);
          hb[3] = spread4(((uint32_t)p1[hb0 + 2] >> ns) & 0xF);
        } else {
          hb[0] = (q00 >> sb) & 0x01010101u;
          hb[1] = (q01 >> sb) & 0x01010101u;
          hb[2] = (q10 >> sb) & 0x01010101u;
          hb[3] = (q11 >> sb) & 0x01010101u;
        }
        const uint32_t a[4] = {((w00 >> sh) & 0x0F0F0F0Fu) | (hb[0] << 4), ((w01 >> sh) & 0x0F0F0F0Fu) | (hb[1] << 4),
                               ((w10 >> sh) & 0x0F0F0F0Fu) | (hb[2] << 4), ((w11 >> sh) & 0x0F0F0F0Fu) | (hb[3] << 4)};
        const int bs = 8 * (sb & 3);
        const uint32_t s0w = sb < 4 ? sl0 : sh0, m0w = sb < 4 ? ml0 : mh0;
        const uint32_t s1w = sb < 4 ? sl1 : sh1, m1w = sb < 4 ? ml1 : mh1;
        const float a0 = d0 * (float)((s0w >> bs) & 0xFF), b0 = m0 * (float)((m0w >> bs) & 0xFF);
        const float a1 = d1 * (float)((s1w >> bs) & 0xFF), b1 = m1 * (float)((m1w >> bs) & 0xFF);
#pragma unroll
        for (int o = 0; o < NOCT; ++o) {
          const int tb = 8 * o + g, te = 8 * o + 2 * t;
          uint32_t bh0, bh1, bl0, bl1;
          b_k32(xp + (size_t)tb * xstride + sb * 80, tb < M, t, bh0, bh1, bl0, bl1);
          int dh[4], dl[4];
          mma_k32_u8s8(dh, a, bh0, bh1);
          mma_k32_u8u8(dl, a, bl0, bl1);
          const TokG e0 = tok_group(xp + (size_t)te * xstride + sb * 80, te < M);
          const TokG e1 = tok_group(xp + (size_t)(te + 1) * xstride + sb * 80, te + 1 < M);
          epi(acc[o], dh, dl, a0, b0, a1, b1, e0, e1, e0.t0 + e0.t1, e1.t0 + e1.t1);
        }
      }
    }
  }

  // Q6_K, ggml layout: element 128n + 32j + l: ql[64n + 32(j&1) + l] nibble
  // (j>>1), qh[32n + l] bits 2j; int8 scale sc[(128n + 32j + l) / 16].
  __device__ static void q6k_ggml(const uint8_t* p0, const uint8_t* p1, const uint8_t* xp, int xstride, int M, int g,
                                  int t, float (&acc)[NOCT][4]) {
    const float d0 = h2f(ld_u16(p0 + 208)), d1 = h2f(ld_u16(p1 + 208));
    uint32_t sc0[4], sc1[4];
    ld_words_unaligned<4>(p0 + 192, sc0);
    ld_words_unaligned<4>(p1 + 192, sc1);
#pragma unroll
    for (int n = 0; n < 2; ++n) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int s16 = 8 * n + 2 * j + h;  // scale index
          const int lo = 64 * n + 32 * (j & 1) + 16 * h + 4 * t, hi = 128 + 32 * n + 16 * h + 4 * t;
          const int ns = 4 * (j >> 1), qs = 2 * j;
          const uint32_t a0 = ((lds32_a2(p0 + lo) >> ns) & 0x0F0F0F0Fu) | (((lds32_a2(p0 + hi) >> qs) & 0x03030303u) << 4);
          const uint32_t a1 = ((lds32_a2(p1 + lo) >> ns) & 0x0F0F0F0Fu) | (((lds32_a2(p1 + hi) >> qs) & 0x03030303u) << 4);
          const float f0 = d0 * (float)(int8_t)((sc0[s16 >> 2] >> (8 * (s16 & 3))) & 0xFF);
          const float f1 = d1 * (float)(int8_t)((sc1[s16 >> 2] >> (8 * (s16 & 3))) & 0xFF);
          const int grp = 4 * n + j;
#pragma unroll
          for (int o = 0; o < NOCT; ++o) {
            const int tb = 8 * o + g, te = 8 * o + 2 * t;
            const uint8_t* rb = xp + (size_t)tb * xstride + grp * 80 + 16 * h + 4 * t;
            const uint32_t bh = tb < M ? lds32(rb) : 0u, bl = tb < M ? lds32(rb + 32) : 0u;
            int dh[4], dl[4];
            mma_k16_u8s8(dh, a0, a1, bh);
            mma_k16_u8u8(dl, a0, a1, bl);
            const TokG e0 = tok_group(xp + (size_t)te * xstride + grp * 80, te < M);
            const TokG e1 = tok_group(xp + (size_t)(te + 1) * xstride + grp * 80, te + 1 < M);
            // weights q - 32: S - 32 * (sum of the half's X)
            const int T0 = 32 * (h ? e0.t1 : e0.t0), T1 = 32 * (h ? e1.t1 : e1.t0);
            epi(acc[o], dh, dl, f0, f0, f1, f1, e0, e1, T0, T1);
          }
        }
      }
    }
  }

  // Q6_K, NodeStor layout (dequant_q6k.comp:50-99): element i: ql[i>>1]
  // nibble (i&1), qh[i>>2] bits 2(i&3); scale (b[192 + (i>>4)] - 128) / 64.
  __device__ static void q6k_nodestor(const uint8_t* p0, const uint8_t* p1, const uint8_t* xp, int xstride, int M,
                                      int g, int t, float (&acc)[NOCT][4]) {
    const float d0 = h2f(ld_u16(p0 + 208)), d1 = h2f(ld_u16(p1 + 208));
    auto wq = [](const uint8_t* p, int s, int t) -> uint32_t {
      const uint32_t v = ld_u16(p + 8 * s + 2 * t);
      const uint32_t tt = __byte_perm(v, 0, 0x1100);
      const uint32_t lo4 = (tt & 0x000F000Fu) | ((tt >> 4) & 0x0F000F00u);
      const uint32_t h = p[128 + 4 * s + t];
      return lo4 | (((h | (h << 6) | (h << 12) | (h << 18)) & 0x03030303u) << 4);
    };
#pragma unroll 4
    for (int s = 0; s < 16; ++s) {
      const uint32_t a0 = wq(p0, s, t), a1 = wq(p1, s, t);
      const float f0 = d0 * ((float)((int)p0[192 + s] - 128) * 0.015625f);
      const float f1 = d1 * ((float)((int)p1[192 + s] - 128) * 0.015625f);
      const int grp = s >> 1, h = s & 1;
#pragma unroll
      for (int o = 0; o < NOCT; ++o) {
        const int tb = 8 * o + g, te = 8 * o + 2 * t;
        const uint8_t* rb = xp + (size_t)tb * xstride + grp * 80 + 16 * h + 4 * t;
        const uint32_t bh = tb < M ? lds32(rb) : 0u, bl = tb < M ? lds32(rb + 32) : 0u;
        int dh[4], dl[4];
        mma_k16_u8s8(dh, a0, a1, bh);
        mma_k16_u8u8(dl, a0, a1, bl);
        const TokG e0 = tok_group(xp + (size_t)te * xstride + grp * 80, te < M);
        const TokG e1 = tok_group(xp + (size_t)(te + 1) * xstride + grp * 80, te + 1 < M);
        const int T0 = 32 * (h ? e0.t1 : e0.t0), T1 = 32 * (h ? e1.t1 : e1.t0);
        epi(acc[o], dh, dl, f0, f0, f1, f1, e0, e1, T0, T1);
      }
    }
  }

  // Q4_0: 8 blocks [d][qs 16]: low nibbles = weights 0..15, high = 16..31,
  // value q - 8 (dequant_q4.comp:40-61).
  __device__ static void q40(const uint8_t* p0, const uint8_t* p1, const uint8_t* xp, int xstride, int M, int g,
                             int t, float (&acc)[NOCT][4]) {
#pragma unroll 2
    for (int bi = 0; bi < 8; ++bi) {
      const uint8_t* b0p = p0 + 18 * bi;
      const uint8_t* b1p = p1 + 18 * bi;
      const float d0 = h2f(ld_u16(b0p)), d1 = h2f(ld_u16(b1p));
      const uint32_t w0 = lds32_a2(b0p + 2 + 4 * t), w1 = lds32_a2(b1p + 2 + 4 * t);
      const uint32_t a[4] = {w0 & 0x0F0F0F0Fu, w1 & 0x0F0F0F0Fu, (w0 >> 4) & 0x0F0F0F0Fu, (w1 >> 4) & 0x0F0F0F0Fu};
#pragma unroll
      for (int o = 0; o < NOCT; ++o) {
        const int tb = 8 * o + g, te = 8 * o + 2 * t;
        uint32_t bh0, bh1, bl0, bl1;
        b_k32(xp + (size_t)tb * xstride + bi * 80, tb < M, t, bh0, bh1, bl0, bl1);
        int dh[4], dl[4];
        mma_k32_u8s8(dh, a, bh0, bh1);
        mma_k32_u8u8(dl, a, bl0, bl1);
        const TokG e0 = tok_group(xp + (size_t)te * xstride + bi * 80, te < M);
        const TokG e1 = tok_group(xp + (size_t)(te + 1) * xstride + bi * 80, te + 1 < M);
        epi(acc[o], dh, dl, d0, d0, d1, d1, e0, e1, 8 * (e0.t0 + e0.t1), 8 * (e1.t0 + e1.t1));
      }
    }
  }

  // Q8_0: 8 blocks [d][qs int8 32] (q8_0.rs:14-28).
  __device__ static void q80(const uint8_t* p0, const uint8_t* p1, const uint8_t* xp, int xstride, int M, int g,
                             int t, float (&acc)[NOCT][4]) {
#pragma unroll 2
    for (int bi = 0; bi < 8; ++bi) {
      const uint8_t* b0p = p0 + 34 * bi;
      const uint8_t* b1p = p1 + 34 * bi;
      const float d0 = h2f(ld_u16(b0p)), d1 = h2f(ld_u16(b1p));
      const uint32_t a[4] = {lds32_a2(b0p + 2 + 4 * t), lds32_a2(b1p + 2 + 4 * t), lds32_a2(b0p + 18 + 4 * t),
                             lds32_a2(b1p + 18 + 4 * t)};
#pragma unroll
      for (int o = 0; o < NOCT; ++o) {
        const int tb = 8 * o + g, te = 8 * o + 2 * t;
        uint32_t bh0, bh1, bl0, bl1;
        b_k32(xp + (size_t)tb * xstride + bi * 80, tb < M, t, bh0, bh1, bl0, bl1);
        int dh[4], dl[4];
        mma_k32_s8s8(dh, a, bh0, bh1);
        mma_k32_s8u8(dl, a, bl0, bl1);
        const TokG e0 = tok_group(xp + (size_t)te * xstride + bi * 80, te < M);
        const TokG e1 = tok_group(xp + (size_t)(te + 1) * xstride + bi * 80, te + 1 < M);
        epi(acc[o], dh, dl, d0, 0.f, d1, 0.f, e0, e1, 0, 0);
      }
    }
  }
};

template <int NOCT, int CODE>
__device__ __forceinline__ void mma_piece(int code, const uint8_t* p0, const uint8_t* p1, const uint8_t* xp,
                                          int xstride, int M, int g, int t, float (&acc)[NOCT][4]) {
  const int c = CODE >= 0 ? CODE : code;
  switch (c) {
    case kMQ4K: MmaPieces<NOCT>::q4k(p0, p1, xp, xstride, M, g, t, acc); break;
    case kMQ6KG: MmaPieces<NOCT>::q6k_ggml(p0, p1, xp, xstride, M, g, t, acc); break;
    case kMQ6KN: MmaPieces<NOCT>::q6k_nodestor(p0, p1, xp, xstride, M, g, t, acc); break;
    case kMQ40: MmaPieces<NOCT>::q40(p0, p1, xp, xstride, M, g, t, acc); break;
    case kMQ5KG: MmaPieces<NOCT>::template q5k<NSQ_Q6K_GGML>(p0, p1, xp, xstride, M, g, t, acc); break;
    case kMQ5KN: MmaPieces<NOCT>::template q5k<NSQ_Q6K_NODESTOR>(p0, p1, xp, xstride, M, g, t, acc); break;
    default: MmaPieces<NOCT>::q80(p0, p1, xp, xstride, M, g, t, acc); break;
  }
}

// Walk of one CTA's rows in blocks of kMmaRows, split at segment ends.
struct MRowCursor {
  int seg;
  int64_t row0, rows;  // segment-local first row, row count
  __device__ int64_t seg_end(const MmaParams& p, int64_t re) const { return min(re, p.seg[seg].row0 + p.seg[seg].N); }
  __device__ bool first(const MmaParams& p, int64_t rb, int64_t re) {
    if (rb >= re) return false;
    seg = 0;
    while (seg < p.nseg - 1 && rb >= p.seg[seg].row0 + p.seg[seg].N) ++seg;
    row0 = rb - p.seg[seg].row0;
    rows = min((int64_t)kMmaRows, seg_end(p, re) - rb);
    return true;
  }
  __device__ bool next(const MmaParams& p, int64_t re) {
    const int64_t g = p.seg[seg].row0 + row0 + rows;  // next row, concatenated space
    if (g >= re) return false;
    if (g >= p.seg[seg].row0 + p.seg[seg].N) {
      ++seg;
      row0 = 0;
    } else {
      row0 += rows;
    }
    rows = min((int64_t)kMmaRows, seg_end(p, re) - g);
    return true;
  }
};

template <int NOCT, int CODE>
__global__ void __launch_bounds__(kMmaThreads, 2) gemv_mma_kernel(const __grid_constant__ MmaParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* stages = smem;
  uint8_t* xbufs = stages + (size_t)p.stage_bytes * p.nstages;  // 2 chunk buffers of activation records
  float* accs = reinterpret_cast<float*>(xbufs + 2 * (size_t)p.xbuf_bytes);  // [max_items][4 warps][32][NOCT*4]
  uint64_t* full = reinterpret_cast<uint64_t*>(accs + (size_t)p.max_items * kMmaConsumers * 32 * NOCT * 4);
  uint64_t* empty = full + p.nstages;
  uint64_t* xfull = empty + p.nstages;
  uint64_t* xempty = xfull + 2;
  __shared__ int s_fail;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t r_begin = min(p.T, (int64_t)kMmaRows * (p.nrb * blockIdx.x / gridDim.x));
  const int64_t r_end = min(p.T, (int64_t)kMmaRows * (p.nrb * (blockIdx.x + 1) / gridDim.x));

  if (tid == 0) {
    s_fail = 0;
    for (int s = 0; s < p.nstages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kMmaConsumers);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&xfull[b], 1);
      mbar_init(&xempty[b], kMmaConsumers);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == 0) {
    MRowCursor rc;
    if (rc.first(p, r_begin, r_end)) {
      auto issue_w = [&](const MRowCursor& it, int c, int s) {
        const MSeg& sg = p.seg[it.seg];
        const int np = min(p.PPS, p.npieces - c * p.PPS);
        // the chunk's byte run of each row, widened to 16-byte bounds (rows
        // start 16-byte aligned, so the widened run stays inside the row)
        const int64_t off = (int64_t)c * p.PPS * sg.pb;
        const int64_t a0 = off & ~int64_t(15), a1 = (off + (int64_t)np * sg.pb + 15) & ~int64_t(15);
        const int cb = (int)(a1 - a0);
        uint8_t* slot = stages + (size_t)s * p.stage_bytes;
        if (lane == 0) mbar_arrive_expect_tx(&full[s], (uint32_t)(it.rows * cb));
        __syncwarp();
        for (int r = lane; r < (int)it.rows; r += 32)
          bulk_g2s(slot + (size_t)r * sg.pitch, sg.w + (it.row0 + r) * sg.RB + a0, cb, &full[s]);
      };
      // the weight copies of chunk 0 do not depend on the previous kernel
      int npre = 0;
      {
        MRowCursor pc = rc;
        bool m = true;
        while (m && npre < p.nstages) {
          issue_w(pc, 0, npre);
          ++npre;
          m = pc.next(p, r_end);
        }
      }
      __syncwarp();
      grid_dep_wait_m();
      grid_dep_launch_m();
      bool ok = true;
      // stage t: slot ts = t % nstages, parity tph = (t / nstages) & 1, counted incrementally
      int t = 0, ts = 0;
      uint32_t tph = 0u;
      for (int c = 0; c < p.nchunks && ok; ++c) {
        const int b = c & 1;
        if (c >= 2 && !mbar_wait_bounded(&xempty[b], (uint32_t)(((c >> 1) - 1) & 1))) {
          ok = false;
          break;
        }
        const int ng = min(p.PPS, p.npieces - c * p.PPS) * 8;
        if (lane == 0) {
          mbar_arrive_expect_tx(&xfull[b], (uint32_t)(p.M * ng * 80));
          for (int m = 0; m < p.M; ++m)
            bulk_g2s(xbufs + (size_t)b * p.xbuf_bytes + (size_t)m * p.xstride,
                     p.xg + (int64_t)m * p.GX + (int64_t)c * p.PPS * 8, ng * 80, &xfull[b]);
        }
        __syncwarp();
        MRowCursor it;
        bool more = it.first(p, r_begin, r_end);
        for (; more; ++t, ts = (ts + 1 == p.nstages) ? 0 : ts + 1, tph ^= (ts == 0) ? 1u : 0u,
                     more = it.next(p, r_end)) {
          if (t < npre) continue;  // issued before the dependency wait
          const int s = ts;
          if (!mbar_wait_bounded(&empty[s], tph ^ 1u)) {
            ok = false;
            break;
          }
          fence_proxy_async_smem();
          issue_w(it, c, s);
        }
      }
      if (!ok) s_fail = 1;
      __syncwarp();
    } else {
      grid_dep_wait_m();
      grid_dep_launch_m();
    }
  } else {
    const int cw = warp - 1;
    const int g = lane >> 2, t4 = lane & 3;
    grid_dep_wait_m();
    grid_dep_launch_m();
    bool ok = true;
    int t = 0, ts = 0;  // stage t: slot ts = t % nstages, parity tph = (t / nstages) & 1
    uint32_t tph = 0u;
    MRowCursor probe;
    const bool any = probe.first(p, r_begin, r_end);
    for (int c = 0; any && c < p.nchunks; ++c) {
      const int b = c & 1;
      if (ok) ok = mbar_wait_bounded(&xfull[b], (uint32_t)((c >> 1) & 1));
      const uint8_t* xc = xbufs + (size_t)b * p.xbuf_bytes;
      const int np = min(p.PPS, p.npieces - c * p.PPS);
      MRowCursor it;
      bool more = it.first(p, r_begin, r_end);
      for (int item = 0; more; ++t, ++item, ts = (ts + 1 == p.nstages) ? 0 : ts + 1, tph ^= (ts == 0) ? 1u : 0u,
                                   more = it.next(p, r_end)) {
        const int s = ts;
        if (ok) ok = mbar_wait_bounded(&full[s], tph);
        if (item >= p.max_items) ok = false;  // the plan bounds the items; never taken
        float acc[NOCT][4];
        float* slot_acc = accs + ((size_t)(item * kMmaConsumers + cw) * 32 + lane) * NOCT * 4;
#pragma unroll
        for (int o = 0; o < NOCT; ++o)
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[o][i] = (c == 0 || !ok) ? 0.f : slot_acc[o * 4 + i];
        const MSeg& sg = p.seg[it.seg];
        if (ok && 16 * cw < it.rows) {
          const int delta = (int)(((int64_t)c * p.PPS * sg.pb) & 15);
          const uint8_t* slot = stages + (size_t)s * p.stage_bytes;
          const uint8_t* r0p = slot + (size_t)(16 * cw + g) * sg.pitch + delta;
          const uint8_t* r1p = r0p + (size_t)8 * sg.pitch;
          for (int j = 0; j < np; ++j)
            mma_piece<NOCT, CODE>(sg.code, r0p + j * sg.pb, r1p + j * sg.pb, xc + j * 8 * 80, p.xstride, p.M, g, t4,
                                  acc);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        if (c == p.nchunks - 1) {
          if (ok) {
#pragma unroll
            for (int o = 0; o < NOCT; ++o)
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const int rr = 16 * cw + g + 8 * (i >> 1), m = 8 * o + 2 * t4 + (i & 1);
                if (rr < it.rows && m < p.M) {
                  if (p.P > 1) {
                    const int64_t idx = (int64_t)m * p.xnfull[it.seg] + p.xrow0[it.seg] + it.row0 + rr;
                    for (int pr = 0; pr < p.P; ++pr)
                      reinterpret_cast<float*>(p.xbuf[pr] + kXchgCtlBytes + p.xoff[it.seg])[idx] = acc[o][i];
                  } else {
                    sg.y[(int64_t)m * sg.N + it.row0 + rr] = acc[o][i];
                  }
                }
              }
          }
        } else if (ok) {
#pragma unroll
          for (int o = 0; o < NOCT; ++o)
#pragma unroll
            for (int i = 0; i < 4; ++i) slot_acc[o * 4 + i] = acc[o][i];
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&xempty[b]);
    }
    if (!ok) s_fail = 1;
  }
  __syncthreads();
  if (p.P > 1 && tid == 0) {
    // publish, as in gemv_fused_kernel (gemv_rows.cu)
    fence_acq_rel_gpu();
    uint32_t* ctl = reinterpret_cast<uint32_t*>(p.xbuf[p.rank]);
    if (atomicAdd(ctl + kXchgDone, 1u) == gridDim.x - 1) {
      fence_acq_rel_gpu();
      ctl[kXchgDone] = 0;
      const uint32_t seq = ctl[kXchgSeq] + 1;
      ctl[kXchgSeq] = seq;
      for (int pr = 0; pr < p.P; ++pr) st_release_sys(reinterpret_cast<uint32_t*>(p.xbuf[pr]) + p.rank, seq);
    }
  }
}

// ---------------------------------------------------------------------------
// Host side
static int mcode(int type, int layout) {
  switch (type) {
    case NSQ_TYPE_Q4_K: return kMQ4K;
    case NSQ_TYPE_Q6_K: return layout == NSQ_Q6K_NODESTOR ? kMQ6KN : kMQ6KG;
    case NSQ_TYPE_Q4_0: return kMQ40;
    case NSQ_TYPE_Q8_0: return kMQ80;
    case NSQ_TYPE_Q5_K: return layout == NSQ_Q6K_NODESTOR ? kMQ5KN : kMQ5KG;
    default: return -2;
  }
}
static int mpiece_bytes(int type) {
  switch (type) {
    case NSQ_TYPE_Q4_K: return 144;
    case NSQ_TYPE_Q6_K: return 210;
    case NSQ_TYPE_Q5_K: return 176;
    case NSQ_TYPE_Q4_0: return 144;
    case NSQ_TYPE_Q8_0: return 272;
    default: return 0;
  }
}

// Smallest M routed to this kernel (env NSQ_MMA_MIN_M).  Measured on B200
// against the dp4a kernel (gemv_rows.cu, 4 tokens per pass): about even at
// M = 8, ahead at M = 16 (Q4_K 2 x [28672 x 8192]: 366 vs 508 us), behind
// below 8, where the per-scale-group fp32 epilogue and the per-chunk
// activation loads are not amortised.  Default 9.
int gemv_mma_min_m() {
  const int m = tune(kTuneMmaMinM, 9);
  return m < 1 ? 1 : m;
}

bool gemv_mma_covers(const nsq_segment* segs, int nseg, int64_t M, int64_t K) {
  if (nseg < 1 || nseg > NSQ_MAX_SEGMENTS || K % 256 || M < 1 || M > 16) return false;
  for (int i = 0; i < nseg; ++i) {
    if (mcode(segs[i].ggml_type, segs[i].q6k_layout) < -1) return false;
    if (((K / 256) * mpiece_bytes(segs[i].ggml_type)) % 16) return false;
  }
  return true;
}

static bool plan_mma(const nsq_segment* segs, int nseg, int64_t M, int64_t K, int num_sms, MmaParams& p, int& blocks,
                     size_t& smem) {
  const int64_t npieces = K / 256;
  int64_t T = 0;
  for (int i = 0; i < nseg; ++i) T += segs[i].N;
  const int noct = M > 8 ? 2 : 1;
  int PPS = tune(kTuneMmaPPS, 2);
  if (PPS < 1) PPS = 1;
  if (PPS > npieces) PPS = (int)npieces;
  int nstages = tune(kTuneMmaStages, 3);
  if (nstages < 2 || nstages > 6) nstages = 3;
  int max_pitch = 0;
  for (int i = 0; i < nseg; ++i) {
    int pitch = (PPS * mpiece_bytes(segs[i].ggml_type) + 14 + 15) & ~15;  // room for the 16-byte widening
    if (((pitch / 16) & 1) == 0) pitch += 16;  // odd multiple of 16 bytes: rows g and g' hit distinct banks
    if (pitch > max_pitch) max_pitch = pitch;
  }
  const int stage_bytes = (kMmaRows * max_pitch + 127) & ~127;
  const int xstride = PPS * 8 * 80 + 16;
  const int xbuf_bytes = ((int)M * xstride + 127) & ~127;
  const int64_t nrb = (T + kMmaRows - 1) / kMmaRows;
  const size_t base = (size_t)stage_bytes * nstages + 2 * (size_t)xbuf_bytes + 16 * (nstages + 2) + 16;
  // CTAs per SM from shared memory, then the partial-sum slots that count implies
  int per_sm = 2, max_items = 0;
  int64_t grid = 1;
  for (int pass = 0; pass < 3; ++pass) {
    smem = base + (size_t)max_items * kMmaConsumers * 32 * noct * 4 * 4;
    per_sm = (int)((220 * 1024) / (smem + 1024));
    if (per_sm > 2) per_sm = 2;
    if (per_sm < 1) per_sm = 1;
    const int64_t gmax = (int64_t)num_sms * per_sm;
    const int64_t per_cta = (nrb + gmax - 1) / gmax;
    grid = (nrb + per_cta - 1) / per_cta;
    const int need = (int)per_cta + nseg;
    if (need <= max_items) break;
    max_items = need;
  }
  if (smem > 220 * 1024) return false;
  for (int i = 0; i < nseg; ++i) {
    MSeg& f = p.seg[i];
    f.w = static_cast<const uint8_t*>(segs[i].w);
    f.y = segs[i].y;
    f.N = segs[i].N;
    f.pb = mpiece_bytes(segs[i].ggml_type);
    f.RB = npieces * f.pb;
    f.code = mcode(segs[i].ggml_type, segs[i].q6k_layout);
    f.pitch = max_pitch;
  }
  int64_t acc_rows = 0;
  for (int i = 0; i < nseg; ++i) {
    p.seg[i].row0 = acc_rows;
    acc_rows += p.seg[i].N;
  }
  p.nseg = nseg;
  p.T = T;
  p.M = (int)M;
  p.K = K;
  p.GX = K / 32;
  p.npieces = (int)npieces;
  p.PPS = PPS;
  p.nchunks = (int)((npieces + PPS - 1) / PPS);
  p.stage_bytes = stage_bytes;
  p.nstages = nstages;
  p.xstride = xstride;
  p.xbuf_bytes = xbuf_bytes;
  p.max_items = max_items;
  p.nrb = nrb;
  p.P = 1;
  blocks = (int)grid;
  return true;
}

template <int NOCT, int CODE>
static cudaError_t launch_mma(const MmaParams& p, int blocks, size_t smem, cudaStream_t st) {
  auto kern = gemv_mma_kernel<NOCT, CODE>;
  static size_t configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || smem > configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) configured[dev] = smem;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)blocks);
  cfg.blockDim = dim3(kMmaThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  note_launch();
  return cudaLaunchKernelEx(&cfg, kern, p);
}

template <int NOCT>
static cudaError_t launch_mma_c(const MmaParams& p, int blocks, size_t smem, cudaStream_t st) {
  int code = p.seg[0].code;
  for (int i = 1; i < p.nseg; ++i)
    if (p.seg[i].code != code) code = kMMixed;
  switch (code) {
    case kMQ4K: return launch_mma<NOCT, kMQ4K>(p, blocks, smem, st);
    case kMQ6KG: return launch_mma<NOCT, kMQ6KG>(p, blocks, smem, st);
    case kMQ6KN: return launch_mma<NOCT, kMQ6KN>(p, blocks, smem, st);
    case kMQ40: return launch_mma<NOCT, kMQ40>(p, blocks, smem, st);
    case kMQ80: return launch_mma<NOCT, kMQ80>(p, blocks, smem, st);
    case kMQ5KG: return launch_mma<NOCT, kMQ5KG>(p, blocks, smem, st);
    case kMQ5KN: return launch_mma<NOCT, kMQ5KN>(p, blocks, smem, st);
    default: return launch_mma<NOCT, kMMixed>(p, blocks, smem, st);
  }
}

// M = 1..16 tokens from prepared records xg [M][K/32]; -1 if not covered.
int run_gemv_mma(const nsq_segment* segs, int nseg, const XGroup* xg, int64_t M, int64_t K, cudaStream_t st,
                 int num_sms, const XchgDesc* xd) {
  if (!gemv_mma_covers(segs, nseg, M, K)) return -1;
  MmaParams p{};
  int blocks;
  size_t smem;
  if (!plan_mma(segs, nseg, M, K, num_sms, p, blocks, smem)) return -1;
  p.xg = xg;
  if (xd && xd->P > 1) {
    p.P = xd->P;
    p.rank = xd->rank;
    for (int r = 0; r < xd->P; ++r) p.xbuf[r] = xd->buf[r];
    for (int i = 0; i < nseg; ++i) {
      p.xrow0[i] = xd->row0[i];
      p.xnfull[i] = xd->nfull[i];
      p.xoff[i] = xd->off[i];
    }
  }
  const cudaError_t e = M > 8 ? launch_mma_c<2>(p, blocks, smem, st) : launch_mma_c<1>(p, blocks, smem, st);
  return e == cudaSuccess ? NSQ_OK : NSQ_ERR_CUDA;
}

}  // namespace nsq
