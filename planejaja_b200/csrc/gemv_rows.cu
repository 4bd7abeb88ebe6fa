// gemv_rows.cu -- decode GEMV, "one lane per weight row" layout (M = 1..4).
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
#include <stdlib.h>

#include "nsq_common.cuh"

namespace nsq {

constexpr int kRowsConsumers = 4;
constexpr int kRowsThreads = 32 * (1 + kRowsConsumers);

struct RowsParams {
  const uint8_t* w;
  const XGroup* xg;
  float* y;
  int64_t N, K, RB;
  int R, KS, PPS;             // rows per CTA, lane groups per warp, pieces per chunk
  int piece_bytes, chunk_bytes, pitch;
  int nchunks, npieces;       // chunks per row, pieces per row (K / 256)
  int xstride;                // bytes of one token's activation records in a stage
  int stage_bytes, nstages;
  int64_t GX;                 // activation groups per token (K / 32)
};

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
template <int LAYOUT, int M>
struct Piece<NSQ_TYPE_Q4_0, LAYOUT, M> {
  __device__ static void run(const uint8_t* pc, const uint8_t* xp, int xstride, float (&acc)[M]) {
#pragma unroll
    for (int g = 0; g < 8; ++g) {
      const uint8_t* blk = pc + 18 * g;
      uint32_t w5[5];
      ld_words_unaligned<5>(blk, w5);  // bytes 0..19 of the block
      const float d = h2f((uint16_t)(w5[0] & 0xFFFF));
      uint32_t q[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t qs = __funnelshift_r(w5[i], w5[i + 1], 16);  // bytes 2+4i .. 5+4i
        q[i] = qs & 0x0F0F0F0Fu;
        q[i + 4] = qs & 0xF0F0F0F0u;  // 16 * high nibble
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
};

// Q8_0: 8 blocks [d][qs int8 32] (q8_0.rs:14-28).
template <int LAYOUT, int M>
struct Piece<NSQ_TYPE_Q8_0, LAYOUT, M> {
  __device__ static void run(const uint8_t* pc, const uint8_t* xp, int xstride, float (&acc)[M]) {
#pragma unroll
    for (int g = 0; g < 8; ++g) {
      const uint8_t* blk = pc + 34 * g;
      uint32_t w9[9];
      ld_words_unaligned<9>(blk, w9);  // bytes 0..35 of the block
      const float d = h2f((uint16_t)(w9[0] & 0xFFFF));
      uint32_t q[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) q[i] = __funnelshift_r(w9[i], w9[i + 1], 16);
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
};

// ---------------------------------------------------------------------------
template <int TYPE, int LAYOUT, int M>
__global__ void __launch_bounds__(kRowsThreads) gemv_rows_kernel(const RowsParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* stages = smem;
  float* red = reinterpret_cast<float*>(smem + (size_t)p.stage_bytes * p.nstages);  // [2][4][32][M]
  uint64_t* full = reinterpret_cast<uint64_t*>(red + 2 * kRowsConsumers * 32 * M);
  uint64_t* empty = full + p.nstages;
  __shared__ int s_fail;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // persistent CTA: a contiguous, balanced range of rows, walked in row
  // blocks of R rows x chunks of K; items (row block, chunk) stream through
  // the stage ring without a break at row-block boundaries
  const int64_t r_begin = p.N * blockIdx.x / gridDim.x, r_end = p.N * (blockIdx.x + 1) / gridDim.x;
  const int nrb = (int)((r_end - r_begin + p.R - 1) / p.R);
  const int nitems = nrb * p.nchunks;
  const int ppc_bytes = p.PPS * p.piece_bytes;

  if (tid == 0) {
    s_fail = 0;
    for (int s = 0; s < p.nstages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kRowsConsumers);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == 0) {
    if (lane == 0) {
      auto issue_w = [&](int t, int s) {
        const int rb = t / p.nchunks, c = t - rb * p.nchunks;
        const int64_t row0 = r_begin + (int64_t)rb * p.R;
        const int rows = (int)min((int64_t)p.R, r_end - row0);
        const int64_t off = (int64_t)c * ppc_bytes;
        const int rbytes = (int)min((int64_t)ppc_bytes, p.RB - off);
        const int ng = (int)(min((int64_t)p.PPS, (int64_t)p.npieces - (int64_t)c * p.PPS)) * 8;
        uint8_t* slot = stages + (size_t)s * p.stage_bytes;
        mbar_arrive_expect_tx(&full[s], (uint32_t)(rows * rbytes + M * ng * 80));
        for (int r = 0; r < rows; ++r) bulk_g2s(slot + r * p.pitch, p.w + (row0 + r) * p.RB + off, rbytes, &full[s]);
      };
      auto issue_x = [&](int t, int s) {
        const int rb = t / p.nchunks, c = t - rb * p.nchunks;
        const int ng = (int)(min((int64_t)p.PPS, (int64_t)p.npieces - (int64_t)c * p.PPS)) * 8;
        uint8_t* xs = stages + (size_t)s * p.stage_bytes + p.R * p.pitch;
        for (int m = 0; m < M; ++m)
          bulk_g2s(xs + m * p.xstride, p.xg + m * p.GX + (int64_t)c * p.PPS * 8, ng * 80, &full[s]);
      };
      // weights of the first stages do not depend on the previous kernel
      const int pre = min(nitems, p.nstages);
      for (int t = 0; t < pre; ++t) issue_w(t, t);
      grid_dep_wait();
      grid_dep_launch();
      for (int t = 0; t < pre; ++t) issue_x(t, t);
      for (int t = pre; t < nitems; ++t) {
        const int s = t % p.nstages;
        if (!mbar_wait_bounded(&empty[s], (uint32_t)(((t / p.nstages) - 1) & 1))) {
          s_fail = 1;
          break;
        }
        fence_proxy_async_smem();
        issue_w(t, s);
        issue_x(t, s);
      }
    }
  } else {
    const int cw = warp - 1;
    const int r = lane % p.R, ks = lane / p.R;
    const int lanes_per_piece = kRowsConsumers * p.KS;
    float acc[M];
#pragma unroll
    for (int m = 0; m < M; ++m) acc[m] = 0.f;
    bool ok = true;
    int par = 0;
    for (int t = 0; t < nitems; ++t) {
      const int rb = t / p.nchunks, c = t - rb * p.nchunks;
      const int64_t row0 = r_begin + (int64_t)rb * p.R;
      const int rows = (int)min((int64_t)p.R, r_end - row0);
      const int s = t % p.nstages;
      // after a failed wait, skip the remaining waits but keep every barrier
      if (ok) ok = mbar_wait_bounded(&full[s], (uint32_t)((t / p.nstages) & 1));
      if (ok) {
        const int np = (int)min((int64_t)p.PPS, (int64_t)p.npieces - (int64_t)c * p.PPS);
        const uint8_t* slot = stages + (size_t)s * p.stage_bytes;
        if (r < rows) {
          for (int j = cw * p.KS + ks; j < np; j += lanes_per_piece) {
            Piece<TYPE, LAYOUT, M>::run(slot + r * p.pitch + j * p.piece_bytes, slot + p.R * p.pitch + j * 8 * 80,
                                        p.xstride, acc);
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
      } else {
        s_fail = 1;
      }
      if (c == p.nchunks - 1) {
        // row block done: reduce lane groups (shuffles) and warps (shared)
        float* rd = red + (size_t)par * kRowsConsumers * 32 * M;
#pragma unroll
        for (int m = 0; m < M; ++m) {
          float v = acc[m];
          for (int o = p.R; o < 32; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
          rd[(cw * 32 + lane) * M + m] = v;
          acc[m] = 0.f;
        }
        asm volatile("bar.sync 1, %0;" ::"r"(kRowsConsumers * 32) : "memory");
        const int ct = tid - 32;
        if (ct < rows * M && s_fail == 0) {
          const int rr = ct / M, m = ct - rr * M;
          float v = 0.f;
#pragma unroll
          for (int w = 0; w < kRowsConsumers; ++w) v += rd[(w * 32 + rr) * M + m];
          p.y[(int64_t)m * p.N + row0 + rr] = v;
        }
        par ^= 1;
      }
    }
  }
  __syncthreads();
}

// ---------------------------------------------------------------------------
// Host side
template <int TYPE>
struct PieceGeom;
template <> struct PieceGeom<NSQ_TYPE_Q4_K> { static constexpr int bytes = 144, align_pieces = 1; };
template <> struct PieceGeom<NSQ_TYPE_Q6_K> { static constexpr int bytes = 210, align_pieces = 8; };
template <> struct PieceGeom<NSQ_TYPE_Q4_0> { static constexpr int bytes = 144, align_pieces = 1; };
template <> struct PieceGeom<NSQ_TYPE_Q8_0> { static constexpr int bytes = 272, align_pieces = 1; };

constexpr int kRowsSmemBudget = 64 * 1024;

static int env_int(const char* name, int dflt) {
  const char* v = getenv(name);
  return (v && v[0]) ? atoi(v) : dflt;
}

// Plans a launch; false if the shape is not covered by this kernel (the
// general kernel in gemv.cu then runs it).
template <int TYPE>
static bool plan_rows(int64_t N, int64_t K, int M, int num_sms, RowsParams& p, int& blocks, size_t& smem) {
  using G = PieceGeom<TYPE>;
  if (K % 256) return false;
  const int64_t npieces = K / 256;
  if (npieces % G::align_pieces) return false;
  const int64_t RB = npieces * G::bytes;
  if (RB % 16) return false;
  // rows per block: 8 (four lane groups per warp split each piece range);
  // small matrices use fewer rows so that every SM gets work.  The
  // NSQ_ROWS_* environment variables override the plan (tuning sweeps).
  int R = env_int("NSQ_ROWS_R", 8);
  if (R != 4 && R != 8 && R != 16 && R != 32) R = 8;
  while (R > 4 && (N + R - 1) / R < (int64_t)num_sms) R >>= 1;
  const int KS = 32 / R;
  int PPS = env_int("NSQ_ROWS_PPSM", 1) * kRowsConsumers * KS;
  if (PPS < 1) PPS = kRowsConsumers * KS;
  if (PPS % G::align_pieces) PPS = ((PPS + G::align_pieces - 1) / G::align_pieces) * G::align_pieces;
  if (PPS > npieces) PPS = (int)npieces;
  const int chunk_bytes = PPS * G::bytes;
  const int pitch = ((chunk_bytes + 15) & ~15) + 16;
  const int xstride = PPS * 8 * 80;
  const int stage_bytes = (R * pitch + M * xstride + 127) & ~127;
  int nstages = env_int("NSQ_ROWS_STAGES", 2);
  if (nstages < 2 || nstages > 8) nstages = 2;
  if ((size_t)stage_bytes * nstages > (size_t)kRowsSmemBudget && nstages > 2) nstages = 2;
  smem = (size_t)stage_bytes * nstages + (size_t)2 * kRowsConsumers * 32 * M * 4 + 16 * nstages + 16;
  if (smem > 200 * 1024) return false;
  const int nchunks = (int)((npieces + PPS - 1) / PPS);
  p.N = N; p.K = K; p.RB = RB;
  p.R = R; p.KS = KS; p.PPS = PPS;
  p.piece_bytes = G::bytes; p.chunk_bytes = chunk_bytes; p.pitch = pitch;
  p.nchunks = nchunks; p.npieces = (int)npieces; p.xstride = xstride;
  p.stage_bytes = stage_bytes; p.nstages = nstages; p.GX = K / 32;
  // persistent grid: as many CTAs as fit on the GPU at once, but no more
  // than there are row blocks
  int per_sm = (int)((220 * 1024) / (smem + 1024));
  if (per_sm > 4) per_sm = 4;
  if (per_sm < 1) per_sm = 1;
  const int cps = env_int("NSQ_ROWS_CPS", 0);
  if (cps >= 1 && cps <= per_sm) per_sm = cps;
  int64_t g = (int64_t)num_sms * per_sm;
  const int64_t nrb = (N + R - 1) / R;
  if (g > nrb) g = nrb;
  blocks = (int)g;
  return true;
}

template <int TYPE, int LAYOUT, int M>
static cudaError_t launch_rows(const RowsParams& p, int blocks, size_t smem, cudaStream_t st) {
  auto kern = gemv_rows_kernel<TYPE, LAYOUT, M>;
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
  cfg.blockDim = dim3(kRowsThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

template <int TYPE, int LAYOUT>
static int run_rows_t(const uint8_t* w, const XGroup* xg, float* y, int64_t M, int64_t N, int64_t K, cudaStream_t st,
                      int num_sms) {
  for (int64_t m0 = 0; m0 < M; m0 += 4) {
    const int mm = (int)((M - m0) < 4 ? (M - m0) : 4);
    RowsParams p{};
    int blocks;
    size_t smem;
    if (!plan_rows<TYPE>(N, K, mm, num_sms, p, blocks, smem)) return -1;
    p.w = w;
    p.xg = xg + m0 * (K / 32);
    p.y = y + m0 * N;
    cudaError_t e;
    switch (mm) {
      case 1: e = launch_rows<TYPE, LAYOUT, 1>(p, blocks, smem, st); break;
      case 2: e = launch_rows<TYPE, LAYOUT, 2>(p, blocks, smem, st); break;
      case 3: e = launch_rows<TYPE, LAYOUT, 3>(p, blocks, smem, st); break;
      default: e = launch_rows<TYPE, LAYOUT, 4>(p, blocks, smem, st); break;
    }
    if (e != cudaSuccess) return NSQ_ERR_CUDA;
  }
  return NSQ_OK;
}

// Returns NSQ_OK / an error, or -1 if the shape is not covered (caller falls
// back to the general kernel).
int run_gemv_rows(const uint8_t* w, int type, int layout, const XGroup* xg, float* y, int64_t M, int64_t N,
                  int64_t K, cudaStream_t st, int num_sms) {
  RowsParams probe{};
  int b;
  size_t sm;
  const int mm = (int)(M < 4 ? M : 4);
  switch (type) {
    case NSQ_TYPE_Q4_K:
      if (!plan_rows<NSQ_TYPE_Q4_K>(N, K, mm, num_sms, probe, b, sm)) return -1;
      return run_rows_t<NSQ_TYPE_Q4_K, 0>(w, xg, y, M, N, K, st, num_sms);
    case NSQ_TYPE_Q6_K:
      if (!plan_rows<NSQ_TYPE_Q6_K>(N, K, mm, num_sms, probe, b, sm)) return -1;
      if (layout == NSQ_Q6K_NODESTOR) return run_rows_t<NSQ_TYPE_Q6_K, NSQ_Q6K_NODESTOR>(w, xg, y, M, N, K, st, num_sms);
      return run_rows_t<NSQ_TYPE_Q6_K, NSQ_Q6K_GGML>(w, xg, y, M, N, K, st, num_sms);
    case NSQ_TYPE_Q4_0:
      if (!plan_rows<NSQ_TYPE_Q4_0>(N, K, mm, num_sms, probe, b, sm)) return -1;
      return run_rows_t<NSQ_TYPE_Q4_0, 0>(w, xg, y, M, N, K, st, num_sms);
    case NSQ_TYPE_Q8_0:
      if (!plan_rows<NSQ_TYPE_Q8_0>(N, K, mm, num_sms, probe, b, sm)) return -1;
      return run_rows_t<NSQ_TYPE_Q8_0, 0>(w, xg, y, M, N, K, st, num_sms);
    default: return -1;
  }
}

}  // namespace nsq
