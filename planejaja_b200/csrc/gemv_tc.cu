// gemv_tc.cu -- batched decode GEMV (M = 2..16 tokens) on 5th-generation
// tensor cores (tcgen05), for Q4_K, Q5_K and Q6_K (ggml and NodeStor layouts),
// Q4_0 and Q8_0.
//
//   y[m, n] = sum_k x[m, k] * W[n, k],   x f32 [M x K], W GGUF blocks [N x K]
//
// The per-32 (Q4_K) or per-16 (Q6_K) weight scale is folded into the MMA's A
// operand, so the fp32 epilogue runs once per 256-weight super-block instead
// of once per scale group (the cost that bounds an integer-MMA design):
//
//   Q4_K  w = d * sc_j * q - dmin * m_j       A = sc_j * q        (<= 945)
//   Q5_K  the same with 5-bit q               A = sc_j * q        (<= 1953)
//   Q6_K  w = d * sc_j * (q - 32)             A = sc_j * (q - 32) (|A| <= 4096)
//         (NodeStor layout: sc_j = b_j - 128 and d / 64 in the epilogue)
//   Q4_0  w = d_b * (q - 8)                   A = fp16(d_b * (q - 8))
//   Q8_0  w = d_b * s                         A = fp16(d_b * s)
//
// A is fp16: Q4_K's products are integers below 2048 and exact; Q6_K's are
// exact up to 2048 in magnitude (every product the quantizer here writes)
// and above that rounded to the nearest even integer (relative error at most
// 2^-12 on those weights).  Q4_0 and Q8_0 carry their per-32 block scale in
// A, rounded once to fp16 (relative error at most 2^-11 per weight; the
// epilogue factor is 1).  x enters as two fp16 operands, hi = fp16(x') and
// lo = fp16(x' - hi), where x' = x * 2^-e_{m,s} with one power of two per
// token and super-block chosen so that |x'| < 2^15: hi + lo carries 22 bits.
// One MMA with N = 32 takes both (the hi and lo tiles are adjacent rows of
// one operand); the epilogue adds the two halves of D.  The tensor cores
// accumulate in fp32 (TMEM); the min
// term sum_j m_j T_j (T_j = the sub-block sums of x') is a second MMA with
// K = 8 (padded to 16) into D2.  Per super-block the epilogue adds
//   y += 2^e * (d * D - 32 * dmin * D2)           (T enters as T / 32)
//
// Work split (stream-K): units are (128-row tile, super-block) pairs in
// tile-major order; CTA i of G takes units [U i / G, U (i+1) / G).  A tile
// that spans CTAs is finished by the last of them to arrive (a counter per
// split tile), which sums the partials in CTA order -- deterministic, and no
// CTA ever waits for another.  A CTA that finds every other partial of the
// tile in place already finishes it from its registers.
//
// The fp16 A operand lives in tensor memory by default: the dequant warps
// write it with tcgen05.st (each warp into its own 32-lane quadrant) and the
// MMA reads it in its A-from-TMEM form, so shared memory carries only the
// raw columns, the x tiles and the min-term tiles (NSQ_TC_A=0 puts A in
// 128B-swizzled shared-memory tiles instead).  TMEM: four accumulator slots
// (D and D2, 64 columns each) and two unit slots of A (128 columns each).
//
// Warp roles (512 threads, one CTA per SM):
//   warp 0      raw producer: one 2-D TMA box [128 rows x one super-block
//               column] of the GGUF bytes per unit (evict-first in L2), the
//               first ones before the setup sync; with a short ring, an L2
//               prefetch of the column that takes the slot next
//   warps 1, 3  MMA issue, one thread each, alternate units (warp 1 owns
//               TMEM).  A thread that issues, commits and waits in turn
//               keeps the tensor pipe busy less than half the time; two
//               issuers overlap each other's waits
//   warp 2      B producer: per unit the four x tiles (hi, lo), the
//               min-term tile and the token scales, from the workspace the
//               preparation kernel wrote
//   warps 4..7  epilogue (TMEM lane quadrant = warp % 4, one row per thread)
//   warps 8..15 dequant: raw bytes -> fp16 A, the min-term A tile and the
//               row's d / dmin; A in TMEM: warp (r, h) writes row 32r + lane
//               (r = warp % 4), K stages 2h and 2h + 1; A in shared memory:
//               warp (q, h) writes K stage q of rows [64h, 64h + 64)
// Every wait is bounded (%globaltimer); a wait that gives up records
// NSQ_ERR_TIMEOUT and the kernel winds down.  With a row-sharded exchange
// (P > 1) the outputs go into every rank's exchange buffer and the grid's
// last CTA publishes the count, as in the fused kernel.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "nsq_common.cuh"
#include "tcgen05.cuh"

namespace nsq {

constexpr int TC_BM = 128;                   // weight rows per tile (UMMA M)
constexpr int TC_BN = 16;                    // UMMA N: tokens, zero-padded
constexpr int TC_THREADS = 512;
constexpr int TC_EPI_WARP0 = 4;
constexpr int TC_DQ_WARP0 = 8;
constexpr int TC_DQ_WARPS = 8;
constexpr int TC_A_BYTES = TC_BM * 128;      // fp16 [128 x 64], 16 KB
constexpr int TC_B_BYTES = 2 * TC_BN * 128;  // fp16 hi [16 x 64] + lo [16 x 64], 4 KB
constexpr int TC_COL_BYTES = 5120;           // workspace stride: B2 hi + lo (4 KB), 16 token scales, pad
constexpr int TC_B2_BYTES = 4096;            // min-term tile (hi + lo) in shared memory
constexpr int TC_UA_BYTES = 4 * TC_A_BYTES;  // a unit's four A stage tiles, 64 KB
constexpr int TC_UB_BYTES = 4 * TC_B_BYTES + TC_B2_BYTES;  // its four x tiles and the min-term tile, 20 KB
constexpr int TC_NACC = 4;                   // units in flight between the MMA and the epilogue
constexpr int TC_MMA_WARPS = 2;              // MMA issuers (warps 1 and 3): unit n -> issuer n % 2
constexpr int TC_ACC_COLS = 64;              // per unit: D (hi | lo, 32 columns) and the min-term D2
constexpr int TC_SCL_STAGES = 16;            // token scales (64 B per unit)
constexpr int TC_GMAX = 256;                 // most CTAs a launch uses
constexpr int TC_TMEM_COLS = TC_NACC * TC_ACC_COLS;
constexpr int TC_A_TMEM_COLS = 128;          // a unit's fp16 A in TMEM: 256 K per lane, two per column
constexpr int TC_TMEM_COLS_A = TC_TMEM_COLS + 2 * TC_A_TMEM_COLS;  // with two unit slots of A in TMEM: 512
constexpr int TC_SMEM_LIMIT = 232448;

enum : int { kTcQ4K = 0, kTcQ6KG = 1, kTcQ40 = 2, kTcQ80 = 3, kTcQ6KN = 4, kTcQ5KG = 5, kTcQ5KN = 6, kTcMixed = -1 };

struct TcSeg {
  const uint8_t* w;
  float* y;
  int64_t N, RB;  // rows, bytes per row
  int code, CB;   // format, bytes per super-block column
  int tile0;      // first tile of this segment in the concatenated tile list
};

struct TcParams {
  CUtensorMap wmap[NSQ_MAX_SEGMENTS];  // W as [N rows x RB/2] u16, box [pitch/2 x 128]
  TcSeg seg[NSQ_MAX_SEGMENTS];
  int nseg, T, NSB, M;
  int64_t U;        // units = T * NSB
  int pitch;        // raw bytes per row per unit in shared memory
  int raw_stages, unit_slots;  // raw columns in flight; units of A and B tiles in shared memory
  const uint8_t* ws_b;    // [NSB * 4][hi 2 KB | lo 2 KB]
  const uint8_t* ws_col;  // [NSB][B2 hi 2 KB | B2 lo 2 KB | 16 f32 scales | pad]
  float* ws_part;         // [2 * TC_GMAX][128 rows][16 tokens]
  uint32_t* ws_cnt;       // [TC_GMAX]
  // Row-sharded exchange (P > 1), as in the fused kernel: every output row
  // goes into the exchange buffer of each of the P ranks (segment s: y[M x
  // xnfull] f32 at byte kXchgCtlBytes + xoff[s], this rank's rows from
  // xrow0[s]), and the grid's last CTA publishes this rank's count.
  int P, rank;
  uint8_t* xbuf[NSQ_MAX_RANKS];
  int64_t xrow0[NSQ_MAX_SEGMENTS], xnfull[NSQ_MAX_SEGMENTS], xoff[NSQ_MAX_SEGMENTS];
};

// Formats with a min term (Q4_K, Q5_K) need the min-term tiles and MMA; a
// single-format launch of Q6_K, Q4_0 or Q8_0 leaves them out, and the shared
// memory they free holds a second unit slot.
template <int CODE>
constexpr bool tc_has_min() {
  return CODE == kTcQ4K || CODE == kTcQ5KG || CODE == kTcQ5KN || CODE == kTcMixed;
}
__host__ __device__ constexpr int tc_ub_bytes(bool has_min) { return has_min ? TC_UB_BYTES : 4 * TC_B_BYTES; }

// Workspace of the batched path: counters, B tiles, min-term tiles, partials.
size_t tc_workspace_bytes(int64_t K) {
  const int64_t nsb = K / 256;
  return 1024 + (size_t)nsb * 4 * TC_B_BYTES + (size_t)nsb * TC_COL_BYTES + (size_t)2 * TC_GMAX * TC_BM * TC_BN * 4;
}

__device__ __forceinline__ void tc_grid_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void tc_grid_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------------------
// Activation preparation: one warp per (token, super-block), 8 values per lane.
__global__ void __launch_bounds__(256) tc_prep_kernel(const float* __restrict__ x, int M, int64_t K, int NSB,
                                                      uint8_t* __restrict__ ws_b, uint8_t* __restrict__ ws_col,
                                                      uint32_t* __restrict__ ws_cnt) {
  tc_grid_wait();  // x comes from the previous kernel; the workspace may still be read by it
  tc_grid_launch();
  if (blockIdx.x == 0)
    for (int i = threadIdx.x; i < TC_GMAX; i += blockDim.x) ws_cnt[i] = 0u;
  const int wg = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
  const int t = wg % TC_BN, c = wg / TC_BN;
  if (c >= NSB) return;
  float v[8];
  if (t < M) {
    const float* src = x + (int64_t)t * K + 256 * (int64_t)c + 8 * lane;
    if ((reinterpret_cast<uintptr_t>(src) & 15) == 0) {
      const float4 a = *reinterpret_cast<const float4*>(src), b = *reinterpret_cast<const float4*>(src + 4);
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = src[i];
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = 0.f;
  }
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
  for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  // e: amax * 2^-e < 2^15 (amax = f * 2^E, f in [0.5, 1)), at least -126
  int e = 0;
  if (amax > 0.f) {
    const int E = (int)((__float_as_uint(amax) >> 23) & 0xFF) - 126;
    e = max(E - 15, -126);
  }
  const float inv = __uint_as_float((uint32_t)(127 - e) << 23);  // 2^-e
  const float scl = __uint_as_float((uint32_t)(127 + e) << 23);  // 2^e
  uint32_t hw[4], lw[4];
  float ts = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float a = v[2 * i] * inv, b = v[2 * i + 1] * inv;
    ts += a;
    ts += b;
    const __half ha = __float2half_rn(a), hb = __float2half_rn(b);
    const __half la = __float2half_rn(a - __half2float(ha)), lb = __float2half_rn(b - __half2float(hb));
    hw[i] = (uint32_t)__half_as_ushort(ha) | ((uint32_t)__half_as_ushort(hb) << 16);
    lw[i] = (uint32_t)__half_as_ushort(la) | ((uint32_t)__half_as_ushort(lb) << 16);
  }
  // B tiles of 64-wide K stage 4c + q: row t, 16-byte chunk k8, 128B swizzle
  const int q = lane >> 3, k8 = lane & 7;
  uint8_t* bt = ws_b + (int64_t)(4 * c + q) * TC_B_BYTES + t * 128 + ((k8 ^ (t & 7)) << 4);
  *reinterpret_cast<uint4*>(bt) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
  *reinterpret_cast<uint4*>(bt + TC_B_BYTES / 2) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
  // sub-block sums T_j (j = lane / 4) as T / 32, split hi / lo, at K = j of the min-term tile
  ts += __shfl_xor_sync(0xffffffffu, ts, 1);
  ts += __shfl_xor_sync(0xffffffffu, ts, 2);
  const float tq = ts * 0.03125f;
  const __half th = __float2half_rn(tq), tl = __float2half_rn(tq - __half2float(th));
  uint8_t* col = ws_col + (int64_t)c * TC_COL_BYTES;
  const int j = lane >> 2;
  if ((lane & 3) == 0) {
    const int off = t * 128 + ((0 ^ (t & 7)) << 4) + 2 * j;
    *reinterpret_cast<__half*>(col + off) = th;
    *reinterpret_cast<__half*>(col + 2048 + off) = tl;
  }
  if (lane == 1) {  // K 8..15 of the min-term tile are zero
    const int off = t * 128 + ((1 ^ (t & 7)) << 4);
    *reinterpret_cast<uint4*>(col + off) = make_uint4(0, 0, 0, 0);
    *reinterpret_cast<uint4*>(col + 2048 + off) = make_uint4(0, 0, 0, 0);
  }
  if (lane == 2) reinterpret_cast<float*>(col + 4096)[t] = t < M ? scl : 0.f;
}

// ---------------------------------------------------------------------------
// Dequant of one row's share of a 64-wide K stage into fp16 A chunks.
// Thread (row, pp) writes chunks {pp, pp + 4} (pair pp) and {pp + 2, pp + 6}
// (pair pp + 2); chunk k8 holds K 8*k8 .. 8*k8 + 7 of the stage in natural
// order.  `raw` points at the row's super-block bytes.
__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 bits_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// (v0, v1) fp16 with v = base + byte: PRMT of two bytes of `bytes` beside the
// constant high byte (0x64 -> 1024 + b, 0x54 -> 64 + b / 16).
__device__ __forceinline__ __half2 magic2(uint32_t bytes, uint32_t hi_bytes, uint32_t sel) {
  return bits_h2(__byte_perm(bytes, hi_bytes, sel));
}

// Q4_K stage q: pair p = bytes qs[32q + 8p .. +8): low nibbles are chunk p
// (sub-block 2q), high nibbles chunk p + 4 (sub-block 2q + 1).
__device__ __forceinline__ void q4k_pair(const uint8_t* raw, int q, int p, __half2 s0, __half2 b0, __half2 s1,
                                         __half2 b1, uint4& lo_chunk, uint4& hi_chunk) {
  const uint2 w = *reinterpret_cast<const uint2*>(raw + 16 + 32 * q + 8 * p);
  const uint32_t L0 = w.x & 0x0F0F0F0Fu, L1 = w.y & 0x0F0F0F0Fu;
  const uint32_t H0 = (w.x >> 4) & 0x0F0F0F0Fu, H1 = (w.y >> 4) & 0x0F0F0F0Fu;
  const uint32_t K64 = 0x64646464u;
  // (1024 + q) * sc - 1024 * sc = sc * q exactly (one rounding of an integer <= 945)
  lo_chunk.x = h2_bits(__hfma2(magic2(L0, K64, 0x4140), s0, b0));
  lo_chunk.y = h2_bits(__hfma2(magic2(L0, K64, 0x4342), s0, b0));
  lo_chunk.z = h2_bits(__hfma2(magic2(L1, K64, 0x4140), s0, b0));
  lo_chunk.w = h2_bits(__hfma2(magic2(L1, K64, 0x4342), s0, b0));
  hi_chunk.x = h2_bits(__hfma2(magic2(H0, K64, 0x4140), s1, b1));
  hi_chunk.y = h2_bits(__hfma2(magic2(H0, K64, 0x4342), s1, b1));
  hi_chunk.z = h2_bits(__hfma2(magic2(H1, K64, 0x4140), s1, b1));
  hi_chunk.w = h2_bits(__hfma2(magic2(H1, K64, 0x4342), s1, b1));
}

// Q5_K stage q, pair p: Q4_K's nibbles (qs at byte 48) widened by the fifth
// bit of each weight -- ggml: bit j of qh[l]; NodeStor (q5_k.rs:57-70): bit
// l % 8 of qh[8 (j >> 1) + 4 (j & 1) + l / 8] (qh at byte 16) -- so that
// A = sc * q (at most 63 * 31 = 1953) stays exact in fp16.
template <bool NODESTOR>
__device__ __forceinline__ void q5k_pair(const uint8_t* raw, int q, int p, __half2 s0, __half2 b0, __half2 s1,
                                         __half2 b1, uint4& lo_chunk, uint4& hi_chunk) {
  const uint2 w = *reinterpret_cast<const uint2*>(raw + 48 + 32 * q + 8 * p);
  uint32_t L0 = w.x & 0x0F0F0F0Fu, L1 = w.y & 0x0F0F0F0Fu;
  uint32_t H0 = (w.x >> 4) & 0x0F0F0F0Fu, H1 = (w.y >> 4) & 0x0F0F0F0Fu;
  if constexpr (NODESTOR) {
    const uint32_t bl = raw[16 + 8 * q + p], bh = raw[16 + 8 * q + 4 + p];
    L0 |= spread4(bl & 0xF) << 4;
    L1 |= spread4(bl >> 4) << 4;
    H0 |= spread4(bh & 0xF) << 4;
    H1 |= spread4(bh >> 4) << 4;
  } else {
    const uint2 hq = *reinterpret_cast<const uint2*>(raw + 16 + 8 * p);
    L0 |= ((hq.x >> (2 * q)) & 0x01010101u) << 4;
    L1 |= ((hq.y >> (2 * q)) & 0x01010101u) << 4;
    H0 |= ((hq.x >> (2 * q + 1)) & 0x01010101u) << 4;
    H1 |= ((hq.y >> (2 * q + 1)) & 0x01010101u) << 4;
  }
  const uint32_t K64 = 0x64646464u;
  lo_chunk.x = h2_bits(__hfma2(magic2(L0, K64, 0x4140), s0, b0));
  lo_chunk.y = h2_bits(__hfma2(magic2(L0, K64, 0x4342), s0, b0));
  lo_chunk.z = h2_bits(__hfma2(magic2(L1, K64, 0x4140), s0, b0));
  lo_chunk.w = h2_bits(__hfma2(magic2(L1, K64, 0x4342), s0, b0));
  hi_chunk.x = h2_bits(__hfma2(magic2(H0, K64, 0x4140), s1, b1));
  hi_chunk.y = h2_bits(__hfma2(magic2(H0, K64, 0x4342), s1, b1));
  hi_chunk.z = h2_bits(__hfma2(magic2(H1, K64, 0x4140), s1, b1));
  hi_chunk.w = h2_bits(__hfma2(magic2(H1, K64, 0x4342), s1, b1));
}

// Q4_K 6-bit scale / min j of the packed 12 bytes (get_scale_min_k4,
// q4_k.rs:120-131): sc in the low byte, m in the next.
__device__ __forceinline__ uint32_t q4k_scale_min(uint32_t S0, uint32_t S1, uint32_t S2, int j) {
  if (j < 4) return ((S0 >> (8 * j)) & 63) | (((S1 >> (8 * j)) & 63) << 8);
  const int sh = 8 * (j - 4);
  const uint32_t b2 = (S2 >> sh) & 0xFF, b0 = (S0 >> sh) & 0xFF, b1 = (S1 >> sh) & 0xFF;
  return ((b2 & 0xF) | ((b0 >> 6) << 4)) | (((b2 >> 4) | ((b1 >> 6) << 4)) << 8);
}

// Q6_K (ggml) stage q = 64 weights of half n = q / 2: chunk k8 = p + 4h is
// group j = 2(q & 1) + h, elements l = 8p .. 8p + 7: ql[64n + 32(j & 1) + l]
// nibble (q & 1), qh[32n + l] bits 2j, scale sc[8n + 2j + l / 16].  The 6-bit
// value enters as fp16 64 + 4q/16 and (4 sc) * v - 288 sc = sc (q - 32).
// The stage's four int8 scales are one word (bytes 8n + 2j0 .. + 3): each
// byte s + 128 beside 0x64 is fp16 1024 + s + 128, less 1152 it is s, and
// 4 s and -288 s are exact in fp16.  `raw` is 2-byte aligned inside the
// column's 16-byte span; ALIGNED4 when it is 4-byte aligned (the same for
// every row of a unit), else the byte runs are read as shifted words.
template <bool ALIGNED4>
__device__ __forceinline__ void q6k_stage(const uint8_t* raw, int q, uint4 (&ch)[8]) {
  const int n = q >> 1, j0 = 2 * (q & 1), sh = 4 * (q & 1);
  uint32_t la[8], lb[8], hh[8], scw;
  if constexpr (ALIGNED4) {
    const uint32_t* w = reinterpret_cast<const uint32_t*>(raw);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      la[i] = w[16 * n + i];
      lb[i] = w[16 * n + 8 + i];
      hh[i] = w[32 + 8 * n + i];
    }
    scw = w[48 + 2 * n + (j0 >> 1)];
  } else {
    uint32_t sw1[1];
    ld_words_unaligned<8>(raw + 64 * n, la);
    ld_words_unaligned<8>(raw + 64 * n + 32, lb);
    ld_words_unaligned<8>(raw + 128 + 32 * n, hh);
    ld_words_unaligned<1>(raw + 192 + 8 * n + 2 * j0, sw1);
    scw = sw1[0];
  }
  const uint32_t sb = scw ^ 0x80808080u;
  const __half2 k1152 = __float2half2_rn(1152.f);
  const __half2 sA = __hsub2(magic2(sb, 0x64646464u, 0x4140), k1152);  // group j0: l < 16, l >= 16
  const __half2 sB = __hsub2(magic2(sb, 0x64646464u, 0x4342), k1152);  // group j0 + 1
  const __half2 s4A = __hmul2(sA, __float2half2_rn(4.f)), s4B = __hmul2(sB, __float2half2_rn(4.f));
  const __half2 cA = __hmul2(sA, __float2half2_rn(-288.f)), cB = __hmul2(sB, __float2half2_rn(-288.f));
  const uint32_t K54 = 0x54545454u;
#pragma unroll
  for (int w = 0; w < 8; ++w) {  // elements 4w .. 4w + 3 of both groups
    const __half2 ma = w < 4 ? __low2half2(s4A) : __high2half2(s4A), ca = w < 4 ? __low2half2(cA) : __high2half2(cA);
    const __half2 mb = w < 4 ? __low2half2(s4B) : __high2half2(s4B), cb = w < 4 ? __low2half2(cB) : __high2half2(cB);
    // 4q as bytes: ((ql >> shift) & 15) << 2 | ((qh >> 2j) & 3) << 6
    const uint32_t qa = (((la[w] >> sh) & 0x0F0F0F0Fu) << 2) | (((hh[w] >> (2 * j0)) & 0x03030303u) << 6);
    const uint32_t qb = (((lb[w] >> sh) & 0x0F0F0F0Fu) << 2) | (((hh[w] >> (2 * j0 + 2)) & 0x03030303u) << 6);
    const uint32_t a01 = h2_bits(__hfma2(magic2(qa, K54, 0x4140), ma, ca));
    const uint32_t a23 = h2_bits(__hfma2(magic2(qa, K54, 0x4342), ma, ca));
    const uint32_t b01 = h2_bits(__hfma2(magic2(qb, K54, 0x4140), mb, cb));
    const uint32_t b23 = h2_bits(__hfma2(magic2(qb, K54, 0x4342), mb, cb));
    if (w & 1) {
      ch[w >> 1].z = a01; ch[w >> 1].w = a23; ch[4 + (w >> 1)].z = b01; ch[4 + (w >> 1)].w = b23;
    } else {
      ch[w >> 1].x = a01; ch[w >> 1].y = a23; ch[4 + (w >> 1)].x = b01; ch[4 + (w >> 1)].y = b23;
    }
  }
}

// Q4_0 / Q8_0 stage q: blocks 2q and 2q + 1 of the 256-weight column, whose
// scale d (fp16) is folded into the operand: A = fp16(d * (q - 8)) or
// fp16(d * s).  The magic 1024 + byte less 1032 (Q4_0) or 1152 (Q8_0, the
// int8 as byte s + 128) is q - 8 or s exactly, and one multiply by d rounds
// once (relative error at most 2^-11 per weight, as for any fp16 weight).
// The column starts 16-byte aligned and blocks are 18 / 34 bytes, so block
// 2q's quants sit 2 bytes past a word boundary and block 2q + 1's are aligned.
// Chunk k8 holds K 8 k8 .. 8 k8 + 7 of the stage.
__device__ __forceinline__ uint32_t q_half2(uint32_t bytes, uint32_t sel, __half2 off, __half2 d) {
  return h2_bits(__hmul2(__hadd2(magic2(bytes, 0x64646464u, sel), off), d));
}
__device__ __forceinline__ uint4 q_chunk(uint32_t w0, uint32_t w1, __half2 off, __half2 d) {
  return make_uint4(q_half2(w0, 0x4140, off, d), q_half2(w0, 0x4342, off, d), q_half2(w1, 0x4140, off, d),
                    q_half2(w1, 0x4342, off, d));
}
__device__ __forceinline__ void q40_stage(const uint8_t* raw, int q, uint4 (&ch)[8]) {
  const uint32_t* w = reinterpret_cast<const uint32_t*>(raw + 36 * q);
  uint32_t v[9];
#pragma unroll
  for (int i = 0; i < 9; ++i) v[i] = w[i];
  const __half2 off = __float2half2_rn(-1032.f);
  // block 2q: d in bytes 0..1, quants 2..17; block 2q + 1: d in 18..19, quants 20..35
  const __half2 dA = __half2half2(__ushort_as_half((unsigned short)(v[0] & 0xFFFFu)));
  const __half2 dB = __half2half2(__ushort_as_half((unsigned short)(v[4] >> 16)));
  uint32_t qa[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) qa[i] = __byte_perm(v[i], v[i + 1], 0x5432);
  const uint32_t L = 0x0F0F0F0Fu;
  ch[0] = q_chunk(qa[0] & L, qa[1] & L, off, dA);                // weights 0..7: low nibbles of quants 0..7
  ch[1] = q_chunk(qa[2] & L, qa[3] & L, off, dA);                // 8..15
  ch[2] = q_chunk((qa[0] >> 4) & L, (qa[1] >> 4) & L, off, dA);  // 16..23: high nibbles of quants 0..7
  ch[3] = q_chunk((qa[2] >> 4) & L, (qa[3] >> 4) & L, off, dA);  // 24..31
  ch[4] = q_chunk(v[5] & L, v[6] & L, off, dB);
  ch[5] = q_chunk(v[7] & L, v[8] & L, off, dB);
  ch[6] = q_chunk((v[5] >> 4) & L, (v[6] >> 4) & L, off, dB);
  ch[7] = q_chunk((v[7] >> 4) & L, (v[8] >> 4) & L, off, dB);
}
__device__ __forceinline__ void q80_stage(const uint8_t* raw, int q, uint4 (&ch)[8]) {
  const uint32_t* w = reinterpret_cast<const uint32_t*>(raw + 68 * q);
  uint32_t v[17];
#pragma unroll
  for (int i = 0; i < 17; ++i) v[i] = w[i];
  const __half2 off = __float2half2_rn(-1152.f);
  const uint32_t F = 0x80808080u;  // int8 s -> byte s + 128
  // block 2q: d in bytes 0..1, quants 2..33; block 2q + 1: d in 34..35, quants 36..67
  const __half2 dA = __half2half2(__ushort_as_half((unsigned short)(v[0] & 0xFFFFu)));
  const __half2 dB = __half2half2(__ushort_as_half((unsigned short)(v[8] >> 16)));
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint32_t a0 = __byte_perm(v[2 * k], v[2 * k + 1], 0x5432) ^ F;
    const uint32_t a1 = __byte_perm(v[2 * k + 1], v[2 * k + 2], 0x5432) ^ F;
    ch[k] = q_chunk(a0, a1, off, dA);
    ch[4 + k] = q_chunk(v[9 + 2 * k] ^ F, v[10 + 2 * k] ^ F, off, dB);
  }
}

// Q6_K, NodeStor layout (dequant_q6k.comp:50-99), stage q = elements
// 64q .. 64q + 63: element i is nibble (i & 1) of ql[i >> 1], bits 2(i & 3) of
// qh[128 + (i >> 2)], scale (b[192 + (i >> 4)] - 128) / 64, d at 208.  With
// sc = b - 128, A = sc * (q - 32) as for the ggml layout (the same fp16
// magic and one hfma2), and the epilogue factor is d / 64.  `raw` is 2-byte
// aligned (210-byte columns).
__device__ __forceinline__ void q6kn_stage(const uint8_t* raw, int q, uint4 (&ch)[8]) {
  uint32_t ql[8], qh[4], scw[1];
  ld_words_unaligned<8>(raw + 32 * q, ql);
  ld_words_unaligned<4>(raw + 128 + 16 * q, qh);
  ld_words_unaligned<1>(raw + 192 + 4 * q, scw);
  const uint32_t K54 = 0x54545454u;
#pragma unroll
  for (int k8 = 0; k8 < 8; ++k8) {
    const int sc = (int)((scw[0] >> (8 * (k8 >> 1))) & 0xFF) - 128;
    const __half2 s4 = __half2half2(__int2half_rn(4 * sc)), c = __half2half2(__int2half_rn(-288 * sc));
    const uint32_t h16 = (qh[k8 >> 1] >> (16 * (k8 & 1))) & 0xFFFFu;
    uint32_t b4[2];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      // elements 4hh .. 4hh + 3 of the chunk: low nibbles spread to bytes, high bits beside them
      const uint32_t tt = __byte_perm(ql[k8] >> (16 * hh), 0, 0x1100);
      const uint32_t lo4 = (tt & 0x000F000Fu) | ((tt >> 4) & 0x0F000F00u);
      const uint32_t h = (h16 >> (8 * hh)) & 0xFFu;
      const uint32_t hi2 = (h | (h << 6) | (h << 12) | (h << 18)) & 0x03030303u;
      b4[hh] = (lo4 | (hi2 << 4)) << 2;  // 4q as bytes
    }
    ch[k8] = make_uint4(h2_bits(__hfma2(magic2(b4[0], K54, 0x4140), s4, c)),
                        h2_bits(__hfma2(magic2(b4[0], K54, 0x4342), s4, c)),
                        h2_bits(__hfma2(magic2(b4[1], K54, 0x4140), s4, c)),
                        h2_bits(__hfma2(magic2(b4[1], K54, 0x4342), s4, c)));
  }
}

// Walk of a CTA's units: segment, tile within it and super-block column of
// unit u0 + n, advanced one unit at a time (the per-unit 64-bit division of a
// direct lookup cost every role's threads more integer work than the dequant
// of a unit's rows).
struct TcCursor {
  int sg = 0, tl = 0, c = 0, t = 0;
  __device__ void init(const TcParams& p, int64_t u) {
    // 32-bit: the host keeps U * (G + 1) below 2^32
    t = (int)((uint32_t)u / (uint32_t)p.NSB);
    c = (int)((uint32_t)u - (uint32_t)t * (uint32_t)p.NSB);
    sg = 0;
    while (sg + 1 < p.nseg && t >= p.seg[sg + 1].tile0) ++sg;
    tl = t - p.seg[sg].tile0;
  }
  __device__ void next(const TcParams& p) {
    if (++c < p.NSB) return;
    c = 0;
    ++t;
    ++tl;
    while (sg + 1 < p.nseg && t >= p.seg[sg + 1].tile0) {
      ++sg;
      tl = t - p.seg[sg].tile0;
    }
  }
};
// Use j of a ring of R slots, one use at a time: slot j % R, phase parity (j / R) & 1.
struct TcRing {
  int R, slot;
  uint32_t par;
  __device__ explicit TcRing(int r) : R(r), slot(0), par(0u) {}
  __device__ void next() {
    if (++slot == R) {
      slot = 0;
      par ^= 1u;
    }
  }
};

// Output y[m, nrow] of segment sg: to the segment's y, or (row-sharded
// exchange) into every rank's exchange buffer.
__device__ __forceinline__ void tc_store_y(const TcParams& p, const TcSeg& S, int sg, int m, int64_t nrow, float v) {
  if (p.P > 1) {
    const int64_t idx = (int64_t)m * p.xnfull[sg] + p.xrow0[sg] + nrow;
    for (int pr = 0; pr < p.P; ++pr) reinterpret_cast<float*>(p.xbuf[pr] + kXchgCtlBytes + p.xoff[sg])[idx] = v;
  } else {
    S.y[(int64_t)m * S.N + nrow] = v;
  }
}

// First unit of CTA i, and the CTA owning unit u (unit ranges [U i / G,
// U (i+1) / G)), in 32-bit arithmetic: the host keeps U * (G + 1) below 2^32.
__device__ __forceinline__ int64_t tc_first(int64_t U, int i, int G) {
  return (int64_t)(((uint32_t)U * (uint32_t)i) / (uint32_t)G);
}
__device__ __forceinline__ int tc_owner(int64_t u, int64_t U, int G) {
  return (int)(((uint32_t)(u + 1) * (uint32_t)G - 1u) / (uint32_t)U);
}

// One row's K stage q (64 weights) of a unit: the fp16 A chunks in natural K
// order (chunk k8 = K 8 k8 .. 8 k8 + 7 of the stage), word q of the row's
// min-term chunk a2c (Q4_K / Q5_K: the mins of sub-blocks 2q and 2q + 1, else
// zero), for q == 0 the row's epilogue factors (d, 32 dmin), and for q == 1
// the zero chunk beside the min-term chunk.
template <int CODE>
__device__ __forceinline__ void tc_stage(int code, const uint8_t* raw, int q, int off16, uint8_t* a2row, int a2c,
                                         int sw, float2* dsc_row, uint4 (&ch)[8]) {
  constexpr bool HM = tc_has_min<CODE>();
  if (code == kTcQ4K || code == kTcQ5KG || code == kTcQ5KN) {
    // Q4_K and Q5_K share the header: d, dmin, the packed 6-bit scales and mins
    const uint4 hdr = *reinterpret_cast<const uint4*>(raw);
    // bytes sc_2q, m_2q, sc_2q+1, m_2q+1 (each below 64): fp16 1024 + byte
    // less 1024 gives each exactly
    const uint32_t smw = q4k_scale_min(hdr.y, hdr.z, hdr.w, 2 * q) | (q4k_scale_min(hdr.y, hdr.z, hdr.w, 2 * q + 1) << 16);
    const __half2 k1024 = __float2half2_rn(1024.f);
    const __half2 scs = __hsub2(magic2(smw, 0x64646464u, 0x4240), k1024);
    const __half2 mns = __hsub2(magic2(smw, 0x64646464u, 0x4341), k1024);
    *reinterpret_cast<uint32_t*>(a2row + ((a2c ^ sw) << 4) + 4 * q) = h2_bits(mns);
    if (q == 0) {
      const float d = h2f((uint16_t)(hdr.x & 0xFFFF)), dmin = h2f((uint16_t)(hdr.x >> 16));
      *dsc_row = make_float2(d, 32.0f * dmin);
    }
    const __half2 s0 = __low2half2(scs), s1 = __high2half2(scs);
    const __half2 bb = __hmul2(scs, __float2half2_rn(-1024.f));
    const __half2 b0 = __low2half2(bb), b1 = __high2half2(bb);
    if (code == kTcQ4K) {
#pragma unroll
      for (int pp = 0; pp < 4; ++pp) q4k_pair(raw, q, pp, s0, b0, s1, b1, ch[pp], ch[pp + 4]);
    } else if (code == kTcQ5KG) {
#pragma unroll
      for (int pp = 0; pp < 4; ++pp) q5k_pair<false>(raw, q, pp, s0, b0, s1, b1, ch[pp], ch[pp + 4]);
    } else {
#pragma unroll
      for (int pp = 0; pp < 4; ++pp) q5k_pair<true>(raw, q, pp, s0, b0, s1, b1, ch[pp], ch[pp + 4]);
    }
  } else if (code == kTcQ6KG) {
    if (HM) *reinterpret_cast<uint32_t*>(a2row + ((a2c ^ sw) << 4) + 4 * q) = 0u;
    if (q == 0) *dsc_row = make_float2(h2f((uint16_t)ld_u16(raw + 208)), 0.f);
    if ((off16 & 3) == 0) q6k_stage<true>(raw, q, ch);
    else q6k_stage<false>(raw, q, ch);
  } else if (code == kTcQ6KN) {
    if (HM) *reinterpret_cast<uint32_t*>(a2row + ((a2c ^ sw) << 4) + 4 * q) = 0u;
    if (q == 0) *dsc_row = make_float2(h2f((uint16_t)ld_u16(raw + 208)) * 0.015625f, 0.f);
    q6kn_stage(raw, q, ch);
  } else {
    // Q4_0 / Q8_0: the block scales are in A, no min term
    if (HM) *reinterpret_cast<uint32_t*>(a2row + ((a2c ^ sw) << 4) + 4 * q) = 0u;
    if (q == 0) *dsc_row = make_float2(1.0f, 0.f);
    if (code == kTcQ40) q40_stage(raw, q, ch);
    else q80_stage(raw, q, ch);
  }
  if (HM && q == 1) *reinterpret_cast<uint4*>(a2row + (((a2c + 1) ^ sw) << 4)) = make_uint4(0, 0, 0, 0);
}

template <int CODE, bool ATM>
__global__ void __launch_bounds__(TC_THREADS, 1) gemv_tc_kernel(const __grid_constant__ TcParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int US = p.unit_slots, RS = p.raw_stages, PITCH = p.pitch;
  // 1024-aligned swizzled tiles first: per unit slot the four A stage tiles
  // and the B tiles (four x stages, then the min-term tile); the min-term A
  // tile (4 accumulator slots, 16 K columns each)
  uint8_t* a_sm = smem;
  constexpr bool HM = tc_has_min<CODE>();
  constexpr int UB = tc_ub_bytes(HM);
  uint8_t* b_sm = a_sm + (ATM ? 0 : US * TC_UA_BYTES);  // A in TMEM: no A tiles here
  uint8_t* a2_sm = b_sm + US * UB;
  float* scl_sm = reinterpret_cast<float*>(a2_sm + (HM ? TC_A_BYTES : 0));  // [16][16]
  float2* dsc = reinterpret_cast<float2*>(scl_sm + TC_SCL_STAGES * TC_BN);  // [4][128] (d, 32 dmin)
  uint8_t* raw_sm = reinterpret_cast<uint8_t*>(dsc + TC_NACC * TC_BM);
  const uint32_t RAW_BYTES = (uint32_t)(TC_BM * PITCH);
  // A unit slot is filled by the dequant warps (afull) and the B producer
  // (bfull) and freed by one commit of its MMA thread (uempty).  The full
  // barriers come one set per MMA thread (unit n fills set n % 2): with one
  // unit slot both threads use its data in turn, but each full barrier is
  // waited on by one thread, in order, so a parity wait never sees a phase
  // two ahead of the one it waits for.
  uint64_t* afull = reinterpret_cast<uint64_t*>(raw_sm + RS * RAW_BYTES);  // [thread][US]
  uint64_t* bfull = afull + TC_MMA_WARPS * US;                             // [thread][US]
  uint64_t* uempty = bfull + TC_MMA_WARPS * US;                            // [US]
  uint64_t* scl_full = uempty + US;
  uint64_t* scl_empty = scl_full + TC_SCL_STAGES;
  uint64_t* a2_full = scl_empty + TC_SCL_STAGES;
  uint64_t* a2_empty = a2_full + TC_NACC;
  uint64_t* acc_full = a2_empty + TC_NACC;
  uint64_t* acc_empty = acc_full + TC_NACC;
  uint64_t* raw_full = acc_empty + TC_NACC;
  uint64_t* raw_empty = raw_full + RS;
  uint64_t* done = raw_empty + RS;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  int* s_last = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = (int)gridDim.x;
  const int64_t u0 = tc_first(p.U, (int)blockIdx.x, G), u1 = tc_first(p.U, (int)blockIdx.x + 1, G);
  const int nunits = (int)(u1 - u0);

  // ---- raw producer (thread 0): per unit one 2-D TMA box [128 rows x one
  // super-block column] of the GGUF bytes, evict-first in L2.  A short ring
  // (fewer than 4 columns) is backed by an L2 prefetch of the column that
  // takes the slot next, so that its copy reads the L2, not HBM; a deep ring
  // is not (the prefetches would double the burst at the start).  The first
  // columns are issued before the block-wide setup sync.
  TcCursor rcur, rahead;
  TcRing rring(RS);
  int rn = 0;
  uint64_t rpol = 0;
  const bool l2_ahead = RS < 4;
  auto raw_issue = [&]() -> bool {
    const int sg = rcur.sg, tl = rcur.tl, c = rcur.c, rs = rring.slot;
    if (!mbar_wait_bounded(&raw_empty[rs], rring.par ^ 1)) return false;
    const int x0 = (int)(((int64_t)c * p.seg[sg].CB) & ~int64_t(15)) / 2;
    mbar_arrive_expect_tx(&raw_full[rs], RAW_BYTES);
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(raw_sm + rs * RAW_BYTES)),
        "l"(reinterpret_cast<uint64_t>(&p.wmap[sg])), "r"(x0), "r"(tl * TC_BM), "r"(smem_u32(&raw_full[rs])),
        "l"(rpol)
        : "memory");
    if (l2_ahead) {
      if (rn + RS < nunits) {
        const int sg2 = rahead.sg, tl2 = rahead.tl, c2 = rahead.c;
        const int x2 = (int)(((int64_t)c2 * p.seg[sg2].CB) & ~int64_t(15)) / 2;
        asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(
                         reinterpret_cast<uint64_t>(&p.wmap[sg2])),
                     "r"(x2), "r"(tl2 * TC_BM)
                     : "memory");
      }
      rahead.next(p);
    }
    ++rn;
    rcur.next(p);
    rring.next();
    return true;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < US; ++s) mbar_init(&uempty[s], 1);
    for (int s = 0; s < TC_MMA_WARPS * US; ++s) {
      mbar_init(&afull[s], TC_DQ_WARPS);
      mbar_init(&bfull[s], 1);
    }
    for (int s = 0; s < TC_SCL_STAGES; ++s) {
      mbar_init(&scl_full[s], 1);
      mbar_init(&scl_empty[s], 4);
    }
    for (int s = 0; s < TC_NACC; ++s) {
      mbar_init(&a2_full[s], TC_DQ_WARPS);
      mbar_init(&a2_empty[s], 4);
      mbar_init(&acc_full[s], 1);
      mbar_init(&acc_empty[s], 4);
    }
    for (int s = 0; s < RS; ++s) {
      mbar_init(&raw_full[s], 1);
      mbar_init(&raw_empty[s], TC_DQ_WARPS);
    }
    mbar_init(done, TC_MMA_WARPS);
    fence_mbar_init();
    // the first columns depend on nothing: their slots are fresh (the empty
    // waits pass at once)
    rpol = l2_policy_evict_first();
    rcur.init(p, u0);
    if (l2_ahead) rahead.init(p, u0 + RS);
    while (rn < nunits && rn < RS) raw_issue();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, ATM ? TC_TMEM_COLS_A : TC_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // The next kernel may launch now: each of ours waits for this grid
  // (griddepcontrol.wait) before it reads or writes anything this one uses,
  // so only its launch latency overlaps this grid's work.
  tc_grid_launch();

  // parity of the k-th use of a ring slot: full waits (k / R) & 1, empty waits its complement
  auto ph = [](int k, int R) { return (uint32_t)((k / R) & 1); };
  // parity of an issuer's own full barrier: use k (per uses per unit) of a
  // ring of R slots.  Slot uses j = k / R come from units j*r .. (r = R /
  // per units per turn of the ring); for odd r they alternate between the
  // issuers, so an issuer sees every other one.
  auto iph = [](int k, int R, int per) {
    const int j = k / R, r = R / per;
    return (uint32_t)((((r & 1) ? (j >> 1) : j)) & 1);
  };

  if (warp == 0) {
    // ---- raw producer: the rest of the columns, as their slots free up
    if (lane == 0)
      while (rn < nunits)
        if (!raw_issue()) break;
  } else if (warp == 1 || warp == 3) {
    // ---- MMA issue: issuer i takes units i, i + 2, ... (accumulators a = n % 4
    // alternate between the issuers)
    if (lane == 0) {
      const int issuer = warp == 1 ? 0 : 1;
      uint64_t* my_afull = afull + issuer * US;
      uint64_t* my_bfull = bfull + issuer * US;
      // N = 32: the hi and lo x tiles are adjacent 16-row tiles, one operand
      constexpr uint32_t IDESC = umma_idesc_f16(TC_BM, 2 * TC_BN);
      const uint32_t a_base = smem_u32(a_sm), b_base = smem_u32(b_sm), a2_base = smem_u32(a2_sm);
      for (int n = issuer; n < nunits; n += TC_MMA_WARPS) {
        const int a = n % TC_NACC, u = n % US;
        const uint32_t dD = tmem + (uint32_t)(TC_ACC_COLS * a), dD2 = dD + 32;
        // the accumulator is free, the unit's A tiles (and its min-term A
        // column, written before the same arrivals) and B tiles are in place
        if (!mbar_wait_bounded(&acc_empty[a], ph(n, TC_NACC) ^ 1) || !mbar_wait_bounded(&my_afull[u], iph(n, US, 1)) ||
            !mbar_wait_bounded(&my_bfull[u], iph(n, US, 1)))
          break;
        tc_fence_after();
        const uint32_t ua = a_base + u * TC_UA_BYTES, ub = b_base + u * UB;
        const uint32_t ta = tmem + (uint32_t)(TC_TMEM_COLS + TC_A_TMEM_COLS * u);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t bd = umma_desc_sw128(ub + q * TC_B_BYTES + kk * 32);
            if constexpr (ATM) {
              // K step 16 q' of the unit: TMEM columns 8 q' .. 8 q' + 7 of its A slot
              tc_mma_ts(dD, ta + (uint32_t)(32 * q + 8 * kk), bd, IDESC, (q | kk) ? 1u : 0u);
            } else {
              const uint64_t ad = umma_desc_sw128(ua + q * TC_A_BYTES + kk * 32);
              tc_mma_bf16(dD, ad, bd, IDESC, (q | kk) ? 1u : 0u);
            }
          }
        }
        // min-term A slot a: K columns 16a .. 16a + 16 of the min-term tile
        if (HM) tc_mma_bf16(dD2, umma_desc_sw128(a2_base + a * 32), umma_desc_sw128(ub + 4 * TC_B_BYTES), IDESC, 0u);
        tc_commit(&uempty[u]);
        tc_commit(&acc_full[a]);
      }
      tc_commit(done);  // every MMA this thread issued has completed when this arrives
    }
  } else if (warp == 2) {
    // ---- B producer: x tiles per K stage; per unit the min-term tile and the token scales
    if (lane == 0) {
      tc_grid_wait();  // the workspace is written by the preparation kernel
      const uint64_t pol = l2_policy_evict_last();
      TcCursor cur;
      cur.init(p, u0);
      TcRing ur(US);
      for (int n = 0; n < nunits; ++n, cur.next(p), ur.next()) {
        const int c = cur.c, u = ur.slot, ss = n % TC_SCL_STAGES;
        // the x tiles of super-block c's four K stages are contiguous in the workspace
        const uint8_t* col = p.ws_col + (int64_t)c * TC_COL_BYTES;
        if (!mbar_wait_bounded(&uempty[u], ur.par ^ 1)) break;
        uint64_t* bf = &bfull[(n % TC_MMA_WARPS) * US + u];
        mbar_arrive_expect_tx(bf, UB);
        uint8_t* dst = b_sm + u * UB;
        bulk_g2s_hint(dst, p.ws_b + (int64_t)(4 * c) * TC_B_BYTES, 4 * TC_B_BYTES, bf, pol);
        if (HM) bulk_g2s_hint(dst + 4 * TC_B_BYTES, col, TC_B2_BYTES, bf, pol);
        if (!mbar_wait_bounded(&scl_empty[ss], ph(n, TC_SCL_STAGES) ^ 1)) break;
        mbar_arrive_expect_tx(&scl_full[ss], TC_BN * 4);
        bulk_g2s_hint(scl_sm + ss * TC_BN, col + TC_B2_BYTES, TC_BN * 4, &scl_full[ss], pol);
      }
    }
  } else if (ATM && warp >= TC_DQ_WARP0) {
    // ---- dequant into TMEM: warp (r, h), r = warp % 4 its TMEM lane
    // quadrant, writes row 32r + lane of every unit, K stages 2h and 2h + 1
    // (one tcgen05.st of 32 columns each) into the unit slot's A columns.
    // The warps of stage q = 0 / 1 also write the row's d / dmin and the
    // min-term chunk's zero half; stage q's writer owns min-term word q.
    // The TMEM stores and the MMAs that read them are ordered through the
    // unit slot's barriers (wait::st, fence, arrive / wait, fence), and the
    // stores into a slot wait for the commit of the MMAs that read it last.
    // The waits' outcomes are made warp-uniform before the .aligned stores.
    const int dw = warp - TC_DQ_WARP0, r = dw & 3, h = dw >> 2;
    const int row = 32 * r + lane, sw = row & 7;
    const uint32_t trow = tmem + ((uint32_t)(32 * r) << 16) + (uint32_t)TC_TMEM_COLS;
    TcCursor cur;
    cur.init(p, u0);
    TcRing rr(RS), ur(US);
    for (int n = 0; n < nunits; ++n, cur.next(p), rr.next(), ur.next()) {
      const int sg = cur.sg, c = cur.c;
      const int code = CODE == kTcMixed ? p.seg[sg].code : CODE;
      const int rs = rr.slot, a = n % TC_NACC, u = ur.slot;
      bool ok = mbar_wait_bounded(&raw_full[rs], rr.par) && mbar_wait_bounded(&a2_empty[a], ph(n, TC_NACC) ^ 1);
      if (!__all_sync(0xFFFFFFFFu, ok)) break;
      const int off16 = (int)(((int64_t)c * p.seg[sg].CB) & 15);
      const uint8_t* raw = raw_sm + rs * RAW_BYTES + row * PITCH + off16;
      uint8_t* a2row = a2_sm + row * 128;
#pragma unroll
      for (int s = 0; s < 2; ++s) {
        const int q = 2 * h + s;
        uint4 ch[8];
        tc_stage<CODE>(code, raw, q, off16, a2row, 2 * a, sw, &dsc[a * TC_BM + row], ch);
        if (s == 0) {
          // the slot's A columns are free once the MMAs of its previous unit have completed
          ok = __all_sync(0xFFFFFFFFu, mbar_wait_bounded(&uempty[u], ur.par ^ 1));
          if (!ok) break;
          tc_fence_after();
        }
        tc_st_32x32b_x32(trow + (uint32_t)(TC_A_TMEM_COLS * u + 32 * q), ch);
      }
      if (!ok) break;
      tc_wait_st();
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&a2_full[a]);
        mbar_arrive(&afull[(n % TC_MMA_WARPS) * US + u]);
        mbar_arrive(&raw_empty[rs]);
      }
    }
  } else if (warp >= TC_DQ_WARP0) {
    // ---- dequant: warp (q, h) produces K stage q of every unit for rows
    // [64h, 64h + 64), rows lane and lane + 32, all 8 chunks of a row in one
    // thread (a quarter-warp is 8 consecutive rows of one chunk, so its
    // 16-byte swizzled stores fall in 8 distinct bank groups).  The four
    // stages of a unit are dequantized at the same time, and each warp meets
    // its barriers once per unit instead of once per stage.  Warp q also
    // writes word q of the unit's min-term chunk (the mins of sub-blocks 2q,
    // 2q + 1); warp 0 the row's d / dmin, warp 1 the zero chunk beside it.
    const int dw = warp - TC_DQ_WARP0, q = dw & 3, h = dw >> 2;
    TcCursor cur;
    cur.init(p, u0);
    TcRing rr(RS), ur(US);
    for (int n = 0; n < nunits; ++n, cur.next(p), rr.next(), ur.next()) {
      const int sg = cur.sg, c = cur.c;
      const int code = CODE == kTcMixed ? p.seg[sg].code : CODE;
      const int rs = rr.slot, a = n % TC_NACC, u = ur.slot;
      if (!mbar_wait_bounded(&raw_full[rs], rr.par)) break;
      if (!mbar_wait_bounded(&a2_empty[a], ph(n, TC_NACC) ^ 1)) break;
      const int off16 = (int)(((int64_t)c * p.seg[sg].CB) & 15);
      const int a2c = 2 * a;  // 16-byte chunks of this unit's 16 K columns of the min-term tile
      bool ok = true;
      // both rows unrolled: their independent integer / half chains interleave
      // (70B gate|up pair at M = 16: 200 -> 187 us)
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int row = 64 * h + 32 * i + lane, sw = row & 7;
        const uint8_t* raw = raw_sm + rs * RAW_BYTES + row * PITCH + off16;
        uint4 ch[8];
        tc_stage<CODE>(code, raw, q, off16, a2_sm + row * 128, a2c, sw, &dsc[a * TC_BM + row], ch);
        // the unit slot is free once the MMAs of its previous unit have completed
        if (i == 0 && !mbar_wait_bounded(&uempty[u], ur.par ^ 1)) {
          ok = false;
          break;
        }
        uint8_t* dst = a_sm + u * TC_UA_BYTES + q * TC_A_BYTES + row * 128;
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) *reinterpret_cast<uint4*>(dst + ((cc ^ sw) << 4)) = ch[cc];
      }
      if (!ok) break;
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&a2_full[a]);
        mbar_arrive(&afull[(n % TC_MMA_WARPS) * US + u]);
        mbar_arrive(&raw_empty[rs]);
      }
    }
  } else if (warp >= TC_EPI_WARP0) {
    // ---- epilogue: one weight row per thread
    const int qd = warp & 3, row = 32 * qd + lane;
    tc_grid_wait();  // y and the partials may still be in use by the previous kernel
    float acc[TC_BN];
#pragma unroll
    for (int t = 0; t < TC_BN; ++t) acc[t] = 0.f;
    int seg_first_c = -1;
    // A wait that gives up stops the work but not the walk: the four warps
    // pass the same named barriers whatever happens.
    bool ok = true;
    TcCursor cur;
    cur.init(p, u0);
    for (int n = 0; n < nunits; ++n, cur.next(p)) {
      const int sg = cur.sg, tl = cur.tl, c = cur.c;
      if (seg_first_c < 0) seg_first_c = c;
      const int a = n % TC_NACC, ss = n % TC_SCL_STAGES;
      if (ok)
        ok = mbar_wait_bounded(&acc_full[a], ph(n, TC_NACC)) && mbar_wait_bounded(&a2_full[a], ph(n, TC_NACC)) &&
             mbar_wait_bounded(&scl_full[ss], ph(n, TC_SCL_STAGES));
      if (ok) {
        tc_fence_after();
        // D and D2, each as hi | lo halves of 16 columns
        float dsum[TC_BN], d2sum[TC_BN];
        const uint32_t taddr = tmem + ((uint32_t)(32 * qd) << 16) + (uint32_t)(TC_ACC_COLS * a);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint32_t v[32];
          if (h == 1 && !HM) {
#pragma unroll
            for (int t = 0; t < TC_BN; ++t) d2sum[t] = 0.f;
            continue;
          }
          tc_ld_32x32b_x32(taddr + 32 * h, v);
#pragma unroll
          for (int t = 0; t < TC_BN; ++t) {
            const float x = __uint_as_float(v[t]) + __uint_as_float(v[t + 16]);
            if (h == 0) dsum[t] = x;
            else d2sum[t] = x;
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[a]);
        const float2 dd = dsc[a * TC_BM + row];
        const float* sct = scl_sm + ss * TC_BN;
#pragma unroll
        for (int t = 0; t < TC_BN; ++t) acc[t] = fmaf(sct[t], fmaf(dd.x, dsum[t], -dd.y * d2sum[t]), acc[t]);
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&a2_empty[a]);
          mbar_arrive(&scl_empty[ss]);
        }
      }
      // end of this CTA's segment of the tile?
      const bool last_of_tile = (c == p.NSB - 1) || (n == nunits - 1);
      if (!last_of_tile) continue;
      const TcSeg& S = p.seg[sg];
      const int t_glob = S.tile0 + tl;
      const int64_t nrow = (int64_t)tl * TC_BM + row;
      const bool row_ok = nrow < S.N;
      if (seg_first_c == 0 && c == p.NSB - 1) {
        if (row_ok && ok) {
#pragma unroll
          for (int m = 0; m < TC_BN; ++m)
            if (m < p.M) tc_store_y(p, S, sg, m, nrow, acc[m]);
        }
      } else {
        const int64_t ut0 = (int64_t)t_glob * p.NSB;
        const int i_first = tc_owner(ut0, p.U, G), i_last = tc_owner(ut0 + p.NSB - 1, p.U, G);
        // Every other CTA of the tile has added its partial already (usual for
        // a CTA's last segment: the next CTA starts with that tile): this CTA
        // finishes the tile from its registers, without a partial of its own,
        // a fence or an arrival.  The sum runs in CTA order either way, so
        // the bits do not depend on the path.
        if (threadIdx.x == TC_EPI_WARP0 * 32)
          *s_last = ld_acquire_gpu(p.ws_cnt + i_first) == (uint32_t)(i_last - i_first) ? 2 : 0;
        asm volatile("bar.sync 1, 128;" ::: "memory");
        const bool fast = *s_last == 2;
        if (!fast) {
          // partial: slot 2i for the first segment of CTA i, 2i + 1 for its last
          const bool first_seg = ut0 <= u0;
          const int slot = 2 * (int)blockIdx.x + (first_seg ? 0 : 1);
          float4* dst = reinterpret_cast<float4*>(p.ws_part + ((int64_t)slot * TC_BM + row) * TC_BN);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            __stcg(dst + i, make_float4(acc[4 * i], acc[4 * i + 1], acc[4 * i + 2], acc[4 * i + 3]));
          __threadfence();
          asm volatile("bar.sync 1, 128;" ::: "memory");
          if (threadIdx.x == TC_EPI_WARP0 * 32) {
            const uint32_t old = atomicAdd(p.ws_cnt + i_first, 1u);
            *s_last = (old == (uint32_t)(i_last - i_first)) ? 1 : 0;
          }
          asm volatile("bar.sync 1, 128;" ::: "memory");
        }
        if (*s_last) {
          __threadfence();
          float sum[TC_BN];
#pragma unroll
          for (int t = 0; t < TC_BN; ++t) sum[t] = 0.f;
          for (int i = i_first; i <= i_last; ++i) {
            if (fast && i == (int)blockIdx.x) {
#pragma unroll
              for (int t = 0; t < TC_BN; ++t) sum[t] += acc[t];
              continue;
            }
            const int64_t ui0 = tc_first(p.U, i, G);
            const int sl = 2 * i + ((i == i_first && ui0 < ut0) ? 1 : 0);
            const float4* src = reinterpret_cast<const float4*>(p.ws_part + ((int64_t)sl * TC_BM + row) * TC_BN);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const float4 f = __ldcg(src + q);
              sum[4 * q] += f.x; sum[4 * q + 1] += f.y; sum[4 * q + 2] += f.z; sum[4 * q + 3] += f.w;
            }
          }
          if (row_ok) {
#pragma unroll
            for (int m = 0; m < TC_BN; ++m)
              if (m < p.M) tc_store_y(p, S, sg, m, nrow, sum[m]);
          }
          if (threadIdx.x == TC_EPI_WARP0 * 32) p.ws_cnt[i_first] = 0u;
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
      }
#pragma unroll
      for (int t = 0; t < TC_BN; ++t) acc[t] = 0.f;
      seg_first_c = -1;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (p.P > 1 && threadIdx.x == 0) {
    // Publish, as the fused kernel does: the fence orders this CTA's peer
    // stores before its count; the grid's last CTA advances the exchange
    // count and writes it to this rank's flag word in every buffer.
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
  if (warp == 1) {
    // both issuers' final commits arrive once every MMA has completed
    mbar_wait_bounded(done, 0);
    tc_fence_after();
    tmem_dealloc(tmem, ATM ? TC_TMEM_COLS_A : TC_TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// Host side
static PFN_cuTensorMapEncodeTiled_v12000 tc_encode_fn() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

static int tc_code(int type, int layout) {
  if (type == NSQ_TYPE_Q4_K) return kTcQ4K;
  if (type == NSQ_TYPE_Q6_K && layout == NSQ_Q6K_GGML) return kTcQ6KG;
  if (type == NSQ_TYPE_Q6_K && layout == NSQ_Q6K_NODESTOR) return kTcQ6KN;
  if (type == NSQ_TYPE_Q5_K) return layout == NSQ_Q6K_NODESTOR ? kTcQ5KN : kTcQ5KG;
  if (type == NSQ_TYPE_Q4_0) return kTcQ40;
  if (type == NSQ_TYPE_Q8_0) return kTcQ80;
  return -2;
}

// True if the batched tensor-core path covers these segments: Q4_K, Q5_K and
// Q6_K (both layouts), Q4_0 or Q8_0, K % 256 == 0, whole 16-byte rows, M in
// [2, 16].
bool tc_covers(const nsq_segment* segs, int nseg, int64_t M, int64_t K) {
  if (M < 2 || M > TC_BN || K % 256 || K <= 0 || nseg < 1 || nseg > NSQ_MAX_SEGMENTS) return false;
  for (int i = 0; i < nseg; ++i) {
    if (tc_code(segs[i].ggml_type, segs[i].q6k_layout) < -1) return false;
    const int64_t rb = K / nsq_block_weights(segs[i].ggml_type) * nsq_block_bytes(segs[i].ggml_type);
    if (rb % 16 || segs[i].N > 0x7FFFFFFF) return false;
  }
  return true;
}

// From 5 tokens the tcgen05 kernel beats the dp4a kernel's passes of 4 tokens
// (B200: Llama-3-8B decode step at M = 5: 4.96 against 5.43 ms, M = 8: 4.98
// against 7.42 ms; at M = 4 the single dp4a pass wins, 3.78 against 4.96 ms).
int tc_min_m() { return tune(kTuneTcMinM, 5); }

template <int CODE, bool ATM>
static cudaError_t launch_tc(const TcParams& p, int blocks, size_t smem, cudaStream_t st) {
  auto kern = gemv_tc_kernel<CODE, ATM>;
  static size_t configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || smem > configured[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) configured[dev] = smem;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)blocks);
  cfg.blockDim = dim3(TC_THREADS);
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

template <bool ATM>
static cudaError_t launch_code(int code, const TcParams& p, int G, size_t smem, cudaStream_t st) {
  switch (code) {
    case kTcQ4K: return launch_tc<kTcQ4K, ATM>(p, G, smem, st);
    case kTcQ6KG: return launch_tc<kTcQ6KG, ATM>(p, G, smem, st);
    case kTcQ40: return launch_tc<kTcQ40, ATM>(p, G, smem, st);
    case kTcQ80: return launch_tc<kTcQ80, ATM>(p, G, smem, st);
    case kTcQ6KN: return launch_tc<kTcQ6KN, ATM>(p, G, smem, st);
    case kTcQ5KG: return launch_tc<kTcQ5KG, ATM>(p, G, smem, st);
    case kTcQ5KN: return launch_tc<kTcQ5KN, ATM>(p, G, smem, st);
    default: return launch_tc<kTcMixed, ATM>(p, G, smem, st);
  }
}

// Batched decode GEMV; -1 if not covered.  workspace: tc_workspace_bytes(K)
// bytes, 16-byte aligned.
int run_gemv_tc(const nsq_segment* segs, int nseg, const float* x, int64_t M, int64_t K, void* workspace,
                cudaStream_t st, int num_sms, const XchgDesc* xd) {
  if (!tc_covers(segs, nseg, M, K)) return -1;
  auto enc = tc_encode_fn();
  if (!enc) return -1;
  TcParams p{};
  const int NSB = (int)(K / 256);
  int pitch = 144, code = -2, tiles = 0;
  for (int i = 0; i < nseg; ++i) {
    TcSeg& s = p.seg[i];
    s.code = tc_code(segs[i].ggml_type, segs[i].q6k_layout);
    // bytes of one 256-weight column: one K-quant super-block, 8 Q4_0 / Q8_0 blocks
    s.CB = (int)(nsq_block_bytes(segs[i].ggml_type) * (256 / nsq_block_weights(segs[i].ggml_type)));
    s.w = static_cast<const uint8_t*>(segs[i].w);
    s.y = segs[i].y;
    s.N = segs[i].N;
    s.RB = (int64_t)NSB * s.CB;
    s.tile0 = tiles;
    tiles += (int)((s.N + TC_BM - 1) / TC_BM);
    code = (i == 0 || code == s.code) ? s.code : kTcMixed;
    if ((s.code == kTcQ6KG || s.code == kTcQ6KN) && pitch < 240) pitch = 240;  // 210-byte columns, any even offset
    if (s.code == kTcQ80) pitch = 272;                   // 272-byte columns, 16-byte aligned
    if ((s.code == kTcQ5KG || s.code == kTcQ5KN) && pitch < 176) pitch = 176;  // 176-byte columns, aligned
  }
  for (int i = 0; i < nseg; ++i) {
    cuuint64_t dims[2] = {(cuuint64_t)(p.seg[i].RB / 2), (cuuint64_t)p.seg[i].N};
    cuuint64_t strides[1] = {(cuuint64_t)p.seg[i].RB};
    cuuint32_t box[2] = {(cuuint32_t)(pitch / 2), (cuuint32_t)TC_BM};
    cuuint32_t estr[2] = {1, 1};
    if (enc(&p.wmap[i], CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<uint8_t*>(p.seg[i].w), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return -1;
  }
  p.nseg = nseg;
  p.P = 1;
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
  p.T = tiles;
  p.NSB = NSB;
  p.M = (int)M;
  p.U = (int64_t)tiles * NSB;
  p.pitch = pitch;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  p.ws_cnt = reinterpret_cast<uint32_t*>(ws);
  p.ws_b = ws + 1024;
  p.ws_col = p.ws_b + (size_t)NSB * 4 * TC_B_BYTES;
  p.ws_part = reinterpret_cast<float*>(const_cast<uint8_t*>(p.ws_col) + (size_t)NSB * TC_COL_BYTES);
  // A in TMEM (the default): two unit slots of A in TMEM beside the
  // accumulators, their B tiles in shared memory, and as many raw columns as
  // fit (up to 8).  A in shared memory: two unit slots of A and B tiles when
  // they fit beside two raw columns, so that the dequant warps and the B
  // producer fill a unit while the MMAs of the one before still read theirs:
  // Q4_K, Q4_0, and a single-format Q6_K launch, which leaves out the
  // min-term tiles; otherwise one unit slot and up to four raw columns.
  const bool hm = code == kTcMixed || code == kTcQ4K || code == kTcQ5KG || code == kTcQ5KN;
  const bool atm = tune(kTuneTcA, 1) != 0;
  auto smem_of = [&](int us, int r) {
    return 1024 + (size_t)us * ((atm ? 0 : TC_UA_BYTES) + tc_ub_bytes(hm)) + (hm ? TC_A_BYTES : 0) +
           (size_t)TC_SCL_STAGES * TC_BN * 4 + (size_t)TC_NACC * TC_BM * 8 + 1024 + (size_t)r * TC_BM * pitch;
  };
  int us = 2, rs = 2;
  if (atm) {
    rs = 8;
    while (smem_of(us, rs) > (size_t)TC_SMEM_LIMIT && rs > 2) --rs;
  } else if (smem_of(us, rs) > (size_t)TC_SMEM_LIMIT) {
    us = 1;
    rs = 4;
    while (smem_of(us, rs) > (size_t)TC_SMEM_LIMIT && rs > 2) --rs;
  }
  const size_t smem = smem_of(us, rs);
  if (smem > (size_t)TC_SMEM_LIMIT) return -1;
  p.raw_stages = rs;
  p.unit_slots = us;
  int G = num_sms > 0 ? num_sms : 148;
  if (G > TC_GMAX) G = TC_GMAX;
  if ((int64_t)G > p.U) G = (int)p.U;
  if (p.U * (G + 1) >= ((int64_t)1 << 32)) return -1;  // the unit arithmetic is 32-bit
  // activations -> fp16 B tiles, min-term tiles, scales; counters zeroed
  {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((TC_BN * NSB + 7) / 8));
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    note_launch();
    if (cudaLaunchKernelEx(&cfg, tc_prep_kernel, x, (int)M, K, NSB, ws + 1024,
                           const_cast<uint8_t*>(p.ws_col), p.ws_cnt) != cudaSuccess)
      return NSQ_ERR_CUDA;
  }
  const cudaError_t e = atm ? launch_code<true>(code, p, G, smem, st) : launch_code<false>(code, p, G, smem, st);
  return e == cudaSuccess ? NSQ_OK : NSQ_ERR_CUDA;
}

}  // namespace nsq
