// gemm_tc.cu -- prefill GEMM on 5th-generation tensor cores (tcgen05).
//
//   y[M x N] (bf16) = x[M x K] (bf16) . W^T,   W: N rows of GGUF blocks
//
// "Swap-AB" tiling: the weights are the UMMA M side (128 rows of W per CTA),
// the tokens the UMMA N side (TOK = 128, 256 or 512 per CTA), so D = W_tile .
// x_tile^T is a [128 x TOK] fp32 accumulator in tensor memory (TOK columns;
// 512 is all of it, filled by two N = 256 MMAs per K step).  The kernel is
// bound by the dequant warps, so a larger token tile, which reuses every
// dequantized weight tile for more tokens, is worth the shallower ring: on
// B200, Q4_K [14336 x 4096] at M = 512 runs 977 TFLOP/s with 512-token tiles
// against 582 with 256.  K advances in blocks of 64 (one 128-byte swizzle
// atom of bf16).
//
// Warp roles (384 threads):
//   warp 0      : TMA producer -- one thread loads the x tile [TOK x 64]
//                 (2-D tiled bulk tensor copy, 128B swizzle) per K block.
//   warp 1      : allocates TMEM; one thread issues 4 tcgen05.mma
//                 (kind::f16, bf16 inputs, fp32 accumulate, K = 16 each)
//                 per K block and commits them to the stage's "empty"
//                 barrier, and finally to the accumulator barrier.
//   warps 4..11 : dequant producers -- 2 threads per W row turn the GGUF
//                 blocks of the K block into bf16 and store them in the
//                 same 128B-swizzled K-major layout TMA uses; then the
//                 epilogue: tcgen05.ld of the accumulator, bf16 convert,
//                 store to y.
// Stages form a 4-deep ring guarded by mbarriers.  Every wait is bounded
// (%globaltimer); a wait that gives up records NSQ_ERR_TIMEOUT and the
// kernel winds down instead of hanging.
//
// Weights are dequantized with the same formulas (and roundings) as the
// standalone dequant, then rounded to bf16.  The reference computes the
// contraction in f32 (crates/nodestor-vulkan/src/pipeline.rs:1256-1268);
// the bf16 operands here bound the error at about 2^-8 relative per term,
// checked at a 2e-2 tolerance.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <stdlib.h>

#include <mutex>

#include "nsq_common.cuh"
#include "tcgen05.cuh"

namespace nsq {

constexpr int GEMM_BM = 128;   // W rows per CTA (UMMA M)
constexpr int GEMM_BK = 64;    // K per stage (bf16: 128 bytes per row)
constexpr int GEMM_RAW_STAGES = 2; // raw GGUF byte stages (256-wide K columns)
constexpr int GEMM_SMEM_LIMIT = 232448;  // opt-in shared memory per CTA on sm_100
constexpr int GEMM_THREADS = 640;
constexpr int GEMM_DQ_WARP0 = 4;  // first dequant / epilogue warp
constexpr int GEMM_DQ_THREADS = 512;

// Raw bytes of one row for one 256-weight column of K: a K-quant
// super-block, or 8 Q4_0 / Q8_0 blocks.  Q6_K columns (210 B) start at any
// even offset, so their copies carry up to 15 bytes of slack on each side.
template <int TYPE> struct RawCol;
template <> struct RawCol<NSQ_TYPE_Q4_K> { static constexpr int bytes = 144, pitch = 144; };
template <> struct RawCol<NSQ_TYPE_Q5_K> { static constexpr int bytes = 176, pitch = 176; };
template <> struct RawCol<NSQ_TYPE_Q4_0> { static constexpr int bytes = 144, pitch = 144; };
template <> struct RawCol<NSQ_TYPE_Q8_0> { static constexpr int bytes = 272, pitch = 272; };
template <> struct RawCol<NSQ_TYPE_Q6_K> { static constexpr int bytes = 210, pitch = 240; };

// bf16 W / x stages (64-wide K blocks): as many as fit beside the raw ring
template <int TYPE, int TOK>
__host__ __device__ constexpr int gemm_stages() {
  constexpr int fixed = 1024 + GEMM_RAW_STAGES * 128 * RawCol<TYPE>::pitch + 256;
  constexpr int per = 128 * 128 + TOK * 128;
  constexpr int n = (GEMM_SMEM_LIMIT - fixed) / per;
  return n > 6 ? 6 : n;
}

// ---------------------------------------------------------------------------
// Dequant of 32 weights of one row for one 64-wide K block, as bf16 pairs in
// K order.  chunk[i] (i < 4) is the 16-byte chunk index (0..7) of the 64-wide
// row segment that pair-group i (8 bf16) belongs to.
__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Byte b of w as the float 2^23 + byte: one byte permute beside the exponent
// byte 0x4B, exact for every byte value.  With it the small integers of the
// quant formats become floats without an integer-to-float conversion, and the
// byte extraction is the permute itself.
constexpr float kTwo23 = 8388608.0f;
__device__ __forceinline__ float byte_magic(uint32_t w, int b) {
  return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7440u | (uint32_t)b));
}

// Dequant of 16 weights of one row for one 64-wide K block q (0..3) of a
// 256-weight column whose raw bytes `raw` sit in shared memory; qq (0..3)
// picks which 16 of the 64 (two 16-byte chunks of the bf16 row segment,
// chunk[0] and chunk[1]).  Same formulas and roundings as dequant.cu.
template <int TYPE, int LAYOUT>
__device__ __forceinline__ void dequant_col_kblock(const uint8_t* raw, int q, int qq, uint32_t (&out)[8],
                                                   int (&chunk)[2]) {
  float v[16];
  if constexpr (TYPE == NSQ_TYPE_Q4_K) {
    // qs[32q + 8qq .. +8): low nibbles -> K 8qq.. (sub-block 2q),
    // high nibbles -> K 32 + 8qq.. (sub-block 2q+1)
    const uint4 hdr = *reinterpret_cast<const uint4*>(raw);
    const uint2 qv = *reinterpret_cast<const uint2*>(raw + 16 + 32 * q + 8 * qq);
    const float d = h2f((uint16_t)(hdr.x & 0xFFFF)), dmin = h2f((uint16_t)(hdr.x >> 16));
    uint32_t sc[2], mn[2];
#pragma unroll
    for (int s2 = 0; s2 < 2; ++s2) {
      const int j = 2 * q + s2;
      if (j < 4) {
        sc[s2] = (hdr.y >> (8 * j)) & 63;
        mn[s2] = (hdr.z >> (8 * j)) & 63;
      } else {
        const int sh = 8 * (j - 4);
        const uint32_t b2 = (hdr.w >> sh) & 0xFF, b0 = (hdr.y >> sh) & 0xFF, b1 = (hdr.z >> sh) & 0xFF;
        sc[s2] = (b2 & 0xF) | ((b0 >> 6) << 4);
        mn[s2] = (b2 >> 4) | ((b1 >> 6) << 4);
      }
    }
    const float d1 = __fmul_rn(d, (float)sc[0]), m1 = __fmul_rn(dmin, (float)mn[0]);
    const float d2 = __fmul_rn(d, (float)sc[1]), m2 = __fmul_rn(dmin, (float)mn[1]);
    // d1*q is exact (<= 21 significant bits), so fma(d1, q, -m1) rounds
    // once, exactly like the reference's d1*q - m1.  (Building q as 2^23 + q
    // by a byte permute, as the other formats do, costs an extra float add
    // here: prefill Q4_K M = 512 869 against 901 TFLOP/s.)
#pragma unroll
    for (int w2 = 0; w2 < 2; ++w2) {
      const uint32_t wv = w2 ? qv.y : qv.x;
      const uint32_t lo = wv & 0x0F0F0F0Fu, hi = (wv >> 4) & 0x0F0F0F0Fu;
#pragma unroll
      for (int b = 0; b < 4; b += 2) {
        const float2 l = __ffma2_rn(make_float2(d1, d1),
                                    make_float2((float)((lo >> (8 * b)) & 0xFF), (float)((lo >> (8 * b + 8)) & 0xFF)),
                                    make_float2(-m1, -m1));
        const float2 h = __ffma2_rn(make_float2(d2, d2),
                                    make_float2((float)((hi >> (8 * b)) & 0xFF), (float)((hi >> (8 * b + 8)) & 0xFF)),
                                    make_float2(-m2, -m2));
        v[4 * w2 + b] = l.x;
        v[4 * w2 + b + 1] = l.y;
        v[8 + 4 * w2 + b] = h.x;
        v[8 + 4 * w2 + b + 1] = h.y;
      }
    }
    chunk[0] = qq;
    chunk[1] = 4 + qq;
  } else if constexpr (TYPE == NSQ_TYPE_Q5_K) {
    // Q4_K's nibbles (qs at byte 48) plus one high bit per weight from
    // qh[32]: ggml: bit 2q (low) / 2q+1 (high) of qh[8qq + i]; NODESTOR
    // (q5_k.rs:57-70): bit i of qh[8q + qq] (low) / qh[8q + 4 + qq] (high)
    const uint4 hdr = *reinterpret_cast<const uint4*>(raw);
    const uint2 qv = *reinterpret_cast<const uint2*>(raw + 48 + 32 * q + 8 * qq);
    const float d = h2f((uint16_t)(hdr.x & 0xFFFF)), dmin = h2f((uint16_t)(hdr.x >> 16));
    uint32_t sc[2], mn[2];
#pragma unroll
    for (int s2 = 0; s2 < 2; ++s2) {
      const int j = 2 * q + s2;
      if (j < 4) {
        sc[s2] = (hdr.y >> (8 * j)) & 63;
        mn[s2] = (hdr.z >> (8 * j)) & 63;
      } else {
        const int sh = 8 * (j - 4);
        const uint32_t b2 = (hdr.w >> sh) & 0xFF, b0 = (hdr.y >> sh) & 0xFF, b1 = (hdr.z >> sh) & 0xFF;
        sc[s2] = (b2 & 0xF) | ((b0 >> 6) << 4);
        mn[s2] = (b2 >> 4) | ((b1 >> 6) << 4);
      }
    }
    const float d1 = __fmul_rn(d, (float)sc[0]), m1 = __fmul_rn(dmin, (float)mn[0]);
    const float d2 = __fmul_rn(d, (float)sc[1]), m2 = __fmul_rn(dmin, (float)mn[1]);
    uint32_t hlo[8], hhi[8];
    if constexpr (LAYOUT == NSQ_Q6K_NODESTOR) {
      const uint32_t bl = raw[16 + 8 * q + qq], bh = raw[16 + 8 * q + 4 + qq];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        hlo[i] = (bl >> i) & 1;
        hhi[i] = (bh >> i) & 1;
      }
    } else {
      const uint2 hv = *reinterpret_cast<const uint2*>(raw + 16 + 8 * qq);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint32_t byte = ((i < 4 ? hv.x : hv.y) >> (8 * (i & 3))) & 0xFF;
        hlo[i] = (byte >> (2 * q)) & 1;
        hhi[i] = (byte >> (2 * q + 1)) & 1;
      }
    }
    // d1*q is exact (<= 22 significant bits): fma rounds once, like d1*q - m1
#pragma unroll
    for (int w2 = 0; w2 < 2; ++w2) {
      const uint32_t wv = w2 ? qv.y : qv.x;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const int i = 4 * w2 + b;
        const uint32_t lo = ((wv >> (8 * b)) & 0x0F) | (hlo[i] << 4);
        const uint32_t hi = ((wv >> (8 * b + 4)) & 0x0F) | (hhi[i] << 4);
        v[i] = __fmaf_rn(d1, (float)lo, -m1);
        v[8 + i] = __fmaf_rn(d2, (float)hi, -m2);
      }
    }
    chunk[0] = qq;
    chunk[1] = 4 + qq;
  } else if constexpr (TYPE == NSQ_TYPE_Q6_K) {
    const float d = h2f((uint16_t)ld_u16(raw + 208));
    if constexpr (LAYOUT == NSQ_Q6K_NODESTOR) {
      // elements e = 64q + 16qq + l: ql[e>>1], qh[e>>2], scale byte [e>>4]
      uint32_t ql[2], qh[1];
      ld_words_unaligned<2>(raw + 32 * q + 8 * qq, ql);
      ld_words_unaligned<1>(raw + 128 + 16 * q + 4 * qq, qh);
      const float sa = __fmul_rn(d, (float)((int)raw[192 + 4 * q + qq] - 128) / 64.0f);
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const uint32_t l2 = (ql[t >> 1] >> (16 * (t & 1))) & 0xFFFF;  // elements 4t .. 4t+3
        const uint32_t hb = (qh[0] >> (8 * t)) & 0xFF;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const uint32_t lo = (l2 >> (4 * e)) & 0xF;
          const uint32_t hi = (hb >> (2 * e)) & 3;
          v[4 * t + e] = __fmul_rn(sa, (float)((int)(lo | (hi << 4)) - 32));
        }
      }
    } else {
      // ggml: n = q>>1, group j = 2(q&1) + (qq>>1), l = 16(qq&1) + i;
      // ql[64n + 32(j&1) + l] nibble (q&1), qh[32n + l] bits 2j, int8 scale
      // sc[8n + (qq&1) + 2j]
      const int n = q >> 1, j = 2 * (q & 1) + (qq >> 1), nib = q & 1, l0 = 16 * (qq & 1);
      uint32_t ql[4], qh[4];
      ld_words_unaligned<4>(raw + 64 * n + 32 * (j & 1) + l0, ql);
      ld_words_unaligned<4>(raw + 128 + 32 * n + l0, qh);
      const float sa = __fmul_rn(d, (float)(int8_t)raw[192 + 8 * n + (qq & 1) + 2 * j]);
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        // the four 6-bit values of word w as bytes; q - 32 exactly from 2^23 + q
        const uint32_t qb = ((ql[w] >> (4 * nib)) & 0x0F0F0F0Fu) | (((qh[w] >> (2 * j)) & 0x03030303u) << 4);
#pragma unroll
        for (int b = 0; b < 4; b += 2) {
          const float2 t = __fmul2_rn(make_float2(sa, sa), __fadd2_rn(make_float2(byte_magic(qb, b), byte_magic(qb, b + 1)),
                                                                      make_float2(-(kTwo23 + 32.0f), -(kTwo23 + 32.0f))));
          v[4 * w + b] = t.x;
          v[4 * w + b + 1] = t.y;
        }
      }
    }
    chunk[0] = 2 * qq;
    chunk[1] = 2 * qq + 1;
  } else if constexpr (TYPE == NSQ_TYPE_Q4_0) {
    // block 2q + (qq>>1); qq&1 picks the low (weights 0..15) or high
    // (16..31) nibbles of its 16 bytes
    const uint8_t* blk = raw + (2 * q + (qq >> 1)) * 18;
    const float d = h2f((uint16_t)ld_u16(blk));
    uint32_t qs[4];
    ld_words_unaligned<4>(blk + 2, qs);
    const int sh = 4 * (qq & 1);
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const uint32_t nb = (qs[w] >> sh) & 0x0F0F0F0Fu;
#pragma unroll
      for (int b = 0; b < 4; b += 2) {
        const float2 t = __fmul2_rn(__fadd2_rn(make_float2(byte_magic(nb, b), byte_magic(nb, b + 1)),
                                               make_float2(-(kTwo23 + 8.0f), -(kTwo23 + 8.0f))),
                                    make_float2(d, d));
        v[4 * w + b] = t.x;
        v[4 * w + b + 1] = t.y;
      }
    }
    chunk[0] = 2 * qq;
    chunk[1] = 2 * qq + 1;
  } else {  // Q8_0: block 2q + (qq>>1), bytes 16(qq&1) .. +16
    const uint8_t* blk = raw + (2 * q + (qq >> 1)) * 34;
    const float d = h2f((uint16_t)ld_u16(blk));
    uint32_t qs[4];
    ld_words_unaligned<4>(blk + 2 + 16 * (qq & 1), qs);
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const uint32_t ub = qs[w] ^ 0x80808080u;  // int8 s as the byte s + 128
#pragma unroll
      for (int b = 0; b < 4; b += 2) {
        const float2 t = __fmul2_rn(make_float2(d, d), __fadd2_rn(make_float2(byte_magic(ub, b), byte_magic(ub, b + 1)),
                                                                  make_float2(-(kTwo23 + 128.0f), -(kTwo23 + 128.0f))));
        v[4 * w + b] = t.x;
        v[4 * w + b + 1] = t.y;
      }
    }
    chunk[0] = 2 * qq;
    chunk[1] = 2 * qq + 1;
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) out[i] = pack_bf16(v[2 * i], v[2 * i + 1]);
}

// ---------------------------------------------------------------------------
struct GemmParams {
  const uint8_t* w;
  __nv_bfloat16* y;
  int64_t M, N, K, RB;
  int wmap_ok;  // 1: raw weight columns come by one 2-D TMA box per column
  int S;        // split-K: CTAs per cluster, each over 1/S of the 256-wide K columns
};

// Split-K cluster helpers (distributed shared memory).
__device__ __forceinline__ uint32_t gemm_cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void gemm_cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t gemm_cluster_map(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ void gemm_st_cluster_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared::cluster.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}

template <int TYPE, int LAYOUT, int TOK>
__global__ void __launch_bounds__(GEMM_THREADS, 1) gemm_tc_kernel(const __grid_constant__ CUtensorMap xmap,
                                                                   const __grid_constant__ CUtensorMap wmap,
                                                                   const GemmParams p) {
  constexpr uint32_t W_STAGE = GEMM_BM * 128;  // bytes
  constexpr uint32_t X_STAGE = TOK * 128;
  constexpr uint32_t RAW_STAGE = GEMM_BM * RawCol<TYPE>::pitch;
  constexpr int CB = RawCol<TYPE>::bytes;
  // UMMA N is at most 256: a 512-token tile is two MMAs per K step into
  // accumulator columns [0, 256) and [256, 512)
  constexpr int NH = TOK > 256 ? 2 : 1;
  constexpr int TN = TOK / NH;
  constexpr uint32_t IDESC = umma_idesc_bf16(GEMM_BM, TN);
  constexpr int GEMM_STAGES = gemm_stages<TYPE, TOK>();
  // When the ring holds a whole 256-wide column (four K stages, TOK = 128),
  // dequant warp (q, h) writes K stage q of rows [32h, 32h + 32) of every
  // column: 64 weights per thread and one set of barrier waits per column,
  // instead of 16 weights per thread and per stage.
  constexpr bool kColumnWarps = GEMM_STAGES >= 4;
  constexpr int kFullArrivals = 1 + (kColumnWarps ? 4 : GEMM_DQ_THREADS / 32);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* w_sm = smem;
  uint8_t* x_sm = smem + GEMM_STAGES * W_STAGE;
  uint8_t* raw_sm = x_sm + GEMM_STAGES * X_STAGE;
  uint64_t* full = reinterpret_cast<uint64_t*>(raw_sm + GEMM_RAW_STAGES * RAW_STAGE);
  uint64_t* empty = full + GEMM_STAGES;
  uint64_t* raw_full = empty + GEMM_STAGES;
  uint64_t* raw_empty = raw_full + GEMM_RAW_STAGES;
  uint64_t* accum = raw_empty + GEMM_RAW_STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // split-K: the S CTAs of a cluster share one output tile, rank r taking
  // 256-wide K columns [c0, c1)
  const int split = p.S > 1 ? p.S : 1;
  const int rank = split > 1 ? (int)gemm_cluster_rank() : 0;
  const int64_t n0 = (int64_t)(blockIdx.x / split) * GEMM_BM;
  const int m0 = (int)blockIdx.y * TOK;
  const int NCOL = (int)(p.K / 256);
  const int c0 = NCOL * rank / split, c1 = NCOL * (rank + 1) / split;
  const int kb0 = 4 * c0, kb1 = 4 * c1;
  const int rows_valid = (int)min((int64_t)GEMM_BM, p.N - n0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < GEMM_STAGES; ++s) {
      mbar_init(&full[s], kFullArrivals);
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < GEMM_RAW_STAGES; ++s) {
      mbar_init(&raw_full[s], 1);
      mbar_init(&raw_empty[s], GEMM_DQ_THREADS / 32);
    }
    mbar_init(accum, 1);
    fence_mbar_init();
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&xmap)) : "memory");
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TOK);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_d = *tmem_slot;
  bool have = false;  // epilogue warps: the accumulator is complete

  if (warp == 0) {
    // ---- x tiles: TMA 2-D, 128B swizzle
    if (lane == 0) {
      for (int kb = kb0; kb < kb1; ++kb) {
        const int s = (kb - kb0) % GEMM_STAGES;
        const uint32_t par = (uint32_t)(((kb - kb0) / GEMM_STAGES) & 1);
        if (!mbar_wait_bounded(&empty[s], par ^ 1)) break;
        mbar_arrive_expect_tx(&full[s], X_STAGE);
#pragma unroll
        for (int h = 0; h < NH; ++h)
          tma_load_2d(x_sm + s * X_STAGE + h * TN * 128, &xmap, kb * GEMM_BK, m0 + h * TN, &full[s]);
      }
    }
  } else if (warp == 1) {
    // ---- MMA issue (one thread)
    if (lane == 0) {
      const uint32_t w_base = smem_u32(w_sm), x_base = smem_u32(x_sm);
      bool ok = true;
      for (int kb = kb0; kb < kb1; ++kb) {
        const int s = (kb - kb0) % GEMM_STAGES;
        const uint32_t par = (uint32_t)(((kb - kb0) / GEMM_STAGES) & 1);
        if (!mbar_wait_bounded(&full[s], par)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < GEMM_BK / 16; ++kk) {
          const uint64_t ad = umma_desc_sw128(w_base + s * W_STAGE + kk * 32);
#pragma unroll
          for (int h = 0; h < NH; ++h) {
            const uint64_t bd = umma_desc_sw128(x_base + s * X_STAGE + h * TN * 128 + kk * 32);
            tc_mma_bf16(tmem_d + (uint32_t)(h * TN), ad, bd, IDESC, (kb != kb0 || kk != 0) ? 1u : 0u);
          }
        }
        tc_commit(&empty[s]);
      }
      if (ok) tc_commit(accum);
    }
  } else if (warp == 2) {
    // ---- raw GGUF bytes of the CTA's 128 rows, one 256-wide column at a time
    const int64_t total = p.N * p.RB;
    const int64_t cap = total & ~int64_t(15);
    for (int c = c0; c < c1; ++c) {
      const int rs = (c - c0) % GEMM_RAW_STAGES;
      if (!mbar_wait_bounded(&raw_empty[rs], (uint32_t)((((c - c0) / GEMM_RAW_STAGES) & 1) ^ 1))) break;
      fence_proxy_async_smem();
      uint8_t* dst = raw_sm + rs * RAW_STAGE;
      if (p.wmap_ok) {
        // rows are 16-byte aligned: one 2-D box [128 rows x pitch bytes]
        // (16-bit elements) starting at the column's 16-byte aligned offset
        if (lane == 0) {
          const int x0 = (int)(((int64_t)c * CB) & ~int64_t(15)) / 2;
          mbar_arrive_expect_tx(&raw_full[rs], RAW_STAGE);
          tma_load_2d(dst, &wmap, x0, (int)n0, &raw_full[rs]);
        }
      } else {
        // one 1-D bulk copy per row (16-byte aligned span of the column)
        uint32_t bytes = 0;
        for (int r = lane; r < rows_valid; r += 32) {
          const int64_t off = (n0 + r) * p.RB + (int64_t)c * CB;
          const int64_t a16 = off & ~int64_t(15);
          int64_t e16 = (off + CB + 15) & ~int64_t(15);
          if (e16 > cap) e16 = cap > a16 ? cap : a16;
          bytes += (uint32_t)(e16 - a16);
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) bytes += __shfl_xor_sync(0xffffffffu, bytes, o);
        if (lane == 0) mbar_expect_tx(&raw_full[rs], bytes);
        __syncwarp();
        for (int r = lane; r < rows_valid; r += 32) {
          const int64_t off = (n0 + r) * p.RB + (int64_t)c * CB;
          const int64_t a16 = off & ~int64_t(15);
          int64_t e16 = (off + CB + 15) & ~int64_t(15);
          if (e16 > cap) {
            // the tensor ends inside this span: copy the tail bytes by hand
            for (int64_t i = cap > a16 ? cap : a16; i < off + CB; ++i)
              dst[r * RawCol<TYPE>::pitch + (i - a16)] = p.w[i];
            e16 = cap > a16 ? cap : a16;
          }
          if (e16 > a16) bulk_g2s(dst + r * RawCol<TYPE>::pitch, p.w + a16, (uint32_t)(e16 - a16), &raw_full[rs]);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&raw_full[rs]);
      }
    }
  } else if (warp >= GEMM_DQ_WARP0) {
    bool ok = true;
    if constexpr (kColumnWarps) {
    // ---- dequant, one warp per (K stage q, 32-row quarter h) of every
    // column; a thread writes all 8 chunks of its row's stage, so a
    // quarter-warp's stores (8 consecutive rows, one chunk) hit 8 distinct
    // bank groups
    const int dw = warp - GEMM_DQ_WARP0, q = dw & 3, r = 32 * (dw >> 2) + lane;
    const bool row_ok = r < rows_valid;
    // stage kb - kb0 = 4 (c - c0) + q: slot and parity advanced by 4 per column
    int s = q, rs = 0;
    uint32_t spar = 0u, rpar = 0u;
    for (int c = c0; c < c1; ++c) {
      if (!mbar_wait_bounded(&raw_full[rs], rpar)) {
        ok = false;
        break;
      }
      uint32_t pk[4][8];
      int chunk[4][2];
      if (row_ok) {
        const int64_t off = (n0 + r) * p.RB + (int64_t)c * CB;
        const uint8_t* raw = raw_sm + rs * RAW_STAGE + r * RawCol<TYPE>::pitch + (int)(off & 15);
#pragma unroll
        for (int qq = 0; qq < 4; ++qq) dequant_col_kblock<TYPE, LAYOUT>(raw, q, qq, pk[qq], chunk[qq]);
      } else {
#pragma unroll
        for (int qq = 0; qq < 4; ++qq) {
#pragma unroll
          for (int i = 0; i < 8; ++i) pk[qq][i] = 0u;
          chunk[qq][0] = 2 * qq;
          chunk[qq][1] = 2 * qq + 1;
        }
      }
      // this column's raw bytes are no longer read by this warp
      __syncwarp();
      if (lane == 0) mbar_arrive(&raw_empty[rs]);
      if (!mbar_wait_bounded(&empty[s], spar ^ 1u)) {
        ok = false;
        break;
      }
      uint8_t* dst = w_sm + s * W_STAGE + r * 128;
#pragma unroll
      for (int qq = 0; qq < 4; ++qq) {
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const int cc = chunk[qq][i] ^ (r & 7);
          *reinterpret_cast<uint4*>(dst + cc * 16) =
              make_uint4(pk[qq][4 * i], pk[qq][4 * i + 1], pk[qq][4 * i + 2], pk[qq][4 * i + 3]);
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&full[s]);
      s += 4;
      if (s >= GEMM_STAGES) {
        s -= GEMM_STAGES;
        spar ^= 1u;
      }
      if (++rs == GEMM_RAW_STAGES) {
        rs = 0;
        rpar ^= 1u;
      }
    }
    } else {
    // ---- dequant: each quarter-warp covers 8 distinct rows of one K
    // quarter, so its 16-byte swizzled stores hit 8 distinct bank groups
    const int t = threadIdx.x - GEMM_DQ_WARP0 * 32;  // 0..511
    const int qq = (t >> 3) & 3;
    const int r = (t & 7) | ((t >> 5) << 3);
    const bool row_ok = r < rows_valid;
    for (int kb = kb0; kb < kb1; ++kb) {
      const int c = kb >> 2, q = kb & 3, rs = (c - c0) % GEMM_RAW_STAGES;
      const int s = (kb - kb0) % GEMM_STAGES;
      if (q == 0 && !mbar_wait_bounded(&raw_full[rs], (uint32_t)(((c - c0) / GEMM_RAW_STAGES) & 1))) {
        ok = false;
        break;
      }
      uint32_t pk[8];
      int chunk[2];
      if (row_ok) {
        const int64_t off = (n0 + r) * p.RB + (int64_t)c * CB;
        const uint8_t* raw = raw_sm + rs * RAW_STAGE + r * RawCol<TYPE>::pitch + (int)(off & 15);
        dequant_col_kblock<TYPE, LAYOUT>(raw, q, qq, pk, chunk);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) pk[i] = 0u;
        chunk[0] = 2 * qq;
        chunk[1] = 2 * qq + 1;
      }
      if (q == 3) {
        // this column's raw bytes are no longer read by this warp
        __syncwarp();
        if (lane == 0) mbar_arrive(&raw_empty[rs]);
      }
      if (!mbar_wait_bounded(&empty[s], (uint32_t)((((kb - kb0) / GEMM_STAGES) & 1) ^ 1))) {
        ok = false;
        break;
      }
      uint8_t* dst = w_sm + s * W_STAGE + r * 128;
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int cc = chunk[i] ^ (r & 7);
        *reinterpret_cast<uint4*>(dst + cc * 16) = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&full[s]);
    }
    }
    // ---- epilogue: warp w reads TMEM lanes 32*(w%4).. (its W rows) for a
    // quarter of the TOK accumulator columns
    have = ok && mbar_wait_bounded(accum, 0);
    if (have) tc_fence_after();
    if (split == 1) {
      if (have) {
        const int qd = warp & 3;
        const int part = (warp - GEMM_DQ_WARP0) >> 2;  // 0..3
        const int64_t n = n0 + 32 * qd + lane;
#pragma unroll 1
        for (int cc = part * (TOK / 4); cc < (part + 1) * (TOK / 4); cc += 32) {
          uint32_t v[32];
          tc_ld_32x32b_x32(tmem_d + ((uint32_t)(32 * qd) << 16) + (uint32_t)cc, v);
          if (n < p.N) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int64_t m = (int64_t)m0 + cc + j;
              if (m < p.M) p.y[m * p.N + n] = __float2bfloat16_rn(__uint_as_float(v[j]));
            }
          }
        }
      }
    }
  }
  if (split > 1) {
    // Split-K reduction through distributed shared memory, in rounds of 32
    // accumulator columns per epilogue warp.  The non-leader ranks store
    // their partial sums into the leader's shared memory (the stage and raw
    // buffers, idle once the MMAs are done; slot [rank - 1][warp][lane][32]
    // f32), the leader adds them in rank order and writes bf16.  Every
    // thread of every CTA passes the same cluster barriers.
    constexpr int kRounds = TOK / 4 / 32;
    float* slots = reinterpret_cast<float*>(smem);
    const bool epi_warp = warp >= GEMM_DQ_WARP0;
    const int qd = warp & 3;
    const int part = (warp - GEMM_DQ_WARP0) >> 2;
    const int ew = warp - GEMM_DQ_WARP0;  // 0..15
    gemm_cluster_sync();  // every CTA of the cluster is past its main loop
#pragma unroll 1
    for (int rd = 0; rd < kRounds; ++rd) {
      const int cc = part * (TOK / 4) + 32 * rd;
      uint32_t v[32];
      if (epi_warp) {
        if (have) {
          tc_ld_32x32b_x32(tmem_d + ((uint32_t)(32 * qd) << 16) + (uint32_t)cc, v);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = 0u;
        }
        if (rank > 0) {
          const uint32_t dst = gemm_cluster_map(slots + ((size_t)((rank - 1) * 16 + ew) * 32 + lane) * 32, 0);
#pragma unroll
          for (int j = 0; j < 32; j += 4) gemm_st_cluster_v4(dst + 4 * j, v[j], v[j + 1], v[j + 2], v[j + 3]);
        }
      }
      gemm_cluster_sync();  // partials of this round have landed in the leader
      if (epi_warp && rank == 0) {
        const int64_t n = n0 + 32 * qd + lane;
        float acc[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[j] = __uint_as_float(v[j]);
        for (int r = 1; r < split; ++r) {
          const float4* src = reinterpret_cast<const float4*>(slots + ((size_t)((r - 1) * 16 + ew) * 32 + lane) * 32);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float4 f = src[j];
            acc[4 * j] += f.x;
            acc[4 * j + 1] += f.y;
            acc[4 * j + 2] += f.z;
            acc[4 * j + 3] += f.w;
          }
        }
        if (n < p.N && have) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int64_t m = (int64_t)m0 + cc + j;
            if (m < p.M) p.y[m * p.N + n] = __float2bfloat16_rn(acc[j]);
          }
        }
      }
      gemm_cluster_sync();  // the leader is done with the slots of this round
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_d, TOK);
  }
}

// ---------------------------------------------------------------------------
// Host side
static PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
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

static int encode_xmap(CUtensorMap* map, const void* x, int64_t M, int64_t K, int box_rows) {
  auto enc = get_encode_fn();
  if (!enc) return NSQ_ERR_CUDA;
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)M};
  cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  cuuint32_t box[2] = {(cuuint32_t)GEMM_BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(x), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? NSQ_OK : NSQ_ERR_CUDA;
}

template <int TYPE, int TOK>
static size_t gemm_smem_bytes() {
  constexpr int S = gemm_stages<TYPE, TOK>();
  return 1024 + (size_t)S * (GEMM_BM * 128 + TOK * 128) + (size_t)GEMM_RAW_STAGES * GEMM_BM * RawCol<TYPE>::pitch +
         (2 * S + 2 * GEMM_RAW_STAGES + 1) * 8 + 16;
}

template <int TYPE, int LAYOUT, int TOK>
static int launch_gemm_t(const void* x, const CUtensorMap& wmap, const GemmParams& p0, cudaStream_t st, int num_sms) {
  auto kern = gemm_tc_kernel<TYPE, LAYOUT, TOK>;
  // the x tensor map's box is the kernel's own token tile (TMA boxes hold
  // at most 256 rows: a 512-token tile is loaded as two boxes)
  alignas(64) CUtensorMap map{};
  const int rc = encode_xmap(&map, x, p0.M, p0.K, TOK > 256 ? 256 : TOK);
  if (rc) return rc;
  const size_t smem = gemm_smem_bytes<TYPE, TOK>();
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return NSQ_ERR_CUDA;
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  GemmParams p = p0;
  const int64_t tiles_n = (p.N + GEMM_BM - 1) / GEMM_BM, tiles_m = (p.M + TOK - 1) / TOK;
  if (tiles_m > 65535) return NSQ_ERR_SHAPE;
  // Split-K when the tiles leave most SMs idle: S CTAs per tile (cluster),
  // as many as the SMs allow, at most 4, each with >= 2 K columns, and no
  // more partial-sum slots than the leader's stage buffers hold.
  constexpr size_t region = (size_t)gemm_stages<TYPE, TOK>() * (GEMM_BM * 128 + TOK * 128) +
                            (size_t)GEMM_RAW_STAGES * GEMM_BM * RawCol<TYPE>::pitch;
  int S = 1;
  const int64_t tiles = tiles_n * tiles_m, ncol = p.K / 256;
  S = tune(kTuneGemmSplit, num_sms > 0 && tiles * 2 <= num_sms ? (int)(num_sms / tiles) : 1);
  if (S > 4) S = 4;
  while (S > 1 && (ncol < 2 * S || (size_t)(S - 1) * 16 * 32 * 32 * 4 > region)) --S;
  if (S < 1) S = 1;
  p.S = S;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(tiles_n * S), (unsigned)tiles_m);
  cfg.blockDim = dim3(GEMM_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)S;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = S > 1 ? 1 : 0;
  note_launch();
  return cudaLaunchKernelEx(&cfg, kern, map, wmap, p) == cudaSuccess ? NSQ_OK : NSQ_ERR_CUDA;
}

template <int TYPE, int LAYOUT>
static int run_gemm_t(const void* x, const GemmParams& p0, int tok, cudaStream_t st, int num_sms) {
  GemmParams p = p0;
  alignas(64) CUtensorMap wmap{};
  p.wmap_ok = 0;
  if (p.RB % 16 == 0 && p.N <= 0x7FFFFFFF) {
    // W viewed as [N rows x RB bytes] of 16-bit elements; box = one column
    auto enc = get_encode_fn();
    if (enc) {
      cuuint64_t dims[2] = {(cuuint64_t)(p.RB / 2), (cuuint64_t)p.N};
      cuuint64_t strides[1] = {(cuuint64_t)p.RB};
      cuuint32_t box[2] = {(cuuint32_t)(RawCol<TYPE>::pitch / 2), (cuuint32_t)GEMM_BM};
      cuuint32_t estr[2] = {1, 1};
      if (enc(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<uint8_t*>(p.w), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS)
        p.wmap_ok = 1;
    }
  }
  if (tok == 128) return launch_gemm_t<TYPE, LAYOUT, 128>(x, wmap, p, st, num_sms);
  if constexpr (gemm_stages<TYPE, 512>() >= 2) {
    if (tok == 512) return launch_gemm_t<TYPE, LAYOUT, 512>(x, wmap, p, st, num_sms);
  }
  return launch_gemm_t<TYPE, LAYOUT, 256>(x, wmap, p, st, num_sms);
}

int run_gemm_bf16(const uint8_t* w, int type, int layout, const void* x, void* y, int64_t M, int64_t N, int64_t K,
                  cudaStream_t st, int num_sms) {
  if (K % 256) return NSQ_ERR_SHAPE;  // whole 256-weight columns
  GemmParams p{};
  p.w = w;
  p.y = static_cast<__nv_bfloat16*>(y);
  p.M = M;
  p.N = N;
  p.K = K;
  p.RB = (K / nsq_block_weights(type)) * nsq_block_bytes(type);
  // tokens per CTA: 128 for short prompts, else 256 or 512 (NSQ_GEMM_TOK
  // overrides); a 512-token tile reuses each dequantized weight tile twice
  // as often, where two 64-wide stages of it fit beside the raw bytes
  int tok = M <= 128 ? 128 : (M >= 512 ? 512 : 256);
  // a short matrix whose 512-token tiles would leave three quarters of the
  // SMs idle takes 256-token tiles (twice the tiles, half the split-K
  // clusters): Q6_K [4096 x 14336] at M = 512, 463 against 431 TFLOP/s
  if (tok == 512 && num_sms > 0 && ((N + 127) / 128) * ((M + 511) / 512) * 4 < num_sms) tok = 256;
  const int te = tune(kTuneGemmTok, 0);
  if (te == 128 || te == 256 || te == 512) tok = te;
  if (M <= 128) tok = 128;
  switch (type) {
    case NSQ_TYPE_Q4_0: return run_gemm_t<NSQ_TYPE_Q4_0, 0>(x, p, tok, st, num_sms);
    case NSQ_TYPE_Q8_0: return run_gemm_t<NSQ_TYPE_Q8_0, 0>(x, p, tok, st, num_sms);
    case NSQ_TYPE_Q4_K: return run_gemm_t<NSQ_TYPE_Q4_K, 0>(x, p, tok, st, num_sms);
    case NSQ_TYPE_Q5_K:
      if (layout == NSQ_Q6K_NODESTOR) return run_gemm_t<NSQ_TYPE_Q5_K, NSQ_Q6K_NODESTOR>(x, p, tok, st, num_sms);
      return run_gemm_t<NSQ_TYPE_Q5_K, NSQ_Q6K_GGML>(x, p, tok, st, num_sms);
    case NSQ_TYPE_Q6_K:
      if (layout == NSQ_Q6K_NODESTOR) return run_gemm_t<NSQ_TYPE_Q6_K, NSQ_Q6K_NODESTOR>(x, p, tok, st, num_sms);
      return run_gemm_t<NSQ_TYPE_Q6_K, NSQ_Q6K_GGML>(x, p, tok, st, num_sms);
    default: return NSQ_ERR_TYPE;
  }
}

}  // namespace nsq
