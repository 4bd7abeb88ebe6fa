// gemv.cu -- decode GEMV over GGUF quant blocks, batch M = 1..16.
//
//   y[m, n] = sum_k x[m, k] * W[n, k]        W: N rows of GGUF blocks
//
// Step 1 (prepare_x_kernel): each run of 32 activations of a token becomes
//   a scale sx and int16 values X split into a signed high byte and an
//   unsigned low byte (x ~= sx * (256*hi + lo)), plus the integer sums of X
//   over each half of 16.  Stored as 80-byte XGroup records in the
//   caller's workspace.
// Step 2 (gemv_kernel): rows of W stream from HBM into a ring of shared
//   memory stages with 1-D bulk async copies (TMA, one elected thread,
//   mbarrier completion).  Each thread owns fixed "units" (32 or 64 weights
//   at fixed K positions) of a row, unpacks nibbles / 6-bit values into
//   bytes, and forms exact integer dot products with dp4a against the two
//   activation bytes.  Per 16 or 32 weights the integer sum is converted
//   once and scaled in fp32 (block scale * sub-block scale * sx).  Partials
//   of a row are reduced with warp shuffles and shared-memory atomics.
//
// Parity: the activation split bounds |x - sx*X| by sx/2 = max|x|/65534 per
// group, i.e. about 3e-5 relative error on y, inside the 1e-3 tolerance
// against the reference's f32 composition (crates/nodestor-vulkan/src/
// pipeline.rs:1256-1268 over the dequant of q4_k.rs / q8_0.rs / the
// dequant_q4 / dequant_q6k shaders).
#include <stdlib.h>

#include "nsq_common.cuh"

namespace nsq {

// ---------------------------------------------------------------------------
// Activation preparation: one warp per (token, group of 32).
__global__ void __launch_bounds__(256) prepare_x_kernel(const float* __restrict__ x, XGroup* __restrict__ xg,
                                                        int64_t n_groups_total, int64_t groups_per_row) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  // launched with programmatic stream serialization: x may come from the
  // previous kernel and the workspace may still be read by it
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  for (int64_t gi = warp; gi < n_groups_total; gi += nwarps) {
    const int64_t m = gi / groups_per_row, g = gi % groups_per_row;
    const float v = x[(m * groups_per_row + g) * 32 + lane];
    float amax = fabsf(v);
#pragma unroll
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float inv = amax > 0.f ? 32767.0f / amax : 0.f;
    int X = __float2int_rn(v * inv);
    X = max(-32767, min(32767, X));
    int hs = X;
#pragma unroll
    for (int o = 8; o; o >>= 1) hs += __shfl_xor_sync(0xffffffffu, hs, o);
    XGroup* r = xg + gi;
    r->hi[lane] = (int8_t)(X >> 8);
    r->lo[lane] = (uint8_t)(X & 0xFF);
    if (lane == 0) {
      r->sx = amax / 32767.0f;
      r->s16[0] = hs;
      r->pad = 0;
    }
    if (lane == 16) r->s16[1] = hs;
  }
}

// ---------------------------------------------------------------------------
// Activation group in registers.
struct XRegs {
  uint32_t hi[8], lo[8];
  float sx;
  int t0, t1;  // s16[0], s16[1]
};

__device__ __forceinline__ void load_xgroup(const XGroup* __restrict__ p, XRegs& r) {
  const uint4* q = reinterpret_cast<const uint4*>(p);
  const uint4 a = __ldg(q + 0), b = __ldg(q + 1), c = __ldg(q + 2), d = __ldg(q + 3), e = __ldg(q + 4);
  r.hi[0] = a.x; r.hi[1] = a.y; r.hi[2] = a.z; r.hi[3] = a.w;
  r.hi[4] = b.x; r.hi[5] = b.y; r.hi[6] = b.z; r.hi[7] = b.w;
  r.lo[0] = c.x; r.lo[1] = c.y; r.lo[2] = c.z; r.lo[3] = c.w;
  r.lo[4] = d.x; r.lo[5] = d.y; r.lo[6] = d.z; r.lo[7] = d.w;
  r.sx = __uint_as_float(e.x);
  r.t0 = (int)e.y;
  r.t1 = (int)e.z;
}

// One decoded group of 32 weights: 8 words of 4 byte-values each, the fp32
// multipliers of the two 16-weight halves, the integer offset subtracted
// from every weight (8 for Q4_0, 32 for Q6_K) and the Q4_K min term.
struct DGroup {
  uint32_t q[8];
  float a0, a1, bmin;
};

template <bool SIGNED_W, int OFF>
__device__ __forceinline__ float group_dot(const DGroup& w, const XRegs& x) {
  int h0 = 0, l0 = 0, h1 = 0, l1 = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if constexpr (SIGNED_W) {
      h0 = dp4a_ss(w.q[i], x.hi[i], h0);
      l0 = dp4a_su(w.q[i], x.lo[i], l0);
      h1 = dp4a_ss(w.q[i + 4], x.hi[i + 4], h1);
      l1 = dp4a_su(w.q[i + 4], x.lo[i + 4], l1);
    } else {
      h0 = dp4a_us(w.q[i], x.hi[i], h0);
      l0 = dp4a_uu(w.q[i], x.lo[i], l0);
      h1 = dp4a_us(w.q[i + 4], x.hi[i + 4], h1);
      l1 = dp4a_uu(w.q[i + 4], x.lo[i + 4], l1);
    }
  }
  int s0 = (h0 << 8) + l0, s1 = (h1 << 8) + l1;
  if constexpr (OFF != 0) {
    s0 -= OFF * x.t0;
    s1 -= OFF * x.t1;
  }
  float r = fmaf(w.a0, (float)s0, w.a1 * (float)s1);
  r = fmaf(-w.bmin, (float)(x.t0 + x.t1), r);
  return x.sx * r;
}

// ---------------------------------------------------------------------------
// Per-format unit decoders.  `blk` points at the unit's block in shared
// memory; `ub` is the unit index inside the block.
template <int TYPE, int LAYOUT>
struct Unit;

template <int LAYOUT>
struct Unit<NSQ_TYPE_Q4_0, LAYOUT> {
  static constexpr int NG = 1, UPB = 1, OFF = 8;
  static constexpr bool SIGNED = false;
  __device__ static int64_t group(int64_t u, int) { return u; }
  __device__ static void decode(const uint8_t* blk, int, DGroup (&g)[NG]) {
    const float d = h2f(ld_u16(blk));
    uint32_t qs[4];
    ld_words_unaligned<4>(blk + 2, qs);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      g[0].q[i] = qs[i] & 0x0F0F0F0Fu;
      g[0].q[i + 4] = (qs[i] >> 4) & 0x0F0F0F0Fu;
    }
    g[0].a0 = d; g[0].a1 = d; g[0].bmin = 0.f;
  }
};

template <int LAYOUT>
struct Unit<NSQ_TYPE_Q8_0, LAYOUT> {
  static constexpr int NG = 1, UPB = 1, OFF = 0;
  static constexpr bool SIGNED = true;
  __device__ static int64_t group(int64_t u, int) { return u; }
  __device__ static void decode(const uint8_t* blk, int, DGroup (&g)[NG]) {
    const float d = h2f(ld_u16(blk));
    ld_words_unaligned<8>(blk + 2, g[0].q);
    g[0].a0 = d; g[0].a1 = d; g[0].bmin = 0.f;
  }
};

template <int LAYOUT>
struct Unit<NSQ_TYPE_Q4_K, LAYOUT> {
  // unit p (0..3) = qs[32p .. 32p+32): low nibbles -> sub-block 2p,
  // high nibbles -> sub-block 2p+1 (q4_k.rs:86-111)
  static constexpr int NG = 2, UPB = 4, OFF = 0;
  static constexpr bool SIGNED = false;
  __device__ static int64_t group(int64_t u, int gi) { return 2 * u + gi; }
  __device__ static void scale_min(uint32_t S0, uint32_t S1, uint32_t S2, int j, uint32_t& sc, uint32_t& m) {
    // get_scale_min_k4 (q4_k.rs:120-131) with the 12 scale bytes in 3 words
    if (j < 4) {
      const int sh = 8 * j;
      sc = (S0 >> sh) & 63;
      m = (S1 >> sh) & 63;
    } else {
      const int sh = 8 * (j - 4);
      const uint32_t b2 = (S2 >> sh) & 0xFF, b0 = (S0 >> sh) & 0xFF, b1 = (S1 >> sh) & 0xFF;
      sc = (b2 & 0xF) | ((b0 >> 6) << 4);
      m = (b2 >> 4) | ((b1 >> 6) << 4);
    }
  }
  __device__ static void decode(const uint8_t* blk, int p, DGroup (&g)[NG]) {
    const uint4 hdr = *reinterpret_cast<const uint4*>(blk);
    const float d = h2f((uint16_t)(hdr.x & 0xFFFF)), dmin = h2f((uint16_t)(hdr.x >> 16));
    uint32_t sc0, m0, sc1, m1;
    scale_min(hdr.y, hdr.z, hdr.w, 2 * p, sc0, m0);
    scale_min(hdr.y, hdr.z, hdr.w, 2 * p + 1, sc1, m1);
    const uint4 qa = *reinterpret_cast<const uint4*>(blk + 16 + 32 * p);
    const uint4 qb = *reinterpret_cast<const uint4*>(blk + 32 + 32 * p);
    const uint32_t qw[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      g[0].q[i] = qw[i] & 0x0F0F0F0Fu;
      g[1].q[i] = (qw[i] >> 4) & 0x0F0F0F0Fu;
    }
    g[0].a0 = g[0].a1 = d * (float)sc0;
    g[0].bmin = dmin * (float)m0;
    g[1].a0 = g[1].a1 = d * (float)sc1;
    g[1].bmin = dmin * (float)m1;
  }
};

// 4 high bits (one per byte, for 4 consecutive weights) from a nibble.

template <int LAYOUT>
struct Unit<NSQ_TYPE_Q5_K, LAYOUT> {
  // Q4_K's units (qs at byte 48) with the fifth bit of every weight from
  // qh[32]: ggml: bit j of qh[l]; NODESTOR (q5_k.rs:57-70): bit l%8 of
  // qh[8(j>>1) + 4(j&1) + l/8], j the sub-block, l the element
  static constexpr int NG = 2, UPB = 4, OFF = 0;
  static constexpr bool SIGNED = false;
  __device__ static int64_t group(int64_t u, int gi) { return 2 * u + gi; }
  __device__ static void decode(const uint8_t* blk, int p, DGroup (&g)[NG]) {
    const uint4 hdr = *reinterpret_cast<const uint4*>(blk);
    const float d = h2f((uint16_t)(hdr.x & 0xFFFF)), dmin = h2f((uint16_t)(hdr.x >> 16));
    uint32_t sc0, m0, sc1, m1;
    Unit<NSQ_TYPE_Q4_K, 0>::scale_min(hdr.y, hdr.z, hdr.w, 2 * p, sc0, m0);
    Unit<NSQ_TYPE_Q4_K, 0>::scale_min(hdr.y, hdr.z, hdr.w, 2 * p + 1, sc1, m1);
    const uint4 qa = *reinterpret_cast<const uint4*>(blk + 48 + 32 * p);
    const uint4 qb = *reinterpret_cast<const uint4*>(blk + 64 + 32 * p);
    const uint32_t qw[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
    uint32_t hl[8], hh[8];
    if constexpr (LAYOUT == NSQ_Q6K_NODESTOR) {
      const uint2 h = *reinterpret_cast<const uint2*>(blk + 16 + 8 * p);  // bytes 8p .. 8p+7
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        hl[i] = spread4(((h.x >> (8 * (i >> 1))) >> (4 * (i & 1))) & 0xF);
        hh[i] = spread4(((h.y >> (8 * (i >> 1))) >> (4 * (i & 1))) & 0xF);
      }
    } else {
      const uint4 ha = *reinterpret_cast<const uint4*>(blk + 16), hb = *reinterpret_cast<const uint4*>(blk + 32);
      const uint32_t hw[8] = {ha.x, ha.y, ha.z, ha.w, hb.x, hb.y, hb.z, hb.w};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        hl[i] = (hw[i] >> (2 * p)) & 0x01010101u;
        hh[i] = (hw[i] >> (2 * p + 1)) & 0x01010101u;
      }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      g[0].q[i] = (qw[i] & 0x0F0F0F0Fu) | (hl[i] << 4);
      g[1].q[i] = ((qw[i] >> 4) & 0x0F0F0F0Fu) | (hh[i] << 4);
    }
    g[0].a0 = g[0].a1 = d * (float)sc0;
    g[0].bmin = dmin * (float)m0;
    g[1].a0 = g[1].a1 = d * (float)sc1;
    g[1].bmin = dmin * (float)m1;
  }
};

template <>
struct Unit<NSQ_TYPE_Q6_K, NSQ_Q6K_GGML> {
  // unit (n, jj), ub = 2n + jj: groups j = jj and j = jj + 2 of half n share
  // the ql bytes ql[64n + 32jj + l] (low / high nibble) and qh[32n + l]
  static constexpr int NG = 2, UPB = 4, OFF = 32;
  static constexpr bool SIGNED = false;
  __device__ static int64_t group(int64_t u, int gi) {
    const int64_t b = u >> 2;
    const int ub = (int)(u & 3), n = ub >> 1, jj = ub & 1;
    return 8 * b + 4 * n + jj + 2 * gi;
  }
  __device__ static void decode(const uint8_t* blk, int ub, DGroup (&g)[NG]) {
    const int n = ub >> 1, jj = ub & 1;
    uint32_t ql[8], qh[8], scw[2];
    ld_words_unaligned<8>(blk + 64 * n + 32 * jj, ql);
    ld_words_unaligned<8>(blk + 128 + 32 * n, qh);
    ld_words_unaligned<2>(blk + 192 + 8 * n + 2 * jj, scw);  // bytes sc[2jj + 0,1,4,5] of half n
    const float d = h2f(ld_u16(blk + 208));
    const int sa = 2 * jj, sb = 2 * jj + 4;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      g[0].q[i] = (ql[i] & 0x0F0F0F0Fu) | (((qh[i] >> sa) & 0x03030303u) << 4);
      g[1].q[i] = ((ql[i] >> 4) & 0x0F0F0F0Fu) | (((qh[i] >> sb) & 0x03030303u) << 4);
    }
    g[0].a0 = d * (float)(int8_t)(scw[0] & 0xFF);
    g[0].a1 = d * (float)(int8_t)((scw[0] >> 8) & 0xFF);
    g[1].a0 = d * (float)(int8_t)(scw[1] & 0xFF);
    g[1].a1 = d * (float)(int8_t)((scw[1] >> 8) & 0xFF);
    g[0].bmin = g[1].bmin = 0.f;
  }
};

template <>
struct Unit<NSQ_TYPE_Q6_K, NSQ_Q6K_NODESTOR> {
  // unit c: elements 64c .. 64c+63 in order (dequant_q6k.comp:50-99):
  // ql[i>>1] nibble (i&1), qh[i>>2] bits 2(i&3), scale byte [i>>4]
  static constexpr int NG = 2, UPB = 4, OFF = 32;
  static constexpr bool SIGNED = false;
  __device__ static int64_t group(int64_t u, int gi) { return 2 * u + gi; }
  __device__ static void decode(const uint8_t* blk, int c, DGroup (&g)[NG]) {
    uint32_t ql[8], qh[4], scw[1];
    ld_words_unaligned<8>(blk + 32 * c, ql);
    ld_words_unaligned<4>(blk + 128 + 16 * c, qh);
    ld_words_unaligned<1>(blk + 192 + 4 * c, scw);
    const float d = h2f(ld_u16(blk + 208));
#pragma unroll
    for (int t = 0; t < 16; ++t) {
      const uint32_t v = (ql[t >> 1] >> (16 * (t & 1))) & 0xFFFFu;
      const uint32_t tt = __byte_perm(v, 0, 0x1100);
      const uint32_t lo4 = (tt & 0x000F000Fu) | ((tt >> 4) & 0x0F000F00u);
      const uint32_t h = (qh[t >> 2] >> (8 * (t & 3))) & 0xFFu;
      const uint32_t s = (h | (h << 6) | (h << 12) | (h << 18)) & 0x03030303u;
      g[t >> 3].q[t & 7] = lo4 | (s << 4);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      g[i].a0 = d * ((float)((int)((scw[0] >> (16 * i)) & 0xFF) - 128) * 0.015625f);
      g[i].a1 = d * ((float)((int)((scw[0] >> (16 * i + 8)) & 0xFF) - 128) * 0.015625f);
      g[i].bmin = 0.f;
    }
  }
};

// ---------------------------------------------------------------------------
struct GemvParams {
  const uint8_t* w;
  const XGroup* xg;
  float* y;
  int64_t N, K, RB, total_bytes;
  int U, UPT, G, P, RT;
  int stage_bytes, nstages;
  int64_t GX;  // x groups per token = K / 32
};

// Issue the bulk copy of stage t (rows [ra, rb)) into slot memory.
__device__ __forceinline__ void issue_stage(const GemvParams& p, uint8_t* slot, uint64_t* bar, int64_t ra,
                                            int64_t rb) {
  const int64_t a = ra * p.RB, b = rb * p.RB;
  const int64_t a16 = a & ~int64_t(15);
  const int64_t b16 = (b + 15) & ~int64_t(15);
  const int64_t cap = p.total_bytes & ~int64_t(15);
  const int64_t cend = b16 < cap ? b16 : cap;
  // bytes past the last 16-byte boundary of the tensor (at most 15, last stage only)
  for (int64_t i = (cend > a16 ? cend : a16); i < b; ++i) slot[i - a16] = p.w[i];
  const uint32_t bytes = cend > a16 ? (uint32_t)(cend - a16) : 0u;
  mbar_arrive_expect_tx(bar, bytes);
  if (bytes) bulk_g2s(slot, p.w + a16, bytes, bar);
}

constexpr int kConsumerWarps = 8;
constexpr int kGemvThreads = 32 * (1 + kConsumerWarps);

template <int TYPE, int LAYOUT, int M, bool XREG, int UMAX>
__global__ void __launch_bounds__(kGemvThreads, 2) gemv_kernel(const GemvParams p) {
  using UT = Unit<TYPE, LAYOUT>;
  constexpr int NG = UT::NG;
  constexpr int BB = Fmt<TYPE>::BB;
  extern __shared__ __align__(128) uint8_t smem[];
  const int red_stride = (p.RT * M + 3) & ~3;
  uint8_t* stages = smem;
  float* red = reinterpret_cast<float*>(smem + (size_t)p.stage_bytes * p.nstages);
  uint64_t* full = reinterpret_cast<uint64_t*>(red + (size_t)red_stride * p.nstages);
  uint64_t* empty = full + p.nstages;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t row_begin = p.N * blockIdx.x / gridDim.x;
  const int64_t row_end = p.N * (blockIdx.x + 1) / gridDim.x;
  const int nst = (int)((row_end - row_begin + p.RT - 1) / p.RT);

  for (int i = tid; i < red_stride * p.nstages; i += blockDim.x) red[i] = 0.f;
  if (tid == 0) {
    for (int s = 0; s < p.nstages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == 0) {
    // ---------------- producer: refills the ring and writes finished rows
    int issued = 0;
    if (lane == 0) {
      for (; issued < nst && issued < p.nstages; ++issued) {
        const int64_t ra = row_begin + (int64_t)issued * p.RT;
        issue_stage(p, stages + (size_t)issued * p.stage_bytes, &full[issued], ra, min(row_end, ra + p.RT));
      }
    }
    issued = __shfl_sync(0xffffffffu, issued, 0);
    bool ok = true;
    for (int t = 0; t < nst; ++t) {
      const int s = t % p.nstages;
      if (!mbar_wait_bounded(&empty[s], (uint32_t)((t / p.nstages) & 1))) {
        ok = false;
        break;
      }
      const int64_t ra = row_begin + (int64_t)t * p.RT;
      const int rows = (int)min((int64_t)p.RT, row_end - ra);
      float* rs = red + (size_t)s * red_stride;
      for (int i = lane; i < rows * M; i += 32) {
        const int r = i / M, m = i - r * M;
        p.y[(int64_t)m * p.N + ra + r] = rs[i];
        rs[i] = 0.f;
      }
      __syncwarp();
      if (lane == 0 && issued < nst) {
        fence_proxy_async_smem();
        const int64_t na = row_begin + (int64_t)issued * p.RT;
        issue_stage(p, stages + (size_t)s * p.stage_bytes, &full[s], na, min(row_end, na + p.RT));
      }
      if (issued < nst) ++issued;
    }
    if (!ok && lane == 0) {
      // wind down: wait (bounded) for the copies still in flight
      for (int t = issued - min(issued, p.nstages); t < issued; ++t)
        (void)mbar_wait_bounded(&full[t % p.nstages], (uint32_t)((t / p.nstages) & 1));
    }
  } else {
    // ---------------- consumers: fixed K units per thread
    const int ct = tid - 32;
    const bool active = ct < p.P * p.G;
    const int prow = ct / p.G;
    const int gsub = ct % p.G;
    const bool warp_rows = (p.G % 32) == 0;

    XRegs xr[XREG ? UMAX * NG : 1];
    if constexpr (XREG) {
#pragma unroll
      for (int i = 0; i < UMAX; ++i) {
        const int64_t u = gsub + (int64_t)i * p.G;
        if (active && i < p.UPT && u < p.U) {
#pragma unroll
          for (int gi = 0; gi < NG; ++gi) load_xgroup(p.xg + UT::group(u, gi), xr[i * NG + gi]);
        }
      }
    }
    for (int t = 0; t < nst; ++t) {
      const int s = t % p.nstages;
      if (!mbar_wait_bounded(&full[s], (uint32_t)((t / p.nstages) & 1))) break;
      const int64_t ra = row_begin + (int64_t)t * p.RT;
      const int rows = (int)min((int64_t)p.RT, row_end - ra);
      const uint8_t* sbase = stages + (size_t)s * p.stage_bytes;
      const int64_t a16 = (ra * p.RB) & ~int64_t(15);
      float* rs = red + (size_t)s * red_stride;
      if (active) {
        for (int r = prow; r < rows; r += p.P) {
          const uint8_t* rowp = sbase + ((ra + r) * p.RB - a16);
          float acc[M];
#pragma unroll
          for (int m = 0; m < M; ++m) acc[m] = 0.f;
#pragma unroll
          for (int i = 0; i < UMAX; ++i) {
            const int64_t u = gsub + (int64_t)i * p.G;
            if (i < p.UPT && u < p.U) {
              const int64_t b = u / UT::UPB;
              const int ub = (int)(u - b * UT::UPB);
              DGroup dg[NG];
              UT::decode(rowp + b * BB, ub, dg);
              if constexpr (XREG) {
#pragma unroll
                for (int gi = 0; gi < NG; ++gi)
                  acc[0] += group_dot<UT::SIGNED, UT::OFF>(dg[gi], xr[i * NG + gi]);
              } else {
#pragma unroll
                for (int gi = 0; gi < NG; ++gi) {
                  const int64_t gx = UT::group(u, gi);
#pragma unroll
                  for (int m = 0; m < M; ++m) {
                    XRegs x1;
                    load_xgroup(p.xg + m * p.GX + gx, x1);
                    acc[m] += group_dot<UT::SIGNED, UT::OFF>(dg[gi], x1);
                  }
                }
              }
            }
          }
          if (warp_rows) {
#pragma unroll
            for (int m = 0; m < M; ++m) {
              float v = acc[m];
#pragma unroll
              for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
              acc[m] = v;
            }
            if (lane == 0) {
#pragma unroll
              for (int m = 0; m < M; ++m) atomicAdd(&rs[r * M + m], acc[m]);
            }
          } else {
#pragma unroll
            for (int m = 0; m < M; ++m) atomicAdd(&rs[r * M + m], acc[m]);
          }
        }
      }
      __threadfence_block();
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
  }
  __syncthreads();
}

// ---------------------------------------------------------------------------
// Host side
template <int TYPE>
static int units_per_row(int64_t K) {
  return (int)(K / Fmt<TYPE>::UW);
}

struct LaunchCfg {
  int threads = 256;
  int blocks = 0;
  size_t smem = 0;
};

template <int TYPE, int LAYOUT, int M, bool XREG, int UMAX>
static cudaError_t launch_gemv_inst(const GemvParams& p, int blocks, size_t smem, cudaStream_t st) {
  auto kern = gemv_kernel<TYPE, LAYOUT, M, XREG, UMAX>;
  static size_t configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || smem > configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) configured[dev] = smem;
  }
  note_launch();
  kern<<<blocks, kGemvThreads, smem, st>>>(p);
  return cudaGetLastError();
}

template <int TYPE, int LAYOUT, int M>
static cudaError_t dispatch_x(const GemvParams& p, int blocks, size_t smem, cudaStream_t st) {
  // UMAX (units per thread) is a template constant so that only the
  // activation registers a launch needs are allocated.
  constexpr bool XR = (M == 1);
  if (p.UPT == 1) return launch_gemv_inst<TYPE, LAYOUT, M, XR, 1>(p, blocks, smem, st);
  if (p.UPT == 2) return launch_gemv_inst<TYPE, LAYOUT, M, XR, 2>(p, blocks, smem, st);
  return launch_gemv_inst<TYPE, LAYOUT, M, false, 4>(p, blocks, smem, st);
}

template <int TYPE, int LAYOUT>
static cudaError_t dispatch_m(const GemvParams& p, int M, int blocks, size_t smem, cudaStream_t st) {
  switch (M) {
    case 1: return dispatch_x<TYPE, LAYOUT, 1>(p, blocks, smem, st);
    case 2: return dispatch_x<TYPE, LAYOUT, 2>(p, blocks, smem, st);
    case 3: return dispatch_x<TYPE, LAYOUT, 3>(p, blocks, smem, st);
    case 4: return dispatch_x<TYPE, LAYOUT, 4>(p, blocks, smem, st);
    default: return cudaErrorNotSupported;
  }
}

// Host-side constants of the launch
constexpr int kThreads = 256;
constexpr int kStageTarget = 24 * 1024;
constexpr int kSmemBudget = 104 * 1024;

template <int TYPE>
static bool plan(int64_t N, int64_t K, int num_sms, GemvParams& p, int& blocks, size_t& smem, int M) {
  const int U = units_per_row<TYPE>(K);
  if (U < 1) return false;
  const int UPT = (U + kThreads - 1) / kThreads;
  if (UPT > 4) return false;
  const int G = (U + UPT - 1) / UPT;
  const int P = kThreads / G;
  const int64_t RB = (K / Fmt<TYPE>::QK) * Fmt<TYPE>::BB;
  int RT = (int)(kStageTarget / RB);
  if (RT < 1) RT = 1;
  // spread small matrices over every SM
  const int64_t want = (N + (int64_t)num_sms * 2 - 1) / ((int64_t)num_sms * 2);
  if (RT > want) RT = (int)(want < 1 ? 1 : want);
  if (RT > P) RT -= RT % P;
  const int stage_bytes = (int)(((int64_t)RT * RB + 32 + 127) & ~int64_t(127));
  int nstages = kSmemBudget / stage_bytes;
  if (nstages > 6) nstages = 6;
  if (nstages < 2) nstages = 2;
  if ((size_t)stage_bytes * nstages > 200 * 1024) return false;
  int64_t nblk = (N + RT - 1) / RT;
  const int64_t cap = (int64_t)num_sms * 2;
  if (nblk > cap) nblk = cap;
  p.N = N; p.K = K; p.RB = RB; p.total_bytes = RB * N;
  p.U = U; p.UPT = UPT; p.G = G; p.P = P; p.RT = RT;
  p.stage_bytes = stage_bytes; p.nstages = nstages; p.GX = K / 32;
  blocks = (int)nblk;
  smem = (size_t)stage_bytes * nstages + (size_t)((RT * M + 3) & ~3) * 4 * nstages + 16 * nstages + 16;
  return true;
}

template <int TYPE, int LAYOUT>
static int run_gemv_t(const uint8_t* w, const XGroup* xg, float* y, int64_t M, int64_t N, int64_t K,
                      cudaStream_t st, int num_sms) {
  // token slices of at most 4 keep the per-thread accumulators in registers
  for (int64_t m0 = 0; m0 < M; m0 += 4) {
    const int mm = (int)((M - m0) < 4 ? (M - m0) : 4);
    GemvParams p{};
    int blocks;
    size_t smem;
    if (!plan<TYPE>(N, K, num_sms, p, blocks, smem, mm)) return NSQ_ERR_SHAPE;
    p.w = w;
    p.xg = xg + m0 * (K / 32);
    p.y = y + m0 * N;
    cudaError_t e = dispatch_m<TYPE, LAYOUT>(p, mm, blocks, smem, st);
    if (e != cudaSuccess) return NSQ_ERR_CUDA;
  }
  return NSQ_OK;
}

int run_gemv_fused(const nsq_segment* segs, int nseg, const float* x, const XGroup* xg, int64_t M, int64_t K,
                   cudaStream_t st, int num_sms, const XchgDesc* xd = nullptr, int epi = 0,
                   const float* const* res = nullptr);
int run_gemv_mma(const nsq_segment* segs, int nseg, const XGroup* xg, int64_t M, int64_t K, cudaStream_t st,
                 int num_sms, const XchgDesc* xd);
int gemv_mma_min_m();

bool gemv_force_general() {
  // NSQ_GEMV_GENERAL=1 forces the general kernel below (the parity tests use
  // it to cover both kernels on the same shapes)
  return tune(kTuneGemvGeneral, 0) == 1;
}

// GEMV on prepared activations: the tensor-core kernel (gemv_mma.cu) for
// M >= gemv_mma_min_m(), else the fused kernel (gemv_rows.cu) in workspace
// mode where the shape allows it, else the general kernel.
int run_gemv(const uint8_t* w, int type, int layout, const XGroup* xg, float* y, int64_t M, int64_t N, int64_t K,
             cudaStream_t st, int num_sms) {
  if (!gemv_force_general()) {
    nsq_segment sg{w, type, layout, N, y};
    int rc = -1;
    if (M >= gemv_mma_min_m()) rc = run_gemv_mma(&sg, 1, xg, M, K, st, num_sms, nullptr);
    if (rc == -1) rc = run_gemv_fused(&sg, 1, nullptr, xg, M, K, st, num_sms);
    if (rc != -1) return rc;
  }
  switch (type) {
    case NSQ_TYPE_Q4_0: return run_gemv_t<NSQ_TYPE_Q4_0, 0>(w, xg, y, M, N, K, st, num_sms);
    case NSQ_TYPE_Q8_0: return run_gemv_t<NSQ_TYPE_Q8_0, 0>(w, xg, y, M, N, K, st, num_sms);
    case NSQ_TYPE_Q4_K: return run_gemv_t<NSQ_TYPE_Q4_K, 0>(w, xg, y, M, N, K, st, num_sms);
    case NSQ_TYPE_Q5_K:
      if (layout == NSQ_Q6K_NODESTOR)
        return run_gemv_t<NSQ_TYPE_Q5_K, NSQ_Q6K_NODESTOR>(w, xg, y, M, N, K, st, num_sms);
      return run_gemv_t<NSQ_TYPE_Q5_K, NSQ_Q6K_GGML>(w, xg, y, M, N, K, st, num_sms);
    case NSQ_TYPE_Q6_K:
      if (layout == NSQ_Q6K_NODESTOR)
        return run_gemv_t<NSQ_TYPE_Q6_K, NSQ_Q6K_NODESTOR>(w, xg, y, M, N, K, st, num_sms);
      return run_gemv_t<NSQ_TYPE_Q6_K, NSQ_Q6K_GGML>(w, xg, y, M, N, K, st, num_sms);
    default: return NSQ_ERR_TYPE;
  }
}

cudaError_t launch_prepare_x(const float* x, XGroup* xg, int64_t M, int64_t K, cudaStream_t st, int num_sms) {
  const int64_t total = M * (K / 32);
  int64_t blocks = (total + 7) / 8;
  const int64_t cap = (int64_t)num_sms * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)blocks);
  cfg.blockDim = dim3(256);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  note_launch();
  return cudaLaunchKernelEx(&cfg, prepare_x_kernel, x, xg, total, K / 32);
}

}  // namespace nsq
