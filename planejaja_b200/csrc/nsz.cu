// nsz.cu -- NSZ (NodeStor Zip, TCA-TBE) lossless tensors: the host tile
// index, the device decoder and ZipGEMM, the fused decompress + GEMV.
//
// Tile bytes (crates/nodestor-formats/src/nsz_format.rs:13-44, written by
// NszTile::to_bytes :291-307): [modal u8][num_res u16][dtype u8][num_near
// u16][2] | match bitmap B | near bitmap B | near deltas ceil(num_near/8) |
// residual exponents num_res | mantissas n*MB | signs B | pad to 64, with
// B = ceil(n/8), MB = 3 / 2 / 1 bytes (FP32 / FP16 / BF16).  Weight i:
// exponent = modal if match bit i, modal +- 1 (next near delta bit) if near
// bit i, else the next residual byte; mantissa and sign verbatim
// (nsz_decoder.rs:19-196).
//
// Device design.  Every warp owns a contiguous run of tiles and keeps
// kDepth of them in flight: lane 0 moves each whole tile (its size from the
// offset table) into a warp-private shared-memory stage with one bulk async
// copy completing on an mbarrier.  A tile is decoded by the 32 lanes at once,
// 16 consecutive weights per lane:
//   * each lane's 16 match / near / sign bits are one 16-bit load;
//   * its first near-delta and residual ranks come from one warp prefix sum
//     of its (near, residual) popcounts;
//   * per group of 4 weights, shared-memory tables turn the 4-bit near and
//     residual masks into byte masks and byte-permute selectors, and the
//     next 4 near-delta bits into a byte mask; the next 4 residual bytes are
//     placed on their weights by one byte permute of the two aligned words
//     around them, so the 4 exponent bytes come out of three word selects;
//   * the lane's mantissas (48 / 32 / 16 bytes) are 8-byte loads; the
//     section's offset modulo 8 is the same for every lane, so a
//     warp-uniform switch picks constant-offset shifts for all 16 fields;
//   * an FP32 weight is assembled by one byte permute (exponent byte to the
//     top) and one funnel shift that brings in the sign bit.
// ZipGEMM splits the output rows evenly over CTAs (a CTA owns rows [r0, r1)
// and writes them once; tiles that straddle its boundary are decoded by both
// neighbours and masked), accumulates each lane's 16 products per token in
// registers while its row stays the same, and adds finished rows into a
// shared-memory row buffer (a warp sum when the warp is on one row).
#include <algorithm>

#include "nsq_common.cuh"

namespace nsq {
int device_check(int* num_sms);  // api.cu

namespace {

constexpr int kNszW = NSQ_NSZ_TILE_WEIGHTS;
constexpr int kNszWarps = 8;
constexpr int kNszDepth = 3;

template <int DT>
struct NszFmt;
// kStage: largest padded tile (8 + 3 * 64 + 512 + 512 * MB + 64, rounded up
// to 64) plus 64 bytes of slack for the decoder's over-reads.
template <>
struct NszFmt<NSQ_NSZ_FP32> {
  static constexpr int MB = 3, kStage = 2432;
};
template <>
struct NszFmt<NSQ_NSZ_FP16> {
  static constexpr int MB = 2, kStage = 1920;
};
template <>
struct NszFmt<NSQ_NSZ_BF16> {
  static constexpr int MB = 1, kStage = 1408;
};

__host__ __device__ __forceinline__ int64_t imin64(int64_t a, int64_t b) { return a < b ? a : b; }
__host__ __device__ __forceinline__ int64_t imax64(int64_t a, int64_t b) { return a > b ? a : b; }

__host__ __device__ constexpr int mant_bytes(int dt) { return dt == NSQ_NSZ_FP32 ? 3 : dt == NSQ_NSZ_FP16 ? 2 : 1; }

__host__ __device__ inline int64_t nsz_tile_bytes(int n, int num_near, int num_res, int dt) {
  const int64_t bm = (n + 7) / 8;
  const int64_t raw = 8 + 2 * bm + (num_near + 7) / 8 + num_res + (int64_t)n * mant_bytes(dt) + bm;
  return (raw + 63) / 64 * 64;
}

__device__ __forceinline__ uint32_t lds_u16_any(const uint8_t* q) {
  if (reinterpret_cast<uintptr_t>(q) & 1) return (uint32_t)q[0] | ((uint32_t)q[1] << 8);
  return *reinterpret_cast<const uint16_t*>(q);
}
// 32 bits starting at byte q (any alignment) from the two aligned words around it.
__device__ __forceinline__ uint32_t lds_u32_any(const uint8_t* q) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(q);
  const uint32_t* w = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
  return __funnelshift_r(w[0], w[1], 8u * (uint32_t)(a & 3));
}

// Shared-memory tables, built once per CTA (indexed by 4-bit masks of the
// weights of one group of 4):
//   m4[b].x: byte-permute selector placing source byte k at the position of
//            the k-th set bit of b (other nibbles 4), popc(b) in bits 16..
//   m4[b].y: byte mask, 0xFF at the set bits of b
//   dx[b * 16 + d]: byte mask, 0xFF at the position of the k-th set bit of b
//            where bit k of d is set (the near deltas placed on the near weights)
struct NszLut {
  uint2 m4[16];
  uint32_t dx[256];
};

__device__ __forceinline__ void init_nsz_lut(NszLut* L) {
  for (int i = threadIdx.x; i < 256; i += blockDim.x) {
    const uint32_t b = (uint32_t)i >> 4, d = (uint32_t)i & 15;
    uint32_t mask = 0, k = 0;
    for (int j = 0; j < 4; ++j)
      if ((b >> j) & 1) {
        if ((d >> k) & 1) mask |= 0xFFu << (8 * j);
        ++k;
      }
    L->dx[i] = mask;
    if (i < 16) {
      uint32_t sel = 0, r = 0;
      for (int j = 0; j < 4; ++j) sel |= ((i >> j) & 1 ? r++ : 4u) << (4 * j);
      L->m4[i] = make_uint2(sel | (r << 16), spread4((uint32_t)i) * 0xFFu);
    }
  }
}

// NB little-endian bytes starting at byte O of the word array W.
template <int O, int NB, int NW>
__device__ __forceinline__ uint32_t bytes_at(const uint32_t (&W)[NW]) {
  constexpr int w = O >> 2, sh = 8 * (O & 3);
  static_assert(w < NW && ((O & 3) + NB <= 4 || w + 1 < NW), "read past the loaded words");
  if constexpr ((O & 3) + NB <= 4) return W[w] >> sh;
  else return __funnelshift_r(W[w], W[w + 1], sh);
}

// The lane's 16 mantissas from its words W (byte D = first mantissa byte);
// FP32 fields keep the bits above 23 (cleared when the weight is assembled).
template <int DT, int D, int NW>
__device__ __forceinline__ void mant_extract(const uint32_t (&W)[NW], uint32_t (&mant)[16]) {
  if constexpr (DT == NSQ_NSZ_FP32) {
#define NSZ_M3(j) mant[j] = bytes_at<D + 3 * (j), 3>(W);  // bits 23.. masked at assembly
    NSZ_M3(0) NSZ_M3(1) NSZ_M3(2) NSZ_M3(3) NSZ_M3(4) NSZ_M3(5) NSZ_M3(6) NSZ_M3(7)
    NSZ_M3(8) NSZ_M3(9) NSZ_M3(10) NSZ_M3(11) NSZ_M3(12) NSZ_M3(13) NSZ_M3(14) NSZ_M3(15)
#undef NSZ_M3
  } else if constexpr (DT == NSQ_NSZ_FP16) {
#define NSZ_M2(j) mant[j] = bytes_at<D + 2 * (j), 2>(W) & 0x3FFu;
    NSZ_M2(0) NSZ_M2(1) NSZ_M2(2) NSZ_M2(3) NSZ_M2(4) NSZ_M2(5) NSZ_M2(6) NSZ_M2(7)
    NSZ_M2(8) NSZ_M2(9) NSZ_M2(10) NSZ_M2(11) NSZ_M2(12) NSZ_M2(13) NSZ_M2(14) NSZ_M2(15)
#undef NSZ_M2
  } else {
#define NSZ_M1(j) mant[j] = bytes_at<D + (j), 1>(W) & 0x7Fu;
    NSZ_M1(0) NSZ_M1(1) NSZ_M1(2) NSZ_M1(3) NSZ_M1(4) NSZ_M1(5) NSZ_M1(6) NSZ_M1(7)
    NSZ_M1(8) NSZ_M1(9) NSZ_M1(10) NSZ_M1(11) NSZ_M1(12) NSZ_M1(13) NSZ_M1(14) NSZ_M1(15)
#undef NSZ_M1
  }
}

// Decodes the 16 weights [16 * lane, 16 * lane + 16) of the n-weight tile at
// p (shared memory, 16-byte aligned) into their original bit patterns (FP16 /
// BF16 in the low half).  vmask: weights that exist (< n).  Warp-collective.
template <int DT, bool FULL>
__device__ __forceinline__ void nsz_decode16(const uint8_t* __restrict__ p, int n_, int lane,
                                             const NszLut& L, uint32_t (&v)[16],
                                             uint32_t& vmask) {
  const int n = FULL ? kNszW : n_;  // FULL: a 512-weight tile, offsets fold to constants
  constexpr int MB = NszFmt<DT>::MB;
  const uint2 h = *reinterpret_cast<const uint2*>(p);
  // counts clamped to the tile size: a malformed header cannot move a read
  // outside the stage
  const uint32_t modal = h.x & 0xFF, nres = min((h.x >> 8) & 0xFFFFu, (uint32_t)kNszW),
                 nnear = min(h.y & 0xFFFFu, (uint32_t)kNszW);
  const int B = (n + 7) >> 3;
  const int nv = FULL ? 16 : min(max(n - 16 * lane, 0), 16);
  const uint32_t vm = nv >= 16 ? 0xFFFFu : ((1u << nv) - 1u);
  const uint32_t M16 = (FULL ? (uint32_t)*reinterpret_cast<const uint16_t*>(p + 8 + 2 * lane)
                             : lds_u16_any(p + 8 + 2 * lane)) & vm;
  // a weight marked both match and near is a match and takes no delta
  const uint32_t N16 = (FULL ? (uint32_t)*reinterpret_cast<const uint16_t*>(p + 8 + B + 2 * lane)
                             : lds_u16_any(p + 8 + B + 2 * lane)) & vm & ~M16;
  const uint32_t R16 = vm & ~(M16 | N16);
  // exclusive prefix over lanes of (near count, residual count << 16)
  const uint32_t cnt = (uint32_t)__popc(N16) | ((uint32_t)__popc(R16) << 16);
  uint32_t inc = cnt;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t t = __shfl_up_sync(0xFFFFFFFFu, inc, o);
    if (lane >= o) inc += t;
  }
  const uint32_t ex = inc - cnt;
  const int nc0 = (int)(ex & 0xFFFF), rc0 = (int)(ex >> 16);
  const int DO = 8 + 2 * B;
  const int RO = DO + (int)((nnear + 7) >> 3);
  const int MO = RO + (int)nres;
  const int SO = MO + MB * n;
  // this lane's near deltas: bits [nc0, nc0 + 16) of the delta stream
  const uint32_t dw = lds_u32_any(p + DO + (nc0 >> 3)) >> (nc0 & 7);
  const uint32_t S16 = lds_u16_any(p + SO + 2 * lane);

  // mantissas: bytes [MO + 16 * MB * lane, + 16 * MB), read as 8-byte words
  // from the 8-aligned address below them; the byte offset d = MO & 7 is the
  // same for every lane, so each d gets its own constant-offset extraction.
  uint32_t mant[16];
  {
    constexpr int LB = 16 * MB, NW = (LB + 8) / 4;
    const uint8_t* base = p + (MO & ~7) + LB * lane;
    uint32_t W[NW];
#pragma unroll
    for (int i = 0; i < NW / 2; ++i) {
      const uint2 q = *reinterpret_cast<const uint2*>(base + 8 * i);
      W[2 * i] = q.x;
      W[2 * i + 1] = q.y;
    }
    switch (MO & 7) {
      case 0: mant_extract<DT, 0>(W, mant); break;
      case 1: mant_extract<DT, 1>(W, mant); break;
      case 2: mant_extract<DT, 2>(W, mant); break;
      case 3: mant_extract<DT, 3>(W, mant); break;
      case 4: mant_extract<DT, 4>(W, mant); break;
      case 5: mant_extract<DT, 5>(W, mant); break;
      case 6: mant_extract<DT, 6>(W, mant); break;
      default: mant_extract<DT, 7>(W, mant); break;
    }
  }

  const uint32_t modal4 = modal * 0x01010101u;
  const uint32_t plus4 = ((modal + 1u) & 0xFFu) * 0x01010101u, minus4 = ((modal - 1u) & 0xFFu) * 0x01010101u;
  int nq = 0, rq = 0;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint32_t n4 = (N16 >> (4 * q)) & 15u, r4 = (R16 >> (4 * q)) & 15u;
    const uint2 ln = L.m4[n4], lr = L.m4[r4];
    // near: modal + 1 where the weight's delta bit is set, else modal - 1
    const uint32_t dm = L.dx[n4 * 16 + ((dw >> nq) & 15u)];
    const uint32_t ne = (dm & plus4) | (~dm & minus4);
    // residual: the next 4 residual bytes (from two aligned words) placed on
    // the residual weights; the other bytes are masked off below
    const int o = RO + rc0 + rq;
    const uint32_t* rw = reinterpret_cast<const uint32_t*>(p + (o & ~3));
    const uint32_t rex = __byte_perm(rw[0], rw[1], lr.x + (uint32_t)(o & 3) * 0x1111u);
    const uint32_t E = (lr.y & rex) | (~lr.y & ((ln.y & ne) | (~ln.y & modal4)));
    nq += (int)(ln.x >> 16);
    rq += (int)(lr.x >> 16);
    if constexpr (DT == NSQ_NSZ_FP32) {
      // byte 0: exponent i, byte 1: sign i (0/1); times 2^23 puts them at
      // bits 23..30 and 31 (the garbage in bytes 2..3 leaves the word)
      const uint32_t sb = spread4((S16 >> (4 * q)) & 15u);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t se = __byte_perm(E, sb, (uint32_t)(i | ((4 + i) << 4)));
        v[4 * q + i] = (mant[4 * q + i] & 0x7FFFFFu) | (se * 8388608u);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int k = 4 * q + i;
        const uint32_t e = (E >> (8 * i)) & 0xFFu, sg = (S16 >> k) & 1u;
        if constexpr (DT == NSQ_NSZ_FP16) {
          v[k] = (sg << 15) | ((e & 0x1Fu) << 10) | mant[k];
        } else {
          v[k] = (sg << 15) | (e << 7) | mant[k];
        }
      }
    }
  }
  vmask = vm;
}

template <int DT>
__device__ __forceinline__ float nsz_value(uint32_t bits) {
  if constexpr (DT == NSQ_NSZ_FP32) return __uint_as_float(bits);
  if constexpr (DT == NSQ_NSZ_FP16) return __half2float(__ushort_as_half((unsigned short)bits));
  return __uint_as_float(bits << 16);
}

// Warp-private tile pipeline: kDepth stages of kStage bytes and their mbarriers.
template <int DT>
struct WarpRing {
  uint8_t* stage;  // kDepth * kStage bytes, 128-byte aligned
  uint64_t* bar;   // kDepth
  __device__ uint8_t* at(int s) const { return stage + s * NszFmt<DT>::kStage; }
  // lane 0 only
  __device__ void issue(const uint8_t* tiles, const uint32_t* off, int64_t t, int s) const {
    const uint64_t o0 = (uint64_t)off[t] * 64, o1 = (uint64_t)off[t + 1] * 64;
    const uint32_t bytes = (uint32_t)(o1 > o0 ? (o1 - o0 < (uint64_t)NszFmt<DT>::kStage - 64 ? o1 - o0 : (uint64_t)NszFmt<DT>::kStage - 64) : 0);
    if (bytes == 0) {
      mbar_arrive(&bar[s]);
      return;
    }
    mbar_arrive_expect_tx(&bar[s], bytes);
    bulk_g2s(at(s), tiles + o0, bytes, &bar[s]);
  }
};

template <int DT>
__device__ __forceinline__ void ring_setup(uint8_t* smem, int warp, WarpRing<DT>& r) {
  r.stage = smem + (size_t)warp * kNszDepth * NszFmt<DT>::kStage;
  r.bar = reinterpret_cast<uint64_t*>(smem + (size_t)kNszWarps * kNszDepth * NszFmt<DT>::kStage) + warp * kNszDepth;
}

// After a timed-out wait: wait (bounded) for this warp's copies still in
// flight, so that none lands in shared memory after the CTA has exited.
template <int DT>
__device__ void ring_drain(const WarpRing<DT>& r, int64_t i0, int64_t n_issued) {
  for (int64_t i = i0; i < n_issued; ++i) mbar_wait_bounded(&r.bar[i % kNszDepth], (uint32_t)((i / kNszDepth) & 1));
}

constexpr size_t ring_bytes(int stage) {
  return (size_t)kNszWarps * kNszDepth * stage + (size_t)kNszWarps * kNszDepth * 8;
}

// ---------------------------------------------------------------------------
// Decode kernel: CTA c decodes tiles [c * per, (c + 1) * per), warp w a
// contiguous eighth of them.
struct DecodeParams {
  const uint8_t* tiles;
  const uint32_t* off;
  void* out;
  int64_t count, ntiles, per_cta;
};

template <int DT>
__global__ void __launch_bounds__(kNszWarps * 32, 3) nsz_decode_kernel(DecodeParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ NszLut lut;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  WarpRing<DT> ring;
  ring_setup<DT>(smem, warp, ring);
  init_nsz_lut(&lut);
  if (lane == 0)
    for (int s = 0; s < kNszDepth; ++s) mbar_init(&ring.bar[s], 1);
  fence_mbar_init();
  __syncthreads();

  const int64_t ta = (int64_t)blockIdx.x * p.per_cta, tb = min(p.ntiles, ta + p.per_cta);
  if (ta >= tb) return;
  const int64_t per_w = (tb - ta + kNszWarps - 1) / kNszWarps;
  const int64_t wa = ta + warp * per_w, wb = min(tb, wa + per_w);
  const int64_t nt = wb - wa;
  if (nt <= 0) return;
  if (lane == 0)
    for (int64_t i = 0; i < imin64(nt, kNszDepth); ++i) ring.issue(p.tiles, p.off, wa + i, (int)i);
  int s = 0;
  uint32_t phase = 0;  // stage s of tile i: i % kNszDepth, phase (i / kNszDepth) & 1
  for (int64_t i = 0; i < nt; ++i, s = s + 1 == kNszDepth ? 0 : s + 1, phase ^= s == 0 ? 1u : 0u) {
    const bool ok = __all_sync(0xFFFFFFFFu, mbar_wait_bounded(&ring.bar[s], phase));
    if (!ok) {
      if (lane == 0) ring_drain<DT>(ring, i + 1, imin64(nt, i + kNszDepth));
      return;
    }
    const int64_t t = wa + i;
    const int n = (int)imin64(kNszW, p.count - t * kNszW);
    uint32_t v[16], vm;
    if (n == kNszW)
      nsz_decode16<DT, true>(ring.at(s), n, lane, lut, v, vm);
    else
      nsz_decode16<DT, false>(ring.at(s), n, lane, lut, v, vm);
    __syncwarp();
    if (lane == 0 && i + kNszDepth < nt) {
      fence_proxy_async_smem();
      ring.issue(p.tiles, p.off, t + kNszDepth, s);
    }
    const int64_t e0 = t * kNszW + 16 * lane;
    if constexpr (DT == NSQ_NSZ_FP32) {
      uint32_t* o = static_cast<uint32_t*>(p.out) + e0;
      if (vm == 0xFFFFu) {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          reinterpret_cast<uint4*>(o)[j] = make_uint4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
      } else {
        for (int j = 0; j < 16; ++j)
          if ((vm >> j) & 1) o[j] = v[j];
      }
    } else {
      uint16_t* o = static_cast<uint16_t*>(p.out) + e0;
      if (vm == 0xFFFFu) {
#pragma unroll
        for (int j = 0; j < 2; ++j)
          reinterpret_cast<uint4*>(o)[j] =
              make_uint4(v[8 * j] | (v[8 * j + 1] << 16), v[8 * j + 2] | (v[8 * j + 3] << 16),
                         v[8 * j + 4] | (v[8 * j + 5] << 16), v[8 * j + 6] | (v[8 * j + 7] << 16));
      } else {
        for (int j = 0; j < 16; ++j)
          if ((vm >> j) & 1) o[j] = (uint16_t)v[j];
      }
    }
  }
}

// ---------------------------------------------------------------------------
// ZipGEMM.  CTA c owns output rows [c * rpc, min(N, (c + 1) * rpc)), i.e.
// weights [r0 * K, r1 * K); its warps split the tiles covering them.
struct ZipParams {
  const uint8_t* tiles;
  const uint32_t* off;
  const float* x;
  float* y;
  int64_t N, K, count;
  int64_t rpc;  // rows per CTA
  int mv;       // tokens in this launch (<= MT); x, y point at the first
};

template <int MT>
__device__ __forceinline__ void flush_rows(float (&acc)[MT], int64_t cur, int64_t next, int lane, float* ys,
                                           int64_t rpc, int64_t r0) {
  const int64_t c0 = __shfl_sync(0xFFFFFFFFu, cur, 0);
  if (__all_sync(0xFFFFFFFFu, cur == c0)) {
    if (c0 >= 0) {
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        float a = acc[m];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xFFFFFFFFu, a, o);
        if (lane == 0) atomicAdd(&ys[m * rpc + (c0 - r0)], a);
      }
    }
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[m] = 0.f;
  } else if (next != cur) {
    if (cur >= 0)
#pragma unroll
      for (int m = 0; m < MT; ++m) atomicAdd(&ys[m * rpc + (cur - r0)], acc[m]);
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[m] = 0.f;
  }
}

// Placement modes.  kRowTile: K % 512 == 0 and x 16-byte aligned: every
// tile is 512 weights of one row, so the row and column of a tile are
// warp-uniform and no weight needs a range check.  kAligned: K % 16 == 0 and
// x 16-byte aligned: a lane's 16 weights lie in one row (x read as float4).
// kGeneral: every weight is placed on its own.
enum : int { kGeneral = 0, kAligned = 1, kRowTile = 2 };

template <int DT, int MT, int MODE>
__global__ void __launch_bounds__(kNszWarps * 32, MT <= 2 ? 3 : 2) zipgemm_kernel(ZipParams p) {
  constexpr bool ALIGNED = MODE == kAligned;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ NszLut lut;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  WarpRing<DT> ring;
  ring_setup<DT>(smem, warp, ring);
  float* ys = reinterpret_cast<float*>(smem + ring_bytes(NszFmt<DT>::kStage));
  const int64_t r0 = (int64_t)blockIdx.x * p.rpc, r1 = min(p.N, r0 + p.rpc);
  if (r0 >= r1) return;  // whole CTA: nothing below synchronizes yet
  init_nsz_lut(&lut);
  if (lane == 0)
    for (int s = 0; s < kNszDepth; ++s) mbar_init(&ring.bar[s], 1);
  for (int64_t i = threadIdx.x; i < MT * p.rpc; i += blockDim.x) ys[i] = 0.f;
  fence_mbar_init();
  __syncthreads();

  const int64_t E0 = r0 * p.K, E1 = r1 * p.K;
  const int64_t ta = E0 / kNszW, tb = (E1 + kNszW - 1) / kNszW;
  const int64_t per_w = (tb - ta + kNszWarps - 1) / kNszWarps;
  const int64_t wa = ta + warp * per_w, wb = min(tb, wa + per_w);
  const int64_t nt = imax64(wb - wa, 0);
  bool ok = true;
  if (nt > 0) {
    if (lane == 0)
      for (int64_t i = 0; i < imin64(nt, kNszDepth); ++i) ring.issue(p.tiles, p.off, wa + i, (int)i);
    float acc[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[m] = 0.f;
    int64_t cur = -1;
    int64_t e0 = wa * kNszW + 16 * lane;
    int64_t row = e0 / p.K, col = e0 - row * p.K;
    // kRowTile: warp-uniform position of the tile: output row (relative to
    // r0) and first column
    const int kt = (int)(p.K / kNszW), K32 = (int)p.K;
    int trow = MODE == kRowTile ? (int)(wa / kt - r0) : 0;
    int tcol = MODE == kRowTile ? (int)(wa % kt) * kNszW : 0;
    bool pending = false;
    auto flush_tile_row = [&]() {
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        float a = acc[m];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xFFFFFFFFu, a, o);
        if (lane == 0 && m < p.mv) atomicAdd(&ys[m * p.rpc + trow], a);
        acc[m] = 0.f;
      }
    };
    int s = 0;
    uint32_t phase = 0;  // stage s of tile i: i % kNszDepth, phase (i / kNszDepth) & 1
    for (int64_t i = 0; i < nt; ++i, s = s + 1 == kNszDepth ? 0 : s + 1, phase ^= s == 0 ? 1u : 0u) {
      if (!__all_sync(0xFFFFFFFFu, mbar_wait_bounded(&ring.bar[s], phase))) {
        if (lane == 0) ring_drain<DT>(ring, i + 1, imin64(nt, i + kNszDepth));
        ok = false;
        break;
      }
      const int64_t t = wa + i;
      uint32_t v[16], vm;
      if constexpr (MODE == kRowTile) {
        nsz_decode16<DT, true>(ring.at(s), kNszW, lane, lut, v, vm);
      } else {
        const int n = (int)imin64(kNszW, p.count - t * kNszW);
        if (n == kNszW)
          nsz_decode16<DT, true>(ring.at(s), n, lane, lut, v, vm);
        else
          nsz_decode16<DT, false>(ring.at(s), n, lane, lut, v, vm);
      }
      __syncwarp();
      if (lane == 0 && i + kNszDepth < nt) {
        fence_proxy_async_smem();
        ring.issue(p.tiles, p.off, t + kNszDepth, s);
      }
      if constexpr (MODE == kRowTile) {
        float w[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) w[j] = nsz_value<DT>(v[j]);
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          if (m < p.mv) {
            const float4* xp = reinterpret_cast<const float4*>(p.x + (size_t)m * K32 + tcol + 16 * lane);
            float a = acc[m];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float4 xv = __ldg(xp + j);
              a = fmaf(w[4 * j], xv.x, a);
              a = fmaf(w[4 * j + 1], xv.y, a);
              a = fmaf(w[4 * j + 2], xv.z, a);
              a = fmaf(w[4 * j + 3], xv.w, a);
            }
            acc[m] = a;
          }
        }
        pending = true;
        tcol += kNszW;
        if (tcol == K32) {
          flush_tile_row();
          pending = false;
          tcol = 0;
          ++trow;
        }
      } else if constexpr (ALIGNED) {
        const bool valid = vm != 0 && e0 >= E0 && e0 < E1;
        const int64_t r = valid ? row : -1;
        if (__any_sync(0xFFFFFFFFu, r != cur)) {
          flush_rows<MT>(acc, cur, r, lane, ys, p.rpc, r0);
          cur = r;
        }
        if (valid) {
          float w[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) w[j] = nsz_value<DT>(v[j]);
#pragma unroll
          for (int m = 0; m < MT; ++m) {
            if (m < p.mv) {
              const float4* xp = reinterpret_cast<const float4*>(p.x + (size_t)m * p.K + col);
              float a = acc[m];
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const float4 xv = __ldg(xp + j);
                a = fmaf(w[4 * j], xv.x, a);
                a = fmaf(w[4 * j + 1], xv.y, a);
                a = fmaf(w[4 * j + 2], xv.z, a);
                a = fmaf(w[4 * j + 3], xv.w, a);
              }
              acc[m] = a;
            }
          }
        }
        e0 += kNszW;
        col += kNszW;
        while (col >= p.K) {
          col -= p.K;
          ++row;
        }
      } else {
        int64_t rr = row, cc = col;
#pragma unroll 1
        for (int j = 0; j < 16; ++j) {
          const int64_t e = e0 + j;
          if (((vm >> j) & 1) && e >= E0 && e < E1) {
            const float w = nsz_value<DT>(v[j]);
            for (int m = 0; m < p.mv; ++m) atomicAdd(&ys[m * p.rpc + (rr - r0)], w * p.x[(size_t)m * p.K + cc]);
          }
          if (++cc == p.K) {
            cc = 0;
            ++rr;
          }
        }
        e0 += kNszW;
        row = e0 / p.K;
        col = e0 - row * p.K;
      }
    }
    if constexpr (ALIGNED) {
      if (ok) flush_rows<MT>(acc, cur, -1, lane, ys, p.rpc, r0);
    }
    if constexpr (MODE == kRowTile) {
      if (ok && pending) flush_tile_row();
    }
  }
  if (!__syncthreads_and(ok)) return;
  const int64_t rows = r1 - r0;
  for (int64_t i = threadIdx.x; i < (int64_t)p.mv * rows; i += blockDim.x) {
    const int64_t m = i / rows, r = i - m * rows;
    p.y[(size_t)m * p.N + r0 + r] = ys[m * p.rpc + r];
  }
}

// ---------------------------------------------------------------------------
// Host side
template <typename K>
static int occupancy_ctas(K kernel, size_t smem, int num_sms) {
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kNszWarps * 32, smem) != cudaSuccess ||
      per_sm < 1)
    per_sm = 1;
  return per_sm * num_sms;
}

template <int DT>
static int run_decode(const uint8_t* tiles, const uint32_t* off, int64_t count, void* out, cudaStream_t st,
                      int num_sms) {
  const int64_t ntiles = (count + kNszW - 1) / kNszW;
  const size_t smem = ring_bytes(NszFmt<DT>::kStage);
  auto kern = nsz_decode_kernel<DT>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return NSQ_ERR_CUDA;
  const int64_t ctas = imax64(1, imin64(occupancy_ctas(kern, smem, num_sms), (ntiles + 7) / 8));
  DecodeParams p{tiles, off, out, count, ntiles, (ntiles + ctas - 1) / ctas};
  const int64_t grid = (ntiles + p.per_cta - 1) / p.per_cta;
  note_launch();
  kern<<<(unsigned)grid, kNszWarps * 32, smem, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? NSQ_OK : NSQ_ERR_CUDA;
}

template <int DT, int MT, int AL>
static int launch_zip(ZipParams p, cudaStream_t st, int num_sms) {
  constexpr size_t kYsMax = 48 * 1024;  // row buffer bound (floats: MT * rpc)
  const size_t base = ring_bytes(NszFmt<DT>::kStage);
  auto kern = zipgemm_kernel<DT, MT, AL>;
  const size_t smem_max = base + kYsMax;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_max) != cudaSuccess)
    return NSQ_ERR_CUDA;
  // one wave of CTAs at the occupancy of a small row buffer, more if the
  // rows would not fit the bound
  int64_t ctas = imax64(1, imin64(p.N, occupancy_ctas(kern, base + 8 * 1024, num_sms)));
  int64_t rpc = (p.N + ctas - 1) / ctas;
  if ((size_t)MT * rpc * 4 > kYsMax) rpc = kYsMax / (4 * MT);
  p.rpc = rpc;
  const int64_t grid = (p.N + rpc - 1) / rpc;
  const size_t smem = base + (size_t)MT * rpc * 4;
  note_launch();
  kern<<<(unsigned)grid, kNszWarps * 32, smem, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? NSQ_OK : NSQ_ERR_CUDA;
}

template <int DT, int AL>
static int launch_zip_m(ZipParams p, int mt, cudaStream_t st, int num_sms) {
  switch (mt) {
    case 1: return launch_zip<DT, 1, AL>(p, st, num_sms);
    case 2: return launch_zip<DT, 2, AL>(p, st, num_sms);
    case 4: return launch_zip<DT, 4, AL>(p, st, num_sms);
    default: return launch_zip<DT, 8, AL>(p, st, num_sms);
  }
}

template <int DT>
static int run_zip(const uint8_t* tiles, const uint32_t* off, const float* x, float* y, int64_t M, int64_t N,
                   int64_t K, cudaStream_t st, int num_sms) {
  const bool xa = !(reinterpret_cast<uintptr_t>(x) & 15);
  const int mode = xa && K % kNszW == 0 && K < (1ll << 30) ? kRowTile : xa && K % 16 == 0 ? kAligned : kGeneral;
  for (int64_t m0 = 0; m0 < M; m0 += 8) {
    const int mv = (int)imin64(8, M - m0);
    const int mt = mv == 1 ? 1 : mv == 2 ? 2 : mv <= 4 ? 4 : 8;
    ZipParams p{tiles, off, x + m0 * K, y + m0 * N, N, K, N * K, 0, mv};
    const int rc = mode == kRowTile  ? launch_zip_m<DT, kRowTile>(p, mt, st, num_sms)
                   : mode == kAligned ? launch_zip_m<DT, kAligned>(p, mt, st, num_sms)
                                      : launch_zip_m<DT, kGeneral>(p, mt, st, num_sms);
    if (rc) return rc;
  }
  return NSQ_OK;
}

static bool dtype_ok(int dt) { return dt == NSQ_NSZ_FP32 || dt == NSQ_NSZ_FP16 || dt == NSQ_NSZ_BF16; }

}  // namespace
}  // namespace nsq

using namespace nsq;

extern "C" {

int64_t nsq_nsz_num_tiles(int64_t num_weights) {
  return num_weights <= 0 ? 0 : (num_weights + kNszW - 1) / kNszW;
}

int nsq_nsz_index(const void* tiles_host, int64_t nbytes, int64_t num_weights, int dtype, uint32_t* offsets) {
  if (!dtype_ok(dtype)) return NSQ_ERR_TYPE;
  if (num_weights < 0 || nbytes < 0) return NSQ_ERR_SHAPE;
  if (!offsets || (!tiles_host && nbytes > 0)) return NSQ_ERR_NULL;
  const uint8_t* d = static_cast<const uint8_t*>(tiles_host);
  int64_t pos = 0, t = 0;
  for (int64_t t0 = 0; t0 < num_weights; t0 += kNszW, ++t) {
    const int n = (int)imin64(kNszW, num_weights - t0);
    if (pos + 8 > nbytes) return NSQ_ERR_FORMAT;
    const uint8_t* h = d + pos;
    const int nres = h[1] | (h[2] << 8), nnear = h[4] | (h[5] << 8);
    if (h[3] != dtype) return NSQ_ERR_FORMAT;
    const int64_t size = nsz_tile_bytes(n, nnear, nres, dtype);
    if (pos + size > nbytes) return NSQ_ERR_FORMAT;
    // the counts in the header must be the ones the bitmaps imply
    const int B = (n + 7) / 8;
    int near = 0, matched_or_near = 0;
    for (int b = 0; b < B; ++b) {
      const uint32_t valid = (b == B - 1 && (n & 7)) ? ((1u << (n & 7)) - 1u) : 0xFFu;
      const uint32_t mt = h[8 + b] & valid, nr = h[8 + B + b] & valid;
      near += __builtin_popcount(nr & ~mt);
      matched_or_near += __builtin_popcount(mt | nr);
    }
    if (near != nnear || n - matched_or_near != nres) return NSQ_ERR_FORMAT;
    if (pos / 64 > 0xFFFFFFFFll) return NSQ_ERR_SHAPE;
    offsets[t] = (uint32_t)(pos / 64);
    pos += size;
  }
  if (pos != nbytes || pos / 64 > 0xFFFFFFFFll) return NSQ_ERR_FORMAT;
  offsets[t] = (uint32_t)(pos / 64);
  return NSQ_OK;
}

int nsq_nsz_decode(const void* tiles, const uint32_t* offsets, int64_t num_weights, int dtype, void* out,
                   void* stream) {
  if (!dtype_ok(dtype)) return NSQ_ERR_TYPE;
  if (num_weights < 0) return NSQ_ERR_SHAPE;
  if (num_weights == 0) return NSQ_OK;
  if (!tiles || !offsets || !out) return NSQ_ERR_NULL;
  if ((reinterpret_cast<uintptr_t>(tiles) & 15) || (reinterpret_cast<uintptr_t>(out) & 15) ||
      (reinterpret_cast<uintptr_t>(offsets) & 3))
    return NSQ_ERR_ALIGN;
  int num_sms = 0, rc = device_check(&num_sms);
  if (rc) return rc;
  const uint8_t* t = static_cast<const uint8_t*>(tiles);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case NSQ_NSZ_FP32: return run_decode<NSQ_NSZ_FP32>(t, offsets, num_weights, out, st, num_sms);
    case NSQ_NSZ_FP16: return run_decode<NSQ_NSZ_FP16>(t, offsets, num_weights, out, st, num_sms);
    default: return run_decode<NSQ_NSZ_BF16>(t, offsets, num_weights, out, st, num_sms);
  }
}

int nsq_zipgemm(const void* tiles, const uint32_t* offsets, int dtype, const float* x, float* y, int64_t M,
                int64_t N, int64_t K, void* stream) {
  if (!dtype_ok(dtype)) return NSQ_ERR_TYPE;
  if (M < 1 || N < 1 || K < 1) return NSQ_ERR_SHAPE;
  if (!tiles || !offsets || !x || !y) return NSQ_ERR_NULL;
  if ((reinterpret_cast<uintptr_t>(tiles) & 15) || (reinterpret_cast<uintptr_t>(offsets) & 3) ||
      (reinterpret_cast<uintptr_t>(x) & 3) || (reinterpret_cast<uintptr_t>(y) & 3))
    return NSQ_ERR_ALIGN;
  int num_sms = 0, rc = device_check(&num_sms);
  if (rc) return rc;
  const uint8_t* t = static_cast<const uint8_t*>(tiles);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case NSQ_NSZ_FP32: return run_zip<NSQ_NSZ_FP32>(t, offsets, x, y, M, N, K, st, num_sms);
    case NSQ_NSZ_FP16: return run_zip<NSQ_NSZ_FP16>(t, offsets, x, y, M, N, K, st, num_sms);
    default: return run_zip<NSQ_NSZ_BF16>(t, offsets, x, y, M, N, K, st, num_sms);
  }
}

}  // extern "C"
