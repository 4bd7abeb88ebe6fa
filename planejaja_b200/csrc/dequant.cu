// dequant.cu -- standalone GGUF block dequantization to f32 / bf16.
//
// One warp per group of 32 weights, one lane per weight: the block header is
// a broadcast read, each lane reads its quant byte(s), and the 32 outputs of
// a warp are one coalesced 128-byte (f32) or 64-byte (bf16) store.
//
// f32 values are bit-exact to the reference (one rounding per element, as
// in the reference; explicit _rn intrinsics keep the operation order):
//   Q8_0  y = d*q                 crates/nodestor-inference/src/dequant/q8_0.rs:14-28
//   Q4_0  y = (q-8)*d             crates/nodestor-vulkan/shaders/dequant_q4.comp:40-61
//   Q4_K  y = (d*sc)*q - dmin*m   crates/nodestor-inference/src/dequant/q4_k.rs:75-131
//   Q5_K  y = (d*sc)*q - dmin*m   q5_k.rs:33-88 (NODESTOR high bits) or ggml's layout
//   Q6_K  y = (d*s)*q             dequant_q6k.comp:50-99 (NODESTOR) or ggml's layout
#include "nsq_common.cuh"

namespace nsq {

__device__ __forceinline__ float q4k_value(const uint8_t* blk, int j, int l) {
  // j: sub-block 0..7, l: 0..31
  const uint8_t* s = blk + 4;
  uint32_t sc, mn;
  if (j < 4) {
    sc = s[j] & 63;
    mn = s[j + 4] & 63;
  } else {
    sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4);
    mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
  }
  const float d = h2f(ld_u16(blk)), dmin = h2f(ld_u16(blk + 2));
  const uint32_t qb = blk[16 + 32 * (j >> 1) + l];
  const uint32_t q = (j & 1) ? (qb >> 4) : (qb & 0xF);
  const float d1 = __fmul_rn(d, (float)sc), m1 = __fmul_rn(dmin, (float)mn);
  return __fsub_rn(__fmul_rn(d1, (float)q), m1);
}

// Q5_K [d][dmin][scales 12][qh 32][qs 128]: sub-block j (0..7), element l:
// nibble (j & 1) of qs[32 (j >> 1) + l] plus 16 * the high bit, which is bit
// j of qh[l] (ggml) or bit l % 8 of qh[8 (j >> 1) + 4 (j & 1) + l / 8]
// (NODESTOR, q5_k.rs:57-70).
__device__ __forceinline__ float q5k_value(const uint8_t* blk, int layout, int j, int l) {
  const uint8_t* s = blk + 4;
  uint32_t sc, mn;
  if (j < 4) {
    sc = s[j] & 63;
    mn = s[j + 4] & 63;
  } else {
    sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4);
    mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
  }
  const float d = h2f(ld_u16(blk)), dmin = h2f(ld_u16(blk + 2));
  const uint32_t qb = blk[48 + 32 * (j >> 1) + l];
  const uint32_t nib = (j & 1) ? (qb >> 4) : (qb & 0xF);
  const uint32_t hb = layout == NSQ_Q6K_NODESTOR ? (blk[16 + 8 * (j >> 1) + 4 * (j & 1) + (l >> 3)] >> (l & 7)) & 1
                                                 : (blk[16 + l] >> j) & 1;
  const float d1 = __fmul_rn(d, (float)sc), m1 = __fmul_rn(dmin, (float)mn);
  return __fsub_rn(__fmul_rn(d1, (float)(nib | (hb << 4))), m1);
}

__device__ __forceinline__ float q6k_value(const uint8_t* blk, int layout, int i) {
  // i: element 0..255 of the super-block
  const float d = h2f(ld_u16(blk + 208));
  if (layout == NSQ_Q6K_NODESTOR) {
    const uint32_t qlb = blk[i >> 1];
    const uint32_t lo = (i & 1) ? (qlb >> 4) : (qlb & 0xF);
    const uint32_t hi = (blk[128 + (i >> 2)] >> ((i & 3) * 2)) & 3;
    const int q = (int)(lo | (hi << 4)) - 32;
    const float s = (float)((int)blk[192 + (i >> 4)] - 128) / 64.0f;  // exact
    return __fmul_rn(__fmul_rn(d, s), (float)q);
  }
  const int n = i >> 7, r = i & 127, j = r >> 5, l = r & 31;
  const uint32_t qlb = blk[64 * n + 32 * (j & 1) + l];
  const uint32_t lo = (j >> 1) ? (qlb >> 4) : (qlb & 0xF);
  const uint32_t hi = (blk[128 + 32 * n + l] >> (2 * j)) & 3;
  const int q = (int)(lo | (hi << 4)) - 32;
  const float sc = (float)(int8_t)blk[192 + 8 * n + (l >> 4) + 2 * j];
  return __fmul_rn(__fmul_rn(d, sc), (float)q);
}

template <int TYPE, typename OutT>
__global__ void __launch_bounds__(256) dequant_kernel(const uint8_t* __restrict__ w, int layout,
                                                      OutT* __restrict__ out, int64_t n_groups) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t g = warp; g < n_groups; g += nwarps) {
    float v;
    if constexpr (TYPE == NSQ_TYPE_Q8_0) {
      const uint8_t* blk = w + g * 34;
      v = __fmul_rn(h2f(ld_u16(blk)), (float)(int8_t)blk[2 + lane]);
    } else if constexpr (TYPE == NSQ_TYPE_Q4_0) {
      const uint8_t* blk = w + g * 18;
      const uint32_t qb = blk[2 + (lane & 15)];
      const int q = (int)((lane < 16) ? (qb & 0xF) : (qb >> 4)) - 8;
      v = __fmul_rn((float)q, h2f(ld_u16(blk)));
    } else if constexpr (TYPE == NSQ_TYPE_Q4_K) {
      const uint8_t* blk = w + (g >> 3) * 144;
      v = q4k_value(blk, (int)(g & 7), lane);
    } else if constexpr (TYPE == NSQ_TYPE_Q5_K) {
      const uint8_t* blk = w + (g >> 3) * 176;
      v = q5k_value(blk, layout, (int)(g & 7), lane);
    } else {
      const uint8_t* blk = w + (g >> 3) * 210;
      v = q6k_value(blk, layout, (int)(g & 7) * 32 + lane);
    }
    if constexpr (sizeof(OutT) == 4) {
      out[g * 32 + lane] = v;
    } else {
      out[g * 32 + lane] = __float2bfloat16_rn(v);
    }
  }
}

template <int TYPE>
static cudaError_t launch_dequant_t(const uint8_t* w, int layout, int out_dtype, void* out, int64_t n_groups,
                                    cudaStream_t st, int num_sms) {
  const int threads = 256;
  int64_t blocks = (n_groups + 7) / 8;
  const int64_t cap = (int64_t)num_sms * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  note_launch();
  if (out_dtype == NSQ_OUT_F32)
    dequant_kernel<TYPE, float><<<(unsigned)blocks, threads, 0, st>>>(w, layout, (float*)out, n_groups);
  else
    dequant_kernel<TYPE, __nv_bfloat16><<<(unsigned)blocks, threads, 0, st>>>(w, layout, (__nv_bfloat16*)out,
                                                                              n_groups);
  return cudaGetLastError();
}

cudaError_t launch_dequant(const uint8_t* w, int type, int layout, int out_dtype, void* out, int64_t n_elems,
                           cudaStream_t st, int num_sms) {
  const int64_t n_groups = n_elems / 32;
  switch (type) {
    case NSQ_TYPE_Q4_0: return launch_dequant_t<NSQ_TYPE_Q4_0>(w, layout, out_dtype, out, n_groups, st, num_sms);
    case NSQ_TYPE_Q8_0: return launch_dequant_t<NSQ_TYPE_Q8_0>(w, layout, out_dtype, out, n_groups, st, num_sms);
    case NSQ_TYPE_Q4_K: return launch_dequant_t<NSQ_TYPE_Q4_K>(w, layout, out_dtype, out, n_groups, st, num_sms);
    case NSQ_TYPE_Q5_K: return launch_dequant_t<NSQ_TYPE_Q5_K>(w, layout, out_dtype, out, n_groups, st, num_sms);
    case NSQ_TYPE_Q6_K: return launch_dequant_t<NSQ_TYPE_Q6_K>(w, layout, out_dtype, out, n_groups, st, num_sms);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace nsq
