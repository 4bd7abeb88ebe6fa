// gemv_rows.cu -- host side of the fused decode GEMV (gemv_rows.cuh):
// launch planning, the per-call entry (run_gemv_fused) and coverage probes.
#include "gemv_rows.cuh"

namespace nsq {

// ---------------------------------------------------------------------------
// Host side
constexpr int kXSelfMaxBytes = 40 * 1024;

static int seg_code(int type, int layout) {
  switch (type) {
    case NSQ_TYPE_Q4_K: return kQ4K;
    case NSQ_TYPE_Q6_K: return layout == NSQ_Q6K_NODESTOR ? kQ6KN : kQ6KG;
    case NSQ_TYPE_Q5_K: return layout == NSQ_Q6K_NODESTOR ? kQ5KN : kQ5KG;
    case NSQ_TYPE_Q4_0: return kQ40;
    case NSQ_TYPE_Q8_0: return kQ80;
    default: return -1;
  }
}
static int piece_bytes_of(int type) {
  switch (type) {
    case NSQ_TYPE_Q4_K: return 144;
    case NSQ_TYPE_Q6_K: return 210;
    case NSQ_TYPE_Q5_K: return 176;
    case NSQ_TYPE_Q4_0: return 144;
    case NSQ_TYPE_Q8_0: return 272;
    default: return 0;
  }
}

// Plans a fused launch; false if a segment's shape is not covered (K % 256,
// Q6_K needs K % 2048, 16-byte row alignment).
static bool plan_fused(const nsq_segment* segs, int nseg, int64_t K, int M, bool xself, int num_sms,
                       int max_clusters, FusedParams& p, int& blocks, size_t& smem, int min_r = 4) {
  if (nseg < 1 || nseg > NSQ_MAX_SEGMENTS || K % 256) return false;
  const int64_t npieces = K / 256;
  bool any_q6k = false, any_b32 = false;
  int64_t T = 0;
  for (int i = 0; i < nseg; ++i) {
    const int t = segs[i].ggml_type;
    if (seg_code(t, segs[i].q6k_layout) < 0) return false;
    if (t == NSQ_TYPE_Q4_0 || t == NSQ_TYPE_Q8_0) any_b32 = true;
    if (t == NSQ_TYPE_Q6_K) {
      any_q6k = true;
      if (npieces % 8) return false;
    }
    if ((npieces * piece_bytes_of(t)) % 16) return false;
    T += segs[i].N;
  }
  // Defaults from measurement on B200 (M = 1): many rows per SM (an FFN
  // input projection) stream best in 16-row blocks of whole 4096-wide rows
  // for the K-quants, but in 8-row blocks for the 32-weight-block formats
  // (Llama-2-7B Q4_0 decode step: 1.33-1.38 against 1.49-1.50 ms); long rows
  // (K >= 8192) gain from sharing the activation quantisation in CTA pairs.
  const bool many_rows = T >= (int64_t)128 * num_sms;
  const bool long_k = K >= 8192;
  int R = tune(kTuneRowsR, many_rows && !any_b32 ? 16 : 8);
  if (R != 4 && R != 8 && R != 16 && R != 32) R = 8;
  if (R < min_r) R = min_r;
  while (R > min_r && (T + R - 1) / R < (int64_t)num_sms) R >>= 1;
  const int KS = 32 / R;
  int PPS = tune(kTuneRowsPPSM, many_rows ? 2 : 1) * kRowsConsumers * KS;
  if (PPS < 1) PPS = kRowsConsumers * KS;
  if (any_q6k && PPS % 8) PPS = (PPS + 7) / 8 * 8;
  if (PPS > npieces) PPS = (int)npieces;
  int nstages = tune(kTuneRowsStages, 2);
  if (nstages < 2 || nstages > 8) nstages = 2;
  const size_t xsm = xself ? (size_t)M * npieces * kXPieceSelf : 0;
  const int min_pps = any_q6k ? 8 : 1;
  int max_pitch = 0, xstride = 0, stage_bytes = 0;
  for (;;) {
    // shrink the chunk until the stages fit in shared memory
    max_pitch = 0;
    for (int i = 0; i < nseg; ++i) {
      const int cb = PPS * piece_bytes_of(segs[i].ggml_type);
      const int pitch = ((cb + 15) & ~15) + 16;
      if (pitch > max_pitch) max_pitch = pitch;
    }
    xstride = PPS * 8 * 80;
    stage_bytes = (R * max_pitch + (xself ? 0 : M * xstride) + 127) & ~127;
    smem = (size_t)stage_bytes * nstages + xsm + (size_t)2 * kRowsConsumers * 32 * M * 4 + 16 * nstages + 16;
    if (smem <= 200 * 1024) break;
    if (PPS / 2 < min_pps || (PPS / 2) % min_pps) return false;
    PPS /= 2;
  }
  for (int i = 0; i < nseg; ++i) {
    FSeg& f = p.seg[i];
    const int pb = piece_bytes_of(segs[i].ggml_type);
    f.w = static_cast<const uint8_t*>(segs[i].w);
    f.y = segs[i].y;
    f.N = segs[i].N;
    f.RB = npieces * pb;
    f.code = seg_code(segs[i].ggml_type, segs[i].q6k_layout);
    f.piece_bytes = pb;
    f.chunk_bytes = PPS * pb;
    f.pitch = ((f.chunk_bytes + 15) & ~15) + 16;
  }
  int64_t acc_rows = 0;
  for (int i = 0; i < nseg; ++i) {
    p.seg[i].row0 = acc_rows;
    acc_rows += p.seg[i].N;
  }
  p.nseg = nseg; p.T = T; p.K = K; p.GX = K / 32;
  p.R = R; p.Rblk = R; p.KS = KS; p.PPS = PPS; p.npieces = (int)npieces; p.nchunks = (int)((npieces + PPS - 1) / PPS);
  p.xstride = xstride; p.stage_bytes = stage_bytes; p.nstages = nstages; p.max_pitch = max_pitch;
  p.npre = tune(kTuneRowsPre, nstages);
  if (p.npre < 0 || p.npre > nstages) p.npre = nstages;
  // weights evict_first: 1.70 against 1.78-1.82 ms per Llama-3-8B decode step (B200)
  p.l2hint = tune(kTuneRowsL2Hint, 1);

  int per_sm = (int)((220 * 1024) / (smem + 1024));
  if (per_sm > 4) per_sm = 4;
  if (per_sm < 1) per_sm = 1;
  const int cps = tune(kTuneRowsCPS, 0);
  if (cps >= 1 && cps <= per_sm) per_sm = cps;
  // clusters share the activation quantisation (self-prepared mode only)
  int C = xself ? tune(kTuneRowsC, long_k ? 2 : 1) : 1;
  if (C != 2 && C != 4 && C != 8) C = 1;
  // grid: as many CTAs as fit at once, then the fewest that give every CTA
  // the same number of whole row blocks (give or take one)
  const int64_t nrb = (T + R - 1) / R;
  int64_t gmax = (int64_t)num_sms * per_sm;
  if (C > 1 && max_clusters > 0 && gmax > (int64_t)max_clusters * C) gmax = (int64_t)max_clusters * C;
  gmax = gmax / C * C;
  if (gmax < C) return false;
  // whole row blocks per CTA for every shape: Llama-3-8B decode step 1.596
  // against 1.638 ms with an even row split for K < 8192
  const bool whole_blocks = tune(kTuneRowsBal, 1) != 0;
  int64_t g = gmax < nrb ? gmax : nrb;
  if (whole_blocks) {
    const int64_t per_cta = (nrb + gmax - 1) / gmax;
    g = (nrb + per_cta - 1) / per_cta;
  }
  g = (g + C - 1) / C * C;
  blocks = (int)g;
  p.C = C;
  p.nrb = whole_blocks ? nrb : 0;
  return true;
}

static cudaError_t launch_fused_e(int epi, int M, const FusedParams& p, bool xself, int blocks, size_t smem,
                                  cudaStream_t st, int* mc) {
  int code = p.seg[0].code;
  for (int i = 1; i < p.nseg; ++i)
    if (p.seg[i].code != code) code = kMixed;
  switch (code) {
    case kQ4K: return launch_fused_code<kQ4K>(xself, epi, M, p, blocks, smem, st, mc);
    case kQ6KG: return launch_fused_code<kQ6KG>(xself, epi, M, p, blocks, smem, st, mc);
    case kQ6KN: return launch_fused_code<kQ6KN>(xself, epi, M, p, blocks, smem, st, mc);
    case kQ40: return launch_fused_code<kQ40>(xself, epi, M, p, blocks, smem, st, mc);
    case kQ80: return launch_fused_code<kQ80>(xself, epi, M, p, blocks, smem, st, mc);
    case kQ5KG: return launch_fused_code<kQ5KG>(xself, epi, M, p, blocks, smem, st, mc);
    case kQ5KN: return launch_fused_code<kQ5KN>(xself, epi, M, p, blocks, smem, st, mc);
    default: return launch_fused_code<kMixed>(xself, epi, M, p, blocks, smem, st, mc);
  }
}

// True if the fused kernel can prepare the activations of M tokens on chip.
bool fused_self_prepare_fits(int64_t M, int64_t K) { return M <= 4 && M * (K / 32) * 80 <= kXSelfMaxBytes; }

// True if preparing the activations on chip is also the faster choice.  One
// token is quantised one group of 32 per consumer thread; when a CTA (or CTA
// pair, K >= 8192) has more groups than threads, the rounds delay every
// consumer and the separate one-warp-per-group kernel is faster (B200, M = 1:
// Llama-3-8B decode step 1.556 against 1.612 ms with its K = 14336 `down`
// launch prepared separately, Llama-2-7B 1.281 against 1.329 ms with
// K = 11008; every K = 4096 launch prepared separately: 1.706 ms).
bool fused_self_prepare_preferred(int64_t M, int64_t K) {
  if (M > 1) return true;  // M = 4, K = 4096: 3.80 on chip against 3.87 ms separately
  const int64_t C = K >= 8192 ? 2 : 1;
  return K / 32 <= C * kRowsConsumers * 32;
}

// Fused decode GEMV.  xg == nullptr: activations are prepared on chip from x
// (requires fused_self_prepare_fits); otherwise xg holds prepared records.
// Returns NSQ_OK / an error, or -1 if a shape is not covered.
// epi: 0 plain; 1 residual add (res[i] per segment, [M x N_i], may alias y);
// 2 SwiGLU (segments gate, up with equal formats and rows; h = silu(gate) *
// up into segment 0's y).
int run_gemv_fused(const nsq_segment* segs, int nseg, const float* x, const XGroup* xg, int64_t M, int64_t K,
                   cudaStream_t st, int num_sms, const XchgDesc* xd, int epi, const float* const* res) {
  const bool xself = (xg == nullptr);
  if (epi == 2 && (nseg != 2 || segs[0].N != segs[1].N || segs[0].ggml_type != segs[1].ggml_type ||
                   segs[0].q6k_layout != segs[1].q6k_layout))
    return -1;
  if (epi == 1 && !res) return -1;
  for (int64_t m0 = 0; m0 < M; m0 += 4) {
    const int mm = (int)((M - m0) < 4 ? (M - m0) : 4);
    nsq_segment sl[NSQ_MAX_SEGMENTS];
    for (int i = 0; i < nseg && i < NSQ_MAX_SEGMENTS; ++i) {
      sl[i] = segs[i];
      sl[i].y = segs[i].y + m0 * segs[i].N;
    }
    int max_clusters = 0;
    cudaError_t e = cudaSuccess;
    for (int attempt = 0; attempt < 2; ++attempt) {
      FusedParams p{};
      int blocks;
      size_t smem;
      if (!plan_fused(sl, nseg, K, mm, xself, num_sms, max_clusters, p, blocks, smem, epi == 2 ? 8 : 4)) return -1;
      if (epi == 2) {
        // walk the gate rows in half blocks; each block also carries up's rows
        if (p.R < 8) return -1;
        p.Rblk = p.R / 2;
        p.T = sl[0].N;
        p.nseg = 1;
      }
      if (epi == 1)
        for (int i = 0; i < nseg; ++i) p.res[i] = res[i] + m0 * segs[i].N;
      p.x = x ? x + m0 * K : nullptr;
      p.xg = xg ? xg + m0 * (K / 32) : nullptr;
      p.P = 1;
      if (xd && xd->P > 1) {
        p.P = xd->P;
        p.rank = xd->rank;
        p.xwait = xd->wait && m0 == 0;
        for (int r = 0; r < xd->P; ++r) p.xbuf[r] = xd->buf[r];
        for (int i = 0; i < nseg; ++i) {
          p.xrow0[i] = xd->row0[i];
          p.xnfull[i] = xd->nfull[i];
          p.xoff[i] = xd->off[i] + m0 * xd->nfull[i] * 4;
        }
      }
      e = launch_fused_e(epi, mm, p, xself, blocks, smem, st, &max_clusters);
      if (e != static_cast<cudaError_t>(kNoRoom)) break;  // else re-plan with fewer clusters
    }
    if (e != cudaSuccess) return NSQ_ERR_CUDA;
  }
  return NSQ_OK;
}

// Probe: would run_gemv_fused accept these segments?
bool fused_covers(const nsq_segment* segs, int nseg, int64_t K) {
  if (nseg < 1 || nseg > NSQ_MAX_SEGMENTS || K % 256) return false;
  const int64_t npieces = K / 256;
  for (int i = 0; i < nseg; ++i) {
    const int t = segs[i].ggml_type;
    if (seg_code(t, segs[i].q6k_layout) < 0) return false;
    if (t == NSQ_TYPE_Q6_K && npieces % 8) return false;
    if ((npieces * piece_bytes_of(t)) % 16) return false;
  }
  return true;
}

}  // namespace nsq
