/*
 * nsq_oracle.c -- CPU restatement of NodeStor's GGUF dequant + matmul path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA library
 * (libnsq): only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
 * reference legs may load it.  The product never calls it.
 *
 * Every function restates one reference routine (paths relative to the
 * reference project root, nodestor/...):
 *
 *   orc_half_to_f32         crates/nodestor-inference/src/dequant/mod.rs:234-260
 *   orc_half_to_f32_shader  crates/nodestor-vulkan/shaders/dequant_q4.comp:27-38
 *                           (same body in dequant_q8.comp:24-35, dequant_q6k.comp:37-48)
 *   orc_dequant_q8_0        crates/nodestor-inference/src/dequant/q8_0.rs:14-28
 *                           (shader twin dequant_q8.comp:37-55 when fp16_mode=1)
 *   orc_dequant_q4_0        crates/nodestor-vulkan/shaders/dequant_q4.comp:40-61
 *   orc_dequant_q4_k        crates/nodestor-inference/src/dequant/q4_k.rs:56-131
 *   orc_dequant_q4_k_avx2   crates/nodestor-inference/src/dequant/simd_x86.rs:84-158
 *                           (timing variant; unfused mul then sub, :131)
 *   orc_dequant_q5_k (layout NODESTOR)
 *                           crates/nodestor-inference/src/dequant/q5_k.rs:33-88
 *   orc_dequant_q5_k (layout GGML)
 *                           third-party: ggml's Q5_K as implemented by gguf-py
 *                           0.19.0 gguf/quants.py class Q5_K.dequantize_blocks
 *   orc_dequant_q6_k (layout NODESTOR)
 *                           crates/nodestor-vulkan/shaders/dequant_q6k.comp:50-99
 *   orc_dequant_q6_k (layout GGML)
 *                           third-party: ggml's Q6_K as implemented by gguf-py
 *                           0.19.0 gguf/quants.py class Q6_K.dequantize_blocks
 *                           (the meaning of Q6_K bytes written by llama.cpp)
 *   orc_matmul_f32          crates/nodestor-vulkan/src/pipeline.rs:1256-1268
 *                           C[i,j] = sum_l A[i*K+l]*B[l*N+j], sequential f32
 *   orc_quant_matmul        composition used by the operator path:
 *                           y = cpu_matmul_f32(x, transpose(dequant(W)))
 *
 * Parity pins: half_to_f32 / Q8_0 / Q4_K known answers from the reference's
 * unit tests (mod.rs:266-283, q8_0.rs:36-61, q4_k.rs:166-222); Q4_0, Q8_0,
 * Q4_K and Q6_K(ggml) against gguf-py 0.19.0 golden vectors (tests/golden).
 * Q6_K(nodestor) and Q4_0 have no reference test: they are pinned only by the
 * shader source restated here.
 *
 * Build: -O2 -ffp-contract=off, no fast-math (see oracle/Makefile).
 */
#include <stdint.h>
#include <string.h>
#include <math.h>
#include <stdlib.h>
#ifdef __AVX2__
#include <immintrin.h>
#endif

#define NSQ_T_Q4_0 2
#define NSQ_T_Q8_0 8
#define NSQ_T_Q4_K 12
#define NSQ_T_Q6_K 14
#define NSQ_T_Q5_K 13

#define Q6K_LAYOUT_GGML 0
#define Q6K_LAYOUT_NODESTOR 1

static inline float bits_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* mod.rs:234-260 -- IEEE half -> f32, subnormals renormalised. */
float orc_half_to_f32(uint16_t bits) {
    uint32_t sign = ((uint32_t)(bits >> 15)) << 31;
    uint32_t exp = (bits >> 10) & 0x1F;
    uint32_t mant = bits & 0x3FF;
    uint32_t e32, m32;
    if (exp == 0) {
        if (mant == 0) { e32 = 0; m32 = 0; }
        else {
            int32_t e = 127 - 14;
            uint32_t m = mant;
            while ((m & 0x400) == 0) { m <<= 1; e -= 1; }
            m &= 0x3FF;
            e32 = (uint32_t)e; m32 = m << 13;
        }
    } else if (exp == 31) { e32 = 255; m32 = mant << 13; }
    else { e32 = exp + 127 - 15; m32 = mant << 13; }
    return bits_f32(sign | (e32 << 23) | m32);
}

/* dequant_q4.comp:27-38 -- the shaders' own conversion.  Normal numbers are
 * exact (pow(2, e-15) is a power of two); subnormals are scaled by an extra
 * 2^-10 (5.96e-8 * m/1024 instead of 5.96e-8 * m). */
float orc_half_to_f32_shader(uint16_t h) {
    uint32_t s = (h >> 15) & 1u, e = (h >> 10) & 0x1Fu, m = h & 0x3FFu;
    float sg = s ? -1.0f : 1.0f;
    if (e == 0u) {
        if (m == 0u) return s ? -0.0f : 0.0f;
        return sg * 5.960464477539063e-8f * ((float)m / 1024.0f);
    } else if (e == 31u) {
        return m == 0u ? sg * INFINITY : NAN;
    }
    return sg * ldexpf(1.0f, (int)e - 15) * (1.0f + (float)m / 1024.0f);
}

static inline float h2f(const uint8_t *p, int fp16_mode) {
    uint16_t b = (uint16_t)(p[0] | (p[1] << 8));
    return fp16_mode ? orc_half_to_f32_shader(b) : orc_half_to_f32(b);
}

/* q8_0.rs:14-28: y[i] = d * (int8)q[i] over 34-byte blocks. */
void orc_dequant_q8_0(const uint8_t *raw, int64_t nblocks, float *out, int fp16_mode) {
    for (int64_t b = 0; b < nblocks; ++b) {
        const uint8_t *blk = raw + b * 34;
        float d = h2f(blk, fp16_mode);
        for (int i = 0; i < 32; ++i) out[b * 32 + i] = d * (float)(int8_t)blk[2 + i];
    }
}

/* dequant_q4.comp:40-61: y[i] = ((q&15)-8)*d, y[i+16] = ((q>>4)-8)*d. */
void orc_dequant_q4_0(const uint8_t *raw, int64_t nblocks, float *out, int fp16_mode) {
    for (int64_t b = 0; b < nblocks; ++b) {
        const uint8_t *blk = raw + b * 18;
        float d = h2f(blk, fp16_mode);
        for (int i = 0; i < 16; ++i) {
            uint8_t v = blk[2 + i];
            out[b * 32 + i] = (float)((int)(v & 0x0F) - 8) * d;
            out[b * 32 + i + 16] = (float)((int)(v >> 4) - 8) * d;
        }
    }
}

/* q4_k.rs:120-131 */
static inline void get_scale_min_k4(int j, const uint8_t *s, uint8_t *d, uint8_t *m) {
    if (j < 4) { *d = s[j] & 0x3F; *m = s[j + 4] & 0x3F; }
    else {
        *d = (uint8_t)((s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4));
        *m = (uint8_t)((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
    }
}

uint32_t orc_get_scale_min_k4(int j, const uint8_t *scales) {
    uint8_t d, m;
    get_scale_min_k4(j, scales, &d, &m);
    return (uint32_t)d | ((uint32_t)m << 8);
}

/* q4_k.rs:56-112: super-block [d][dmin][scales 12][qs 128]. */
void orc_dequant_q4_k(const uint8_t *raw, int64_t nblocks, float *out, int fp16_mode) {
    for (int64_t b = 0; b < nblocks; ++b) {
        const uint8_t *blk = raw + b * 144;
        float d = h2f(blk, fp16_mode), dmin = h2f(blk + 2, fp16_mode);
        const uint8_t *scales = blk + 4, *qs = blk + 16;
        float *o = out + b * 256;
        int is = 0, qo = 0;
        for (int chunk = 0; chunk < 4; ++chunk) {
            uint8_t sc0, m0, sc1, m1b;
            get_scale_min_k4(is, scales, &sc0, &m0);
            float d1 = d * (float)sc0, m1 = dmin * (float)m0;
            get_scale_min_k4(is + 1, scales, &sc1, &m1b);
            float d2 = d * (float)sc1, m2 = dmin * (float)m1b;
            for (int l = 0; l < 32; ++l) *o++ = d1 * (float)(qs[qo + l] & 0x0F) - m1;
            for (int l = 0; l < 32; ++l) *o++ = d2 * (float)(qs[qo + l] >> 4) - m2;
            qo += 32; is += 2;
        }
    }
}

/* simd_x86.rs:84-158: 8-wide AVX2 mul then sub (same values as scalar). */
void orc_dequant_q4_k_avx2(const uint8_t *raw, int64_t nblocks, float *out) {
#ifdef __AVX2__
    for (int64_t b = 0; b < nblocks; ++b) {
        const uint8_t *blk = raw + b * 144;
        float d = orc_half_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
        float dmin = orc_half_to_f32((uint16_t)(blk[2] | (blk[3] << 8)));
        const uint8_t *scales = blk + 4, *qs = blk + 16;
        __m256 d_v = _mm256_set1_ps(d), dmin_v = _mm256_set1_ps(dmin);
        float *o = out + b * 256;
        int is = 0, qo = 0;
        for (int chunk = 0; chunk < 4; ++chunk) {
            uint8_t sc0, m0, sc1, m1;
            get_scale_min_k4(is, scales, &sc0, &m0);
            get_scale_min_k4(is + 1, scales, &sc1, &m1);
            __m256 s0 = _mm256_mul_ps(d_v, _mm256_set1_ps((float)sc0));
            __m256 s1 = _mm256_mul_ps(d_v, _mm256_set1_ps((float)sc1));
            __m256 mn0 = _mm256_mul_ps(dmin_v, _mm256_set1_ps((float)m0));
            __m256 mn1 = _mm256_mul_ps(dmin_v, _mm256_set1_ps((float)m1));
            __m256i mask = _mm256_set1_epi32(0x0F);
            for (int l = 0; l < 32; l += 8) {
                __m256i i32s = _mm256_cvtepu8_epi32(_mm_loadl_epi64((const __m128i *)(qs + qo + l)));
                __m256 f = _mm256_cvtepi32_ps(_mm256_and_si256(i32s, mask));
                _mm256_storeu_ps(o, _mm256_sub_ps(_mm256_mul_ps(s0, f), mn0));
                o += 8;
            }
            for (int l = 0; l < 32; l += 8) {
                __m256i i32s = _mm256_cvtepu8_epi32(_mm_loadl_epi64((const __m128i *)(qs + qo + l)));
                __m256 f = _mm256_cvtepi32_ps(_mm256_and_si256(_mm256_srli_epi32(i32s, 4), mask));
                _mm256_storeu_ps(o, _mm256_sub_ps(_mm256_mul_ps(s1, f), mn1));
                o += 8;
            }
            qo += 32; is += 2;
        }
    }
#else
    orc_dequant_q4_k(raw, nblocks, out, 0);
#endif
}

/*
 * Q5_K, 176-byte block: d(f16) | dmin(f16) | scales[12] | qh[32] | qs[128].
 * Weight (chunk c, half h, l) = d * sc(2c+h) * q - dmin * m(2c+h), with
 * q = nibble h of qs[32c + l] plus 16 * the high bit:
 *   NODESTOR (q5_k.rs:57-70): bit l%8 of qh[8c + 4h + l/8];
 *   GGML (gguf-py Q5_K):      bit 2c+h of qh[l].
 */
void orc_dequant_q5_k(const uint8_t *raw, int64_t nblocks, float *out, int layout, int fp16_mode) {
    for (int64_t b = 0; b < nblocks; ++b) {
        const uint8_t *blk = raw + b * 176;
        float d = h2f(blk, fp16_mode), dmin = h2f(blk + 2, fp16_mode);
        const uint8_t *scales = blk + 4, *qh = blk + 16, *qs = blk + 48;
        float *o = out + b * 256;
        for (int c = 0; c < 4; ++c) {
            for (int h = 0; h < 2; ++h) {
                uint8_t sc, m;
                get_scale_min_k4(2 * c + h, scales, &sc, &m);
                float d1 = d * (float)sc, m1 = dmin * (float)m;
                for (int l = 0; l < 32; ++l) {
                    uint32_t nib = h ? (uint32_t)(qs[32 * c + l] >> 4) : (uint32_t)(qs[32 * c + l] & 0x0F);
                    uint32_t hb = layout == Q6K_LAYOUT_NODESTOR ? (qh[8 * c + 4 * h + l / 8] >> (l % 8)) & 1u
                                                                : (qh[l] >> (2 * c + h)) & 1u;
                    *o++ = d1 * (float)(nib | (hb << 4)) - m1;
                }
            }
        }
    }
}

/* Q6_K, 210-byte block: ql[128] | qh[64] | scales[16] | d(f16) at 208. */
void orc_dequant_q6_k(const uint8_t *raw, int64_t nblocks, float *out, int layout, int fp16_mode) {
    for (int64_t b = 0; b < nblocks; ++b) {
        const uint8_t *blk = raw + b * 210;
        const uint8_t *ql = blk, *qh = blk + 128, *sc = blk + 192;
        float d = h2f(blk + 208, fp16_mode);
        float *o = out + b * 256;
        if (layout == Q6K_LAYOUT_NODESTOR) {
            /* dequant_q6k.comp:50-99 */
            for (int i = 0; i < 256; ++i) {
                uint32_t qlb = ql[i >> 1];
                uint32_t lo = (i & 1) == 0 ? (qlb & 0x0Fu) : ((qlb >> 4) & 0x0Fu);
                uint32_t hi = (qh[i >> 2] >> ((i & 3) * 2)) & 0x3u;
                int q = (int)(lo | (hi << 4)) - 32;
                float scale = (float)((int)sc[i >> 4] - 128) / 64.0f;
                o[i] = d * scale * (float)q;
            }
        } else {
            /* ggml Q6_K (gguf-py quants.py Q6_K.dequantize_blocks) */
            for (int n = 0; n < 2; ++n) {
                const uint8_t *l8 = ql + 64 * n, *h8 = qh + 32 * n;
                const int8_t *s8 = (const int8_t *)(sc + 8 * n);
                float *y = o + 128 * n;
                for (int l = 0; l < 32; ++l) {
                    int is = l / 16;
                    int q1 = (int)((l8[l] & 0xF) | (((h8[l] >> 0) & 3) << 4)) - 32;
                    int q2 = (int)((l8[l + 32] & 0xF) | (((h8[l] >> 2) & 3) << 4)) - 32;
                    int q3 = (int)((l8[l] >> 4) | (((h8[l] >> 4) & 3) << 4)) - 32;
                    int q4 = (int)((l8[l + 32] >> 4) | (((h8[l] >> 6) & 3) << 4)) - 32;
                    y[l + 0] = d * (float)s8[is + 0] * (float)q1;
                    y[l + 32] = d * (float)s8[is + 2] * (float)q2;
                    y[l + 64] = d * (float)s8[is + 4] * (float)q3;
                    y[l + 96] = d * (float)s8[is + 6] * (float)q4;
                }
            }
        }
    }
}

int64_t orc_block_weights(int type) {
    switch (type) {
    case NSQ_T_Q4_0: case NSQ_T_Q8_0: return 32;
    case NSQ_T_Q4_K: case NSQ_T_Q5_K: case NSQ_T_Q6_K: return 256;
    default: return 0;
    }
}

int64_t orc_block_bytes(int type) {
    switch (type) {
    case NSQ_T_Q4_0: return 18;
    case NSQ_T_Q8_0: return 34;
    case NSQ_T_Q4_K: return 144;
    case NSQ_T_Q5_K: return 176;
    case NSQ_T_Q6_K: return 210;
    default: return 0;
    }
}

/* Dispatch over the four formats; returns 0 or -1 for an unknown type. */
int orc_dequant(const uint8_t *raw, int type, int layout, int64_t nblocks, float *out, int fp16_mode) {
    switch (type) {
    case NSQ_T_Q4_0: orc_dequant_q4_0(raw, nblocks, out, fp16_mode); return 0;
    case NSQ_T_Q8_0: orc_dequant_q8_0(raw, nblocks, out, fp16_mode); return 0;
    case NSQ_T_Q4_K: orc_dequant_q4_k(raw, nblocks, out, fp16_mode); return 0;
    case NSQ_T_Q5_K: orc_dequant_q5_k(raw, nblocks, out, layout, fp16_mode); return 0;
    case NSQ_T_Q6_K: orc_dequant_q6_k(raw, nblocks, out, layout, fp16_mode); return 0;
    default: return -1;
    }
}

/* pipeline.rs:1256-1268: naive i-j-l loop, B is [K x N] row-major. */
void orc_matmul_f32(const float *a, const float *b, float *c, int64_t m, int64_t k, int64_t n) {
    for (int64_t i = 0; i < m; ++i)
        for (int64_t j = 0; j < n; ++j) {
            float sum = 0.0f;
            for (int64_t l = 0; l < k; ++l) sum += a[i * k + l] * b[l * n + j];
            c[i * n + j] = sum;
        }
}

/* Same contraction with a double accumulator (diagnosis only). */
void orc_matmul_f64(const float *a, const float *b, double *c, int64_t m, int64_t k, int64_t n) {
    for (int64_t i = 0; i < m; ++i)
        for (int64_t j = 0; j < n; ++j) {
            double sum = 0.0;
            for (int64_t l = 0; l < k; ++l) sum += (double)a[i * k + l] * (double)b[l * n + j];
            c[i * n + j] = sum;
        }
}

/*
 * y[M x N] = cpu_matmul_f32(x[M x K], transpose(dequant(W[N x K])))
 * Rows [n0, n1) only.  Row n of W is dequantised once into `wrow` (K floats)
 * and the dot product runs in cpu_matmul_f32's order (l ascending, f32 sum),
 * so the values equal those of the explicit transpose + matmul.
 */
int orc_quant_matmul_rows(const uint8_t *w, int type, int layout, const float *x, float *y,
                          int64_t M, int64_t N, int64_t K, int64_t n0, int64_t n1, float *wrow) {
    int64_t qk = orc_block_weights(type), bb = orc_block_bytes(type);
    if (qk == 0 || K % qk) return -1;
    int64_t nb = K / qk;
    for (int64_t n = n0; n < n1; ++n) {
        if (orc_dequant(w + n * nb * bb, type, layout, nb, wrow, 0)) return -1;
        for (int64_t i = 0; i < M; ++i) {
            float sum = 0.0f;
            const float *xr = x + i * K;
            for (int64_t l = 0; l < K; ++l) sum += xr[l] * wrow[l];
            y[i * N + n] = sum;
        }
    }
    return 0;
}

int orc_quant_matmul(const uint8_t *w, int type, int layout, const float *x, float *y,
                     int64_t M, int64_t N, int64_t K) {
    float *wrow = (float *)malloc(sizeof(float) * (size_t)K);
    if (!wrow) return -2;
    int rc = orc_quant_matmul_rows(w, type, layout, x, y, M, N, K, 0, N, wrow);
    free(wrow);
    return rc;
}

/* Multi-threaded row split of orc_quant_matmul (identical values). */
#include <pthread.h>
#include <unistd.h>
typedef struct {
    const uint8_t *w; int type, layout; const float *x; float *y;
    int64_t M, N, K, n0, n1; int rc;
} orc_mt_job;

static void *orc_mt_worker(void *p) {
    orc_mt_job *j = (orc_mt_job *)p;
    float *wrow = (float *)malloc(sizeof(float) * (size_t)j->K);
    if (!wrow) { j->rc = -2; return NULL; }
    j->rc = orc_quant_matmul_rows(j->w, j->type, j->layout, j->x, j->y, j->M, j->N, j->K, j->n0, j->n1, wrow);
    free(wrow);
    return NULL;
}

int orc_num_threads(void) {
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    return n > 0 ? (int)n : 1;
}

int orc_quant_matmul_mt(const uint8_t *w, int type, int layout, const float *x, float *y,
                        int64_t M, int64_t N, int64_t K, int nthreads) {
    if (nthreads <= 0) nthreads = orc_num_threads();
    if (nthreads > 256) nthreads = 256;
    pthread_t th[256];
    orc_mt_job jobs[256];
    int rc = 0;
    for (int t = 0; t < nthreads; ++t) {
        jobs[t] = (orc_mt_job){w, type, layout, x, y, M, N, K, N * t / nthreads, N * (t + 1) / nthreads, 0};
        if (pthread_create(&th[t], NULL, orc_mt_worker, &jobs[t]) != 0) { orc_mt_worker(&jobs[t]); th[t] = 0; }
    }
    for (int t = 0; t < nthreads; ++t) {
        if (th[t]) pthread_join(th[t], NULL);
        rc |= jobs[t].rc;
    }
    return rc;
}
