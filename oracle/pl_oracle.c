/*
 * pl_oracle.c -- CPU oracle (test infrastructure only; see pl_oracle.h).
 *
 * Every function restates one piece of picolm's arithmetic, with the
 * reference file:line it follows.  Build flags match the reference Makefile
 * (picolm/Makefile:2: -O2 -std=c11), plus an explicit -ffp-contract=off so
 * that no multiply-add is fused: the reference's loops are compiled without
 * FMA, and bit-exact K rows depend on that.
 */
#define _GNU_SOURCE
#include "pl_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ---- FP16 decode: picolm/quant.c:11-39 (exact, subnormals renormalised) */
float orc_fp16_to_fp32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1Fu;
    uint32_t m = h & 0x3FFu;
    uint32_t bits;
    if (e == 0x1Fu) {
        bits = sign | 0x7F800000u | (m << 13);
    } else if (e != 0) {
        bits = sign | ((e + 112u) << 23) | (m << 13);
    } else if (m == 0) {
        bits = sign;
    } else {
        /* subnormal: shift the leading one up to the implicit-bit position */
        uint32_t shifts = 0;
        while (!(m & 0x400u)) { m <<= 1; ++shifts; }
        bits = sign | ((113u - shifts) << 23) | ((m & 0x3FFu) << 13);
    }
    float f;
    memcpy(&f, &bits, sizeof f);
    return f;
}

/* ---- FP16 encode: picolm/quant.c:41-78.
 * Normal range: add half an FP16 ulp (bit 12) to the 23-bit mantissa and
 * truncate, i.e. round half AWAY from zero (not to even).  A carry out of
 * the mantissa bumps the exponent; reaching exponent 31 gives infinity.
 * FP32 zero/subnormal -> signed zero; NaN -> sign|0x7E00; Inf -> sign|0x7C00;
 * FP16-subnormal results also round half up.                             */
uint16_t orc_fp32_to_fp16(float f) {
    uint32_t b;
    memcpy(&b, &f, sizeof b);
    uint16_t s = (uint16_t)((b >> 16) & 0x8000u);
    uint32_t E = (b >> 23) & 0xFFu;
    uint32_t m = b & 0x7FFFFFu;
    if (E == 0) return s;
    if (E == 0xFFu) return (uint16_t)(s | 0x7C00u | (m ? 0x0200u : 0u));
    int e = (int)E - 112;                      /* FP16 biased exponent */
    if (e >= 31) return (uint16_t)(s | 0x7C00u);
    if (e <= 0) {
        if (e < -10) return s;
        uint32_t full = m | 0x800000u;
        uint32_t sh = (uint32_t)(14 - e);
        return (uint16_t)(s | ((full + (1u << (sh - 1))) >> sh));
    }
    /* exponent and mantissa side by side, so the rounding carry propagates */
    uint32_t r = ((((uint32_t)e << 23) | m) + 0x1000u) >> 13;
    if (r >= 0x7C00u) return (uint16_t)(s | 0x7C00u);
    return (uint16_t)(s | r);
}

void orc_fp32_to_fp16_array(const float *src, uint16_t *dst, long n) {
    for (long i = 0; i < n; ++i) dst[i] = orc_fp32_to_fp16(src[i]);
}

void orc_fp16_to_fp32_array(const uint16_t *src, float *dst, long n) {
    for (long i = 0; i < n; ++i) dst[i] = orc_fp16_to_fp32(src[i]);
}

/* ---- RoPE tables: picolm/model.c:545-556 (FP32 libm, built once) ------- */
void orc_rope_tables(float *cos_tab, float *sin_tab, int max_seq, int head_dim,
                     float freq_base) {
    int half = head_dim / 2;
    for (int p = 0; p < max_seq; ++p) {
        for (int i = 0; i < half; ++i) {
            float inv = powf(freq_base, (float)(2 * i) / (float)head_dim);
            float theta = (float)p / inv;
            cos_tab[(long)p * half + i] = cosf(theta);
            sin_tab[(long)p * half + i] = sinf(theta);
        }
    }
}

/* ---- RoPE: picolm/tensor.c:533-603.  Each rotated element is two rounded
 * products and one rounded add/sub (no FMA).                              */
static void rotate_heads(float *x, int n, int head_dim, const float *cs,
                         const float *sn, int rope_type) {
    int half = head_dim / 2;
    for (int h = 0; h < n; ++h) {
        float *xh = x + (long)h * head_dim;
        for (int i = 0; i < half; ++i) {
            int a = rope_type == 1 ? i : 2 * i;          /* Qwen: (i, i+half) */
            int b = rope_type == 1 ? i + half : 2 * i + 1; /* LLaMA: (2i, 2i+1) */
            float x0 = xh[a], x1 = xh[b];
            float t0 = x0 * cs[i];
            float t1 = x1 * sn[i];
            float t2 = x0 * sn[i];
            float t3 = x1 * cs[i];
            xh[a] = t0 - t1;
            xh[b] = t2 + t3;
        }
    }
}

void orc_rope(float *q, float *k, int head_dim, int n_heads, int n_kv_heads,
              const float *cos_pos, const float *sin_pos, int rope_type) {
    rotate_heads(q, n_heads, head_dim, cos_pos, sin_pos, rope_type);
    rotate_heads(k, n_kv_heads, head_dim, cos_pos, sin_pos, rope_type);
}

/* ---- Attention inner loop: picolm/model.c:848-892.
 * Per query head h (KV head h / kv_mul): single-pass online softmax over
 * rows t = 0..pos, score = (sum_d q[d]*K[t][d]) / sqrtf(hd) accumulated
 * sequentially, strict '>' for a new maximum, max initialised to -1e30f,
 * libm expf, out = acc * (1/sum).                                         */
void orc_attn_core(const orc_cfg *c, const uint16_t *kc, const uint16_t *vc,
                   int pos, const float *q, float *out) {
    int hd = c->head_dim;
    int kv_dim = c->n_kv_heads * hd;
    int kv_mul = c->n_heads / c->n_kv_heads;
    float acc[256];
    for (int h = 0; h < c->n_heads; ++h) {
        const float *qh = q + (long)h * hd;
        int g = h / kv_mul;
        float best = -1e30f;
        float denom = 0.0f;
        for (int d = 0; d < hd; ++d) acc[d] = 0.0f;
        for (int t = 0; t <= pos; ++t) {
            const uint16_t *kt = kc + (long)t * kv_dim + (long)g * hd;
            const uint16_t *vt = vc + (long)t * kv_dim + (long)g * hd;
            float sc = 0.0f;
            for (int d = 0; d < hd; ++d) sc += qh[d] * orc_fp16_to_fp32(kt[d]);
            sc /= sqrtf((float)hd);
            if (sc > best) {
                float corr = expf(best - sc);
                denom = denom * corr + 1.0f;
                for (int d = 0; d < hd; ++d)
                    acc[d] = acc[d] * corr + orc_fp16_to_fp32(vt[d]);
                best = sc;
            } else {
                float w = expf(sc - best);
                denom += w;
                for (int d = 0; d < hd; ++d)
                    acc[d] += w * orc_fp16_to_fp32(vt[d]);
            }
        }
        float inv = 1.0f / denom;
        for (int d = 0; d < hd; ++d) out[(long)h * hd + d] = acc[d] * inv;
    }
}

/* RoPE + FP16 append of one position: model.c:820-826 (decode) and
 * model.c:1039-1051 (prefill). */
static void rope_and_append(const orc_cfg *c, uint16_t *kc, uint16_t *vc,
                            int pos, float *q, float *k, const float *v,
                            const float *cos_tab, const float *sin_tab) {
    int half = c->head_dim / 2;
    int kv_dim = c->n_kv_heads * c->head_dim;
    orc_rope(q, k, c->head_dim, c->n_heads, c->n_kv_heads,
             cos_tab + (long)pos * half, sin_tab + (long)pos * half,
             c->rope_type);
    uint16_t *krow = kc + (long)pos * kv_dim;
    uint16_t *vrow = vc + (long)pos * kv_dim;
    for (int d = 0; d < kv_dim; ++d) {
        krow[d] = orc_fp32_to_fp16(k[d]);
        vrow[d] = orc_fp32_to_fp16(v[d]);
    }
}

/* ---- Decode step: picolm/model.c:802-892 ------------------------------ */
void orc_attn_decode(const orc_cfg *c, uint16_t *kc, uint16_t *vc, int pos,
                     float *q, float *k, const float *v,
                     const float *cos_tab, const float *sin_tab, float *out) {
    rope_and_append(c, kc, vc, pos, q, k, v, cos_tab, sin_tab);
    orc_attn_core(c, kc, vc, pos, q, out);
}

/* ---- Prefill: picolm/model.c:1019-1090.  Strictly position by position:
 * position bi is rotated and appended before its attention runs, so it sees
 * rows [0, start_pos+bi] and nothing later (causal).                     */
void orc_attn_prefill(const orc_cfg *c, uint16_t *kc, uint16_t *vc,
                      int start_pos, int n_tok, float *q, float *k,
                      const float *v, const float *cos_tab,
                      const float *sin_tab, float *out, int out_stride) {
    int q_dim = c->n_heads * c->head_dim;
    int kv_dim = c->n_kv_heads * c->head_dim;
    for (int bi = 0; bi < n_tok; ++bi) {
        int pos = start_pos + bi;
        float *qp = q + (long)bi * q_dim;
        rope_and_append(c, kc, vc, pos, qp, k + (long)bi * kv_dim,
                        v + (long)bi * kv_dim, cos_tab, sin_tab);
        orc_attn_core(c, kc, vc, pos, qp, out + (long)bi * out_stride);
    }
}

/* ---- Batched decode over independent sequences ------------------------ */
typedef struct {
    const orc_cfg *c;
    int s0, s1;
    uint16_t *kc, *vc;
    long seq_stride;
    const int *pos;
    float *q, *k;
    const float *v, *cos_tab, *sin_tab;
    float *out;
} seq_job;

static void *seq_worker(void *arg) {
    seq_job *j = (seq_job *)arg;
    int q_dim = j->c->n_heads * j->c->head_dim;
    int kv_dim = j->c->n_kv_heads * j->c->head_dim;
    for (int s = j->s0; s < j->s1; ++s)
        orc_attn_decode(j->c, j->kc + s * j->seq_stride, j->vc + s * j->seq_stride,
                        j->pos[s], j->q + (long)s * q_dim, j->k + (long)s * kv_dim,
                        j->v + (long)s * kv_dim, j->cos_tab, j->sin_tab,
                        j->out + (long)s * q_dim);
    return NULL;
}

void orc_attn_decode_seqs(const orc_cfg *c, int n_seq, uint16_t *kc,
                          uint16_t *vc, long seq_stride, const int *pos,
                          float *q, float *k, const float *v,
                          const float *cos_tab, const float *sin_tab,
                          float *out, int n_threads) {
    if (n_threads < 1) n_threads = 1;
    if (n_threads > n_seq) n_threads = n_seq;
    if (n_threads > 256) n_threads = 256;
    seq_job jobs[256];
    pthread_t tid[256];
    for (int t = 0; t < n_threads; ++t) {
        seq_job j = {c, (int)((long)n_seq * t / n_threads),
                     (int)((long)n_seq * (t + 1) / n_threads), kc, vc,
                     seq_stride, pos, q, k, v, cos_tab, sin_tab, out};
        jobs[t] = j;
    }
    for (int t = 1; t < n_threads; ++t)
        pthread_create(&tid[t], NULL, seq_worker, &jobs[t]);
    seq_worker(&jobs[0]);
    for (int t = 1; t < n_threads; ++t) pthread_join(tid[t], NULL);
}

void orc_matvec(const float *W, const float *x, float *out, int n, int d) {
    for (int i = 0; i < d; ++i) {
        float s = 0.0f;
        for (int j = 0; j < n; ++j) s += W[(long)i * n + j] * x[j];
        out[i] = s;
    }
}

/* ==================================================================
 * The projections on either side of the attention path (model.c:779-817,
 * 894-897): vec_dot per GGUF type, matmul, rmsnorm.  The summation orders
 * are those of the reference as compiled for plain x86-64: the scalar
 * branches of the quantised dots (quant.c:496-505, 583-617, 695-709) and
 * the SSE2 branch of the F32 dot (quant.c:366-377).
 * ================================================================== */

static float orc_sse2_dot(const float *w, const float *x, int n) {
    /* quant.c:366-377: two 4-wide accumulators over steps of 8, the
     * horizontal sum of their sum (hsum_sse, quant.h:23-29), then the tail */
    float a0[4] = {0, 0, 0, 0}, a1[4] = {0, 0, 0, 0};
    int i = 0;
    for (; i + 7 < n; i += 8)
        for (int l = 0; l < 4; ++l) {
            a0[l] = a0[l] + w[i + l] * x[i + l];
            a1[l] = a1[l] + w[i + 4 + l] * x[i + 4 + l];
        }
    float v[4];
    for (int l = 0; l < 4; ++l) v[l] = a0[l] + a1[l];
    float sum = (v[0] + v[2]) + (v[1] + v[3]);
    for (; i < n; i++) sum += w[i] * x[i];
    return sum;
}

static void orc_scale_min_k4(int j, const uint8_t *q, uint8_t *sc, uint8_t *mn) {
    /* quant.c:82-90 */
    if (j < 4) {
        *sc = q[j] & 63;
        *mn = q[j + 4] & 63;
    } else {
        *sc = (uint8_t)((q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4));
        *mn = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
    }
}

static float orc_dot_q4_K(const uint8_t *src, const float *x, int n) {
    /* quant.c:390-512, scalar branch; block {d, dmin, scales[12], qs[128]} */
    float sumf = 0.0f;
    for (int i = 0; i < n / 256; i++) {
        const uint8_t *b = src + (size_t)i * 144;
        uint16_t dh, mh;
        memcpy(&dh, b, 2);
        memcpy(&mh, b + 2, 2);
        const float d = orc_fp16_to_fp32(dh), dmin = orc_fp16_to_fp32(mh);
        const uint8_t *scales = b + 4, *q = b + 16;
        const float *xp = x + i * 256;
        for (int j = 0, is = 0; j < 4; j++, is += 2, xp += 64, q += 32) {
            uint8_t sc, mn;
            orc_scale_min_k4(is, scales, &sc, &mn);
            const float d1 = d * (float)sc, m1 = dmin * (float)mn;
            orc_scale_min_k4(is + 1, scales, &sc, &mn);
            const float d2 = d * (float)sc, m2 = dmin * (float)mn;
            float sum_qx1 = 0.0f, sum_x1 = 0.0f, sum_qx2 = 0.0f, sum_x2 = 0.0f;
            for (int l = 0; l < 32; l++) {
                sum_qx1 += (float)(q[l] & 0xF) * xp[l];
                sum_x1 += xp[l];
                sum_qx2 += (float)(q[l] >> 4) * xp[l + 32];
                sum_x2 += xp[l + 32];
            }
            sumf += d1 * sum_qx1 - m1 * sum_x1 + d2 * sum_qx2 - m2 * sum_x2;
        }
    }
    return sumf;
}

static float orc_dot_q6_K(const uint8_t *src, const float *x, int n) {
    /* quant.c:517-625, scalar branch; block {ql[128], qh[64], scales[16], d} */
    float sumf = 0.0f;
    for (int i = 0; i < n / 256; i++) {
        const uint8_t *b = src + (size_t)i * 210;
        const uint8_t *ql = b, *qh = b + 128;
        const int8_t *sc = (const int8_t *)(b + 192);
        uint16_t dh;
        memcpy(&dh, b + 208, 2);
        const float d = orc_fp16_to_fp32(dh);
        const float *xp = x + i * 256;
        float sums[16] = {0};
        for (int chunk = 0; chunk < 2; chunk++) {
            const int is = chunk * 8;
            const uint8_t *qlc = ql + chunk * 64, *qhc = qh + chunk * 32;
            const float *xc = xp + chunk * 128;
            for (int half = 0; half < 2; half++)
                for (int l = half * 16; l < half * 16 + 16; l++) {
                    const int q1 = (int)((qlc[l] & 0xF) | (((qhc[l] >> 0) & 3) << 4)) - 32;
                    const int q2 = (int)((qlc[l + 32] & 0xF) | (((qhc[l] >> 2) & 3) << 4)) - 32;
                    const int q3 = (int)((qlc[l] >> 4) | (((qhc[l] >> 4) & 3) << 4)) - 32;
                    const int q4 = (int)((qlc[l + 32] >> 4) | (((qhc[l] >> 6) & 3) << 4)) - 32;
                    sums[is + half + 0] += (float)q1 * xc[l];
                    sums[is + half + 2] += (float)q2 * xc[l + 32];
                    sums[is + half + 4] += (float)q3 * xc[l + 64];
                    sums[is + half + 6] += (float)q4 * xc[l + 96];
                }
        }
        for (int j = 0; j < 16; j++) sumf += d * (float)sc[j] * sums[j];
    }
    return sumf;
}

static float orc_dot_q8_0(const uint8_t *src, const float *x, int n) {
    /* quant.c:627-711, scalar branch; block {d, qs[32]} */
    float sumf = 0.0f;
    for (int i = 0; i < n / 32; i++) {
        const uint8_t *b = src + (size_t)i * 34;
        uint16_t dh;
        memcpy(&dh, b, 2);
        const float d = orc_fp16_to_fp32(dh);
        const int8_t *qs = (const int8_t *)(b + 2);
        float sum = 0.0f;
        for (int j = 0; j + 1 < 32; j += 2)
            sum += (float)qs[j] * x[j] + (float)qs[j + 1] * x[j + 1];
        sumf += d * sum;
        x += 32;
    }
    return sumf;
}

float orc_vec_dot(const void *src, const float *x, int n, int type) {
    /* quant.c:713-730 */
    switch (type) {
        case 12: return orc_dot_q4_K((const uint8_t *)src, x, n);
        case 14: return orc_dot_q6_K((const uint8_t *)src, x, n);
        case 8: return orc_dot_q8_0((const uint8_t *)src, x, n);
        case 0: return orc_sse2_dot((const float *)src, x, n);
        case 1: {
            /* default branch: dequantize_row_f16 (quant.c:254-259), then the
             * F32 dot */
            float *buf = (float *)malloc((size_t)n * sizeof(float));
            const uint16_t *h = (const uint16_t *)src;
            for (int i = 0; i < n; i++) buf[i] = orc_fp16_to_fp32(h[i]);
            const float s = orc_sse2_dot(buf, x, n);
            free(buf);
            return s;
        }
        default: return NAN;
    }
}

long orc_row_bytes(int type, int n) {
    /* gguf_type_row_size (quant.c:322-330) for the types above */
    switch (type) {
        case 0: return (long)n * 4;
        case 1: return (long)n * 2;
        case 8: return (long)(n / 32) * 34;
        case 12: return (long)(n / 256) * 144;
        case 14: return (long)(n / 256) * 210;
        default: return -1;
    }
}

void orc_matmul(float *out, const float *x, const void *W, int n, int d, int type) {
    /* tensor.c:202-227: one vec_dot per output row (the thread split does
     * not change any row's arithmetic) */
    const long rb = orc_row_bytes(type, n);
    for (int i = 0; i < d; i++)
        out[i] = orc_vec_dot((const uint8_t *)W + (size_t)i * (size_t)rb, x, n, type);
}

void orc_rmsnorm(float *out, const float *x, const float *weight, int size, float eps) {
    /* tensor.c:425-490, SSE2 branch (4-wide sum of squares, hsum_sse, tail);
     * the scale is applied as (x * ss) * w */
    float a[4] = {0, 0, 0, 0};
    int i = 0;
    for (; i + 3 < size; i += 4)
        for (int l = 0; l < 4; ++l) a[l] = a[l] + x[i + l] * x[i + l];
    float ss = (a[0] + a[2]) + (a[1] + a[3]);
    for (; i < size; i++) ss += x[i] * x[i];
    ss = 1.0f / sqrtf(ss / (float)size + eps);
    for (i = 0; i < size; i++) out[i] = x[i] * ss * weight[i];
}
