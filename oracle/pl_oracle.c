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
