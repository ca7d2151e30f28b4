/*
 * ref_shim.c -- TEST INFRASTRUCTURE: a thin harness around the GENUINE
 * picolm sources, compiled in place from the reference tree by
 * oracle/Makefile (target `ref`) into oracle/_ref/libpicoref.so.
 *
 * This translation unit #includes the reference's model.c (it is not copied
 * into this repository; the include path points at the reference tree) so
 * that its file-static functions -- allocate_run_state, init_rope_tables,
 * model_forward_ex -- can be driven directly on an in-memory one-layer FP32
 * model.  quant.c and tensor.c are compiled as their own objects, exactly
 * as the reference Makefile does, so fp16_to_fp32 / fp32_to_fp16 / rope stay
 * out-of-line calls like in the real binary.
 *
 * Exported entry points (used by tests/golden/make_golden.py and by
 * bench.py --impl reference):
 *   ref_rope_tables      model.c:545-556 (the reference's init_rope_tables)
 *   ref_decode_layer     model.c:746-925 model_forward_ex, 1 layer, Wo = I,
 *                        FFN/logits zero; returns q,k,v as the layer computed
 *                        them, the attention output (s->xb2) and the cache.
 *   ref_prefill_layer    model.c:939-1144 model_forward_prefill, 1 layer;
 *                        returns q,k,v rows and the cache rows it appended.
 *   ref_attn_decode_seqs the decode attention loop of model.c:848-892 for
 *                        many independent sequences on POSIX threads.  The
 *                        loop is inline in model_forward_ex, so it cannot be
 *                        called alone; it is restated below with the same
 *                        order of operations, calling the reference's own
 *                        compiled fp16_to_fp32 / fp32_to_fp16 / rope.  The
 *                        golden tests pin it against model_forward_ex bit
 *                        for bit.
 */
#include "model.c"   /* resolved with -I <reference>/picolm */

#include <pthread.h>

static void fill_ones(float *p, long n) { for (long i = 0; i < n; ++i) p[i] = 1.0f; }

/* A one-layer FP32 model whose output projection is the identity, so that
 * s->xb2 after model_forward_ex equals the attention output exactly (each
 * xb2[i] is a dot product with exactly one nonzero term, 1.0f * xb[i]).  */
typedef struct {
    model_t m;
    float *blob;
} ref_model;

static int ref_model_init(ref_model *rm, int n_heads, int n_kv_heads,
                          int head_dim, int max_seq, float rope_base,
                          int rope_type, const float *embd, int vocab,
                          const float *wq, const float *wk, const float *wv) {
    memset(rm, 0, sizeof *rm);
    model_config_t *c = &rm->m.config;
    int dim = n_heads * head_dim;
    int kv_dim = n_kv_heads * head_dim;
    int n_ffn = 8;
    c->n_embd = dim;
    c->n_ffn = n_ffn;
    c->n_heads = n_heads;
    c->n_kv_heads = n_kv_heads;
    c->n_layers = 1;
    c->vocab_size = vocab;
    c->max_seq_len = max_seq;
    c->head_dim = head_dim;
    c->rope_freq_base = rope_base;
    c->rms_norm_eps = 1e-5f;
    c->rope_type = rope_type ? ROPE_TYPE_QWEN : ROPE_TYPE_LLAMA;
    c->alignment = 32;
    c->weight_type = GGUF_TYPE_F32;

    long n_norm = 3L * dim;
    long n_wo = (long)dim * dim;
    long n_ffn_w = 3L * n_ffn * dim;
    long n_out = (long)vocab * dim;
    long total = n_norm + n_wo + n_ffn_w + n_out;
    rm->blob = (float *)calloc((size_t)total, sizeof(float));
    if (!rm->blob) return -1;
    float *p = rm->blob;
    float *attn_norm = p; p += dim;
    float *ffn_norm = p; p += dim;
    float *out_norm = p; p += dim;
    float *wo = p; p += n_wo;
    float *ffn = p; p += n_ffn_w;
    float *wout = p;
    fill_ones(attn_norm, dim);
    fill_ones(ffn_norm, dim);
    fill_ones(out_norm, dim);
    for (int i = 0; i < dim; ++i) wo[(long)i * dim + i] = 1.0f;

    model_weights_t *w = &rm->m.weights;
    w->token_embd = embd;          w->type_token_embd = GGUF_TYPE_F32;
    w->output_norm = out_norm;     w->type_output_norm = GGUF_TYPE_F32;
    w->output = wout;              w->type_output = GGUF_TYPE_F32;
    layer_weights_t *lw = &w->layers[0];
    lw->attn_norm = attn_norm;     lw->type_attn_norm = GGUF_TYPE_F32;
    lw->attn_q = wq;               lw->type_attn_q = GGUF_TYPE_F32;
    lw->attn_k = wk;               lw->type_attn_k = GGUF_TYPE_F32;
    lw->attn_v = wv;               lw->type_attn_v = GGUF_TYPE_F32;
    lw->attn_output = wo;          lw->type_attn_output = GGUF_TYPE_F32;
    lw->ffn_norm = ffn_norm;       lw->type_ffn_norm = GGUF_TYPE_F32;
    lw->ffn_gate = ffn;            lw->type_ffn_gate = GGUF_TYPE_F32;
    lw->ffn_up = ffn + (long)n_ffn * dim; lw->type_ffn_up = GGUF_TYPE_F32;
    lw->ffn_down = ffn + 2L * n_ffn * dim; lw->type_ffn_down = GGUF_TYPE_F32;
    (void)kv_dim;
    if (allocate_run_state(&rm->m) != 0) { free(rm->blob); return -1; }
    return 0;
}

static void ref_model_free(ref_model *rm) {
    model_free(&rm->m);
    free(rm->blob);
}

/* ---- model.c:545-556, the reference's own table builder ---------------- */
int ref_rope_tables(float *cos_tab, float *sin_tab, int max_seq, int head_dim,
                    float freq_base) {
    model_config_t c;
    run_state_t s;
    memset(&c, 0, sizeof c);
    memset(&s, 0, sizeof s);
    c.max_seq_len = max_seq;
    c.head_dim = head_dim;
    c.rope_freq_base = freq_base;
    s.rope_cos = cos_tab;
    s.rope_sin = sin_tab;
    init_rope_tables(&s, &c);
    return 0;
}

/* ---- One genuine decode layer at `pos`.
 * x [dim]: the layer input (token 0's embedding row).
 * kc/vc [max_seq][kv_dim]: cache contents before the step (rows < pos used);
 *   overwritten with the cache after the step.
 * q_out [dim], k_out/v_out [kv_dim]: q, k, v as the layer computes them
 *   (before RoPE), recomputed here with the same reference calls.
 * attn_out [dim]: the attention output of model.c:848-892.
 * cos_tab/sin_tab, if not NULL, receive the layer's RoPE tables.          */
int ref_decode_layer(int n_heads, int n_kv_heads, int head_dim, int max_seq,
                     float rope_base, int rope_type, const float *x,
                     const float *wq, const float *wk, const float *wv,
                     uint16_t *kc, uint16_t *vc, int pos, float *q_out,
                     float *k_out, float *v_out, float *attn_out,
                     float *cos_tab, float *sin_tab) {
    ref_model rm;
    if (ref_model_init(&rm, n_heads, n_kv_heads, head_dim, max_seq, rope_base,
                       rope_type, x, 1, wq, wk, wv) != 0)
        return -1;
    model_config_t *c = &rm.m.config;
    run_state_t *s = &rm.m.state;
    int dim = c->n_embd;
    int kv_dim = n_kv_heads * head_dim;
    size_t cache_elems = (size_t)max_seq * kv_dim;
    memcpy(s->key_cache, kc, cache_elems * sizeof(uint16_t));
    memcpy(s->val_cache, vc, cache_elems * sizeof(uint16_t));

    /* q, k, v exactly as model.c:777-789 computes them */
    float *xb = (float *)malloc(sizeof(float) * (size_t)dim);
    rmsnorm(xb, x, s->attn_norm_w[0], dim, c->rms_norm_eps);
    matmul_bias(q_out, xb, rm.m.weights.layers[0].attn_q, s->attn_q_bias[0],
                dim, n_heads * head_dim, GGUF_TYPE_F32, GGUF_TYPE_F32,
                s->dequant_scratch);
    matmul_dual(k_out, v_out, xb, wk, wv, dim, kv_dim, GGUF_TYPE_F32,
                GGUF_TYPE_F32);
    free(xb);

    model_forward_ex(&rm.m, 0, pos, 1);
    memcpy(attn_out, s->xb2, sizeof(float) * (size_t)dim);
    memcpy(kc, s->key_cache, cache_elems * sizeof(uint16_t));
    memcpy(vc, s->val_cache, cache_elems * sizeof(uint16_t));
    if (cos_tab)
        memcpy(cos_tab, s->rope_cos, sizeof(float) * (size_t)max_seq * (head_dim / 2));
    if (sin_tab)
        memcpy(sin_tab, s->rope_sin, sizeof(float) * (size_t)max_seq * (head_dim / 2));
    ref_model_free(&rm);
    return 0;
}

/* ---- One genuine prefill layer (model_forward_prefill, 1 layer).
 * embd [n_tok][dim]: the n_tok token rows (token id bi -> row bi).
 * kc/vc as above (rows < start_pos used, rows appended are returned).
 * q_out [n_tok][dim], k_out/v_out [n_tok][kv_dim]: the batched projections
 * as model.c:990-1000 computes them (before RoPE).                         */
int ref_prefill_layer(int n_heads, int n_kv_heads, int head_dim, int max_seq,
                      float rope_base, int rope_type, const float *embd,
                      int n_tok, int start_pos, const float *wq,
                      const float *wk, const float *wv, uint16_t *kc,
                      uint16_t *vc, float *q_out, float *k_out, float *v_out) {
    ref_model rm;
    if (ref_model_init(&rm, n_heads, n_kv_heads, head_dim, max_seq, rope_base,
                       rope_type, embd, n_tok, wq, wk, wv) != 0)
        return -1;
    model_config_t *c = &rm.m.config;
    run_state_t *s = &rm.m.state;
    int dim = c->n_embd;
    int kv_dim = n_kv_heads * head_dim;
    size_t cache_elems = (size_t)max_seq * kv_dim;
    memcpy(s->key_cache, kc, cache_elems * sizeof(uint16_t));
    memcpy(s->val_cache, vc, cache_elems * sizeof(uint16_t));

    float *xb = (float *)malloc(sizeof(float) * (size_t)dim * n_tok);
    for (int bi = 0; bi < n_tok; ++bi)
        rmsnorm(xb + (size_t)bi * dim, embd + (size_t)bi * dim, s->attn_norm_w[0],
                dim, c->rms_norm_eps);
    matmul_batch(q_out, xb, n_tok, wq, dim, n_heads * head_dim, GGUF_TYPE_F32);
    matmul_dual_batch(k_out, v_out, xb, n_tok, wk, wv, dim, kv_dim,
                      GGUF_TYPE_F32, GGUF_TYPE_F32);
    free(xb);

    int *tokens = (int *)malloc(sizeof(int) * (size_t)n_tok);
    for (int bi = 0; bi < n_tok; ++bi) tokens[bi] = bi;
    model_forward_prefill(&rm.m, tokens, n_tok, start_pos);
    free(tokens);
    memcpy(kc, s->key_cache, cache_elems * sizeof(uint16_t));
    memcpy(vc, s->val_cache, cache_elems * sizeof(uint16_t));
    ref_model_free(&rm);
    return 0;
}

/* ---- Decode attention for many independent sequences ------------------
 * Restatement of model.c:820-826 and 848-892 with the same order of
 * floating-point operations (the loop is inline in model_forward_ex),
 * calling the reference's own compiled rope / fp32_to_fp16 / fp16_to_fp32.  One sequence runs on one thread, as
 * in picolm; independent sequences are spread over n_threads threads.    */
static void ref_decode_one(int n_heads, int n_kv_heads, int head_dim,
                           uint16_t *kc, uint16_t *vc, int pos, float *q,
                           float *k, const float *v, const float *cs,
                           const float *sn, float *out) {
    int kv_dim = n_kv_heads * head_dim;
    int group = n_heads / n_kv_heads;
    float acc[256];
    /* model.c:820-826: rotate q and k, append k and v as FP16 at row pos */
    rope(q, k, head_dim, n_heads, n_kv_heads, cs, sn, ROPE_TYPE_LLAMA);
    for (int d = 0; d < kv_dim; ++d) {
        kc[(size_t)pos * kv_dim + d] = fp32_to_fp16(k[d]);
        vc[(size_t)pos * kv_dim + d] = fp32_to_fp16(v[d]);
    }
    /* model.c:848-892: one online-softmax pass per query head */
    for (int h = 0; h < n_heads; ++h) {
        const float *qh = q + (size_t)h * head_dim;
        size_t col = (size_t)(h / group) * head_dim;
        float best = -1e30f, denom = 0.0f;
        for (int d = 0; d < head_dim; ++d) acc[d] = 0.0f;
        for (int t = 0; t <= pos; ++t) {
            const uint16_t *kr = kc + (size_t)t * kv_dim + col;
            const uint16_t *vr = vc + (size_t)t * kv_dim + col;
            float sc = 0.0f;
            for (int d = 0; d < head_dim; ++d) sc += qh[d] * fp16_to_fp32(kr[d]);
            sc /= sqrtf((float)head_dim);
            if (sc > best) {
                float corr = expf(best - sc);
                denom = denom * corr + 1.0f;
                for (int d = 0; d < head_dim; ++d)
                    acc[d] = acc[d] * corr + fp16_to_fp32(vr[d]);
                best = sc;
            } else {
                float w = expf(sc - best);
                denom += w;
                for (int d = 0; d < head_dim; ++d) acc[d] += w * fp16_to_fp32(vr[d]);
            }
        }
        float inv = 1.0f / denom;
        for (int d = 0; d < head_dim; ++d) out[(size_t)h * head_dim + d] = acc[d] * inv;
    }
}

typedef struct {
    int n_heads, n_kv_heads, head_dim, s0, s1;
    uint16_t *kc, *vc;
    long seq_stride;
    const int *pos;
    float *q, *k;
    const float *v, *cos_tab, *sin_tab;
    float *out;
} ref_job;

static void *ref_worker(void *arg) {
    ref_job *j = (ref_job *)arg;
    int q_dim = j->n_heads * j->head_dim;
    int kv_dim = j->n_kv_heads * j->head_dim;
    int half = j->head_dim / 2;
    for (int s = j->s0; s < j->s1; ++s)
        ref_decode_one(j->n_heads, j->n_kv_heads, j->head_dim,
                       j->kc + s * j->seq_stride, j->vc + s * j->seq_stride,
                       j->pos[s], j->q + (size_t)s * q_dim, j->k + (size_t)s * kv_dim,
                       j->v + (size_t)s * kv_dim,
                       j->cos_tab + (size_t)j->pos[s] * half,
                       j->sin_tab + (size_t)j->pos[s] * half,
                       j->out + (size_t)s * q_dim);
    return NULL;
}

int ref_attn_decode_seqs(int n_heads, int n_kv_heads, int head_dim, int n_seq,
                         uint16_t *kc, uint16_t *vc, long seq_stride,
                         const int *pos, float *q, float *k, const float *v,
                         const float *cos_tab, const float *sin_tab, float *out,
                         int n_threads) {
    if (n_threads < 1) n_threads = 1;
    if (n_threads > n_seq) n_threads = n_seq;
    if (n_threads > 256) n_threads = 256;
    ref_job jobs[256];
    pthread_t tid[256];
    for (int t = 0; t < n_threads; ++t) {
        ref_job j = {n_heads, n_kv_heads, head_dim,
                     (int)((long)n_seq * t / n_threads),
                     (int)((long)n_seq * (t + 1) / n_threads), kc, vc, seq_stride,
                     pos, q, k, v, cos_tab, sin_tab, out};
        jobs[t] = j;
    }
    for (int t = 1; t < n_threads; ++t) pthread_create(&tid[t], NULL, ref_worker, &jobs[t]);
    ref_worker(&jobs[0]);
    for (int t = 1; t < n_threads; ++t) pthread_join(tid[t], NULL);
    return 0;
}

/* ---- Causal prefill attention of independent sequences (or layers) ----
 * model.c:1039-1089 per position: position start_pos + i is rotated,
 * appended and attends rows [0, start_pos + i], the positions one after
 * another as model_forward_prefill runs them (the same per-position steps
 * as decode, ref_decode_one).  Sequence s has cache slab kc + s*seq_stride,
 * q [n_tok][n_heads*head_dim], k/v [n_tok][kv_dim] at s*n_tok rows, out
 * likewise.  Independent sequences (for the CPU baseline: the independent
 * layers of a prefill) are spread over n_threads threads; each sequence
 * runs on one thread, as picolm's loop does.                              */
typedef struct {
    int n_heads, n_kv_heads, head_dim, n_tok, start_pos, s0, s1;
    uint16_t *kc, *vc;
    long seq_stride;
    float *q, *k;
    const float *v, *cos_tab, *sin_tab;
    float *out;
} ref_pf_job;

static void *ref_pf_worker(void *arg) {
    ref_pf_job *j = (ref_pf_job *)arg;
    int q_dim = j->n_heads * j->head_dim;
    int kv_dim = j->n_kv_heads * j->head_dim;
    int half = j->head_dim / 2;
    for (int s = j->s0; s < j->s1; ++s)
        for (int i = 0; i < j->n_tok; ++i) {
            size_t row = (size_t)s * j->n_tok + i;
            int pos = j->start_pos + i;
            ref_decode_one(j->n_heads, j->n_kv_heads, j->head_dim,
                           j->kc + s * j->seq_stride, j->vc + s * j->seq_stride, pos,
                           j->q + row * q_dim, j->k + row * kv_dim, j->v + row * kv_dim,
                           j->cos_tab + (size_t)pos * half, j->sin_tab + (size_t)pos * half,
                           j->out + row * q_dim);
        }
    return NULL;
}

int ref_attn_prefill_seqs(int n_heads, int n_kv_heads, int head_dim, int n_seq,
                          uint16_t *kc, uint16_t *vc, long seq_stride, int start_pos,
                          int n_tok, float *q, float *k, const float *v,
                          const float *cos_tab, const float *sin_tab, float *out,
                          int n_threads) {
    if (n_threads < 1) n_threads = 1;
    if (n_threads > n_seq) n_threads = n_seq;
    if (n_threads > 256) n_threads = 256;
    ref_pf_job jobs[256];
    pthread_t tid[256];
    for (int t = 0; t < n_threads; ++t) {
        ref_pf_job j = {n_heads, n_kv_heads, head_dim, n_tok, start_pos,
                        (int)((long)n_seq * t / n_threads),
                        (int)((long)n_seq * (t + 1) / n_threads), kc, vc, seq_stride,
                        q, k, v, cos_tab, sin_tab, out};
        jobs[t] = j;
    }
    for (int t = 1; t < n_threads; ++t) pthread_create(&tid[t], NULL, ref_pf_worker, &jobs[t]);
    ref_pf_worker(&jobs[0]);
    for (int t = 1; t < n_threads; ++t) pthread_join(tid[t], NULL);
    return 0;
}

/* ---- Array forms of the reference's FP16 conversions (quant.c:11-78), so
 * that bit patterns (NaN payloads included) never pass through a host
 * language's float type on the way in or out.                           */
void ref_fp32_to_fp16_array(const float *src, uint16_t *dst, long n) {
    for (long i = 0; i < n; ++i) dst[i] = fp32_to_fp16(src[i]);
}

void ref_fp16_to_fp32_array(const uint16_t *src, float *dst, long n) {
    for (long i = 0; i < n; ++i) dst[i] = fp16_to_fp32(src[i]);
}
