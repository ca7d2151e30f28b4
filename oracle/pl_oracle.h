/*
 * pl_oracle.h -- CPU oracle for the picolm attention hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (libpl_attn.so, the
 * picolm_b200 package) links, loads or calls this code.  It is used by the
 * test-suite, by __graft_entry__.smoke() and by bench.py's CPU-baseline leg,
 * always as the checker, never as the thing measured or shipped.
 *
 * It restates, in plain C11 compiled with the reference's flags
 * (-O2 -std=c11, which implies -ffp-contract=off: no FMA contraction),
 * the arithmetic of picolm's attention block:
 *
 *   orc_fp16_to_fp32        picolm/quant.c:11-39   exact FP16 decode
 *   orc_fp32_to_fp16        picolm/quant.c:41-78   FP16 encode, ties AWAY from zero
 *   orc_rope_tables         picolm/model.c:545-556 cos/sin tables (libm powf/cosf/sinf)
 *   orc_rope                picolm/tensor.c:533-603 LLaMA pairwise / Qwen half-split
 *   orc_attn_decode         picolm/model.c:802-892 RoPE, FP16 append, online softmax
 *   orc_attn_prefill        picolm/model.c:1019-1090 the same, position by position
 *
 * Parity pin: tests/golden/ holds vectors produced by the genuine reference
 * (model_forward_ex / rope / fp32_to_fp16 compiled from the reference's own
 * sources by oracle/Makefile into oracle/_ref/), and tests/test_oracle.py
 * checks this restatement against them bit for bit.
 *
 * KV layout, as in picolm (model.c:802-805): one layer of one sequence is
 * [max_seq][kv_dim] uint16 FP16 words, kv_dim = n_kv_heads * head_dim.
 */
#ifndef PL_ORACLE_H
#define PL_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct orc_cfg {
    int n_heads;      /* query heads H          */
    int n_kv_heads;   /* KV heads Hk (GQA)      */
    int head_dim;     /* hd, <= 256             */
    int max_seq;      /* rows per layer in the cache */
    int rope_type;    /* 0 = LLaMA pairwise, 1 = Qwen half-split */
} orc_cfg;

float    orc_fp16_to_fp32(uint16_t h);
uint16_t orc_fp32_to_fp16(float f);
void     orc_fp32_to_fp16_array(const float *src, uint16_t *dst, long n);
void     orc_fp16_to_fp32_array(const uint16_t *src, float *dst, long n);

void orc_rope_tables(float *cos_tab, float *sin_tab, int max_seq, int head_dim,
                     float freq_base);

void orc_rope(float *q, float *k, int head_dim, int n_heads, int n_kv_heads,
              const float *cos_pos, const float *sin_pos, int rope_type);

/* One decode step at `pos` for one layer of one sequence.
 * q [H*hd] and k [kv_dim] are rotated IN PLACE (as model.c does), k and v are
 * appended as FP16 at row `pos`, out [H*hd] receives the attention output. */
void orc_attn_decode(const orc_cfg *c, uint16_t *kc, uint16_t *vc, int pos,
                     float *q, float *k, const float *v,
                     const float *cos_tab, const float *sin_tab, float *out);

/* Attention over rows [0, pos] of an already-filled cache for an already
 * rotated q (no RoPE, no append): the inner loop model.c:848-892 alone. */
void orc_attn_core(const orc_cfg *c, const uint16_t *kc, const uint16_t *vc,
                   int pos, const float *q, float *out);

/* Causal prefill of n_tok positions starting at start_pos (model.c:1019-1090).
 * q [n_tok][H*hd], k/v [n_tok][kv_dim]; q and k rotated in place;
 * out row bi at out + bi*out_stride. */
void orc_attn_prefill(const orc_cfg *c, uint16_t *kc, uint16_t *vc,
                      int start_pos, int n_tok, float *q, float *k,
                      const float *v, const float *cos_tab,
                      const float *sin_tab, float *out, int out_stride);

/* Batched decode over independent sequences (the batched-decode config):
 * sequence s uses the layer view kc + s*seq_stride (elements), position
 * pos[s], q + s*H*hd, k/v + s*kv_dim, out + s*H*hd.  Sequences are spread
 * over n_threads POSIX threads; each sequence is still the reference's
 * single-threaded loop. */
void orc_attn_decode_seqs(const orc_cfg *c, int n_seq, uint16_t *kc,
                          uint16_t *vc, long seq_stride, const int *pos,
                          float *q, float *k, const float *v,
                          const float *cos_tab, const float *sin_tab,
                          float *out, int n_threads);

/* out[d] = sum_i W[d][i] * x[i], plain sequential FP32 (input generation). */
void orc_matvec(const float *W, const float *x, float *out, int n, int d);

/* The projections around the attention path.  vec_dot (quant.c:713-730) for
 * GGUF types F32 (0), F16 (1), Q8_0 (8), Q4_K (12), Q6_K (14) in the
 * reference's plain x86-64 summation order; matmul (tensor.c:202-227) over
 * d rows of raw GGUF bytes; rmsnorm (tensor.c:425-490).  orc_row_bytes is
 * gguf_type_row_size for those types (-1 otherwise). */
float orc_vec_dot(const void *src, const float *x, int n, int type);
long  orc_row_bytes(int type, int n);
void  orc_matmul(float *out, const float *x, const void *W, int n, int d, int type);
void  orc_rmsnorm(float *out, const float *x, const float *weight, int size, float eps);

#ifdef __cplusplus
}
#endif
#endif /* PL_ORACLE_H */
