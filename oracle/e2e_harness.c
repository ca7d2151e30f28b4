/* e2e_harness.c -- greedy-decoding driver for the end-to-end check (config 2).
 *
 * Test infrastructure.  It stands in for picolm's main (picolm.c:91-318)
 * without the tokenizer: it loads a GGUF file with picolm's model_load,
 * feeds a prompt of random token ids through model_forward_prefill, then
 * generates greedily with model_forward, taking the argmax of the logits as
 * sampler_sample does at temperature 0 (sampler.c:43-51).  The same source
 * is linked twice: with picolm's unmodified model.c (the CPU reference), and
 * with the copy of model.c whose attention blocks call the B200 module
 * (built with -DUSE_PL_ATTN), and with the copy whose whole attention
 * sub-blocks, projections included, call it (-DUSE_PL_BLOCK as well; the
 * layers' attention weights are uploaded once after model_load).  Each
 * generated token is printed with the margin between the best and the
 * second-best logit.
 *
 * usage: e2e MODEL.gguf N_PROMPT N_GEN SEED THREADS [--save F] [--load F]
 *   --load F  kvcache_load(F) first (model.c:1199-1259) and skip the cached
 *             prompt positions in the prefill, as picolm.c:214-236 does;
 *             the last prompt token is always recomputed for its logits
 *   --save F  kvcache_save(F) of the whole prompt (model.c:1158-1196):
 *             after the prefill, or, with --load, right after the load
 */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "model.h"
#include "tensor.h"
#ifdef USE_PL_ATTN
#include "pl_attn.h"
#endif

static uint64_t splitmix64(uint64_t *s) {
    uint64_t z = (*s += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

static double now_s(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (double)ts.tv_sec + 1e-9 * (double)ts.tv_nsec;
}

int main(int argc, char **argv) {
    const char *save_path = NULL, *load_path = NULL;
    for (int i = 6; i + 1 < argc; i += 2) {
        if (strcmp(argv[i], "--save") == 0) save_path = argv[i + 1];
        else if (strcmp(argv[i], "--load") == 0) load_path = argv[i + 1];
        else argc = -1;
    }
    if (argc < 6 || (argc - 6) % 2) {
        fprintf(stderr, "usage: %s MODEL.gguf N_PROMPT N_GEN SEED THREADS [--save F] [--load F]\n",
                argv[0]);
        return 2;
    }
    const char *path = argv[1];
    const int n_prompt = atoi(argv[2]), n_gen = atoi(argv[3]), threads = atoi(argv[5]);
    uint64_t seed = (uint64_t)strtoull(argv[4], NULL, 10);
    tensor_set_threads(threads);

    model_t model;
    if (model_load(&model, path, 0) != 0) {
        fprintf(stderr, "model_load failed\n");
        return 1;
    }
    const model_config_t *c = &model.config;
    if (n_prompt < 1 || n_gen < 1 || n_prompt + n_gen > c->max_seq_len) {
        fprintf(stderr, "prompt + generation exceeds the context (%d)\n", c->max_seq_len);
        return 2;
    }
#ifdef USE_PL_ATTN
    int rc = pl_attn_init(c->n_layers, c->n_heads, c->n_kv_heads, c->head_dim, c->max_seq_len,
                          c->rope_freq_base, c->rope_type, 1, 0);
    if (rc == PL_OK)
        rc = pl_attn_set_rope(model.state.rope_cos, model.state.rope_sin, c->max_seq_len,
                              c->head_dim / 2);
    /* the run-state block holds s->q, k_tmp, v_tmp and s->xb (model.c:593-627):
       page-locked once, the decode calls DMA them without staging */
    if (rc == PL_OK)
        rc = pl_attn_host_register(model.state.mem_block,
                                   model.state.mem_size - model.state.kv_size);
#ifdef USE_PL_BLOCK
    /* each layer's attention weights (model.h:39-72) in their GGUF types,
     * with the F32 norm weights and biases picolm prepared at load
     * (model.c:640-712) */
    for (int l = 0; l < c->n_layers && rc == PL_OK; l++) {
        const layer_weights_t *lw = &model.weights.layers[l];
        const run_state_t *s = &model.state;
        rc = pl_attn_set_layer(l, c->n_embd, s->attn_norm_w[l], c->rms_norm_eps,
                               lw->attn_q, lw->type_attn_q, lw->attn_k, lw->type_attn_k,
                               lw->attn_v, lw->type_attn_v, lw->attn_output,
                               lw->type_attn_output,
                               lw->attn_q_b ? s->attn_q_bias[l] : NULL,
                               lw->attn_k_b ? s->attn_k_bias[l] : NULL,
                               lw->attn_v_b ? s->attn_v_bias[l] : NULL,
                               lw->attn_output_b ? s->attn_output_bias[l] : NULL,
                               lw->attn_q_norm ? s->attn_q_norm_w[l] : NULL,
                               lw->attn_q_norm ? s->attn_k_norm_w[l] : NULL);
    }
#endif
    if (rc != PL_OK) {
        fprintf(stderr, "pl_attn: %s\n", pl_attn_strerror(rc));
        return 1;
    }
#endif
    int *prompt = (int *)malloc((size_t)n_prompt * sizeof(int));
    for (int i = 0; i < n_prompt; i++)
        prompt[i] = 3 + (int)(splitmix64(&seed) % (uint64_t)(c->vocab_size - 3));

    int cache_pos = 0;
    if (load_path) {
        cache_pos = kvcache_load(&model, load_path);
        if (cache_pos <= 0) {
            fprintf(stderr, "kvcache_load failed\n");
            return 1;
        }
        if (save_path && kvcache_save(&model, save_path, cache_pos) != 0) return 1;
        if (cache_pos > n_prompt - 1) cache_pos = n_prompt - 1;
    }
    const double t0 = now_s();
    model_forward_prefill(&model, prompt + cache_pos, n_prompt - cache_pos, cache_pos);
    const double t1 = now_s();
    if (save_path && !load_path && kvcache_save(&model, save_path, n_prompt) != 0) return 1;
    const float *logits = model.state.logits;
    int pos = n_prompt - 1;
    for (int i = 0; i < n_gen; i++) {
        int best = 0, second = -1;
        for (int v = 1; v < c->vocab_size; v++) {
            if (logits[v] > logits[best]) {
                second = best;
                best = v;
            } else if (second < 0 || logits[v] > logits[second]) {
                second = v;
            }
        }
        printf("T %d %d %.9g\n", i, best, (double)(logits[best] - logits[second]));
        if (i + 1 < n_gen) {
            pos++;
            logits = model_forward(&model, best, pos);
        }
    }
    const double t2 = now_s();
    printf("S prefill_tokens=%d prefill_s=%.6f decode_tokens=%d decode_s=%.6f threads=%d\n",
           n_prompt - cache_pos, t1 - t0, n_gen - 1, t2 - t1, threads);
    fflush(stdout);
#ifdef USE_PL_ATTN
    pl_attn_host_unregister(model.state.mem_block);
    pl_attn_shutdown();
#endif
    free(prompt);
    model_free(&model);
    return 0;
}
