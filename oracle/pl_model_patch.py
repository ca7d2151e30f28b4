"""Build step: a copy of picolm's model.c whose attention calls the B200 module.

Test infrastructure for the end-to-end check.  Reads REF/model.c, finds the
two attention blocks by their text (not by line number, so a different
reference revision fails loudly instead of being mis-patched) and writes
the copy with each block replaced by one C-ABI call:

* decode (model.c:820-892): from the RoPE call `rope(s->q, k_tmp, ...)`
  through the end of the online-softmax loop, up to `/* Output projection */`
  -> pl_attn_decode(0, l, pos, s->q, k_tmp, v_tmp, s->xb);
* prefill (model.c:1019-1090): the per-position QK-norm / RoPE / KV store /
  attention loop, up to `/* f. Batch output projection */`
  -> the QK-norm (Qwen3 only) on the host, then
     pl_attn_prefill(0, l, start_pos, n_tokens, q_batch, k_batch, v_batch,
                     xb_batch, dim).
* kvcache_save (model.c:1158-1196): before the file is written, every
  layer's first n_pos cache rows are downloaded from the device into
  picolm's host cache arrays (pl_kv_download), so the KVCP file keeps its
  exact format;
* kvcache_load (model.c:1199-1259): after the rows are read into the host
  arrays, they are uploaded to the device (pl_kv_upload).
A failing call prints pl_attn_strerror and exits: there is no CPU fallback.
The copy is written to a temporary directory by the oracle Makefile and
deleted after compiling.

With --block the whole attention sub-block goes to the device instead,
projections included (the harness uploads each layer's weights with
pl_attn_set_layer):

* decode (model.c:779-897): from `rmsnorm(s->xb, s->x, s->attn_norm_w[l], ...)`
  through the residual `vec_add(s->x, s->xb2, dim)`
  -> pl_attn_block_decode(l, 1, &seq, &pos, s->x);
* prefill (model.c:990-1100): from `/* a. Batch RMSNorm */` up to
  `/* h. Batch FFN RMSNorm */`
  -> pl_attn_block_prefill(0, l, start_pos, n_tokens, x_batch).

usage: python pl_model_patch.py [--block] REF/model.c OUT/model_pl.c
"""
import sys

DECODE_CALL = """\
        /* RoPE, FP16 KV append and attention of this token on the B200 */
        {
            int pl_rc = pl_attn_decode(0, l, pos, s->q, k_tmp, v_tmp, s->xb);
            if (pl_rc != PL_OK) {
                fprintf(stderr, "pl_attn_decode: %s\\n", pl_attn_strerror(pl_rc));
                exit(1);
            }
        }
"""

PREFILL_CALL = """\
        /* e. QK-norm (Qwen3) on the host, then RoPE, KV append and causal
         *    attention of all positions on the B200 */
        if (lw->attn_q_norm) {
            for (int bi = 0; bi < n_tokens; bi++) {
                float *qb = q_batch + bi * q_dim, *kb = k_batch + bi * kv_dim;
                for (int h = 0; h < n_heads; h++)
                    rmsnorm(qb + h * head_dim, qb + h * head_dim,
                            s->attn_q_norm_w[l], head_dim, c->rms_norm_eps);
                for (int h = 0; h < n_kv_heads; h++)
                    rmsnorm(kb + h * head_dim, kb + h * head_dim,
                            s->attn_k_norm_w[l], head_dim, c->rms_norm_eps);
            }
        }
        {
            int pl_rc = pl_attn_prefill(0, l, start_pos, n_tokens, q_batch, k_batch,
                                        v_batch, xb_batch, dim);
            if (pl_rc != PL_OK) {
                fprintf(stderr, "pl_attn_prefill: %s\\n", pl_attn_strerror(pl_rc));
                exit(1);
            }
        }

"""


KV_SAVE_SYNC = """\
    /* the cache lives on the B200: bring its rows into the host arrays */
    for (int pl_l = 0; pl_l < c->n_layers; pl_l++) {
        int pl_rc = pl_kv_download(0, pl_l, 0, n_pos,
                                   m->state.key_cache + (size_t)pl_l * seq_len * kv_dim,
                                   m->state.val_cache + (size_t)pl_l * seq_len * kv_dim);
        if (pl_rc != PL_OK) {
            fprintf(stderr, "pl_kv_download: %s\\n", pl_attn_strerror(pl_rc));
            return -1;
        }
    }
"""

KV_LOAD_SYNC = """\
    /* the cache lives on the B200: send the rows just read there */
    for (int pl_l = 0; pl_l < c->n_layers; pl_l++) {
        int pl_rc = pl_kv_upload(0, pl_l, 0, n_pos,
                                 m->state.key_cache + (size_t)pl_l * seq_len * kv_dim,
                                 m->state.val_cache + (size_t)pl_l * seq_len * kv_dim);
        if (pl_rc != PL_OK) {
            fprintf(stderr, "pl_kv_upload: %s\\n", pl_attn_strerror(pl_rc));
            fclose(f);
            return 0;
        }
    }
"""


BLOCK_DECODE_CALL = """\
        /* the attention sub-block on the B200: RMSNorm, Q/K/V projections,
         * QK-norm, RoPE, FP16 KV append, attention, output projection and
         * the residual add, s->x updated in place */
        {
            int pl_seq = 0;
            int pl_rc = pl_attn_block_decode(l, 1, &pl_seq, &pos, s->x);
            if (pl_rc != PL_OK) {
                fprintf(stderr, "pl_attn_block_decode: %s\\n", pl_attn_strerror(pl_rc));
                exit(1);
            }
        }
"""

BLOCK_PREFILL_CALL = """\
        /* a.-g. the attention sub-block of every position on the B200,
         *       x_batch updated in place */
        {
            int pl_rc = pl_attn_block_prefill(0, l, start_pos, n_tokens, x_batch);
            if (pl_rc != PL_OK) {
                fprintf(stderr, "pl_attn_block_prefill: %s\\n", pl_attn_strerror(pl_rc));
                exit(1);
            }
        }

"""


def find(lines, pred, start=0):
    for i in range(start, len(lines)):
        if pred(lines[i]):
            return i
    raise SystemExit(f"pl_model_patch: anchor not found after line {start + 1}")


def main():
    args = sys.argv[1:]
    whole_block = "--block" in args
    src, dst = [a for a in args if a != "--block"]
    lines = open(src).read().split("\n")

    ds = find(lines, lambda s: "rope(s->q, k_tmp," in s)
    de = find(lines, lambda s: s.strip() == "/* Output projection */", ds)
    block = "\n".join(lines[ds:de])
    for must in ("fp32_to_fp16(k_tmp[d])", "Flash Attention", "acc[d] * inv_sum"):
        if must not in block:
            raise SystemExit(f"pl_model_patch: decode block does not contain {must!r}")

    ps = find(lines, lambda s: s.strip().startswith("/* e. Per-position: QK-norm, RoPE, KV store"), de)
    pe = find(lines, lambda s: s.strip() == "/* f. Batch output projection */", ps)
    block = "\n".join(lines[ps:pe])
    for must in ("rope(q_pos, k_pos", "fp32_to_fp16(k_pos[d])", "xb_batch + bi * dim"):
        if must not in block:
            raise SystemExit(f"pl_model_patch: prefill block does not contain {must!r}")

    # kvcache_save: after its n_pos check; kvcache_load: before its success message
    ss = find(lines, lambda s: s.startswith("int kvcache_save("), pe)
    sc = find(lines, lambda s: s.strip() == "if (n_pos <= 0 || n_pos > seq_len) return -1;", ss)
    ls = find(lines, lambda s: s.startswith("int kvcache_load("), sc)
    lm = find(lines, lambda s: 'fprintf(stderr, "KV cache loaded:' in s, ls)
    for must, blk in (("m->state.key_cache", lines[ss:sc + 40]), ("m->state.key_cache", lines[ls:lm])):
        if must not in "\n".join(blk):
            raise SystemExit("pl_model_patch: kvcache block does not read the host cache")
    inc = find(lines, lambda s: s.strip() == '#include "model.h"')
    if whole_block:
        # widen both blocks to the whole attention sub-block
        ds = find(lines, lambda s: s.strip().startswith(
            "rmsnorm(s->xb, s->x, s->attn_norm_w[l]"), inc)
        de = find(lines, lambda s: s.strip() == "vec_add(s->x, s->xb2, dim);", ds) + 1
        ps = find(lines, lambda s: s.strip().startswith("/* a. Batch RMSNorm"), de)
        pe = find(lines, lambda s: s.strip().startswith("/* h. Batch FFN RMSNorm"), ps)
        for must, blk in (("matmul_dual(k_tmp, v_tmp", lines[ds:de]),
                          ("lw->attn_output", lines[ds:de]),
                          ("matmul_dual_batch(k_batch", lines[ps:pe]),
                          ("xbi[d] += xoi[d]", lines[ps:pe])):
            if must not in "\n".join(blk):
                raise SystemExit(f"pl_model_patch: block does not contain {must!r}")
        dec, pre = BLOCK_DECODE_CALL, BLOCK_PREFILL_CALL
    else:
        dec, pre = DECODE_CALL, PREFILL_CALL
    out = (lines[:inc + 1] + ['#include "pl_attn.h"'] + lines[inc + 1:ds]
           + dec.split("\n") + lines[de:ps] + pre.split("\n")
           + lines[pe:sc + 1] + KV_SAVE_SYNC.split("\n") + lines[sc + 1:lm - 1]
           + KV_LOAD_SYNC.split("\n") + lines[lm - 1:])
    with open(dst, "w") as f:
        f.write("\n".join(out))


if __name__ == "__main__":
    main()
