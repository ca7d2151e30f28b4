/*
 * pl_attn.h -- C-ABI of the B200 attention module for picolm.
 *
 * picolm runs its attention block inline in model.c, twice:
 *   decode  : model_forward_ex      picolm/model.c:802-892
 *             (RoPE 820, FP16 KV append 822-826, GQA online softmax 848-892)
 *   prefill : model_forward_prefill picolm/model.c:1019-1090
 *             (per position: RoPE 1040-1041, append 1044-1051,
 *              causal attention 1054-1089)
 * and its only device backend, gpu.h, offloads matmuls alone
 * (picolm/gpu.h:23-26).  This header adds the missing attention entry points
 * in gpu.h's style: plain C, int status (0 = success, negative = failure),
 * one module-global context, inline stubs when the backend is compiled out
 * (picolm/gpu.h:33-42).  Unlike gpu_try_matmul there is NO CPU fallback:
 * a failing call returns a negative code, pl_attn_strerror() names it, and
 * the caller reports it and stops.
 *
 * KV cache.  It lives in device HBM, owned by the module, laid out as
 * picolm's host cache (model.c:612-619, 802-805) with a sequence slot in
 * front: [seq][layer][max_seq][n_kv_heads][head_dim] FP16 words.  Rows are
 * written with picolm's own FP32->FP16 rounding (quant.c:41-78, ties away
 * from zero), so the cache is bit-identical to the one model.c would hold.
 *
 * Threading.  One host thread drives the module.  Host-buffer calls are
 * synchronous: caller buffers are read and written before return.
 * Device-pointer calls (suffix _dev) are asynchronous on the given stream.
 *
 * Supported shapes: head_dim 64 or 128 (model.c:856 accepts up to 256);
 * n_kv_heads in {1, 2, 4, 8}; n_heads / n_kv_heads in {1, 2, 4, 8}; LLaMA
 * (pairwise) or Qwen (half-split) RoPE.  Other shapes are rejected with
 * PL_EUNSUPPORTED at pl_attn_init.
 */
#ifndef PL_ATTN_H
#define PL_ATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- Status codes (0 = success, as gpu.h's int returns) ---- */
#define PL_OK             0
#define PL_EFAIL         -1   /* generic failure                              */
#define PL_EARG          -2   /* argument out of range (seq, layer, pos, ...) */
#define PL_ENOMEM        -3   /* device or pinned-host allocation failed      */
#define PL_ECUDA         -4   /* CUDA runtime / driver error                  */
#define PL_ETIMEOUT      -5   /* a bounded device-side wait gave up           */
#define PL_ESTATE        -6   /* not initialised, or initialised twice        */
#define PL_EDEVICE       -7   /* no usable sm_100 device                      */
#define PL_EUNSUPPORTED  -8   /* shape not supported by the kernels           */

#define PL_ROPE_LLAMA 0       /* pairs (2i, 2i+1)   -- tensor.c:558-601 */
#define PL_ROPE_QWEN  1       /* pairs (i, i+hd/2)  -- tensor.c:537-557 */

#define PL_SPLIT_SEQS 0       /* pl_attn_init_devices: slots spread over devices */
#define PL_SPLIT_KV   1       /* pl_attn_init_devices: every slot's rows spread  */

#ifndef PL_ATTN_DISABLED

/* ---- Lifecycle (cf. gpu_init / gpu_available / gpu_shutdown,
 *      picolm/gpu.h:9-29; called where picolm.c:186-193 and 312-314 call them) */

/* Create the module context on CUDA device `device`: allocate the device KV
 * cache for `n_seqs` independent sequences (slot 0 is the one model.c uses),
 * zero it, and build the RoPE tables from rope_freq_base exactly as
 * init_rope_tables does (model.c:545-556).  Replaces the KV calloc of
 * allocate_run_state (model.c:612-619) for the attention path. */
int  pl_attn_init(int n_layers, int n_heads, int n_kv_heads, int head_dim,
                  int max_seq_len, float rope_freq_base, int rope_type,
                  int n_seqs, int device);

/* The same context over n_devices GPUs of this process (1..16; an id may
 * repeat, which runs the split on one GPU).  The host-buffer entry points
 * below, pl_kv_download / pl_kv_upload, pl_attn_set_rope, pl_attn_rope,
 * pl_attn_status, pl_attn_set_wait_limit and the profiling calls fan out to
 * the devices internally, from the one host thread that drives the module;
 * peer access is enabled between every pair.  No counterpart in the
 * reference, whose gpu.c drives one device (picolm/gpu.c:34-83).
 *   PL_SPLIT_SEQS  slots [d*n_seqs/D, (d+1)*n_seqs/D) live on devices[d];
 *                  a batch is split by slot owner and each device runs its
 *                  part with no exchange (independent sequences).
 *   PL_SPLIT_KV    every slot's cache rows are spread over the devices in
 *                  blocks of 512 positions (block b on devices[b % D]).  A
 *                  decode step runs a partial over each device's rows in
 *                  parallel and merges the (max, sum, output) triples on
 *                  devices[0] with a log-sum-exp combine that reads the
 *                  other devices' partials over NVLink; a prefill gathers
 *                  the earlier rows onto devices[0], runs there, and returns
 *                  each new row to its owner.  Memory per device: about
 *                  1/D of the cache.
 * The device-pointer (_dev), KV-exchange (xfer) and projection (block)
 * entry points need a single-device context and return PL_EUNSUPPORTED on
 * a multi-device one.  pl_attn_init is pl_attn_init_devices with one device. */
int  pl_attn_init_devices(int n_layers, int n_heads, int n_kv_heads,
                          int head_dim, int max_seq_len, float rope_freq_base,
                          int rope_type, int n_seqs, int n_devices,
                          const int *devices, int split);

/* Replace the device RoPE tables with host tables [n_rows][half_dim]
 * (model.c's s->rope_cos / s->rope_sin), copied once. */
int  pl_attn_set_rope(const float *cos_tab, const float *sin_tab, int n_rows,
                      int half_dim);

/* 1 if pl_attn_init succeeded and the context is usable (gpu.h:20-21). */
int  pl_attn_available(void);

/* Release every device and host resource (gpu.h:28-29). */
void pl_attn_shutdown(void);

/* Static text for a status code. */
const char *pl_attn_strerror(int rc);

/* ---- Host-buffer entry points (the drop-in for model.c) ---- */

/* Decode step for one sequence: replaces model.c:820-892.
 * q [n_heads*head_dim] and k, v [n_kv_heads*head_dim] are the layer's FP32
 * projections BEFORE RoPE (model.c's s->q, k_tmp, v_tmp); out
 * [n_heads*head_dim] receives the attention output (model.c's s->xb).
 * Rotates q and k by the RoPE of `pos`, appends k and v as FP16 at row pos
 * of (seq, layer), attends rows [0, pos].  q, k, v are not modified. */
int  pl_attn_decode(int seq, int layer, int pos, const float *q,
                    const float *k, const float *v, float *out);

/* n independent decode steps in one launch: sequence slot seqs[i] at
 * position pos[i] with q + i*q_dim, k/v + i*kv_dim, out + i*q_dim.  Slots
 * must be distinct. */
int  pl_attn_decode_batch(int layer, int n, const int *seqs, const int *pos,
                          const float *q, const float *k, const float *v,
                          float *out);

/* Causal prefill of n_tok positions start_pos .. start_pos+n_tok-1 for one
 * sequence: replaces model.c:1039-1089.  q [n_tok][n_heads*head_dim],
 * k, v [n_tok][n_kv_heads*head_dim] before RoPE; output row i is written at
 * out + i*out_stride (model.c's xb_batch, out_stride = n_embd).  Position
 * start_pos+i attends rows [0, start_pos+i], rows below start_pos being
 * whatever the cache already holds (a loaded KV file, picolm.c:214-230). */
int  pl_attn_prefill(int seq, int layer, int start_pos, int n_tok,
                     const float *q, const float *k, const float *v,
                     float *out, int out_stride);

/* Page-lock a caller buffer for the host-buffer calls above: an input or
 * output that lies inside a registered range moves directly between it and
 * the device, without the copy through the module's staging area.  model.c
 * allocates s->q, s->k, s->v and s->xb once (model.c:597-619) and can
 * register them after pl_attn_init.  Ranges must not overlap (PL_EARG); a
 * range is unregistered by its start address, and must be before the memory
 * is freed (pl_attn_shutdown unregisters what is left).  No counterpart in
 * the reference: picolm has no device memory. */
int  pl_attn_host_register(void *ptr, size_t bytes);
int  pl_attn_host_unregister(void *ptr);

/* RoPE alone, in place on host buffers, bit-identical to rope()
 * (tensor.c:533-603): q [n_tok][n_heads*head_dim], k [n_tok][kv_dim]
 * (either may be NULL), position of row i = pos0 + i. */
int  pl_attn_rope(int pos0, int n_tok, float *q, float *k);

/* Copy FP16 cache rows [pos0, pos0+n_pos) of (seq, layer) out of / into
 * device HBM; k and v are [n_pos][kv_dim] FP16 words.  With these,
 * kvcache_save / kvcache_load (model.c:1158-1259) keep the KVCP file format
 * while the cache lives on the device. */
int  pl_kv_download(int seq, int layer, int pos0, int n_pos, uint16_t *k,
                    uint16_t *v);
int  pl_kv_upload(int seq, int layer, int pos0, int n_pos, const uint16_t *k,
                  const uint16_t *v);

/* ---- Device-pointer entry points (asynchronous on `stream`, a
 *      cudaStream_t passed as void*; NULL = the CUDA default stream) ----
 *
 * One stream at a time.  These calls use scratch that belongs to the
 * context (the split-KV partials and segment table, the error word, the
 * prefill's work counters and FP16 q staging), so calls that could overlap
 * on the GPU -- on two streams with no ordering between them -- race on it.
 * Issue them on one stream, or order the streams with events.  The current
 * device must be the context's.  Any of them may grow that scratch with a
 * cudaMalloc on first use (the device-wide synchronisation that implies
 * included); pl_attn_decode_batch_dev_noalloc never does.  A device-side
 * failure (a bounded wait that gave up, a slot or position out of range)
 * is reported by pl_attn_status. */

/* pl_attn_decode_batch with every array already in device memory.
 * max_pos must bound every d_pos[i] (it sizes the KV split).  The decode
 * grid is launched with programmatic dependent launch, so it may start its
 * set-up while the kernel queued before it on `stream` finishes; arrays that
 * kernel writes are still read correctly (after griddepcontrol.wait). */
int  pl_attn_decode_batch_dev(int layer, int n, const int *d_seqs,
                              const int *d_pos, int max_pos, const float *d_q,
                              const float *d_k, const float *d_v, float *d_out,
                              void *stream);

/* pl_attn_prefill with device arrays.  d_q, d_k, d_v and d_out must be
 * 16-byte aligned and out_stride a multiple of 4 (PL_EARG otherwise). */
int  pl_attn_prefill_dev(int seq, int layer, int start_pos, int n_tok,
                         const float *d_q, const float *d_k, const float *d_v,
                         float *d_out, int out_stride, void *stream);

/* One shard of a KV-split decode (a long sequence whose cache rows are
 * spread over several devices).  This device holds global positions
 * [row0, row0 + n_rows) of sequence slot `seq` in its local rows
 * [0, n_rows).  q is rotated by the RoPE of global position `pos`; if
 * `append` is nonzero, k is rotated too and k, v are appended at local row
 * pos - row0 (which must be < n_rows).  Attends local rows [0, n_rows) and
 * writes, per query head h, the partial triple in a block of head_dim+4
 * floats (16-byte aligned):
 *   d_part[h*(head_dim+4) + 0]        m_h: running max, log2 domain
 *   d_part[h*(head_dim+4) + 1]        l_h: sum of 2^(s - m_h)
 *   d_part[h*(head_dim+4) + 4 + d]    o_h[d]: unnormalised sum of p * V
 * with s = (q.k) * log2(e) / sqrt(head_dim).  An empty shard (n_rows = 0)
 * writes m = -inf, l = 0, o = 0.  Merge shards with pl_attn_combine_dev. */
int  pl_attn_decode_partial_dev(int seq, int layer, int pos, int row0,
                                int n_rows, int append, const float *d_q,
                                const float *d_k, const float *d_v,
                                float *d_part, void *stream);

/* Log-sum-exp merge of n_part (1..16) partial blocks laid out back to back
 * (n_part * n_heads*(head_dim+4) floats) into out [n_heads*head_dim]:
 *   M = max_g m_g, L = sum_g l_g 2^(m_g - M),
 *   out = sum_g 2^(m_g - M) o_g / L. */
int  pl_attn_combine_dev(int n_part, const float *d_parts, float *d_out,
                         void *stream);

/* Device address of the FP16 cache rows of (seq, layer): K at *d_k, V at
 * *d_v, each [max_seq][kv_dim].  For engines that share the cache. */
int  pl_attn_kv_ptr(int seq, int layer, uint16_t **d_k, uint16_t **d_v);

/* ---- KV-split merge over NVLink peer memory (one process per GPU).  No
 *      counterpart in the reference, which runs on one CPU; this is the
 *      multi-GPU form of the merge that pl_attn_combine_dev does locally. ---- */

/* Bytes of the handle pl_attn_xfer_setup writes (a CUDA IPC handle). */
int  pl_attn_xfer_handle_bytes(void);

/* Allocate this rank's receive buffer for a split over `world` (1..8)
 * ranks and write its IPC handle to handle_out.  Once per context. */
int  pl_attn_xfer_setup(int world, int rank, void *handle_out);

/* Map every other rank's buffer: `handles` holds world handles back to back,
 * in rank order (exchange them between the processes first). */
int  pl_attn_xfer_connect(const void *handles);

/* Push this rank's partial block d_part (as pl_attn_decode_partial_dev
 * writes it) to every rank over NVLink, wait (bounded) for all ranks'
 * blocks of the same merge, and write the merged attention output to d_out
 * [n_heads*head_dim].  Every rank calls it once per merge, in the same
 * order; the merges are numbered on the device, so a captured CUDA graph
 * of these calls can be replayed. */
int  pl_attn_combine_p2p_dev(const float *d_part, float *d_out, void *stream);

/* pl_attn_decode_partial_dev followed by pl_attn_combine_p2p_dev in one
 * call, without the intermediate partial: each block of the grid that
 * merges this rank's segments stores its merged head straight into every
 * rank's buffer, waits (bounded) for that head from every rank and writes
 * the merged output of the head to d_out [n_heads*head_dim].  Arguments as
 * pl_attn_decode_partial_dev (n_rows = 0: an empty shard, which still takes
 * part in the exchange); calling rules as pl_attn_combine_p2p_dev.  One
 * kernel launch fewer per layer than the two calls. */
int  pl_attn_decode_p2p_dev(int seq, int layer, int pos, int row0, int n_rows,
                            int append, const float *d_q, const float *d_k,
                            const float *d_v, float *d_out, void *stream);

/* pl_attn_decode_batch_dev for callers that cannot allow the library to
 * allocate device memory.  No counterpart in the reference: picolm's
 * attention runs on the CPU and allocates nothing per step.
 * pl_attn_decode_batch_dev may cudaMalloc a larger buffer for its split
 * partials the first time a launch needs one; serving engines that reserve
 * the whole device in their own pool, or latency-critical loops where an
 * allocation's implicit device synchronisation would stall other streams,
 * cannot accept that.  This entry point runs the same kernels with their
 * scratch (split partials and the per-sequence segment table) in one fixed
 * file-scope device array of 4 MiB + 8 KiB, which every GPU that loads the
 * library holds until the process exits; it calls no cudaMalloc, cudaFree
 * or other allocating routine.  Limits: n <= 1024 sequences, and at most
 * 4 MiB / (n_heads * (head_dim + 4) * 4 bytes) partial slots, one per CTA
 * plus one per sequence (32 query heads: 481 slots at head_dim 64, 248 at
 * head_dim 128), so the KV split is capped to fit (fewer, longer CTAs); an
 * n that leaves no slot for a CTA fails with PL_EARG and a message on
 * stderr.  The current device must be the module's (PL_EDEVICE otherwise).
 * The first call on a
 * device looks up the array's device address (cudaGetSymbolAddress); make
 * that first call before any stream capture.  All calls share the one
 * array, so calls that overlap on the GPU (e.g. on two streams at once)
 * race; each call writes every scratch word it later reads, so nothing has
 * to be cleared between calls. */
int  pl_attn_decode_batch_dev_noalloc(int layer, int n, const int *d_seqs,
                                      const int *d_pos, int max_pos,
                                      const float *d_q, const float *d_k,
                                      const float *d_v, float *d_out,
                                      void *stream);

/* ---- The whole attention sub-block, projections included ----
 *
 * The calls above take q, k, v already projected.  These take the residual
 * stream instead and run, per layer, everything model.c does between the
 * two residual adds on the device: RMSNorm (attn_norm), the Q, K, V
 * projections and their biases, QK-norm, RoPE, the FP16 KV append,
 * attention, the output projection, its bias and the residual add.  The
 * weights stay on the device in their GGUF quantisation. */

/* GGUF tensor types the projections take (picolm/quant.h:49-63) */
#define PL_GGUF_F32   0
#define PL_GGUF_F16   1
#define PL_GGUF_Q8_0  8
#define PL_GGUF_Q4_K 12
#define PL_GGUF_Q6_K 14

/* Upload one layer's attention weights, the tensors model.c:779-817 and
 * 894-897 read (layer_weights_t, model.h:39-72): wq [n_heads*head_dim rows]
 * x [dim], wk and wv [n_kv_heads*head_dim] x [dim], wo [dim] x
 * [n_heads*head_dim], each as raw GGUF rows of type type_* (F32, F16, Q8_0,
 * Q4_K or Q6_K; a row length must be a multiple of the type's block,
 * PL_EUNSUPPORTED otherwise).  attn_norm [dim] and rms_eps are the RMSNorm
 * applied to x first (s->attn_norm_w[l], c->rms_norm_eps; NULL: none).
 * Biases bq, bk, bv, bo are F32 (s->attn_q_bias[l] ...; NULL: none).
 * q_norm and k_norm [head_dim] are the QK-norm weights (Qwen3,
 * s->attn_q_norm_w[l]; both NULL or both set).  The data are copied; a
 * second call for the same layer replaces the first. */
int  pl_attn_set_layer(int layer, int dim, const float *attn_norm,
                       float rms_eps, const void *wq, int type_q,
                       const void *wk, int type_k, const void *wv,
                       int type_v, const void *wo, int type_o,
                       const float *bq, const float *bk, const float *bv,
                       const float *bo, const float *q_norm,
                       const float *k_norm);

/* Decode: replaces model.c:779-897 for n sequences, sequence slot seqs[i]
 * at position pos[i] (distinct slots).  x [n][dim] is the residual stream
 * (model.c's s->x), updated in place: x += attention sub-block(x).  The K
 * and V rows appended to the cache are picolm's FP16 encoding of k and v
 * as this module computes them; the projections sum in a different order
 * than the CPU, so they agree with picolm's to FP32 rounding. */
int  pl_attn_block_decode(int layer, int n, const int *seqs, const int *pos,
                          float *x);

/* Prefill: replaces model.c:990-1100 (RMSNorm through the residual add) for
 * n_tok positions start_pos.. of one sequence; x [n_tok][dim] in place. */
int  pl_attn_block_prefill(int seq, int layer, int start_pos, int n_tok,
                           float *x);

/* The same with x in device memory (16-byte aligned), on `stream`. */
int  pl_attn_block_decode_dev(int layer, int n, const int *d_seqs,
                              const int *d_pos, int max_pos, float *d_x,
                              void *stream);
int  pl_attn_block_prefill_dev(int seq, int layer, int start_pos, int n_tok,
                               float *d_x, void *stream);

/* One uploaded projection alone, matmul_bias (tensor.c:230-238) on n input
 * rows: y[i] = W x[i] + b for which = 0 (Wq), 1 (Wk), 2 (Wv), 3 (Wo); x
 * [n][dim] (Wo: [n][n_heads*head_dim]), y [n][rows of W].  No RMSNorm. */
int  pl_attn_proj(int layer, int which, int n, const float *x, float *y);

/* ---- Status and failure detection ---- */

/* Wait for the work queued on `stream` (a cudaStream_t as void*; NULL = the
 * CUDA default stream), then read and clear the module's device error word:
 * PL_ETIMEOUT if a device-side wait gave up since the last check (a TMA
 * tile, a tensor-core commit, or another rank's partial in
 * pl_attn_combine_p2p_dev), PL_EARG if a kernel found a slot or position
 * out of range in a device array, PL_OK otherwise.  The module stays usable after either.  Host-buffer calls
 * check the word themselves; callers of the _dev entry points use this.
 * No counterpart in the reference, whose Vulkan backend waits on a fence
 * with a 5 s timeout (picolm/gpu.c:693-698). */
int  pl_attn_status(void *stream);

/* Bound on every device-side wait, in seconds (1e-4 .. 60; default 2,
 * restored by pl_attn_init).  A healthy wait lasts microseconds; the bound
 * only turns a lost peer or a stalled pipeline into PL_ETIMEOUT instead of
 * a hang.  A multi-GPU engine with its own failure detector may shorten it
 * so that a rank that left is noticed within its heartbeat period. */
int  pl_attn_set_wait_limit(double seconds);

/* ---- Profiling (cf. picolm's timing stats, picolm.c:285-302) ---- */

/* Enable (1) or disable (0) device timing: every later call records CUDA
 * events immediately before and after its attention kernel, on the stream
 * that kernel runs on, and counts the module's kernel launches.  Enabling
 * clears previous records. */
int  pl_attn_profile(int enable);

/* Total device time (ms) of the attention kernels recorded since the last
 * read or enable, the number of those kernels, and the number of all module
 * kernels launched (attention, prologue, combine, RoPE).  Waits for the
 * recorded events; clears the records. */
int  pl_attn_profile_read(double *attn_ms, long *attn_launches,
                          long *all_launches);

#else /* PL_ATTN_DISABLED: inline stubs for every entry point, as gpu.h does
        without USE_VULKAN (picolm/gpu.h:33-42).  pl_attn_init reports
        PL_EDEVICE, so a caller keeps its CPU loops; nothing else is
        reachable without it and reports PL_ESTATE. */
static inline int pl_attn_init(int n_layers, int n_heads, int n_kv_heads,
                               int head_dim, int max_seq_len,
                               float rope_freq_base, int rope_type, int n_seqs,
                               int device) {
    (void)n_layers; (void)n_heads; (void)n_kv_heads; (void)head_dim;
    (void)max_seq_len; (void)rope_freq_base; (void)rope_type; (void)n_seqs;
    (void)device; return PL_EDEVICE;
}
static inline int pl_attn_init_devices(int n_layers, int n_heads,
                                       int n_kv_heads, int head_dim,
                                       int max_seq_len, float rope_freq_base,
                                       int rope_type, int n_seqs,
                                       int n_devices, const int *devices,
                                       int split) {
    (void)n_layers; (void)n_heads; (void)n_kv_heads; (void)head_dim;
    (void)max_seq_len; (void)rope_freq_base; (void)rope_type; (void)n_seqs;
    (void)n_devices; (void)devices; (void)split; return PL_EDEVICE;
}
static inline int pl_attn_set_rope(const float *cos_tab, const float *sin_tab,
                                   int n_rows, int half_dim) {
    (void)cos_tab; (void)sin_tab; (void)n_rows; (void)half_dim;
    return PL_ESTATE;
}
static inline int pl_attn_available(void) { return 0; }
static inline void pl_attn_shutdown(void) {}
static inline const char *pl_attn_strerror(int rc) {
    (void)rc; return "attention backend compiled out (PL_ATTN_DISABLED)";
}
static inline int pl_attn_decode(int seq, int layer, int pos, const float *q,
                                 const float *k, const float *v, float *out) {
    (void)seq; (void)layer; (void)pos; (void)q; (void)k; (void)v; (void)out;
    return PL_ESTATE;
}
static inline int pl_attn_decode_batch(int layer, int n, const int *seqs,
                                       const int *pos, const float *q,
                                       const float *k, const float *v,
                                       float *out) {
    (void)layer; (void)n; (void)seqs; (void)pos; (void)q; (void)k; (void)v;
    (void)out; return PL_ESTATE;
}
static inline int pl_attn_prefill(int seq, int layer, int start_pos, int n_tok,
                                  const float *q, const float *k,
                                  const float *v, float *out, int out_stride) {
    (void)seq; (void)layer; (void)start_pos; (void)n_tok; (void)q; (void)k;
    (void)v; (void)out; (void)out_stride; return PL_ESTATE;
}
static inline int pl_attn_host_register(void *ptr, size_t bytes) {
    (void)ptr; (void)bytes; return PL_ESTATE;
}
static inline int pl_attn_host_unregister(void *ptr) {
    (void)ptr; return PL_ESTATE;
}
static inline int pl_attn_rope(int pos0, int n_tok, float *q, float *k) {
    (void)pos0; (void)n_tok; (void)q; (void)k; return PL_ESTATE;
}
static inline int pl_kv_download(int seq, int layer, int pos0, int n_pos,
                                 uint16_t *k, uint16_t *v) {
    (void)seq; (void)layer; (void)pos0; (void)n_pos; (void)k; (void)v;
    return PL_ESTATE;
}
static inline int pl_kv_upload(int seq, int layer, int pos0, int n_pos,
                               const uint16_t *k, const uint16_t *v) {
    (void)seq; (void)layer; (void)pos0; (void)n_pos; (void)k; (void)v;
    return PL_ESTATE;
}
static inline int pl_attn_decode_batch_dev(int layer, int n, const int *d_seqs,
                                           const int *d_pos, int max_pos,
                                           const float *d_q, const float *d_k,
                                           const float *d_v, float *d_out,
                                           void *stream) {
    (void)layer; (void)n; (void)d_seqs; (void)d_pos; (void)max_pos; (void)d_q;
    (void)d_k; (void)d_v; (void)d_out; (void)stream; return PL_ESTATE;
}
static inline int pl_attn_prefill_dev(int seq, int layer, int start_pos,
                                      int n_tok, const float *d_q,
                                      const float *d_k, const float *d_v,
                                      float *d_out, int out_stride,
                                      void *stream) {
    (void)seq; (void)layer; (void)start_pos; (void)n_tok; (void)d_q; (void)d_k;
    (void)d_v; (void)d_out; (void)out_stride; (void)stream; return PL_ESTATE;
}
static inline int pl_attn_decode_partial_dev(int seq, int layer, int pos,
                                             int row0, int n_rows, int append,
                                             const float *d_q,
                                             const float *d_k,
                                             const float *d_v, float *d_part,
                                             void *stream) {
    (void)seq; (void)layer; (void)pos; (void)row0; (void)n_rows; (void)append;
    (void)d_q; (void)d_k; (void)d_v; (void)d_part; (void)stream;
    return PL_ESTATE;
}
static inline int pl_attn_combine_dev(int n_part, const float *d_parts,
                                      float *d_out, void *stream) {
    (void)n_part; (void)d_parts; (void)d_out; (void)stream; return PL_ESTATE;
}
static inline int pl_attn_kv_ptr(int seq, int layer, uint16_t **d_k,
                                 uint16_t **d_v) {
    (void)seq; (void)layer; (void)d_k; (void)d_v; return PL_ESTATE;
}
static inline int pl_attn_xfer_handle_bytes(void) { return 0; }
static inline int pl_attn_xfer_setup(int world, int rank, void *handle_out) {
    (void)world; (void)rank; (void)handle_out; return PL_ESTATE;
}
static inline int pl_attn_xfer_connect(const void *handles) {
    (void)handles; return PL_ESTATE;
}
static inline int pl_attn_combine_p2p_dev(const float *d_part, float *d_out,
                                          void *stream) {
    (void)d_part; (void)d_out; (void)stream; return PL_ESTATE;
}
static inline int pl_attn_decode_p2p_dev(int seq, int layer, int pos, int row0,
                                         int n_rows, int append,
                                         const float *d_q, const float *d_k,
                                         const float *d_v, float *d_out,
                                         void *stream) {
    (void)seq; (void)layer; (void)pos; (void)row0; (void)n_rows; (void)append;
    (void)d_q; (void)d_k; (void)d_v; (void)d_out; (void)stream;
    return PL_ESTATE;
}
static inline int pl_attn_decode_batch_dev_noalloc(int layer, int n,
                                                   const int *d_seqs,
                                                   const int *d_pos,
                                                   int max_pos,
                                                   const float *d_q,
                                                   const float *d_k,
                                                   const float *d_v,
                                                   float *d_out, void *stream) {
    (void)layer; (void)n; (void)d_seqs; (void)d_pos; (void)max_pos; (void)d_q;
    (void)d_k; (void)d_v; (void)d_out; (void)stream; return PL_ESTATE;
}
static inline int pl_attn_set_layer(int layer, int dim, const float *attn_norm,
                                    float rms_eps, const void *wq, int type_q,
                                    const void *wk, int type_k, const void *wv,
                                    int type_v, const void *wo, int type_o,
                                    const float *bq, const float *bk,
                                    const float *bv, const float *bo,
                                    const float *q_norm, const float *k_norm) {
    (void)layer; (void)dim; (void)attn_norm; (void)rms_eps; (void)wq;
    (void)type_q; (void)wk; (void)type_k; (void)wv; (void)type_v; (void)wo;
    (void)type_o; (void)bq; (void)bk; (void)bv; (void)bo; (void)q_norm;
    (void)k_norm; return PL_ESTATE;
}
static inline int pl_attn_block_decode(int layer, int n, const int *seqs,
                                       const int *pos, float *x) {
    (void)layer; (void)n; (void)seqs; (void)pos; (void)x; return PL_ESTATE;
}
static inline int pl_attn_block_prefill(int seq, int layer, int start_pos,
                                        int n_tok, float *x) {
    (void)seq; (void)layer; (void)start_pos; (void)n_tok; (void)x;
    return PL_ESTATE;
}
static inline int pl_attn_block_decode_dev(int layer, int n, const int *d_seqs,
                                           const int *d_pos, int max_pos,
                                           float *d_x, void *stream) {
    (void)layer; (void)n; (void)d_seqs; (void)d_pos; (void)max_pos; (void)d_x;
    (void)stream; return PL_ESTATE;
}
static inline int pl_attn_block_prefill_dev(int seq, int layer, int start_pos,
                                            int n_tok, float *d_x, void *stream)
{
    (void)seq; (void)layer; (void)start_pos; (void)n_tok; (void)d_x;
    (void)stream; return PL_ESTATE;
}
static inline int pl_attn_proj(int layer, int which, int n, const float *x,
                               float *y) {
    (void)layer; (void)which; (void)n; (void)x; (void)y; return PL_ESTATE;
}
static inline int pl_attn_status(void *stream) {
    (void)stream; return PL_ESTATE;
}
static inline int pl_attn_set_wait_limit(double seconds) {
    (void)seconds; return PL_ESTATE;
}
static inline int pl_attn_profile(int enable) {
    (void)enable; return PL_ESTATE;
}
static inline int pl_attn_profile_read(double *attn_ms, long *attn_launches,
                                       long *all_launches) {
    (void)attn_ms; (void)attn_launches; (void)all_launches; return PL_ESTATE;
}

#endif /* PL_ATTN_DISABLED */

#ifdef __cplusplus
}
#endif
#endif /* PL_ATTN_H */
