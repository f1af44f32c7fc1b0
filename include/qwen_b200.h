/*
 * libqwenb200 -- B200 (sm_100a) implementation of the speculative-decode hot
 * path of the hybrid Qwen C engine (Julien-Bui/Qwen3.8-27B-in-C).
 *
 * Drop-in boundary.  The entry points below keep the names, argument meaning
 * and return conventions of the reference headers, so a caller written
 * against include/model.h and include/kernels.h recompiles against this
 * header (through include/shim) with no source edit; src/main.c does:
 *
 *   model_init / model_free            include/model.h:117-118
 *   attention_layer / gdn_layer        include/model.h:121-122
 *   model_forward                      include/model.h:125
 *   model_forward_batch                include/model.h:130-131
 *   model_rollback_to                  include/model.h:136
 *   mtp_forward / mtp_forward_batch    include/model.h:139-145
 *   model_sample_greedy                include/model.h:148
 *   gemv_rows / gemv / gemv_rows_batch / gemv_batch
 *                                      include/kernels.h:11-26
 *   gemv_multi / gemv_multi_batch      include/kernels.h:28-34
 *   rmsnorm / l2norm / silu_inplace / sigmoid_inplace / softplus_inplace /
 *   softmax_inplace                    include/kernels.h:36-44
 *   pool_create / pool_destroy / pool_run   include/threadpool.h:9-15
 *   sampler_init / sampler_free / sampler_sample   include/sampler.h:16-19
 *
 * All pointers in these calls are HOST pointers, as in the reference; the
 * library owns the CUDA device memory (weights, KV caches, recurrent states
 * and their rollback slots) and mirrors the fields a caller reads or writes
 * (logits, logits_b, h_save, mtp_h, x, pos) in host memory.  The pool
 * argument is accepted and ignored: all work runs on one CUDA stream per
 * model.  Functions that return void in the reference record failures in
 * qb_last_error(); nothing falls back to a CPU computation.
 *
 * The qb_* entry points at the end run whole loops on the device (prefill,
 * greedy decode, greedy MTP speculation with on-device argmax, acceptance
 * and rollback) with no host round trip per token.
 */
#ifndef QWEN_B200_H
#define QWEN_B200_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- types shared with the reference headers (same layout) ----
 * When the reference gguf.h was included first (a relinked reference caller),
 * its identical definitions are used instead. */
#ifndef GGUF_H

/* include/gguf.h:40-64 */
typedef enum {
    GGML_F32 = 0, GGML_F16 = 1, GGML_Q4_0 = 2, GGML_Q4_1 = 3, GGML_Q5_0 = 6, GGML_Q5_1 = 7,
    GGML_Q8_0 = 8, GGML_Q2_K = 10, GGML_Q3_K = 11, GGML_Q4_K = 12, GGML_Q5_K = 13, GGML_Q6_K = 14,
    GGML_Q8_K = 15, GGML_IQ2_XXS = 16, GGML_IQ2_XS = 17, GGML_IQ3_XXS = 18, GGML_IQ1_S = 19,
    GGML_IQ4_NL = 20, GGML_IQ3_S = 21, GGML_IQ2_S = 22, GGML_IQ4_XS = 23, GGML_IQ1_M = 24,
    GGML_BF16 = 25
} ggml_type_t;

/* include/gguf.h:66-73 */
typedef struct {
    char name[64];
    uint32_t n_dims;
    uint64_t ne[4];        /* ne[0] = innermost (input) dimension */
    ggml_type_t type;
    uint64_t offset;
    const void *data;      /* host pointer to the GGUF row-major blocks */
} gguf_tensor_info_t;

/* include/gguf.h:75-97 */
typedef struct {
    uint32_t n_embd, n_head, n_head_kv, head_dim, n_layer, n_ff, vocab_size, context_len;
    float rope_theta;
    uint32_t rope_dim_count;
    uint32_t rope_sections[4];
    float rms_norm_eps;
    bool tie_word_embeddings;
    uint32_t full_attn_interval, ssm_state_size, ssm_conv_kernel, ssm_inner_size, ssm_group_count;
    uint32_t nextn_layers;
} qwen_config_t;

#endif /* GGUF_H */

/* include/model.h:10-31 */
typedef struct {
    uint32_t n_embd, n_ff, n_layer, n_attn_layer, n_recr_layer;
    uint32_t n_head, n_kv_head, head_dim;
    uint32_t rope_sections[4];
    uint32_t n_v_heads, n_k_heads, head_k_dim, head_v_dim, d_inner, conv_dim, d_conv, d_state;
} qwen_dims_t;

/* The model handle.  The named fields mean what they mean in the reference
 * qwen_model_t (include/model.h:60-111); they are host mirrors of device
 * state, refreshed by the calls that produce them:
 *   logits    [vocab]            model_forward, mtp_forward(want_logits=1)
 *   logits_b  [PREFILL_MAX_B][vocab]  model_forward_batch, mtp_forward_batch(want)
 *   h_save    [PREFILL_MAX_B][n_embd] model_forward_batch (pre-norm hidden)
 *   x         [n_embd]           model_forward (pre-norm hidden of the token)
 *   mtp_h     [n_embd]           read by mtp_forward (caller may write it,
 *                                src/main.c:220), written back after it
 *   pos                          next position, as in the reference */
/* One backbone layer as the layer functions below take it (include/model.h:33-57
 * names the reference's fields; its weights live on the device here, so a
 * caller only reads which layer it is and whether it is recurrent). */
typedef struct qwen_layer {
    uint32_t index;
    bool is_recurrent;
} qwen_layer_t;

typedef struct qwen_model {
    qwen_config_t cfg;
    qwen_dims_t dims;
    float *mtp_h;
    float *x;
    float *logits;
    float *logits_b;
    float *h_save;
    uint32_t n_ctx;
    uint32_t pos;
    qwen_layer_t *layers;  /* [dims.n_layer], as m->layers in the reference */
    void *eng;             /* device engine (opaque) */
#ifdef GGUF_H
    /* Only when the reference gguf.h was included first (a relinked reference
     * caller): the file's parsed GGUF context, opened on the host by the
     * model_init wrapper below, for callers that read metadata from it
     * (src/main.c:93 hands it to tokenizer_init).  The library never reads it;
     * as the last member it leaves the offsets of every field the library
     * touches unchanged. */
    gguf_context_t gguf;
#endif
} qwen_model_t;

typedef struct pool pool_t;
typedef void (*pool_fn_t)(void *arg, int tid, int ntotal);

#define SPEC_MAX_B 4       /* verify width: k = 3 drafts (the reference ships 3) */
#define PREFILL_MAX_B 8
#define GEMV_MAX_B 8

/* ---- include/threadpool.h:9-15 (kept for source compatibility) ---- */
pool_t *pool_create(int n_threads, int pin);
void pool_destroy(pool_t *p);
void pool_run(pool_t *p, pool_fn_t fn, void *arg);

/* ---- include/model.h:117-148 ---- */
int model_init(qwen_model_t *m, const char *path, uint32_t n_ctx);
void model_free(qwen_model_t *m);
/* include/model.h:121-122: one layer of one token on the hidden state m->x
 * (host mirror, read and written): the gated-attention block at position pos,
 * or the Gated DeltaNet block on the current recurrent state, each with its
 * SwiGLU FFN and both residuals (src/model.c:418-485, 617-695).  Runs on the
 * device; L is &m->layers[il]. */
void attention_layer(qwen_model_t *m, qwen_layer_t *L, pool_t *pool, uint32_t pos);
void gdn_layer(qwen_model_t *m, qwen_layer_t *L, pool_t *pool);
void model_forward(qwen_model_t *m, pool_t *pool, uint32_t token, uint32_t pos);
void model_forward_batch(qwen_model_t *m, pool_t *pool, const uint32_t *tokens, uint32_t pos,
                         uint32_t B, int ckpt);
int model_snapshot_states(qwen_model_t *m);
void model_rollback_states(qwen_model_t *m);
void model_rollback_to(qwen_model_t *m, uint32_t b);
int mtp_forward(qwen_model_t *m, pool_t *pool, uint32_t token, uint32_t pos, int want_logits);
int mtp_forward_batch(qwen_model_t *m, pool_t *pool, const uint32_t *tokens, uint32_t pos,
                      uint32_t B, int want_logits);
uint32_t model_sample_greedy(const float *logits, uint32_t vocab_size);

#ifdef GGUF_H
/* A reference caller that reaches into m->gguf (include/model.h:60-61) gets it
 * through these wrappers: model_init also opens the GGUF on the host with the
 * reference's own gguf_open (include/gguf.h:109), model_free closes it first.
 * The device engine does not use that context; it parses the file itself. */
static inline int qb_model_init_with_gguf(qwen_model_t *m, const char *path, uint32_t n_ctx) {
    if (model_init(m, path, n_ctx) != 0) return -1;
    if (gguf_open(&m->gguf, path) != 0) {
        model_free(m);
        return -1;
    }
    return 0;
}
static inline void qb_model_free_with_gguf(qwen_model_t *m) {
    if (m->eng) gguf_close(&m->gguf);
    model_free(m);
}
#define model_init qb_model_init_with_gguf
#define model_free qb_model_free_with_gguf
#endif

/* ---- include/kernels.h:11-44 (host pointers; weights uploaded on first use
 *      and cached on the current device, keyed by W->data) ---- */
void gemv_rows(const gguf_tensor_info_t *W, const float *x, float *out, uint64_t r0, uint64_t r1);
void gemv(pool_t *pool, const gguf_tensor_info_t *W, const float *x, float *out);
void gemv_rows_batch(const gguf_tensor_info_t *W, const float *x, uint64_t ldx, int n, float *out,
                     uint64_t ldo, uint64_t r0, uint64_t r1);
void gemv_batch(pool_t *pool, const gguf_tensor_info_t *W, const float *x, uint64_t ldx, int n,
                float *out, uint64_t ldo);
void gemv_multi(pool_t *pool, const gguf_tensor_info_t *const *Ws, const float *x, float *const *outs,
                int n_mat);
void gemv_multi_batch(pool_t *pool, const gguf_tensor_info_t *const *Ws, const float *x, uint64_t ldx,
                      int n, float *const *outs, const uint64_t *ldos, int n_mat);
void rmsnorm(float *out, const float *x, const float *weight, uint64_t n, float eps);
void l2norm(float *out, const float *x, uint64_t n, float eps);
void silu_inplace(float *x, uint64_t n);
void sigmoid_inplace(float *x, uint64_t n);
void softplus_inplace(float *x, uint64_t n);
void softmax_inplace(float *x, uint64_t n);

/* ---- include/sampler.h (non-greedy sampling, src/sampler.c:49-162) ----
 * Same struct, names and behaviour; the draw runs on the GPU.  sampler_sample
 * takes HOST logits as the reference does, penalises them in place (the same
 * float operations, copied back) and advances s->rng_state.  A seeded stream
 * gives the reference's tokens: each term's exp is the correctly rounded one
 * (the reference uses glibc's expf, one ulp away on about 0.06 % of inputs),
 * and exact ties inside the top-k list are taken in index order. */
#ifndef SAMPLER_H
typedef struct {
    float temp;
    float top_p;
    uint32_t top_k;
    float repeat_penalty;
    uint32_t repeat_last_n;
    uint64_t rng_state;
} sampler_t;
#endif
sampler_t *sampler_init(float temp, float top_p, uint32_t top_k, float repeat_penalty, uint64_t seed);
void sampler_free(sampler_t *s);
uint32_t sampler_sample(sampler_t *s, float *logits, uint32_t vocab_size, const uint32_t *tokens, size_t n_tokens);

/* include/model.h:151-152: per-section timers of the CPU engine's
 * model_forward.  Exported so reference callers (src/main.c:256-263) link; the
 * device engine leaves them at zero and qwen_prof_calls at 0, so the CLI skips
 * its profile line.  Device timings come from qb_last_loop_ms / qb_bench. */
extern double qwen_prof_embed, qwen_prof_gdn, qwen_prof_attn, qwen_prof_head;
extern uint64_t qwen_prof_calls;

/* ---- device-resident loops (no counterpart function in the reference: they
 *      run the loops of src/main.c on the device) ---- */

/* Last error of this thread: 0 = none.  qb_last_error_str() describes it. */
int qb_last_error(void);
const char *qb_last_error_str(void);
void qb_clear_error(void);

/* src/main.c:132-152: batched prefill, plus the MTP cache fill when spec != 0;
 * afterwards m->logits holds the logits of the last prompt token.  The prompt
 * is copied to the device once and the chunks run back to back (one graph
 * replay per full chunk, no host wait in between): chunks of 32 tokens while
 * more than 32 remain (one GPU), then of PREFILL_MAX_B, the last one with the
 * output head; qb_last_loop_ms then gives their device time.  Each token's
 * arithmetic does not depend on the chunk it is in.  Returns 0 or -1. */
int qb_prefill(qwen_model_t *m, const uint32_t *tokens, uint32_t n, int spec);

/* src/main.c:158-225: greedy MTP speculation with n_spec drafts.  Drafts,
 * verify, argmax, acceptance, rollback and the MTP anchor all run on the
 * device; the host only waits between batches of cycles.  When n_forced > 0
 * the accept length of cycle c is forced[c % n_forced] (clamped to n_spec)
 * instead of the first-mismatch rule.  Writes up to n_predict tokens to
 * out_tokens and the accept length of each cycle to out_j (may be NULL,
 * else room for max_cycles entries).  Returns the number of tokens, or -1. */
int qb_spec_generate(qwen_model_t *m, uint32_t n_predict, uint32_t n_spec, const uint32_t *forced,
                     uint32_t n_forced, uint32_t *out_tokens, uint32_t *out_j, uint32_t max_cycles,
                     uint32_t *n_cycles);

/* src/main.c:232-248 at temperature 0: token 0 = argmax(m->logits), then
 * n_predict-1 single-token forwards, each fed its own device argmax.
 * Returns the number of tokens, or -1. */
int qb_greedy_generate(qwen_model_t *m, uint32_t n_predict, uint32_t *out_tokens);

/* src/main.c:232-248 with a sampler (temperature / top-k / top-p / repetition
 * penalty): token 0 is drawn from m->logits, then n_predict-1 forwards, each
 * followed by a draw on the device, with no host round trip per token.
 * tokens[0..n_tokens) is the history the repetition penalty sees (the prompt
 * and earlier output); s->rng_state advances as sampler_sample's would, and
 * m->logits holds the last forward's logits as the last draw left them.
 * Returns the number of tokens, or -1. */
int qb_sample_generate(qwen_model_t *m, sampler_t *s, uint32_t n_predict, const uint32_t *tokens,
                       size_t n_tokens, uint32_t *out_tokens);

/* Device argmax of the last model_forward_batch row b (no host scan). */
uint32_t qb_last_argmax(qwen_model_t *m, uint32_t b);

/* Timing helper for benchmarks: CUDA-event time of the last qb_* loop
 * (qb_prefill, qb_spec_generate, qb_greedy_generate, qb_sample_generate), ms. */
float qb_last_loop_ms(qwen_model_t *m);

/* Copy the recurrent state of backbone layer il (0 conv, 1 ssm) or the KV
 * cache (2 k, 3 v; il == n_layer selects the MTP block) to host memory, for
 * state comparisons against the reference.  Returns the float count. */
int64_t qb_read_state(qwen_model_t *m, uint32_t il, int which, float *dst, int64_t max_floats);

/* Start a new sequence on the same weights: recurrent states and mtp_h to
 * zero, rollback slot 0, pos = 0.  Returns 0 or -1. */
int qb_reset(qwen_model_t *m);

/* Multi-sequence speculative decode (no counterpart in the reference, which
 * decodes one sequence per process).  qb_seq_init gives the model n_seq
 * (1..8) sequences on the same weights, each with its own recurrent slots, KV
 * caches (n_ctx positions), control block and MTP hidden row, all zero.
 * qb_seq_prefill runs qb_prefill(spec = 1) on sequence `seq`.  qb_seq_generate
 * then runs n_cycles cycles of src/main.c:158-225 on all sequences at once:
 * the MTP drafts at n_seq rows, the verify at n_seq * (n_spec + 1) rows (at
 * most 32), acceptance and rollback per sequence, one CUDA graph per cycle;
 * forced accept lengths (as in qb_spec_generate) apply to every sequence.
 * Sequence s's tokens go to out_tokens[s * cap ..] (out_counts[s] of them,
 * at most cap), its accept lengths to out_j[s * n_cycles ..] (may be NULL).
 * Each sequence emits the tokens it would emit alone.  One GPU, default GEMV
 * paths (no QB_TC / QB_FUSE).  After qb_seq_init the single-sequence calls act
 * on the sequence last named by qb_seq_prefill (0 at first).  Return 0 / -1,
 * or (qb_seq_generate) the cycles run, which is fewer than n_cycles only when
 * a sequence would pass n_ctx. */
int qb_seq_init(qwen_model_t *m, uint32_t n_seq);
/* Keep a tcgen05 tile copy of every IQ4_XS matrix (13 GB more for the 64-layer
 * model), so that GEMV inputs of more than 8 rows run IQ4_XS 32 rows per weight
 * sweep: qb_prefill's 32-token chunks and the multi-sequence verify
 * (qb_seq_init does this itself from 3 sequences on).  One GPU.  0 / -1. */
int qb_enable_wide(qwen_model_t *m);
int qb_seq_prefill(qwen_model_t *m, uint32_t seq, const uint32_t *tokens, uint32_t n);
int qb_seq_generate(qwen_model_t *m, uint32_t n_cycles, uint32_t n_spec, const uint32_t *forced,
                    uint32_t n_forced, uint32_t *out_tokens, uint32_t cap, uint32_t *out_counts,
                    uint32_t *out_j);

/* Device time (ms, CUDA events on the model's stream, mean of `iters`) of one
 * component: what = 0 verify forward of `arg` tokens with checkpoints, 1 the
 * fused FFN gate+up GEMV at N = arg rotated over all layers, 2 one MTP draft
 * with logits, 3 the output-head GEMV at N = arg, 5 / 6 / 7 the down, out- and
 * in-projection GEMVs at N = arg, 8 one FFN up matrix alone at N = arg, 10 the
 * same on the wide tcgen05 GEMM at N = arg <= 32 (every one of these rotated
 * over all layers); what = 4 returns instead
 * the number of kernels one speculative cycle launches (after a
 * qb_spec_generate call).  *bytes receives the algorithmic bytes of one
 * run.  Overwrites KV / recurrent state.  -1 on error. */
float qb_bench(qwen_model_t *m, int what, uint32_t arg, uint32_t iters, double *bytes);

/* Copy internal activation buffer `id` ([PREFILL_MAX_B][width] rows of the
 * last forward: 0 residual, 1 raw mixer projection, 2 conv output, 3 z,
 * 4 beta, 5 alpha, 6 GDN output, 7 gated-norm output, 8 q, 9 k|v, 10
 * attention output, 11 ffn gate, 12 ffn up, 13 SwiGLU, 14 MTP embedding, 15
 * MTP residual, 16 h_save) to host.  Returns the float count, -1 on error. */
int64_t qb_read_buffer(qwen_model_t *m, int id, float *dst, int64_t max_floats);

/* ---- tensor parallelism (no counterpart function in the reference; it
 *      splits the rows of every GEMV as src/kernels.c:608-613 splits them
 *      over CPU threads, here over GPUs) ----
 *
 * One process per GPU.  Every rank loads the same GGUF with
 * qb_model_init_tp(m, path, n_ctx, rank, world) (world <= 8; model_init is
 * world = 1) and keeps its share of the heads: its DeltaNet k-heads with their
 * v-heads, its attention q-heads with their kv-heads, its FFN columns (whole
 * 256-column blocks) and its rows of the output head.  The mixers and the
 * SwiGLU run on local data; the out-projections and the down projection write
 * partial sums that every rank adds in rank order (NVLink loads of the peers'
 * tagged words), so all ranks hold identical activations, logits and tokens.
 * Waits on other ranks give up after 2 s (the call then returns its error).
 *
 * Set-up: qb_tp_handle() writes this rank's 64-byte IPC handle of its
 * activation arena; the caller exchanges the handles of all ranks (any host
 * channel) and passes them, rank-ordered `stride` bytes apart, to
 * qb_tp_connect().  Then every rank calls the same sequence of model API
 * functions with the same arguments.  Before model_free, synchronise the
 * ranks on the host so that no rank still writes into a freed peer.
 * Returns: init / connect 0 or -1; handle the byte count or -1. */
int qb_model_init_tp(qwen_model_t *m, const char *gguf_path, uint32_t n_ctx, int rank, int world);
int64_t qb_tp_handle(qwen_model_t *m, void *out, int64_t cap);
int qb_tp_connect(qwen_model_t *m, const void *handles, int64_t stride);
/* The row range [*r0, *r1) of a rows-row matrix held by rank of world:
 * whole 32-row tile pairs, split as evenly as possible. */
void qb_tp_rows(int rows, int rank, int world, int *r0, int *r1);

/* ---- allocation-free entry point (no counterpart in the reference) ----
 *
 * For callers that cannot allocate device memory at call time: a runtime that
 * owns all GPU memory through its own arena, or code on a latency-critical
 * path where cudaMalloc would synchronise the device or fail under memory
 * pressure.  Greedy argmax of `rows` fp32 logit rows that are already on the
 * device (row r at logits + r * ld, n < 2^31 entries); the index of row r
 * is the one model_sample_greedy (src/model.c:746-756) returns for that row,
 * NaN and signed zeros included: the first maximum wins, -0 equals +0, a NaN
 * is never the maximum unless it is entry 0 (then entry 0 is returned, as the
 * reference's scan does).  The index of row r goes to the
 * device array out[r].  Work is enqueued on `stream` (a cudaStream_t; NULL is
 * the legacy default stream) and the call returns without waiting.
 *
 * The scratch is a fixed static device array of QB_ARGMAX_NOALLOC_MAX_ROWS
 * 64-bit keys (256 bytes); rows above that limit are rejected with an error.
 * The function allocates nothing.  The first call on each device does a
 * one-time set-up (a symbol-address lookup that may load the module): make
 * it with that device current and before any stream capture.  The address
 * found then is kept for the life of the process: after cudaDeviceReset (or
 * any teardown of the device's primary context) the module may load at
 * another address, so do not call this function on that device again.  All calls on a
 * device share the one array, so calls that overlap on the GPU (e.g. on two
 * streams without ordering between them) race.  Returns 0, or -1 with
 * qb_last_error() set. */
#define QB_ARGMAX_NOALLOC_MAX_ROWS 32
int qb_argmax_rows_noalloc(const float *logits, int64_t ld, uint32_t n, uint32_t rows, uint32_t *out,
                           void *stream);

#ifdef __cplusplus
}
#endif
#endif /* QWEN_B200_H */
