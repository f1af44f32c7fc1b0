/*
 * Oracle harness around the compiled reference engine.
 *
 * TEST INFRASTRUCTURE ONLY: this file is linked with the unmodified reference
 * sources (src/gguf.c, quant.c, kernels.c, threadpool.c, model.c) into
 * oracle/_ref/libqwenref.so by oracle/Makefile.  Only tests/, the smoke check
 * and bench.py's CPU-baseline leg load that library, as the checker.
 *
 * The reference has no library entry point for its generation loops (they
 * live in main()); the drivers below restate them with token ids instead of
 * the tokenizer:
 *   ref_prefill          <- src/main.c:132-152 (batched prefill, chunks of
 *                           PREFILL_MAX_B, + mtp_forward_batch when spec on)
 *   ref_spec_generate    <- src/main.c:158-225 (greedy MTP speculation), plus
 *                           an optional forced accept length per cycle
 *   ref_sample_generate  <- src/main.c:232-248 with a sampler (sampler_sample
 *                           after each model_forward; EOS omitted)
 *   ref_greedy_generate  <- src/main.c:232-248 with temperature 0 (the
 *                           sampler's greedy branch is an argmax, identical to
 *                           model_sample_greedy, src/model.c:746-756)
 * EOS handling (src/main.c:179) is omitted: synthetic runs have no tokenizer.
 */
#define _POSIX_C_SOURCE 200809L
#include "model.h"
#include "kernels.h"
#include "sampler.h"
#include "quant.h"
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>
#include <unistd.h>

typedef struct {
    qwen_model_t m;
    pool_t *pool;
} ref_t;

ref_t *ref_open(const char *path, uint32_t n_ctx, int n_threads) {
    ref_t *r = calloc(1, sizeof *r);
    if (!r) return NULL;
    if (model_init(&r->m, path, n_ctx) != 0) { free(r); return NULL; }
    if (n_threads <= 0) n_threads = (int)sysconf(_SC_NPROCESSORS_ONLN);
    r->pool = pool_create(n_threads, 0);
    if (!r->pool) { model_free(&r->m); free(r); return NULL; }
    return r;
}

void ref_close(ref_t *r) {
    if (!r) return;
    pool_destroy(r->pool);
    model_free(&r->m);
    free(r);
}

int ref_spec_max_b(void) { return SPEC_MAX_B; }
qwen_model_t *ref_model(ref_t *r) { return &r->m; }
float *ref_logits(ref_t *r) { return r->m.logits; }
float *ref_logits_b(ref_t *r) { return r->m.logits_b; }
float *ref_h_save(ref_t *r) { return r->m.h_save; }
float *ref_mtp_h(ref_t *r) { return r->m.mtp_h; }
float *ref_x(ref_t *r) { return r->m.x; }
float *ref_bx(ref_t *r) { return r->m.bx; }
uint32_t ref_get_pos(ref_t *r) { return r->m.pos; }
void ref_set_pos(ref_t *r, uint32_t p) { r->m.pos = p; }
uint32_t ref_vocab(ref_t *r) { return r->m.cfg.vocab_size; }
uint32_t ref_n_embd(ref_t *r) { return r->m.dims.n_embd; }
uint32_t ref_n_layer(ref_t *r) { return r->m.dims.n_layer; }
int ref_is_recurrent(ref_t *r, uint32_t il) { return r->m.layers[il].is_recurrent ? 1 : 0; }

/* which: 0 conv_state, 1 ssm_state, 2 kv_k, 3 kv_v ; il == n_layer -> MTP layer */
float *ref_layer_state(ref_t *r, uint32_t il, int which) {
    qwen_layer_t *L = il == r->m.dims.n_layer ? &r->m.mtp_layer : &r->m.layers[il];
    switch (which) {
    case 0: return L->conv_state;
    case 1: return L->ssm_state;
    case 2: return L->kv_k;
    case 3: return L->kv_v;
    default: return NULL;
    }
}

const gguf_tensor_info_t *ref_find_tensor(ref_t *r, const char *name) {
    return gguf_find_tensor(&r->m.gguf, name);
}

void ref_forward(ref_t *r, uint32_t tok, uint32_t pos) { model_forward(&r->m, r->pool, tok, pos); }
void ref_forward_batch(ref_t *r, const uint32_t *toks, uint32_t pos, uint32_t B, int ckpt) {
    model_forward_batch(&r->m, r->pool, toks, pos, B, ckpt);
}
void ref_rollback_to(ref_t *r, uint32_t b) { model_rollback_to(&r->m, b); }
/* one layer on m->x: attention_layer / gdn_layer (include/model.h:121-122) */
void ref_layer(ref_t *r, uint32_t il, uint32_t pos) {
    qwen_layer_t *L = &r->m.layers[il];
    if (L->is_recurrent) gdn_layer(&r->m, L, r->pool);
    else attention_layer(&r->m, L, r->pool, pos);
}
void ref_mtp_forward(ref_t *r, uint32_t tok, uint32_t pos, int want_logits) {
    mtp_forward(&r->m, r->pool, tok, pos, want_logits);
}
void ref_mtp_forward_batch(ref_t *r, const uint32_t *toks, uint32_t pos, uint32_t B, int want) {
    mtp_forward_batch(&r->m, r->pool, toks, pos, B, want);
}
uint32_t ref_argmax(const float *x, uint32_t n) { return model_sample_greedy(x, n); }

int ref_prefill(ref_t *r, const uint32_t *toks, uint32_t n, int spec) {
    qwen_model_t *m = &r->m;
    uint32_t pos = 0, lastB = 0;
    while (pos < n) {
        uint32_t B = n - pos;
        if (B > PREFILL_MAX_B) B = PREFILL_MAX_B;
        model_forward_batch(m, r->pool, toks + pos, pos, B, 0);
        if (spec) mtp_forward_batch(m, r->pool, toks + pos, pos, B, 0);
        pos += B;
        lastB = B;
    }
    if (lastB > 0)
        memcpy(m->logits, m->logits_b + (size_t)(lastB - 1) * m->cfg.vocab_size,
               (size_t)m->cfg.vocab_size * sizeof(float));
    return 0;
}

/* Returns the number of emitted tokens.  forced (may be NULL) gives the accept
 * length j of cycle c as forced[c % n_forced], clamped to the draft count k.
 * out_j[c] records j; out_cand0/argmax help diagnose divergences. */
uint32_t ref_spec_generate(ref_t *r, uint32_t n_predict, uint32_t n_spec,
                           const uint32_t *forced, uint32_t n_forced,
                           uint32_t *out_tokens, uint32_t *out_j, uint32_t max_cycles,
                           uint32_t *n_cycles_out) {
    qwen_model_t *m = &r->m;
    const uint32_t V = m->cfg.vocab_size;
    if (n_spec > SPEC_MAX_B - 1) n_spec = SPEC_MAX_B - 1;
    const float *last_logits = m->logits;
    uint32_t generated = 0, n_cycles = 0;
    while (generated < n_predict && n_cycles < max_cycles) {
        const uint32_t P = m->pos - 1;
        const uint32_t room = m->n_ctx - 1 - P;
        if (room < 1) break;
        const uint32_t k = (n_spec < room - 1) ? n_spec : room - 1;
        uint32_t cand[SPEC_MAX_B];
        cand[0] = model_sample_greedy(last_logits, V);
        for (uint32_t s = 1; s <= k; s++) {
            mtp_forward(m, r->pool, cand[s - 1], P + s, 1);
            cand[s] = model_sample_greedy(m->logits, V);
        }
        const uint32_t B = k + 1;
        model_forward_batch(m, r->pool, cand, P + 1, B, 1);
        uint32_t j = k;
        for (uint32_t i = 0; i < k; i++) {
            const uint32_t v = model_sample_greedy(m->logits_b + (size_t)i * V, V);
            if (v != cand[i + 1]) { j = i; break; }
        }
        if (forced && n_forced) {
            j = forced[n_cycles % n_forced];
            if (j > k) j = k;
        }
        for (uint32_t i = 0; i <= j && generated < n_predict; i++)
            out_tokens[generated++] = cand[i];
        if (out_j) out_j[n_cycles] = j;
        n_cycles++;
        if (m->pos >= m->n_ctx) break;
        if (j < k) {
            model_rollback_to(m, j);
            m->pos = P + j + 2;
        }
        memcpy(m->mtp_h, m->h_save + (size_t)j * m->dims.n_embd, m->dims.n_embd * sizeof(float));
        mtp_forward(m, r->pool, cand[j], P + j + 1, 0);
        last_logits = m->logits_b + (size_t)j * V;
    }
    /* keep the next cycle's logits in m->logits for callers that continue */
    if (last_logits != m->logits) memcpy(m->logits, last_logits, (size_t)V * sizeof(float));
    if (n_cycles_out) *n_cycles_out = n_cycles;
    return generated;
}

uint32_t ref_greedy_generate(ref_t *r, uint32_t n_predict, uint32_t *out_tokens) {
    qwen_model_t *m = &r->m;
    const uint32_t V = m->cfg.vocab_size;
    if (n_predict == 0) return 0;
    uint32_t cur = model_sample_greedy(m->logits, V);
    out_tokens[0] = cur;
    uint32_t generated = 1;
    for (uint32_t i = 1; i < n_predict; i++) {
        if (m->pos >= m->n_ctx) break;
        model_forward(m, r->pool, cur, m->pos);
        cur = model_sample_greedy(m->logits, V);
        out_tokens[generated++] = cur;
    }
    return generated;
}

/* gguf_tensor_info_t built around caller memory (for gemv calls from tests). */
gguf_tensor_info_t *ref_make_tensor(const void *data, int type, uint64_t ne0, uint64_t ne1) {
    gguf_tensor_info_t *t = calloc(1, sizeof *t);
    if (!t) return NULL;
    snprintf(t->name, sizeof t->name, "tensor");
    t->n_dims = 2;
    t->ne[0] = ne0;
    t->ne[1] = ne1;
    t->ne[2] = t->ne[3] = 1;
    t->type = (ggml_type_t)type;
    t->data = data;
    return t;
}
void ref_free_tensor(gguf_tensor_info_t *t) { free(t); }

static pool_t *g_pool;
static int g_pool_n;
static pool_t *get_pool(int n) {
    if (n <= 0) n = (int)sysconf(_SC_NPROCESSORS_ONLN);
    if (!g_pool || g_pool_n != n) {
        if (g_pool) pool_destroy(g_pool);
        g_pool = pool_create(n, 0);
        g_pool_n = n;
    }
    return g_pool;
}

/* gemv_batch for any n: the reference caps one call at GEMV_MAX_B vectors
 * (include/kernels.h:19); larger n runs as chunks of GEMV_MAX_B, which is
 * bit-identical because batch == single-token (src/kernels.c:323-327). */
void ref_gemv_batch_any(const gguf_tensor_info_t *W, const float *x, uint64_t ldx, int n,
                        float *out, uint64_t ldo, int n_threads) {
    pool_t *p = get_pool(n_threads);
    for (int t0 = 0; t0 < n; t0 += GEMV_MAX_B) {
        const int nn = n - t0 < GEMV_MAX_B ? n - t0 : GEMV_MAX_B;
        gemv_batch(p, W, x + (size_t)t0 * ldx, ldx, nn, out + (size_t)t0 * ldo, ldo);
    }
}
void ref_gemv(const gguf_tensor_info_t *W, const float *x, float *out, int n_threads) {
    gemv(get_pool(n_threads), W, x, out);
}

double ref_now(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (double)ts.tv_sec + (double)ts.tv_nsec * 1e-9;
}

uint32_t ref_sample_generate(ref_t *r, sampler_t *smp, uint32_t n_predict, uint32_t *all_tokens, uint32_t n_all,
                             uint32_t *out_tokens) {
    qwen_model_t *m = &r->m;
    const uint32_t V = m->cfg.vocab_size;
    if (n_predict == 0) return 0;
    uint32_t cur = sampler_sample(smp, m->logits, V, all_tokens, n_all);
    all_tokens[n_all++] = cur;
    out_tokens[0] = cur;
    uint32_t generated = 1;
    for (uint32_t i = 1; i < n_predict; i++) {
        if (m->pos >= m->n_ctx) break;
        model_forward(m, r->pool, cur, m->pos);
        cur = sampler_sample(smp, m->logits, V, all_tokens, n_all);
        all_tokens[n_all++] = cur;
        out_tokens[generated++] = cur;
    }
    return generated;
}
