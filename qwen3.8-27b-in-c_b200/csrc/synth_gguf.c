/*
 * Seeded synthetic GGUF writer for the hybrid Qwen decoder (Gated DeltaNet +
 * gated GQA + one MTP "nextn" block).
 *
 * The real 14.7 GB IQ4_XS checkpoint is not available, so every test and the
 * benchmark run on weights produced here.  The file follows the layout that
 * the reference parser accepts (reference src/gguf.c:185-305): GGUF v3,
 * general.architecture + general.alignment, "<arch>.*" hyper-parameter keys
 * (src/gguf.c:91-110), rope.dimension_sections as a uint32 array
 * (src/gguf.c:135-150), tensor infos, then 32-byte aligned tensor data.
 * Tensor names and shapes follow the lookups of src/model.c:85-147 (backbone)
 * and src/model.c:245-279 (blk.<n_layer>.* MTP block, nextn.* tensors).
 *
 * Randomness is counter based (splitmix64 of seed, tensor index and block
 * index), so the bytes do not depend on the number of writer threads.
 *
 * Field distributions (per quant block; sigma chosen per tensor so that the
 * row dot products of unit-RMS inputs are O(gain)):
 *   IQ4_XS : d = fp16(|N(0,1)| * sigma), 6-bit sub-scales uniform 0..63,
 *            4-bit indices uniform 0..15 into the 16-entry kvalues table.
 *   Q6_K   : d = fp16(|N| * sigma), int8 sub-scales uniform, 6-bit q uniform.
 *   Q8_0   : d = fp16(|N| * sigma), int8 q uniform.
 *   Q4_K/Q5_K : d, dmin = fp16(|N| * sigma), 6-bit scale/min uniform, q uniform.
 *   F32 norms : 1 + N(0, 0.02).  conv1d taps N(0, 0.5).  dt_bias N(0, 0.5).
 *   ssm_a  : -(0.5 + 1.5 U[0,1))  (negative, so the GDN decay is < 1).
 */
#define _GNU_SOURCE
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <math.h>
#include <fcntl.h>
#include <unistd.h>
#include <pthread.h>
#include <sys/mman.h>
#include <sys/stat.h>

#include "synth_gguf.h"

/* ggml type ids (same numbering as GGUF files use) */
enum { T_F32 = 0, T_Q8_0 = 8, T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14, T_IQ4_XS = 23 };

static uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

typedef struct { uint64_t s; } rng_t;
static inline uint64_t rng_next(rng_t *r) { r->s = mix64(r->s); return r->s; }
static inline double rng_unit(rng_t *r) {          /* (0, 1) */
    return ((double)(rng_next(r) >> 11) + 0.5) * (1.0 / 9007199254740992.0);
}
static inline double rng_normal(rng_t *r) {
    const double u1 = rng_unit(r), u2 = rng_unit(r);
    return sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
}
static inline void rng_bytes(rng_t *r, uint8_t *dst, size_t n) {
    size_t i = 0;
    for (; i + 8 <= n; i += 8) { uint64_t v = rng_next(r); memcpy(dst + i, &v, 8); }
    if (i < n) { uint64_t v = rng_next(r); memcpy(dst + i, &v, n - i); }
}

/* fp32 -> fp16, round to nearest even, subnormals kept. */
uint16_t qb_f32_to_f16(float f) {
    uint32_t x; memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u : 0));
    if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);           /* overflow -> inf */
    if (ax < 0x33000001u) return (uint16_t)sign;                         /* < 2^-25 -> 0    */
    int e = (int)(ax >> 23) - 127;
    uint32_t m = (ax & 0x7FFFFFu) | 0x800000u;
    if (e < -14) {                                                       /* subnormal half  */
        const int shift = -14 - e + 13;
        uint32_t q = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (q & 1))) q++;
        return (uint16_t)(sign | q);
    }
    uint32_t q = m >> 13;
    const uint32_t rem = m & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1))) q++;
    uint32_t h = ((uint32_t)(e + 15) << 10) + (q - 0x400u);            /* carry bumps exp */
    return (uint16_t)(sign | h);
}

static size_t type_block_bytes(int t) {
    switch (t) {
    case T_F32: return 4;
    case T_Q8_0: return 34;
    case T_Q4_K: return 144;
    case T_Q5_K: return 176;
    case T_Q6_K: return 210;
    case T_IQ4_XS: return 136;
    default: return 0;
    }
}
static size_t type_block_elems(int t) {
    switch (t) {
    case T_F32: return 1;
    case T_Q8_0: return 32;
    default: return 256;
    }
}

/* RMS of one dequantised weight for sigma = 1 (used to pick sigma). */
static double type_unit_rms(int t) {
    switch (t) {
    case T_IQ4_XS: return 18.48 * 67.44;   /* rms(ls-32) * rms(kvalues)          */
    case T_Q6_K:   return 73.9 * 18.48;    /* rms(int8 scale) * rms(q-32)        */
    case T_Q8_0:   return 73.9;            /* rms(int8)                          */
    case T_Q4_K:   return 36.4 * 8.8;      /* rms(6-bit scale) * rms(4-bit q)    */
    case T_Q5_K:   return 36.4 * 18.2;
    default:       return 1.0;
    }
}

/* Fill one quant block (or one float for F32 handled elsewhere). */
static void fill_block(int t, uint8_t *b, rng_t *r, float sigma) {
    switch (t) {
    case T_IQ4_XS: {
        const uint16_t d = qb_f32_to_f16((float)(fabs(rng_normal(r)) * sigma));
        memcpy(b, &d, 2);
        rng_bytes(r, b + 2, 134);          /* scales_h(2) scales_l(4) qs(128) */
        break;
    }
    case T_Q6_K: {
        rng_bytes(r, b, 208);              /* ql(128) qh(64) scales(16) */
        const uint16_t d = qb_f32_to_f16((float)(fabs(rng_normal(r)) * sigma));
        memcpy(b + 208, &d, 2);
        break;
    }
    case T_Q8_0: {
        const uint16_t d = qb_f32_to_f16((float)(fabs(rng_normal(r)) * sigma));
        memcpy(b, &d, 2);
        rng_bytes(r, b + 2, 32);
        break;
    }
    case T_Q4_K:
    case T_Q5_K: {
        const uint16_t d = qb_f32_to_f16((float)(fabs(rng_normal(r)) * sigma));
        const uint16_t dm = qb_f32_to_f16((float)(fabs(rng_normal(r)) * sigma * 0.25));
        memcpy(b, &d, 2);
        memcpy(b + 2, &dm, 2);
        rng_bytes(r, b + 4, type_block_bytes(t) - 4);
        break;
    }
    default: break;
    }
}

/* ------------------------------------------------------------------------ */

enum { INIT_QUANT = 0, INIT_NORM, INIT_CONV, INIT_DTBIAS, INIT_SSMA };

typedef struct {
    char name[64];
    int type;
    uint32_t n_dims;
    uint64_t ne[2];
    int init;
    float sigma;
    uint64_t offset;   /* relative to data start */
    uint64_t nbytes;
} tdesc_t;

typedef struct {
    tdesc_t *t;
    int n, cap;
} tlist_t;

static tdesc_t *tl_add(tlist_t *L, const char *name, int type, uint32_t nd, uint64_t ne0,
                       uint64_t ne1, int init) {
    if (L->n == L->cap) {
        L->cap = L->cap ? 2 * L->cap : 256;
        L->t = realloc(L->t, (size_t)L->cap * sizeof *L->t);
    }
    tdesc_t *d = &L->t[L->n++];
    memset(d, 0, sizeof *d);
    snprintf(d->name, sizeof d->name, "%s", name);
    d->type = type;
    d->n_dims = nd;
    d->ne[0] = ne0;
    d->ne[1] = nd > 1 ? ne1 : 1;
    d->init = init;
    return d;
}

static void add_proj(tlist_t *L, const char *name, int type, uint64_t ne0, uint64_t ne1, float gain) {
    tdesc_t *d = tl_add(L, name, type, 2, ne0, ne1, INIT_QUANT);
    d->sigma = (float)(gain / (type_unit_rms(type) * sqrt((double)ne0)));
}

static void add_attn_block(tlist_t *L, const qb_synth_cfg_t *c, uint32_t il, int ty_q, int ty_kv,
                           int ty_o) {
    char nm[64];
    const uint64_t E = c->n_embd, hd = c->head_dim;
    snprintf(nm, sizeof nm, "blk.%u.attn_q.weight", il);
    add_proj(L, nm, ty_q, E, 2 * c->n_head * hd, c->gain);
    snprintf(nm, sizeof nm, "blk.%u.attn_k.weight", il);
    add_proj(L, nm, ty_kv, E, c->n_kv_head * hd, c->gain);
    snprintf(nm, sizeof nm, "blk.%u.attn_v.weight", il);
    add_proj(L, nm, ty_kv, E, c->n_kv_head * hd, c->gain);
    snprintf(nm, sizeof nm, "blk.%u.attn_q_norm.weight", il);
    tl_add(L, nm, T_F32, 1, hd, 1, INIT_NORM);
    snprintf(nm, sizeof nm, "blk.%u.attn_k_norm.weight", il);
    tl_add(L, nm, T_F32, 1, hd, 1, INIT_NORM);
    snprintf(nm, sizeof nm, "blk.%u.attn_output.weight", il);
    add_proj(L, nm, ty_o, c->n_head * hd, E, c->gain);
}

static void add_ffn_block(tlist_t *L, const qb_synth_cfg_t *c, uint32_t il, int ty_gate, int ty_up,
                          int ty_down) {
    char nm[64];
    snprintf(nm, sizeof nm, "blk.%u.ffn_gate.weight", il);
    add_proj(L, nm, ty_gate, c->n_embd, c->n_ff, c->gain);
    snprintf(nm, sizeof nm, "blk.%u.ffn_up.weight", il);
    add_proj(L, nm, ty_up, c->n_embd, c->n_ff, c->gain);
    snprintf(nm, sizeof nm, "blk.%u.ffn_down.weight", il);
    add_proj(L, nm, ty_down, c->n_ff, c->n_embd, c->gain);
}

static void build_tensor_list(const qb_synth_cfg_t *c, tlist_t *L) {
    char nm[64];
    const int mixed = c->profile == QB_SYNTH_MIXED;
    const int P = T_IQ4_XS;
    const uint64_t E = c->n_embd;
    const uint64_t d_inner = (uint64_t)c->ssm_v_heads * c->ssm_state;
    const uint64_t conv_dim = 2ull * c->ssm_groups * c->ssm_state + d_inner;

    tl_add(L, "token_embd.weight", mixed ? T_Q4_K : T_Q6_K, 2, E, c->vocab, INIT_QUANT);
    L->t[L->n - 1].sigma = (float)(c->gain / (type_unit_rms(L->t[L->n - 1].type) * sqrt((double)E)));
    tl_add(L, "output_norm.weight", T_F32, 1, E, 1, INIT_NORM);
    add_proj(L, "output.weight", T_Q6_K, E, c->vocab, c->gain);

    for (uint32_t il = 0; il < c->n_layer; il++) {
        const int recurrent = ((il + 1) % c->full_attn_interval) != 0;
        snprintf(nm, sizeof nm, "blk.%u.attn_norm.weight", il);
        tl_add(L, nm, T_F32, 1, E, 1, INIT_NORM);
        snprintf(nm, sizeof nm, "blk.%u.post_attention_norm.weight", il);
        tl_add(L, nm, T_F32, 1, E, 1, INIT_NORM);
        if (recurrent) {
            snprintf(nm, sizeof nm, "blk.%u.attn_qkv.weight", il);
            add_proj(L, nm, mixed ? T_Q5_K : P, E, conv_dim, c->gain);
            snprintf(nm, sizeof nm, "blk.%u.attn_gate.weight", il);
            add_proj(L, nm, P, E, d_inner, c->gain);
            snprintf(nm, sizeof nm, "blk.%u.ssm_conv1d.weight", il);
            tl_add(L, nm, T_F32, 2, c->d_conv, conv_dim, INIT_CONV);
            snprintf(nm, sizeof nm, "blk.%u.ssm_dt.bias", il);
            tl_add(L, nm, T_F32, 1, c->ssm_v_heads, 1, INIT_DTBIAS);
            snprintf(nm, sizeof nm, "blk.%u.ssm_a", il);
            tl_add(L, nm, T_F32, 1, c->ssm_v_heads, 1, INIT_SSMA);
            snprintf(nm, sizeof nm, "blk.%u.ssm_beta.weight", il);
            add_proj(L, nm, mixed ? T_Q8_0 : P, E, c->ssm_v_heads, c->gain);
            snprintf(nm, sizeof nm, "blk.%u.ssm_alpha.weight", il);
            add_proj(L, nm, mixed ? T_Q8_0 : P, E, c->ssm_v_heads, c->gain);
            snprintf(nm, sizeof nm, "blk.%u.ssm_norm.weight", il);
            tl_add(L, nm, T_F32, 1, c->ssm_state, 1, INIT_NORM);
            snprintf(nm, sizeof nm, "blk.%u.ssm_out.weight", il);
            add_proj(L, nm, mixed ? T_Q6_K : P, d_inner, E, c->gain);
        } else {
            add_attn_block(L, c, il, mixed ? T_Q5_K : P, mixed ? T_Q8_0 : P, mixed ? T_Q4_K : P);
        }
        add_ffn_block(L, c, il, mixed ? T_Q4_K : P, P, mixed ? T_Q6_K : P);
    }
    /* MTP block blk.<n_layer> */
    const uint32_t im = c->n_layer;
    snprintf(nm, sizeof nm, "blk.%u.attn_norm.weight", im);
    tl_add(L, nm, T_F32, 1, E, 1, INIT_NORM);
    snprintf(nm, sizeof nm, "blk.%u.post_attention_norm.weight", im);
    tl_add(L, nm, T_F32, 1, E, 1, INIT_NORM);
    add_attn_block(L, c, im, P, P, P);
    add_ffn_block(L, c, im, P, P, P);
    snprintf(nm, sizeof nm, "blk.%u.nextn.eh_proj.weight", im);
    add_proj(L, nm, T_Q8_0, 2 * E, E, c->gain);
    snprintf(nm, sizeof nm, "blk.%u.nextn.enorm.weight", im);
    tl_add(L, nm, T_F32, 1, E, 1, INIT_NORM);
    snprintf(nm, sizeof nm, "blk.%u.nextn.hnorm.weight", im);
    tl_add(L, nm, T_F32, 1, E, 1, INIT_NORM);
    snprintf(nm, sizeof nm, "blk.%u.nextn.shared_head_norm.weight", im);
    tl_add(L, nm, T_F32, 1, E, 1, INIT_NORM);
}

/* ---------------- metadata serialisation ---------------- */

typedef struct { uint8_t *p; size_t n, cap; } buf_t;
static void bput(buf_t *b, const void *src, size_t n) {
    if (b->n + n > b->cap) {
        b->cap = (b->n + n) * 2 + 4096;
        b->p = realloc(b->p, b->cap);
    }
    memcpy(b->p + b->n, src, n);
    b->n += n;
}
static void bput_u32(buf_t *b, uint32_t v) { bput(b, &v, 4); }
static void bput_u64(buf_t *b, uint64_t v) { bput(b, &v, 8); }
static void bput_str(buf_t *b, const char *s) { bput_u64(b, strlen(s)); bput(b, s, strlen(s)); }

enum { G_U32 = 4, G_F32 = 6, G_BOOL = 7, G_STR = 8, G_ARR = 9, G_U64 = 10 };

static void kv_u32(buf_t *b, const char *arch, const char *suffix, uint32_t v) {
    char k[160]; snprintf(k, sizeof k, "%s%s", arch, suffix);
    bput_str(b, k); bput_u32(b, G_U32); bput_u32(b, v);
}
static void kv_f32(buf_t *b, const char *arch, const char *suffix, float v) {
    char k[160]; snprintf(k, sizeof k, "%s%s", arch, suffix);
    bput_str(b, k); bput_u32(b, G_F32); bput(b, &v, 4);
}

/* ---------------- threaded data fill ---------------- */

typedef struct {
    const tlist_t *L;
    uint8_t *data;
    uint64_t seed;
    uint64_t total_units, next;
    pthread_mutex_t mu;
} fill_job_t;

#define UNIT_BLOCKS 4096ull   /* blocks per work unit */

static void fill_range(const tdesc_t *d, int ti, uint8_t *base, uint64_t seed, uint64_t b0,
                       uint64_t b1) {
    const uint64_t tkey = mix64(seed ^ mix64(0xA5A5A5A5ull + (uint64_t)ti));
    if (d->type == T_F32) {
        float *f = (float *)base;
        for (uint64_t i = b0; i < b1; i++) {
            rng_t r = { mix64(tkey ^ (i * 0xD1B54A32D192ED03ull)) };
            double v;
            switch (d->init) {
            case INIT_NORM:   v = 1.0 + 0.02 * rng_normal(&r); break;
            case INIT_CONV:   v = 0.5 * rng_normal(&r); break;
            case INIT_DTBIAS: v = 0.5 * rng_normal(&r); break;
            case INIT_SSMA:   v = -(0.5 + 1.5 * rng_unit(&r)); break;
            default:          v = rng_normal(&r); break;
            }
            f[i] = (float)v;
        }
        return;
    }
    const size_t bb = type_block_bytes(d->type);
    for (uint64_t i = b0; i < b1; i++) {
        rng_t r = { mix64(tkey ^ (i * 0xD1B54A32D192ED03ull)) };
        fill_block(d->type, base + i * bb, &r, d->sigma);
    }
}

static uint64_t tensor_blocks(const tdesc_t *d) {
    return d->ne[0] * d->ne[1] / type_block_elems(d->type);
}

static void *fill_worker(void *arg) {
    fill_job_t *J = arg;
    for (;;) {
        pthread_mutex_lock(&J->mu);
        const uint64_t u = J->next++;
        pthread_mutex_unlock(&J->mu);
        if (u >= J->total_units) break;
        /* locate unit u */
        uint64_t acc = 0;
        for (int ti = 0; ti < J->L->n; ti++) {
            const tdesc_t *d = &J->L->t[ti];
            const uint64_t nb = tensor_blocks(d);
            const uint64_t nu = (nb + UNIT_BLOCKS - 1) / UNIT_BLOCKS;
            if (u < acc + nu) {
                const uint64_t k = u - acc;
                const uint64_t b0 = k * UNIT_BLOCKS;
                const uint64_t b1 = b0 + UNIT_BLOCKS < nb ? b0 + UNIT_BLOCKS : nb;
                fill_range(d, ti, J->data + d->offset, J->seed, b0, b1);
                break;
            }
            acc += nu;
        }
    }
    return NULL;
}

static void fill_all(const tlist_t *L, uint8_t *data, uint64_t seed, int n_threads) {
    fill_job_t J;
    memset(&J, 0, sizeof J);
    J.L = L;
    J.data = data;
    J.seed = seed;
    for (int ti = 0; ti < L->n; ti++)
        J.total_units += (tensor_blocks(&L->t[ti]) + UNIT_BLOCKS - 1) / UNIT_BLOCKS;
    pthread_mutex_init(&J.mu, NULL);
    if (n_threads < 1) n_threads = 1;
    if (n_threads > 256) n_threads = 256;
    pthread_t th[256];
    for (int i = 0; i < n_threads; i++) pthread_create(&th[i], NULL, fill_worker, &J);
    for (int i = 0; i < n_threads; i++) pthread_join(th[i], NULL);
    pthread_mutex_destroy(&J.mu);
}

static int cfg_check(const qb_synth_cfg_t *c) {
    if (!c->n_embd || !c->n_ff || !c->n_layer || !c->vocab || !c->n_head || !c->n_kv_head) return -1;
    if (c->n_embd % 256 || c->n_ff % 256) return -1;
    if ((c->n_head * c->head_dim) % 256) return -1;
    if (((uint64_t)c->ssm_v_heads * c->ssm_state) % 256) return -1;
    if (c->head_dim % 8 || c->ssm_state % 8 || c->n_head % c->n_kv_head) return -1;
    if (c->d_conv != 4 || c->full_attn_interval == 0) return -1;
    if (c->ssm_v_heads % c->ssm_groups) return -1;
    if (c->rope_dim > c->head_dim || c->rope_dim % 2) return -1;
    if (c->tokenizer && c->vocab < 266) return -1;   /* 256 bytes, 6 merged, 3 specials, one more */
    return 0;
}

int qb_synth_write(const char *path, const qb_synth_cfg_t *c) {
    if (!path || !c || cfg_check(c)) return -1;
    tlist_t L = {0};
    build_tensor_list(c, &L);

    const char *arch = "qwen35";
    const uint32_t align = 32;
    buf_t h = {0};
    uint32_t magic = 0x46554747u, version = 3;
    bput_u32(&h, magic);
    bput_u32(&h, version);
    bput_u64(&h, (uint64_t)L.n);
    const size_t kv_count_at = h.n;
    bput_u64(&h, 0);                       /* patched below */
    uint64_t n_kv = 0;
    bput_str(&h, "general.architecture"); bput_u32(&h, G_STR); bput_str(&h, arch);
    bput_str(&h, "general.alignment"); bput_u32(&h, G_U32); bput_u32(&h, align);
    kv_u32(&h, arch, ".embedding_length", c->n_embd);
    kv_u32(&h, arch, ".attention.head_count", c->n_head);
    kv_u32(&h, arch, ".attention.head_count_kv", c->n_kv_head);
    kv_u32(&h, arch, ".attention.key_length", c->head_dim);
    kv_u32(&h, arch, ".block_count", c->n_layer + 1);
    kv_u32(&h, arch, ".feed_forward_length", c->n_ff);
    kv_u32(&h, arch, ".vocab_size", c->vocab);
    kv_u32(&h, arch, ".context_length", c->n_ctx_train ? c->n_ctx_train : 262144);
    kv_f32(&h, arch, ".rope.freq_base", c->rope_theta);
    kv_u32(&h, arch, ".rope.dimension_count", c->rope_dim);
    {
        char k[160]; snprintf(k, sizeof k, "%s.rope.dimension_sections", arch);
        bput_str(&h, k); bput_u32(&h, G_ARR); bput_u32(&h, G_U32); bput_u64(&h, 4);
        const uint32_t secs[4] = { c->rope_dim / 2 - c->rope_dim / 4, c->rope_dim / 4, 0, 0 };
        for (int i = 0; i < 4; i++) bput_u32(&h, secs[i]);
    }
    kv_f32(&h, arch, ".attention.layer_norm_rms_epsilon", c->rms_eps);
    kv_u32(&h, arch, ".full_attention_interval", c->full_attn_interval);
    kv_u32(&h, arch, ".ssm.state_size", c->ssm_state);
    kv_u32(&h, arch, ".ssm.conv_kernel", c->d_conv);
    kv_u32(&h, arch, ".ssm.inner_size", c->ssm_v_heads * c->ssm_state);
    kv_u32(&h, arch, ".ssm.group_count", c->ssm_groups);
    kv_u32(&h, arch, ".nextn_predict_layers", 1);
    bput_str(&h, "qb.synth.seed"); bput_u32(&h, G_U64); bput_u64(&h, c->seed);
    n_kv = 21;   /* 2 general.* + 18 <arch>.* + qb.synth.seed */
    if (c->tokenizer) {
        /* Byte-level vocabulary: token b < 256 is byte b in the GPT-2 byte-to-unicode
         * form (printable bytes as themselves, the others from U+0100 on, in byte
         * order), then six merged pairs, <tN> fillers, and the chat specials at the
         * end (<|im_end|> the last id: the end-of-sequence token). */
        bput_str(&h, "tokenizer.ggml.tokens"); bput_u32(&h, G_ARR); bput_u32(&h, G_STR);
        bput_u64(&h, c->vocab);
        /* a few BPE merges (the reference tokenizer needs a merge table), their
         * results right after the bytes; U+0120 is the space byte */
        static const char* const merged[6] = {"th", "he", "in", "er", "an", "\xc4\xa0t"};
        static const char* const merges[6] = {"t h", "h e", "i n", "e r", "a n", "\xc4\xa0 t"};
        int extra = 0;
        for (uint32_t id = 0; id < c->vocab; id++) {
            char t[32];
            if (id >= 256 && id < 262) {
                snprintf(t, sizeof t, "%s", merged[id - 256]);
            } else if (id < 256) {
                const uint32_t b = id;
                const int printable = (b >= '!' && b <= '~') || (b >= 0xA1 && b <= 0xAC) || (b >= 0xAE && b <= 0xFF);
                const uint32_t cp = printable ? b : 256 + (uint32_t)extra++;
                if (cp < 0x80) { t[0] = (char)cp; t[1] = 0; }
                else { t[0] = (char)(0xC0 | (cp >> 6)); t[1] = (char)(0x80 | (cp & 0x3F)); t[2] = 0; }
            } else if (id == c->vocab - 3) {
                snprintf(t, sizeof t, "<|endoftext|>");
            } else if (id == c->vocab - 2) {
                snprintf(t, sizeof t, "<|im_start|>");
            } else if (id == c->vocab - 1) {
                snprintf(t, sizeof t, "<|im_end|>");
            } else {
                snprintf(t, sizeof t, "<t%u>", id);
            }
            bput_str(&h, t);
        }
        bput_str(&h, "tokenizer.ggml.merges"); bput_u32(&h, G_ARR); bput_u32(&h, G_STR); bput_u64(&h, 6);
        for (int i = 0; i < 6; i++) bput_str(&h, merges[i]);
        n_kv += 2;
    }
    memcpy(h.p + kv_count_at, &n_kv, 8);

    uint64_t off = 0;
    for (int i = 0; i < L.n; i++) {
        tdesc_t *d = &L.t[i];
        d->nbytes = tensor_blocks(d) * type_block_bytes(d->type);
        off = (off + align - 1) / align * align;
        d->offset = off;
        off += d->nbytes;
        bput_str(&h, d->name);
        bput_u32(&h, d->n_dims);
        for (uint32_t k = 0; k < d->n_dims; k++) bput_u64(&h, d->ne[k]);
        bput_u32(&h, (uint32_t)d->type);
        bput_u64(&h, d->offset);
    }
    const uint64_t data_start = (h.n + align - 1) / align * align;
    const uint64_t file_size = data_start + off;

    int fd = open(path, O_RDWR | O_CREAT | O_TRUNC, 0644);
    if (fd < 0) { free(h.p); free(L.t); return -2; }
    if (ftruncate(fd, (off_t)file_size) != 0) { close(fd); free(h.p); free(L.t); return -3; }
    uint8_t *map = mmap(NULL, file_size, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
    if (map == MAP_FAILED) { close(fd); free(h.p); free(L.t); return -4; }
    memset(map, 0, data_start);
    memcpy(map, h.p, h.n);
    int nt = c->n_threads ? (int)c->n_threads : (int)sysconf(_SC_NPROCESSORS_ONLN);
    fill_all(&L, map + data_start, c->seed, nt);
    munmap(map, file_size);
    close(fd);
    free(h.p);
    free(L.t);
    return 0;
}

uint64_t qb_synth_file_size(const qb_synth_cfg_t *c) {
    if (!c || cfg_check(c)) return 0;
    tlist_t L = {0};
    build_tensor_list(c, &L);
    uint64_t off = 0;
    for (int i = 0; i < L.n; i++) {
        off = (off + 31) / 32 * 32;
        off += tensor_blocks(&L.t[i]) * type_block_bytes(L.t[i].type);
    }
    free(L.t);
    return off;
}

/* Stand-alone IQ4_XS matrix [rows][K] for the gemv micro benchmark: d uses
 * sigma = d_sigma directly (0.02 in the benchmark configuration). */
int qb_synth_iq4xs_matrix(void *dst, uint64_t rows, uint64_t K, uint64_t seed, float d_sigma) {
    if (!dst || K % 256) return -1;
    tdesc_t d;
    memset(&d, 0, sizeof d);
    d.type = T_IQ4_XS;
    d.ne[0] = K;
    d.ne[1] = rows;
    d.sigma = d_sigma;
    fill_range(&d, 0, (uint8_t *)dst, seed, 0, rows * (K / 256));
    return 0;
}

int qb_synth_quant_matrix(void *dst, int type, uint64_t rows, uint64_t K, uint64_t seed,
                          float d_sigma) {
    const size_t be = type_block_elems(type);
    if (!dst || !type_block_bytes(type) || (type != T_F32 && K % be)) return -1;
    tdesc_t d;
    memset(&d, 0, sizeof d);
    d.type = type;
    d.ne[0] = K;
    d.ne[1] = rows;
    d.sigma = d_sigma;
    d.init = INIT_QUANT;
    fill_range(&d, 1, (uint8_t *)dst, seed, 0, rows * K / be);
    return 0;
}

void qb_synth_normal_f32(float *dst, uint64_t n, uint64_t seed) {
    for (uint64_t i = 0; i < n; i++) {
        rng_t r = { mix64(seed ^ mix64(i + 0x1234567ull)) };
        dst[i] = (float)rng_normal(&r);
    }
}
