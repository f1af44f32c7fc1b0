/* Seeded synthetic GGUF writer (see synth_gguf.c for the field distributions). */
#ifndef QB_SYNTH_GGUF_H
#define QB_SYNTH_GGUF_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { QB_SYNTH_DEFAULT = 0, QB_SYNTH_MIXED = 1 };

typedef struct {
    uint32_t n_embd, n_ff, n_layer, vocab;        /* n_layer = backbone layers (MTP added) */
    uint32_t n_head, n_kv_head, head_dim, rope_dim;
    uint32_t full_attn_interval;
    uint32_t ssm_state, ssm_groups, ssm_v_heads, d_conv;
    uint32_t n_ctx_train;
    float rope_theta, rms_eps;
    uint64_t seed;
    uint32_t profile;     /* QB_SYNTH_DEFAULT: IQ4_XS projections, Q6_K embd/head, Q8_0 eh_proj;
                             QB_SYNTH_MIXED: also Q4_K / Q5_K / Q6_K / Q8_0 projections */
    float gain;           /* target RMS of a projection output for unit-RMS input */
    uint32_t n_threads;   /* 0 = all online CPUs */
    uint32_t tokenizer;   /* 1: a byte-level tokenizer vocabulary (tokenizer.ggml.tokens), so the
                             reference CLI can encode prompts and print tokens */
} qb_synth_cfg_t;

int qb_synth_write(const char *path, const qb_synth_cfg_t *cfg);
uint64_t qb_synth_file_size(const qb_synth_cfg_t *cfg);
int qb_synth_iq4xs_matrix(void *dst, uint64_t rows, uint64_t K, uint64_t seed, float d_sigma);
int qb_synth_quant_matrix(void *dst, int ggml_type, uint64_t rows, uint64_t K, uint64_t seed,
                          float d_sigma);
void qb_synth_normal_f32(float *dst, uint64_t n, uint64_t seed);
uint16_t qb_f32_to_f16(float f);

#ifdef __cplusplus
}
#endif
#endif
