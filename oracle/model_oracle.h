/*
 * model_oracle.h -- CPU oracle of the Qwen3-4B-shaped Q4_K (or Q4_K_M) decode step.
 * TEST INFRASTRUCTURE ONLY; see model_oracle.c.
 */
#ifndef ABRA_MODEL_ORACLE_H
#define ABRA_MODEL_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    int32_t n_layers, hidden, n_heads, n_kv_heads, head_dim, ffn, vocab, max_ctx;
    float rope_theta, eps;
    uint64_t seed;
    int32_t centered; /* 1: centred Q4_K variant (orc_gen_q4k_ex flag 1) */
    int32_t mix;      /* 1: the Q4_K_M type map (orc_q6k_layer), 0: all Q4_K */
} orc_model_config;

typedef struct orc_model orc_model;

void orc_model_default_config(orc_model_config *c);
/* Seeded tensor ids: layer -1 -> which (1 embedding/output, 2 out_norm);
 * layer l -> 100 + 16 l + which (0 attn_norm, 1 wqkv, 2 q_norm, 3 k_norm,
 * 4 wo, 5 ffn_norm, 6 wgate, 7 wup, 8 wdown). */
uint64_t orc_tensor_id(int32_t layer, int32_t which);
/* Q4_K_M type map: layer l of n keeps attn_v and ffn_down in Q6_K when
 * l < n/8, l >= 7n/8 or (l - n/8) % 3 == 2 (llama.cpp's use_more_bits; for
 * Qwen3-4B-Q4_K_M that is layers 0-3, 6, 9, ..., 30, 31-35, the census in
 * the reference's bench/results/m3/qwen3-q4k-tensor-map.json); the tied
 * embedding/output is Q6_K, every other linear weight Q4_K.  With the map
 * the V rows of layer l come from tensor 1 as Q6_K rows (same row indices)
 * and ffn_down from tensor 8 as Q6_K. */
int32_t orc_q6k_layer(int32_t layer, int32_t n_layers);
void orc_rope_table(float *out, int32_t ctx, int32_t head_dim, float theta);

orc_model *orc_model_create(const orc_model_config *cfg);
void orc_model_destroy(orc_model *m);
int32_t orc_model_step(orc_model *m, int32_t token, int32_t pos, float *logits_out,
                       int32_t nthreads);
/* One decode step on llama.cpp's CPU path (Q8_K activations for every Q4_K
 * GEMV): the timed CPU baseline of bench.py, not a parity target.  All-Q4_K
 * models only (returns -1 otherwise); returns the greedy pick. */
int32_t orc_model_step_cpu(orc_model *m, int32_t token, int32_t pos, int32_t nthreads);
void orc_model_generate(orc_model *m, const int32_t *prompt, int32_t n_prompt, int32_t n_gen,
                        int32_t *out, int32_t nthreads);
const float *orc_model_hidden(const orc_model *m);

/* canonical pieces, exposed for unit tests */
void orc_add_rmsnorm_quantize(float *h, const float *delta, const float *w, float eps,
                              uint8_t *xq, int64_t K);
void orc_qk_norm_rope(const float *qkv, const float *q_norm, const float *k_norm, float eps,
                      const float *cs_row, int n_heads, int n_kv, int hd, float *q_out,
                      uint16_t *k_out, uint16_t *v_out);
void orc_attention_head(const float *q, const uint16_t *K, const uint16_t *V, int L, int hd,
                        float scale, float *out);
int32_t orc_argmax(const float *x, int64_t n);

#ifdef __cplusplus
}
#endif
#endif
