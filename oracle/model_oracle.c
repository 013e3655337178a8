/*
 * model_oracle.c -- CPU oracle of the Qwen3-4B-shaped Q4_K (or Q4_K_M) decode step.
 *
 * TEST INFRASTRUCTURE ONLY (the reference result for tests/ and the smoke entry).  It
 * evaluates the same random-init model as abra_b200's decode runtime, every
 * operation in the same fp32 order as the CUDA kernels, so greedy tokens and
 * logits can be compared bit for bit.  Compiled with -ffp-contract=off.
 *
 * The architecture (36 layers, hidden 2560, 32 q / 8 kv heads of 128, SwiGLU
 * 9728, QK-RMSNorm, NEOX RoPE theta 1e6, tied 151936 vocabulary, fp16 KV) is
 * the model the reference runs through llama.cpp (Qwen3-4B); the reference
 * contains no forward pass of its own.  Its attention matvec
 * (kernels/q4k/abra-attention.cuh:3-57) fixes the head grouping: kv head =
 * q head / 4.
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "model_oracle.h"
#include "q4k_oracle.h"
#include "q6k_oracle.h"

#define Q4K_BYTES 144
#define Q81_BYTES 36
/* Q6K_BYTES (210) comes from q6k_oracle.h */
#define ATT_CHUNK 256

struct orc_model {
    orc_model_config cfg;
    uint8_t *embd;  /* vocab x hidden Q4_K (Q6_K with the Q4_K_M map), tied with the output */
    float *out_norm;
    struct layer {
        float *attn_norm, *q_norm, *k_norm, *ffn_norm;
        uint8_t *wqkv, *wo, *wgate, *wup, *wdown;
        uint8_t *wv6; /* Q6_K V rows (q6 layers; wqkv then holds q|k only) */
        int q6;       /* attn_v and ffn_down in Q6_K */
    } *L;
    uint16_t *kcache, *vcache; /* [layer][kv head][ctx][head_dim] fp16 */
    float *rope;               /* [ctx][head_dim/2][2] cos, sin */
    /* work buffers */
    float *h, *delta, *qkv, *q, *att, *act, *logits, *tmp;
    uint8_t *xq, *aq;
    float *xn;   /* fp32 normalized activation (the llama.cpp CPU path) */
    uint8_t *yk; /* its Q8_K blocks */
};



void orc_model_default_config(orc_model_config *c) {
    c->n_layers = 36;
    c->hidden = 2560;
    c->n_heads = 32;
    c->n_kv_heads = 8;
    c->head_dim = 128;
    c->ffn = 9728;
    c->vocab = 151936;
    c->max_ctx = 4096;
    c->rope_theta = 1000000.0f;
    c->eps = 1e-6f;
    c->seed = 0;
    c->centered = 0;
    c->mix = 0;
}

int32_t orc_q6k_layer(int32_t layer, int32_t n_layers) {
    const int32_t a = n_layers / 8, b = 7 * n_layers / 8;
    return layer < a || layer >= b || (layer - a) % 3 == 2;
}

uint64_t orc_tensor_id(int32_t layer, int32_t which) {
    if (layer < 0) return (uint64_t)which; /* 1 = embedding/output, 2 = out_norm */
    return 100u + 16u * (uint64_t)layer + (uint64_t)which;
}

static uint8_t *gen_q4k_tensor(int64_t rows, int64_t cols, uint64_t seed, uint64_t tid,
                               int32_t flags) {
    const int64_t nb = rows * (cols / 256);
    uint8_t *p = (uint8_t *)malloc((size_t)nb * Q4K_BYTES);
    const int64_t chunk = 1 << 16;
#pragma omp parallel for schedule(static)
    for (int64_t b = 0; b < nb; b += chunk) {
        const int64_t n = nb - b < chunk ? nb - b : chunk;
        orc_gen_q4k_ex(p + b * Q4K_BYTES, n, seed, tid, b, flags);
    }
    return p;
}

/* rows [row0, row0 + rows) of a Q6_K tensor of `cols` columns */
static uint8_t *gen_q6k_tensor(int64_t row0, int64_t rows, int64_t cols, uint64_t seed,
                               uint64_t tid) {
    const int64_t nsb = cols / 256, nb = rows * nsb;
    uint8_t *p = (uint8_t *)malloc((size_t)nb * Q6K_BYTES);
    const int64_t chunk = 1 << 16;
#pragma omp parallel for schedule(static)
    for (int64_t b = 0; b < nb; b += chunk) {
        const int64_t n = nb - b < chunk ? nb - b : chunk;
        orc_gen_q6k(p + b * Q6K_BYTES, n, seed, tid, row0 * nsb + b);
    }
    return p;
}

/* RMSNorm weights: +-U(0.8, 1.2) with a random sign (orc_gen_norm_f32). */
static float *gen_norm(int64_t n, uint64_t seed, uint64_t tid) {
    float *p = (float *)malloc((size_t)n * sizeof(float));
    orc_gen_norm_f32(p, n, seed, tid);
    return p;
}

void orc_rope_table(float *out, int32_t ctx, int32_t head_dim, float theta) {
    const int32_t half = head_dim / 2;
    for (int32_t p = 0; p < ctx; ++p)
        for (int32_t i = 0; i < half; ++i) {
            const double freq = pow((double)theta, -2.0 * (double)i / (double)head_dim);
            const double ang = (double)p * freq;
            out[((int64_t)p * half + i) * 2 + 0] = (float)cos(ang);
            out[((int64_t)p * half + i) * 2 + 1] = (float)sin(ang);
        }
}

orc_model *orc_model_create(const orc_model_config *cfg) {
    orc_model *m = (orc_model *)calloc(1, sizeof *m);
    m->cfg = *cfg;
    const orc_model_config *c = &m->cfg;
    const uint64_t s = c->seed;
    const int64_t qkv_rows = (int64_t)(c->n_heads + 2 * c->n_kv_heads) * c->head_dim;
    const int64_t qk_rows = (int64_t)(c->n_heads + c->n_kv_heads) * c->head_dim;
    const int64_t kvd = (int64_t)c->n_kv_heads * c->head_dim;
    m->embd = c->mix ? gen_q6k_tensor(0, c->vocab, c->hidden, s, orc_tensor_id(-1, 1))
                     : gen_q4k_tensor(c->vocab, c->hidden, s, orc_tensor_id(-1, 1), c->centered);
    m->out_norm = gen_norm(c->hidden, s, orc_tensor_id(-1, 2));
    m->L = calloc((size_t)c->n_layers, sizeof *m->L);
    for (int l = 0; l < c->n_layers; ++l) {
        struct layer *y = &m->L[l];
        y->attn_norm = gen_norm(c->hidden, s, orc_tensor_id(l, 0));
        y->q6 = c->mix && orc_q6k_layer(l, c->n_layers);
        y->wqkv = gen_q4k_tensor(y->q6 ? qk_rows : qkv_rows, c->hidden, s, orc_tensor_id(l, 1), c->centered);
        if (y->q6) y->wv6 = gen_q6k_tensor(qk_rows, kvd, c->hidden, s, orc_tensor_id(l, 1));
        y->q_norm = gen_norm(c->head_dim, s, orc_tensor_id(l, 2));
        y->k_norm = gen_norm(c->head_dim, s, orc_tensor_id(l, 3));
        y->wo = gen_q4k_tensor(c->hidden, (int64_t)c->n_heads * c->head_dim, s, orc_tensor_id(l, 4), c->centered);
        y->ffn_norm = gen_norm(c->hidden, s, orc_tensor_id(l, 5));
        y->wgate = gen_q4k_tensor(c->ffn, c->hidden, s, orc_tensor_id(l, 6), c->centered);
        y->wup = gen_q4k_tensor(c->ffn, c->hidden, s, orc_tensor_id(l, 7), c->centered);
        y->wdown = y->q6 ? gen_q6k_tensor(0, c->hidden, c->ffn, s, orc_tensor_id(l, 8))
                         : gen_q4k_tensor(c->hidden, c->ffn, s, orc_tensor_id(l, 8), c->centered);
    }
    const size_t kv = (size_t)c->n_layers * c->n_kv_heads * c->max_ctx * c->head_dim;
    m->kcache = (uint16_t *)calloc(kv, 2);
    m->vcache = (uint16_t *)calloc(kv, 2);
    m->rope = (float *)malloc((size_t)c->max_ctx * c->head_dim * sizeof(float));
    orc_rope_table(m->rope, c->max_ctx, c->head_dim, c->rope_theta);
    const int64_t qd = (int64_t)c->n_heads * c->head_dim;
    m->h = calloc((size_t)c->hidden, 4);
    m->delta = calloc((size_t)c->hidden, 4);
    m->qkv = calloc((size_t)qkv_rows, 4);
    m->q = calloc((size_t)qd, 4);
    m->att = calloc((size_t)qd, 4);
    m->act = calloc((size_t)c->ffn, 4);
    m->logits = calloc((size_t)c->vocab, 4);
    int64_t mx = c->hidden > c->ffn ? c->hidden : c->ffn;
    if (qd > mx) mx = qd;
    m->tmp = calloc((size_t)mx * 2, 4);
    m->xq = calloc((size_t)(mx / 32) * Q81_BYTES, 1);
    m->aq = calloc((size_t)(mx / 32) * Q81_BYTES, 1);
    m->xn = calloc((size_t)mx, 4);
    m->yk = calloc((size_t)(mx / 256) * 292, 1);
    return m;
}

void orc_model_destroy(orc_model *m) {
    if (!m) return;
    for (int l = 0; l < m->cfg.n_layers; ++l) {
        struct layer *y = &m->L[l];
        free(y->attn_norm); free(y->wqkv); free(y->q_norm); free(y->k_norm); free(y->wo);
        free(y->ffn_norm); free(y->wgate); free(y->wup); free(y->wdown); free(y->wv6);
    }
    free(m->L); free(m->embd); free(m->out_norm); free(m->kcache); free(m->vcache);
    free(m->rope); free(m->h); free(m->delta); free(m->qkv); free(m->q); free(m->att);
    free(m->act); free(m->logits); free(m->tmp); free(m->xq); free(m->aq);
    free(m->xn); free(m->yk);
    free(m);
}

/* ---- canonical pieces ---------------------------------------------------- */

/* h = h + delta (when delta != NULL), then Q8_1 of RMSNorm(h) * w. */
void orc_add_rmsnorm_quantize(float *h, const float *delta, const float *w, float eps,
                              uint8_t *xq, int64_t K) {
    if (delta)
        for (int64_t i = 0; i < K; ++i) h[i] = h[i] + delta[i];
    orc_rmsnorm_quantize_q8_1(h, w, eps, xq, NULL, K, 1);
}

/* Per-head RMSNorm over head_dim = 128 in the canonical warp order (lane t
 * accumulates elements 4t..4t+3 with fmaf, then an xor butterfly 16..1),
 * then NEOX RoPE with the host table row cs[head_dim/2][2]. */
static void head_norm_rope(const float *x, const float *w, float eps, const float *cs,
                           float *out, int hd) {
    float lane[32], tmp[32];
    for (int t = 0; t < 32; ++t) {
        float acc = 0.0f;
        for (int i = 0; i < hd / 32; ++i) acc = fmaf(x[t * (hd / 32) + i], x[t * (hd / 32) + i], acc);
        lane[t] = acc;
    }
    for (int msk = 16; msk >= 1; msk >>= 1) {
        for (int t = 0; t < 32; ++t) tmp[t] = lane[t] + lane[t ^ msk];
        memcpy(lane, tmp, sizeof lane);
    }
    const float r = 1.0f / sqrtf(lane[0] / (float)hd + eps);
    float y[256];
    for (int i = 0; i < hd; ++i) y[i] = (x[i] * r) * w[i];
    const int half = hd / 2;
    for (int i = 0; i < half; ++i) {
        const float c = cs[2 * i], s = cs[2 * i + 1];
        const float x0 = y[i], x1 = y[i + half];
        out[i] = fmaf(x0, c, -(x1 * s));
        out[i + half] = fmaf(x0, s, x1 * c);
    }
}

void orc_qk_norm_rope(const float *qkv, const float *q_norm, const float *k_norm, float eps,
                      const float *cs_row, int n_heads, int n_kv, int hd, float *q_out,
                      uint16_t *k_out, uint16_t *v_out) {
    float tmp[256];
    for (int h = 0; h < n_heads; ++h) head_norm_rope(qkv + h * hd, q_norm, eps, cs_row, q_out + h * hd, hd);
    for (int g = 0; g < n_kv; ++g) {
        head_norm_rope(qkv + (n_heads + g) * hd, k_norm, eps, cs_row, tmp, hd);
        for (int i = 0; i < hd; ++i) {
            k_out[g * hd + i] = orc_f32_to_f16(tmp[i]);
            v_out[g * hd + i] = orc_f32_to_f16(qkv[(n_heads + n_kv + g) * hd + i]);
        }
    }
}

/* Attention of one q head over positions [0, L), K/V fp16 rows of hd.
 * Chunks of 256 positions; inside a chunk slot t = 32 w + lane:
 *   s = (sequential fmaf over d of q[d] * k[d]) * scale
 *   m = max s;  e = exp(s - m) (0 for slots past L)
 *   l = per-warp xor butterfly of e, then warps 0..7 added in order
 *   o[d] = per warp: sequential fmaf of e * v[d] over its valid slots;
 *          then warps 0..7 added in order
 * Merge over chunks c in order: M = max m_c, w_c = exp(m_c - M),
 *   Lsum = fmaf(l_c, w_c, Lsum), O[d] = fmaf(o_c[d], w_c, O[d]); out = O / Lsum. */
void orc_attention_head(const float *q, const uint16_t *K, const uint16_t *V, int L, int hd,
                        float scale, float *out) {
    const int nch = (L + ATT_CHUNK - 1) / ATT_CHUNK;
    float *mc = malloc((size_t)nch * 4), *lc = malloc((size_t)nch * 4);
    float *oc = malloc((size_t)nch * hd * 4);
    float s[ATT_CHUNK], e[ATT_CHUNK];
    for (int c = 0; c < nch; ++c) {
        const int j0 = c * ATT_CHUNK;
        float m = -INFINITY;
        for (int t = 0; t < ATT_CHUNK; ++t) {
            const int j = j0 + t;
            if (j < L) {
                float acc = 0.0f;
                for (int d = 0; d < hd; ++d) acc = fmaf(q[d], orc_f16_to_f32(K[(int64_t)j * hd + d]), acc);
                s[t] = acc * scale;
                if (s[t] > m) m = s[t];
            }
        }
        for (int t = 0; t < ATT_CHUNK; ++t) e[t] = (j0 + t < L) ? orc_expf(s[t] - m) : 0.0f;
        float lsum = 0.0f;
        for (int w = 0; w < ATT_CHUNK / 32; ++w) {
            float v[32], tmp[32];
            memcpy(v, e + 32 * w, sizeof v);
            for (int msk = 16; msk >= 1; msk >>= 1) {
                for (int t = 0; t < 32; ++t) tmp[t] = v[t] + v[t ^ msk];
                memcpy(v, tmp, sizeof v);
            }
            lsum = (w == 0) ? v[0] : lsum + v[0];
        }
        for (int d = 0; d < hd; ++d) {
            float tot = 0.0f;
            for (int w = 0; w < ATT_CHUNK / 32; ++w) {
                float acc = 0.0f;
                for (int t = 0; t < 32; ++t) {
                    const int j = j0 + 32 * w + t;
                    if (j < L) acc = fmaf(e[32 * w + t], orc_f16_to_f32(V[(int64_t)j * hd + d]), acc);
                }
                tot = (w == 0) ? acc : tot + acc;
            }
            oc[(int64_t)c * hd + d] = tot;
        }
        mc[c] = m;
        lc[c] = lsum;
    }
    float M = mc[0];
    for (int c = 1; c < nch; ++c)
        if (mc[c] > M) M = mc[c];
    float Ls = 0.0f;
    float *wc = malloc((size_t)nch * 4);
    for (int c = 0; c < nch; ++c) {
        wc[c] = orc_expf(mc[c] - M);
        Ls = fmaf(lc[c], wc[c], Ls);
    }
    for (int d = 0; d < hd; ++d) {
        float O = 0.0f;
        for (int c = 0; c < nch; ++c) O = fmaf(oc[(int64_t)c * hd + d], wc[c], O);
        out[d] = O / Ls;
    }
    free(mc); free(lc); free(oc); free(wc);
}

int32_t orc_argmax(const float *x, int64_t n) {
    int64_t best = 0;
    for (int64_t i = 1; i < n; ++i)
        if (x[i] > x[best]) best = i; /* ties keep the lowest index */
    return (int32_t)best;
}

/* ---- one decode step ------------------------------------------------------ */
int32_t orc_model_step(orc_model *m, int32_t token, int32_t pos, float *logits_out,
                       int32_t nthreads) {
    const orc_model_config *c = &m->cfg;
    const int hd = c->head_dim, H = c->hidden;
    const int64_t qd = (int64_t)c->n_heads * hd;
    const int64_t qkv_rows = (int64_t)(c->n_heads + 2 * c->n_kv_heads) * hd;
    const float scale = (float)(1.0 / sqrt((double)hd));
    const int64_t kvstride = (int64_t)c->max_ctx * hd; /* per (layer, kv head) */
    if (c->mix)
        orc_dequant_q6k(m->embd + (int64_t)token * (H / 256) * Q6K_BYTES, m->h, H / 256);
    else
        orc_dequant_q4k(m->embd + (int64_t)token * (H / 256) * Q4K_BYTES, m->h, H / 256);
    int have_delta = 0;
    for (int l = 0; l < c->n_layers; ++l) {
        struct layer *y = &m->L[l];
        orc_add_rmsnorm_quantize(m->h, have_delta ? m->delta : NULL, y->attn_norm, c->eps, m->xq, H);
        if (y->q6) { /* q|k Q4_K, then v Q6_K on the same Q8_1 activation */
            const int64_t qk_rows = qkv_rows - (int64_t)c->n_kv_heads * hd;
            orc_q4k_gemv(y->wqkv, m->xq, m->qkv, qk_rows, H, 1, nthreads);
            orc_q6k_gemv(y->wv6, m->xq, m->qkv + qk_rows, qkv_rows - qk_rows, H, 1, nthreads);
        } else {
            orc_q4k_gemv(y->wqkv, m->xq, m->qkv, qkv_rows, H, 1, nthreads);
        }
        uint16_t kt[8 * 256], vt[8 * 256];
        orc_qk_norm_rope(m->qkv, y->q_norm, y->k_norm, c->eps, m->rope + (int64_t)pos * hd,
                         c->n_heads, c->n_kv_heads, hd, m->q, kt, vt);
        for (int g = 0; g < c->n_kv_heads; ++g) {
            const int64_t base = ((int64_t)l * c->n_kv_heads + g) * kvstride + (int64_t)pos * hd;
            memcpy(m->kcache + base, kt + g * hd, (size_t)hd * 2);
            memcpy(m->vcache + base, vt + g * hd, (size_t)hd * 2);
        }
        const int gq = c->n_heads / c->n_kv_heads;
#pragma omp parallel for num_threads(nthreads) schedule(static)
        for (int h = 0; h < c->n_heads; ++h) {
            const int g = h / gq;
            const int64_t base = ((int64_t)l * c->n_kv_heads + g) * kvstride;
            orc_attention_head(m->q + (int64_t)h * hd, m->kcache + base, m->vcache + base, pos + 1,
                               hd, scale, m->att + (int64_t)h * hd);
        }
        orc_quantize_q8_1(m->att, m->xq, qd, 1);
        orc_q4k_gemv(y->wo, m->xq, m->delta, H, qd, 1, nthreads);
        orc_add_rmsnorm_quantize(m->h, m->delta, y->ffn_norm, c->eps, m->xq, H);
        orc_q4k_gemv(y->wgate, m->xq, m->tmp, c->ffn, H, 1, nthreads);
        orc_q4k_gemv(y->wup, m->xq, m->tmp + c->ffn, c->ffn, H, 1, nthreads);
        orc_swiglu(m->tmp, m->tmp + c->ffn, m->act, c->ffn);
        orc_quantize_q8_1(m->act, m->aq, c->ffn, 1);
        if (y->q6)
            orc_q6k_gemv(y->wdown, m->aq, m->delta, H, c->ffn, 1, nthreads);
        else
            orc_q4k_gemv(y->wdown, m->aq, m->delta, H, c->ffn, 1, nthreads);
        have_delta = 1;
    }
    orc_add_rmsnorm_quantize(m->h, have_delta ? m->delta : NULL, m->out_norm, c->eps, m->xq, H);
    if (c->mix)
        orc_q6k_gemv(m->embd, m->xq, m->logits, c->vocab, H, 1, nthreads);
    else
        orc_q4k_gemv(m->embd, m->xq, m->logits, c->vocab, H, 1, nthreads);
    if (logits_out) memcpy(logits_out, m->logits, (size_t)c->vocab * 4);
    return orc_argmax(m->logits, c->vocab);
}

/* ---- the same step on llama.cpp's CPU path (timed baseline) -------------
 * The decode the reference runs when its model is on the host: every Q4_K
 * matrix-vector product takes its activation as Q8_K blocks (ggml's CPU
 * vec_dot_q4_K_q8_K, restated as orc_q4k_q8k_gemv) instead of Q8_1; norms,
 * RoPE, fp16 KV and attention as in orc_model_step.  All-Q4_K models only.
 * Its logits differ from the canonical step in the last bits; it times the
 * CPU path and is not a parity target. */
static void q8k_gemv(orc_model *m, const uint8_t *w, const float *x, float *y, int64_t N, int64_t K,
                     int32_t nthreads) {
    orc_quantize_q8_K(x, m->yk, K, 1);
    orc_q4k_q8k_gemv(w, m->yk, y, N, K, 1, nthreads);
}

int32_t orc_model_step_cpu(orc_model *m, int32_t token, int32_t pos, int32_t nthreads) {
    const orc_model_config *c = &m->cfg;
    if (c->mix) return -1;
    const int hd = c->head_dim, H = c->hidden;
    const int64_t qd = (int64_t)c->n_heads * hd;
    const int64_t qkv_rows = (int64_t)(c->n_heads + 2 * c->n_kv_heads) * hd;
    const float scale = (float)(1.0 / sqrt((double)hd));
    const int64_t kvstride = (int64_t)c->max_ctx * hd;
    orc_dequant_q4k(m->embd + (int64_t)token * (H / 256) * Q4K_BYTES, m->h, H / 256);
    int have_delta = 0;
    for (int l = 0; l < c->n_layers; ++l) {
        struct layer *y = &m->L[l];
        if (have_delta)
            for (int64_t i = 0; i < H; ++i) m->h[i] = m->h[i] + m->delta[i];
        orc_rmsnorm_quantize_q8_1(m->h, y->attn_norm, c->eps, m->xq, m->xn, H, 1);
        q8k_gemv(m, y->wqkv, m->xn, m->qkv, qkv_rows, H, nthreads);
        uint16_t kt[8 * 256], vt[8 * 256];
        orc_qk_norm_rope(m->qkv, y->q_norm, y->k_norm, c->eps, m->rope + (int64_t)pos * hd,
                         c->n_heads, c->n_kv_heads, hd, m->q, kt, vt);
        for (int g = 0; g < c->n_kv_heads; ++g) {
            const int64_t base = ((int64_t)l * c->n_kv_heads + g) * kvstride + (int64_t)pos * hd;
            memcpy(m->kcache + base, kt + g * hd, (size_t)hd * 2);
            memcpy(m->vcache + base, vt + g * hd, (size_t)hd * 2);
        }
        const int gq = c->n_heads / c->n_kv_heads;
#pragma omp parallel for num_threads(nthreads) schedule(static)
        for (int h = 0; h < c->n_heads; ++h) {
            const int g = h / gq;
            const int64_t base = ((int64_t)l * c->n_kv_heads + g) * kvstride;
            orc_attention_head(m->q + (int64_t)h * hd, m->kcache + base, m->vcache + base, pos + 1,
                               hd, scale, m->att + (int64_t)h * hd);
        }
        q8k_gemv(m, y->wo, m->att, m->delta, H, qd, nthreads);
        for (int64_t i = 0; i < H; ++i) m->h[i] = m->h[i] + m->delta[i];
        orc_rmsnorm_quantize_q8_1(m->h, y->ffn_norm, c->eps, m->xq, m->xn, H, 1);
        q8k_gemv(m, y->wgate, m->xn, m->tmp, c->ffn, H, nthreads);
        orc_q4k_q8k_gemv(y->wup, m->yk, m->tmp + c->ffn, c->ffn, H, 1, nthreads);
        orc_swiglu(m->tmp, m->tmp + c->ffn, m->act, c->ffn);
        q8k_gemv(m, y->wdown, m->act, m->delta, H, c->ffn, nthreads);
        have_delta = 1;
    }
    if (have_delta)
        for (int64_t i = 0; i < H; ++i) m->h[i] = m->h[i] + m->delta[i];
    orc_rmsnorm_quantize_q8_1(m->h, m->out_norm, c->eps, m->xq, m->xn, H, 1);
    q8k_gemv(m, m->embd, m->xn, m->logits, c->vocab, H, nthreads);
    return orc_argmax(m->logits, c->vocab);
}

const float *orc_model_hidden(const orc_model *m) { return m->h; }

/* Greedy generation: feed prompt[0..n_prompt), then generate n_gen tokens.
 * out[0..n_gen) receives the generated ids. */
void orc_model_generate(orc_model *m, const int32_t *prompt, int32_t n_prompt, int32_t n_gen,
                        int32_t *out, int32_t nthreads) {
    int32_t tok = 0;
    for (int32_t i = 0; i < n_prompt; ++i) tok = orc_model_step(m, prompt[i], i, NULL, nthreads);
    for (int32_t i = 0; i < n_gen; ++i) {
        out[i] = tok;
        if (i + 1 < n_gen) tok = orc_model_step(m, tok, n_prompt + i, NULL, nthreads);
    }
}
