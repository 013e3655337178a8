// model.cu -- native decode runtime of the Qwen3-4B-shaped Q4_K model
// behind the C ABI (include/abra_b200.h, abra_model_*).
//
// One decode step is recorded once into a CUDA graph and replayed per
// token.  The position, the token history and the prompt length live in
// device memory: the embedding kernel reads tokens[pos], the argmax kernel
// appends the greedy pick and advances pos, so prompt feeding and generation
// are the same graph replayed N times with no host round trip per token.
//
// Per layer (reference model: Qwen3-4B via llama.cpp; this file is the B200
// equivalent of its decode graph):
//   residual + RMSNorm + Q8_1        (quantize once for q|k|v)
//   MMVQ q|k|v (fused 6144 x 2560)
//   QK-RMSNorm + NEOX RoPE + fp16 KV append
//   chunked attention + merge + Q8_1
//   MMVQ o
//   residual + RMSNorm + Q8_1        (quantize once for gate and up)
//   fused gate/up SwiGLU MMVQ
//   Q8_1 of the SwiGLU output
//   MMVQ down
// then residual + RMSNorm + Q8_1, the tied output MMVQ and argmax.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <new>
#include <vector>

#include "../../include/abra_b200.h"
#include "common.cuh"
#include "decode.cuh"
#include "kernels.cuh"

namespace abra {

struct LayerW {
    float *attn_norm, *q_norm, *k_norm, *ffn_norm;
    uint8_t *wqkv, *wo, *wgate, *wup, *wdown;
};

struct Model {
    abra_model_config cfg;
    int device = 0;
    std::vector<void *> allocs;
    uint8_t *embd = nullptr;
    float *out_norm = nullptr;
    std::vector<LayerW> layers;
    __half *kc = nullptr, *vc = nullptr;
    float *rope = nullptr;
    float *h, *h2;  // residual stream, ping-pong: each fused MMVQ reads one, writes the other
    float *delta, *qkv, *q, *att, *part_m, *part_l, *part_o, *act, *logits;
    uint8_t *xq, *oq, *aq;
    int32_t *tokens, *picks, *pos, *nprompt;
    unsigned long long *amax = nullptr;  // argmax key of the output MMVQ
    int max_chunks = 0;
    cudaStream_t stream = nullptr;
    cudaGraphExec_t graph = nullptr;
    size_t weight_bytes = 0, kv_bytes = 0;
    int32_t host_pos = 0;      // position after the queued steps (mirrors *pos)
    int32_t *pinned = nullptr; // 2 pinned ints for the streaming loop
};

static uint64_t tensor_id(int layer, int which) {
    return layer < 0 ? static_cast<uint64_t>(which) : 100u + 16u * layer + which;
}

#define TRY(expr)                                          \
    do {                                                   \
        cudaError_t _e = (expr);                           \
        if (_e != cudaSuccess) return _e;                  \
    } while (0)

template <typename T>
static cudaError_t alloc(Model &m, T **p, size_t bytes) {
    void *v = nullptr;
    TRY(cudaMalloc(&v, bytes));
    m.allocs.push_back(v);
    *p = static_cast<T *>(v);
    return cudaSuccess;
}

static size_t q4k_bytes(int64_t rows, int64_t cols) {
    return static_cast<size_t>(rows) * (cols / QK_K) * Q4K_BYTES;
}

static cudaError_t build(Model &m) {
    const abra_model_config &c = m.cfg;
    const int flags = c.centered ? 1 : 0;
    const uint64_t s = c.seed;
    const int64_t qkv_rows = static_cast<int64_t>(c.n_heads + 2 * c.n_kv_heads) * c.head_dim;
    const int64_t qd = static_cast<int64_t>(c.n_heads) * c.head_dim;
    cudaStream_t st = m.stream;
    auto q4k = [&](uint8_t **p, int64_t rows, int64_t cols, uint64_t tid) -> cudaError_t {
        const size_t b = q4k_bytes(rows, cols);
        TRY(alloc(m, p, b));
        m.weight_bytes += b;
        return launch_gen_q4k_ex(*p, rows * (cols / QK_K), s, tid, 0, flags, st);
    };
    auto norm = [&](float **p, int64_t n, uint64_t tid) -> cudaError_t {
        TRY(alloc(m, p, n * sizeof(float)));
        return launch_gen_norm_f32(*p, n, s, tid, st);
    };
    TRY(q4k(&m.embd, c.vocab, c.hidden, tensor_id(-1, 1)));
    TRY(norm(&m.out_norm, c.hidden, tensor_id(-1, 2)));
    m.layers.resize(c.n_layers);
    for (int l = 0; l < c.n_layers; ++l) {
        LayerW &y = m.layers[l];
        TRY(norm(&y.attn_norm, c.hidden, tensor_id(l, 0)));
        TRY(q4k(&y.wqkv, qkv_rows, c.hidden, tensor_id(l, 1)));
        TRY(norm(&y.q_norm, c.head_dim, tensor_id(l, 2)));
        TRY(norm(&y.k_norm, c.head_dim, tensor_id(l, 3)));
        TRY(q4k(&y.wo, c.hidden, qd, tensor_id(l, 4)));
        TRY(norm(&y.ffn_norm, c.hidden, tensor_id(l, 5)));
        TRY(q4k(&y.wgate, c.ffn, c.hidden, tensor_id(l, 6)));
        TRY(q4k(&y.wup, c.ffn, c.hidden, tensor_id(l, 7)));
        TRY(q4k(&y.wdown, c.hidden, c.ffn, tensor_id(l, 8)));
    }
    const size_t kv = static_cast<size_t>(c.n_layers) * c.n_kv_heads * c.max_ctx * c.head_dim * 2;
    TRY(alloc(m, &m.kc, kv));
    TRY(alloc(m, &m.vc, kv));
    TRY(cudaMemsetAsync(m.kc, 0, kv, st));
    TRY(cudaMemsetAsync(m.vc, 0, kv, st));
    m.kv_bytes = 2 * kv;
    // RoPE table in double precision on the host: cos/sin(pos * theta^(-2i/d)).
    const int half = c.head_dim / 2;
    std::vector<float> rope(static_cast<size_t>(c.max_ctx) * c.head_dim);
    for (int p = 0; p < c.max_ctx; ++p)
        for (int i = 0; i < half; ++i) {
            const double freq = std::pow(static_cast<double>(c.rope_theta),
                                         -2.0 * static_cast<double>(i) / static_cast<double>(c.head_dim));
            const double ang = static_cast<double>(p) * freq;
            rope[(static_cast<size_t>(p) * half + i) * 2 + 0] = static_cast<float>(std::cos(ang));
            rope[(static_cast<size_t>(p) * half + i) * 2 + 1] = static_cast<float>(std::sin(ang));
        }
    TRY(alloc(m, &m.rope, rope.size() * sizeof(float)));
    TRY(cudaMemcpyAsync(m.rope, rope.data(), rope.size() * sizeof(float), cudaMemcpyHostToDevice, st));
    m.max_chunks = (c.max_ctx + 255) / 256;
    int64_t mx = c.hidden > c.ffn ? c.hidden : c.ffn;
    if (qd > mx) mx = qd;
    TRY(alloc(m, &m.h, c.hidden * 4));
    TRY(alloc(m, &m.h2, c.hidden * 4));
    TRY(alloc(m, &m.delta, c.hidden * 4));
    TRY(alloc(m, &m.qkv, qkv_rows * 4));
    TRY(alloc(m, &m.q, qd * 4));
    TRY(alloc(m, &m.att, qd * 4));
    TRY(alloc(m, &m.part_m, static_cast<size_t>(c.n_heads) * m.max_chunks * 4));
    TRY(alloc(m, &m.part_l, static_cast<size_t>(c.n_heads) * m.max_chunks * 4));
    TRY(alloc(m, &m.part_o, static_cast<size_t>(c.n_heads) * m.max_chunks * c.head_dim * 4));
    TRY(alloc(m, &m.act, c.ffn * 4));
    TRY(alloc(m, &m.logits, static_cast<size_t>(c.vocab) * 4));
    TRY(alloc(m, &m.xq, (mx / QK8_1) * Q81_BYTES));
    TRY(alloc(m, &m.oq, (qd / QK8_1) * Q81_BYTES));
    TRY(alloc(m, &m.aq, (c.ffn / QK8_1) * Q81_BYTES));
    TRY(alloc(m, &m.tokens, (c.max_ctx + 1) * 4));
    TRY(alloc(m, &m.picks, (c.max_ctx + 1) * 4));
    TRY(alloc(m, &m.pos, 4));
    TRY(alloc(m, &m.nprompt, 4));
    TRY(alloc(m, &m.amax, 8));
    TRY(cudaMemsetAsync(m.amax, 0, 8, st));
    TRY(cudaMemsetAsync(m.tokens, 0, (c.max_ctx + 1) * 4, st));
    TRY(cudaMemsetAsync(m.picks, 0, (c.max_ctx + 1) * 4, st));
    TRY(cudaMemsetAsync(m.pos, 0, 4, st));
    TRY(cudaMemsetAsync(m.nprompt, 0, 4, st));
    return cudaStreamSynchronize(st);
}

static cudaError_t mmvq(const Model &m, const void *w, const void *w2, const void *x, float *y,
                        int64_t N, int64_t K, bool pdl, cudaStream_t st,
                        unsigned long long *amax = nullptr) {
    const int id = abra_tune_get(N, K, 1, w2 ? 2 : 1);
    const MmvqConfig *cfg = mmvq_candidate_by_id(id);
    if (!cfg) return cudaErrorInvalidValue;
    return launch_mmvq_q4k(*cfg, w, w2, x, y, N, K, 1, N, pdl ? MMVQ_PDL : 0, st, amax);
}

// The decode step for the token at tokens[*pos] (recorded into the graph).
static cudaError_t record_step(const Model &m, cudaStream_t st) {
    const abra_model_config &c = m.cfg;
    const bool pdl = (c.flags & ABRA_MODEL_NO_PDL) == 0;
    const int64_t qkv_rows = static_cast<int64_t>(c.n_heads + 2 * c.n_kv_heads) * c.head_dim;
    const int64_t qd = static_cast<int64_t>(c.n_heads) * c.head_dim;
    const size_t kv_layer = static_cast<size_t>(c.n_kv_heads) * c.max_ctx * c.head_dim;
    const float scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(c.head_dim)));
    DeltaSet none = {}, one = {};
    none.G = 0;
    one.p[0] = m.delta;
    one.G = 1;
    // residual stream ping-pong: every MMVQ with a fused RMSNorm prologue
    // reads h[cur] (+ the pending delta) and CTA 0 writes the sum to h[cur^1]
    float *h[2] = {m.h, m.h2};
    int cur = 0;
    auto fused = [&](const void *w, const void *w2, const DeltaSet &ds, const float *norm,
                     float *y, int64_t N, unsigned long long *amax) -> cudaError_t {
        const MmvqConfig *cfg = mmvq_candidate_by_id(abra_tune_get(N, c.hidden, 1, w2 ? 2 : 1));
        if (!cfg) return cudaErrorInvalidValue;
        MmvqXin xin = {h[cur], h[cur ^ 1], ds, norm, c.eps};
        cur ^= 1;
        return launch_mmvq_q4k_xin(*cfg, w, w2, xin, y, N, c.hidden, pdl ? MMVQ_PDL : 0, st, amax);
    };
    TRY(launch_embed(m.embd, c.hidden, m.tokens, m.pos, h[cur], pdl, st));
    for (int l = 0; l < c.n_layers; ++l) {
        const LayerW &y = m.layers[l];
        // residual + RMSNorm + Q8_1 fused into the q|k|v MMVQ
        TRY(fused(y.wqkv, nullptr, l == 0 ? none : one, y.attn_norm, m.qkv, qkv_rows, nullptr));
        TRY(launch_qk_norm_rope_kv(m.qkv, y.q_norm, y.k_norm, c.eps, m.rope, m.pos, m.q,
                                   m.kc + l * kv_layer, m.vc + l * kv_layer, c.n_heads,
                                   c.n_kv_heads, c.max_ctx, pdl, st));
        TRY(launch_attention(m.q, m.kc + l * kv_layer, m.vc + l * kv_layer, m.pos, scale,
                             c.n_heads, c.n_kv_heads, c.max_ctx, m.part_m, m.part_l, m.part_o,
                             m.att, m.oq, pdl, st));
        TRY(mmvq(m, y.wo, nullptr, m.oq, m.delta, c.hidden, qd, pdl, st));
        // residual + RMSNorm + Q8_1 fused into the gate/up SwiGLU MMVQ
        TRY(fused(y.wgate, y.wup, one, y.ffn_norm, m.act, c.ffn, nullptr));
        TRY(launch_quantize_q8_1(m.act, m.aq, c.ffn, 1, st));
        TRY(mmvq(m, y.wdown, nullptr, m.aq, m.delta, c.hidden, c.ffn, pdl, st));
    }
    // final residual + RMSNorm fused into the tied output MMVQ, which also
    // reduces the greedy argmax (ties to the lowest id)
    TRY(fused(m.embd, nullptr, c.n_layers > 0 ? one : none, m.out_norm, m.logits, c.vocab, m.amax));
    return launch_argmax_finish(m.amax, m.tokens, m.picks, m.pos, m.nprompt, c.max_ctx, pdl, st);
}

static cudaError_t prepare(const Model &m) {
    const abra_model_config &c = m.cfg;
    const int64_t qkv_rows = static_cast<int64_t>(c.n_heads + 2 * c.n_kv_heads) * c.head_dim;
    const int64_t qd = static_cast<int64_t>(c.n_heads) * c.head_dim;
    // {N, K, nmat, fused RMSNorm input}
    const int64_t shapes[5][4] = {{qkv_rows, c.hidden, 1, 1}, {c.hidden, qd, 1, 0},
                                  {c.ffn, c.hidden, 2, 1}, {c.hidden, c.ffn, 1, 0},
                                  {c.vocab, c.hidden, 1, 1}};
    for (const auto &sh : shapes) {
        const MmvqConfig *cfg = mmvq_candidate_by_id(abra_tune_get(sh[0], sh[1], 1, static_cast<int>(sh[2])));
        if (!cfg) return cudaErrorInvalidValue;
        TRY(prepare_mmvq(*cfg, 1, static_cast<int>(sh[2]), sh[3] != 0));
    }
    return cudaSuccess;
}

static cudaError_t capture(Model &m) {
    if (m.graph) return cudaSuccess;
    TRY(prepare(m));  // kernel attributes are set outside the capture
    if (m.cfg.flags & ABRA_MODEL_EAGER) return cudaSuccess;
    cudaGraph_t g = nullptr;
    TRY(cudaStreamBeginCapture(m.stream, cudaStreamCaptureModeThreadLocal));
    cudaError_t e = record_step(m, m.stream);
    cudaError_t e2 = cudaStreamEndCapture(m.stream, &g);
    if (e != cudaSuccess) {
        if (g) cudaGraphDestroy(g);
        return e;
    }
    TRY(e2);
    e = cudaGraphInstantiate(&m.graph, g, 0);
    cudaGraphDestroy(g);
    return e;
}

}  // namespace abra

using abra::Model;

namespace {
thread_local char g_model_err[256] = "";
int model_fail(int code, const char *what, cudaError_t e) {
    snprintf(g_model_err, sizeof g_model_err, "%s: %s", what, e == cudaSuccess ? "" : cudaGetErrorString(e));
    return code;
}
}  // namespace

extern "C" {

int abra_model_default_config(abra_model_config *c) {
    if (!c) return ABRA_E_INVALID;
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
    c->flags = 0;
    return ABRA_OK;
}

const char *abra_model_last_error(void) { return g_model_err; }

int abra_model_create(const abra_model_config *cfg, void **out) {
    if (!cfg || !out) return model_fail(ABRA_E_INVALID, "null pointer", cudaSuccess);
    const abra_model_config &c = *cfg;
    if (c.head_dim != 128 || c.n_heads <= 0 || c.n_kv_heads <= 0 || c.n_heads % c.n_kv_heads ||
        c.n_heads / c.n_kv_heads > 8 || c.hidden % 256 || c.ffn % 256 ||
        (c.n_heads * c.head_dim) % 256 || c.vocab <= 0 || c.max_ctx <= 0 || c.n_layers < 0 ||
        c.hidden > 16384)
        return model_fail(ABRA_E_UNSUPPORTED, "unsupported model configuration", cudaSuccess);
    Model *m = new (std::nothrow) Model();
    if (!m) return model_fail(ABRA_E_INVALID, "out of host memory", cudaSuccess);
    m->cfg = c;
    cudaGetDevice(&m->device);
    cudaError_t e = cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = abra::build(*m);
    if (e != cudaSuccess) {
        abra_model_destroy(m);
        return model_fail(ABRA_E_CUDA, "model build", e);
    }
    *out = m;
    return ABRA_OK;
}

int abra_model_destroy(void *model) {
    Model *m = static_cast<Model *>(model);
    if (!m) return ABRA_OK;
    if (m->stream) cudaStreamSynchronize(m->stream);
    if (m->graph) cudaGraphExecDestroy(m->graph);
    if (m->pinned) cudaFreeHost(m->pinned);
    for (void *p : m->allocs) cudaFree(p);
    if (m->stream) cudaStreamDestroy(m->stream);
    delete m;
    return ABRA_OK;
}

int abra_model_reset(void *model, const int32_t *prompt, int32_t n_prompt) {
    Model *m = static_cast<Model *>(model);
    if (!m || !prompt || n_prompt < 1 || n_prompt > m->cfg.max_ctx)
        return model_fail(ABRA_E_INVALID, "bad prompt", cudaSuccess);
    for (int i = 0; i < n_prompt; ++i)
        if (prompt[i] < 0 || prompt[i] >= m->cfg.vocab)
            return model_fail(ABRA_E_INVALID, "token id out of range", cudaSuccess);
    const int32_t zero = 0;
    cudaError_t e = cudaMemcpyAsync(m->tokens, prompt, n_prompt * 4, cudaMemcpyHostToDevice, m->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(m->pos, &zero, 4, cudaMemcpyHostToDevice, m->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(m->nprompt, &n_prompt, 4, cudaMemcpyHostToDevice, m->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
    if (e == cudaSuccess) m->host_pos = 0;
    return e == cudaSuccess ? ABRA_OK : model_fail(ABRA_E_CUDA, "reset", e);
}

int abra_model_step(void *model, int32_t n_steps) {
    Model *m = static_cast<Model *>(model);
    if (!m || n_steps < 0) return model_fail(ABRA_E_INVALID, "bad arguments", cudaSuccess);
    if (static_cast<int64_t>(m->host_pos) + n_steps > m->cfg.max_ctx)
        return model_fail(ABRA_E_INVALID, "steps would pass max_ctx", cudaSuccess);
    m->host_pos += n_steps;
    cudaError_t e = abra::capture(*m);
    if (e != cudaSuccess) return model_fail(ABRA_E_CUDA, "graph capture", e);
    for (int i = 0; i < n_steps; ++i) {
        e = m->graph ? cudaGraphLaunch(m->graph, m->stream) : abra::record_step(*m, m->stream);
        if (e != cudaSuccess) return model_fail(ABRA_E_CUDA, "step", e);
    }
    return ABRA_OK;
}

int abra_model_sync(void *model) {
    Model *m = static_cast<Model *>(model);
    if (!m) return ABRA_E_INVALID;
    cudaError_t e = cudaStreamSynchronize(m->stream);
    return e == cudaSuccess ? ABRA_OK : model_fail(ABRA_E_CUDA, "sync", e);
}

int abra_model_read(void *model, int32_t *tokens, int32_t n_tokens, float *logits,
                    int32_t *pos) {
    Model *m = static_cast<Model *>(model);
    if (!m || n_tokens < 0 || n_tokens > m->cfg.max_ctx + 1)
        return model_fail(ABRA_E_INVALID, "bad arguments", cudaSuccess);
    cudaError_t e = cudaStreamSynchronize(m->stream);
    if (e == cudaSuccess && tokens && n_tokens)
        e = cudaMemcpy(tokens, m->tokens, n_tokens * 4, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && logits)
        e = cudaMemcpy(logits, m->logits, static_cast<size_t>(m->cfg.vocab) * 4, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && pos) e = cudaMemcpy(pos, m->pos, 4, cudaMemcpyDeviceToHost);
    return e == cudaSuccess ? ABRA_OK : model_fail(ABRA_E_CUDA, "read", e);
}

int abra_model_generate(void *model, const int32_t *prompt, int32_t n_prompt, int32_t n_gen,
                        int32_t *out) {
    Model *m = static_cast<Model *>(model);
    if (!m || !out || n_gen < 1 || n_prompt + n_gen > m->cfg.max_ctx + 1)
        return model_fail(ABRA_E_INVALID, "bad arguments", cudaSuccess);
    int rc = abra_model_reset(model, prompt, n_prompt);
    if (rc) return rc;
    rc = abra_model_step(model, n_prompt + n_gen - 1);
    if (rc) return rc;
    std::vector<int32_t> all(n_prompt + n_gen);
    rc = abra_model_read(model, all.data(), n_prompt + n_gen, nullptr, nullptr);
    if (rc) return rc;
    std::memcpy(out, all.data() + n_prompt, n_gen * 4);
    return ABRA_OK;
}

int abra_model_decode_streaming(void *model, int32_t n, int32_t *out) {
    Model *m = static_cast<Model *>(model);
    if (!m || !out || n < 1) return model_fail(ABRA_E_INVALID, "bad arguments", cudaSuccess);
    if (static_cast<int64_t>(m->host_pos) + n > m->cfg.max_ctx)
        return model_fail(ABRA_E_INVALID, "steps would pass max_ctx", cudaSuccess);
    cudaError_t e = abra::capture(*m);
    if (e != cudaSuccess) return model_fail(ABRA_E_CUDA, "graph capture", e);
    if (!m->pinned) {
        e = cudaHostAlloc(reinterpret_cast<void **>(&m->pinned), 2 * sizeof(int32_t), cudaHostAllocDefault);
        if (e != cudaSuccess) return model_fail(ABRA_E_CUDA, "pinned buffer", e);
    }
    int32_t *in = m->pinned, *pick = m->pinned + 1;
    // the token the next step consumes
    e = cudaMemcpyAsync(in, m->tokens + m->host_pos, 4, cudaMemcpyDeviceToHost, m->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
    for (int32_t i = 0; i < n && e == cudaSuccess; ++i) {
        const int32_t p = m->host_pos;
        e = cudaMemcpyAsync(m->tokens + p, in, 4, cudaMemcpyHostToDevice, m->stream);
        if (e == cudaSuccess)
            e = m->graph ? cudaGraphLaunch(m->graph, m->stream) : abra::record_step(*m, m->stream);
        if (e == cudaSuccess) e = cudaMemcpyAsync(pick, m->picks + p, 4, cudaMemcpyDeviceToHost, m->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
        if (e == cudaSuccess) {
            out[i] = *pick;
            *in = *pick;
            m->host_pos = p + 1;
        }
    }
    return e == cudaSuccess ? ABRA_OK : model_fail(ABRA_E_CUDA, "streaming decode", e);
}

int abra_model_info(void *model, void **stream, uint64_t *weight_bytes, uint64_t *kv_bytes) {
    Model *m = static_cast<Model *>(model);
    if (!m) return ABRA_E_INVALID;
    if (stream) *stream = m->stream;
    if (weight_bytes) *weight_bytes = m->weight_bytes;
    if (kv_bytes) *kv_bytes = m->kv_bytes;
    return ABRA_OK;
}

}  // extern "C"
