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
//
// With ABRA_MODEL_Q4_K_M the weights follow the real Qwen3-4B-Q4_K_M type
// map: the tied table is Q6_K, and layers with q6k_layer() keep attn_v and
// ffn_down in Q6_K.  There the fused MMVQ covers q|k only and also exports
// its Q8_1 activation, which the Q6_K V MMVQ reads; ffn_down runs the Q6_K
// MMVQ on the SwiGLU's Q8_1; the output is a residual + RMSNorm + Q8_1
// kernel followed by the Q6_K MMVQ with the argmax keys.
#include <algorithm>
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
    uint8_t *wv = nullptr;  // Q6_K V rows (q6 layers; wqkv then holds q|k only)
    bool q6 = false;        // attn_v and ffn_down in Q6_K
};

// Q4_K_M type map (llama.cpp's use_more_bits rule): attn_v and ffn_down stay
// Q6_K in layer l of n when l < n/8, l >= 7n/8 or (l - n/8) % 3 == 2 -- for
// 36 layers: 0-3, 6, 9, ..., 30 and 31-35, as in the Qwen3-4B-Q4_K_M census
// the reference records (bench/results/m3/qwen3-q4k-tensor-map.json).
static bool q6k_layer(int l, int n) {
    const int a = n / 8, b = 7 * n / 8;
    return l < a || l >= b || (l - a) % 3 == 2;
}

// What one rank of a tensor-parallel group holds (world == 1: everything).
// K-sharded layers (o, down) are cut on canonical K-slice boundaries, so the
// ranks' partial sums combine, in the fixed slice tree, to the bits of the
// unsharded layer; every other layer is split by output rows.
static int tp_shard(const abra_model_config &c, int rank, int world, abra_tp_shard &s) {
    if (!(world == 1 || world == 2 || world == 4 || world == 8) || rank < 0 || rank >= world)
        return ABRA_E_INVALID;
    if (c.n_heads % world || c.n_kv_heads % world || c.vocab < world) return ABRA_E_UNSUPPORTED;
    const int per = 8 / world;
    const int qd = c.n_heads * c.head_dim;
    const int nsb_o = qd / QK_K, nsb_f = c.ffn / QK_K;
    s.rank = rank;
    s.world = world;
    s.q_heads = c.n_heads / world;
    s.kv_heads = c.n_kv_heads / world;
    s.q_head_lo = rank * s.q_heads;
    s.kv_head_lo = rank * s.kv_heads;
    s.sl_base = rank * per;
    s.sl_cnt = per;
    // o: this rank's heads must be exactly its canonical slices of K
    for (int r = 0; r <= world; ++r)
        if (slice_start(nsb_o, r * per) * QK_K != r * (qd / world)) return ABRA_E_UNSUPPORTED;
    s.ffn_lo = slice_start(nsb_f, rank * per) * QK_K;
    s.ffn_hi = slice_start(nsb_f, (rank + 1) * per) * QK_K;
    if (s.ffn_hi <= s.ffn_lo) return ABRA_E_UNSUPPORTED;
    s.vocab_lo = static_cast<int64_t>(c.vocab) * rank / world;
    s.vocab_hi = static_cast<int64_t>(c.vocab) * (rank + 1) / world;
    return ABRA_OK;
}

struct Model {
    abra_model_config cfg;
    abra_tp_shard sh = {};
    int device = 0;
    // tensor-parallel exchange arena (world > 1), one cudaMalloc shared by
    // IPC: recv[2 * n_layers][world][hidden] fp32 partial sums (slot 2l: o of
    // layer l, 2l+1: down), then u64 words: rank arrivals cnt[2 * n_layers + 1]
    // (the last for the argmax keys), the combined argmax key, the step
    // epoch, and this GPU's own CTA counters ccnt[2 * n_layers + 1].
    uint8_t *arena = nullptr;
    size_t arena_recv = 0, arena_bytes = 0;
    uint8_t *peer[8] = {};  // every rank's arena as mapped here (peer[rank] == arena)
    bool connected = false;
    std::vector<void *> allocs;
    uint8_t *embd = nullptr;
    bool mix = false;  // the Q4_K_M type map (embd is Q6_K)
    float *out_norm = nullptr;
    std::vector<LayerW> layers;
    __half *kc = nullptr, *vc = nullptr;
    float *rope = nullptr;
    float *h, *h2;  // residual stream, ping-pong: each fused MMVQ reads one, writes the other
    float *delta, *qkv, *q, *att, *part_m, *part_l, *part_o, *act, *logits;
    uint8_t *xq, *oq, *aq;
    int32_t *tokens, *picks, *pos, *nprompt;
    unsigned long long *amax = nullptr;  // argmax key of the output MMVQ
    // batched decode (batch > 1): sequences in lockstep at one shared
    // position; activations, KV cache and tokens are per sequence
    int batch = 1;
    float *gbuf = nullptr, *ubuf = nullptr;  // gate and up outputs
    float *tc_ws = nullptr;                  // k-part scratch of the tensor-core MMVQ
    int max_chunks = 0;
    cudaStream_t stream = nullptr;
    cudaGraphExec_t graph = nullptr;
    // prefill (batch-1 model): up to kPrefillMax prompt tokens of one
    // sequence per step as the columns of the tensor-core GEMVs; buffers
    // allocated on first use, one graph per chunk size (a multiple of 32)
    float *ph = nullptr, *pdelta = nullptr, *pqkv = nullptr, *pq = nullptr, *pg = nullptr, *pu = nullptr;
    float *ppart_m = nullptr, *ppart_l = nullptr, *ppart_o = nullptr, *pws = nullptr;
    uint8_t *pxq = nullptr, *poq = nullptr, *paq = nullptr;
    cudaGraphExec_t pgraph[8] = {};  // chunk size 32 (i + 1)
    int32_t host_nprompt = 0;
    // draft verification: 32 columns with logits and per-column greedy picks
    float *plogits = nullptr;
    int32_t *vpick = nullptr;   // device, 32
    int32_t *vhost = nullptr;   // pinned, 64
    cudaGraphExec_t vgraph = nullptr;
    size_t weight_bytes = 0, kv_bytes = 0;
    int32_t host_pos = 0;      // position after the queued steps (mirrors *pos)
    int32_t *pinned = nullptr; // 2 pinned ints for the streaming loop
    // persistent decode step (batch 1, one GPU, all-Q4_K, unless
    // ABRA_MODEL_KERNEL_CHAIN): one cooperative kernel per token
    bool persist = false;
    bool persist_eager = false;  // the cooperative launch could not be captured
    PersistLayer *players = nullptr;
    void *psync = nullptr;

    // Exchange arena: [slot 0 .. 2L)[rank][batch][hidden] fp32 partials, then
    // the counters: arrivals per slot (2L + 1: o and down of each layer, the
    // output), the argmax key word of each sequence, the step epoch, this
    // rank's CTA count per slot.
    float *recv(int q, int slot) const {  // rank q's partial in slot, in peer[..]'s layout
        return reinterpret_cast<float *>(arena) +
               (static_cast<size_t>(slot) * sh.world + q) * static_cast<size_t>(batch) * cfg.hidden;
    }
    float *recv_of(uint8_t *base, int q, int slot) const {
        return reinterpret_cast<float *>(base) +
               (static_cast<size_t>(slot) * sh.world + q) * static_cast<size_t>(batch) * cfg.hidden;
    }
    unsigned long long *cnt_of(uint8_t *base, int slot) const {
        return reinterpret_cast<unsigned long long *>(base + arena_recv) + slot;
    }
    unsigned long long *key_of(uint8_t *base, int b = 0) const { return cnt_of(base, 2 * cfg.n_layers + 1 + b); }
    unsigned long long *epoch() const { return cnt_of(arena, 2 * cfg.n_layers + 1 + batch); }
    unsigned long long *cta_cnt(int slot) const { return cnt_of(arena, 2 * cfg.n_layers + 2 + batch + slot); }
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

static size_t q6k_bytes(int64_t rows, int64_t cols) {
    return static_cast<size_t>(rows) * (cols / QK_K) * 210;
}

static cudaError_t build(Model &m) {
    const abra_model_config &c = m.cfg;
    const abra_tp_shard &sh = m.sh;
    const int flags = c.centered ? 1 : 0;
    const uint64_t s = c.seed;
    const int64_t hd = c.head_dim;
    const int64_t qd = static_cast<int64_t>(c.n_heads) * hd, kvd = static_cast<int64_t>(c.n_kv_heads) * hd;
    const int64_t qd_l = sh.q_heads * hd, kvd_l = sh.kv_heads * hd, qkv_l = qd_l + 2 * kvd_l;
    const int64_t ffn_l = sh.ffn_hi - sh.ffn_lo, vocab_l = sh.vocab_hi - sh.vocab_lo;
    const int64_t nsb_h = c.hidden / QK_K, nsb_o = qd / QK_K, nsb_f = c.ffn / QK_K;
    cudaStream_t st = m.stream;
    auto walloc = [&](uint8_t **p, int64_t rows, int64_t cols, bool q6 = false) -> cudaError_t {
        const size_t b = q6 ? q6k_bytes(rows, cols) : q4k_bytes(rows, cols);
        TRY(alloc(m, p, b));
        m.weight_bytes += b;
        return cudaSuccess;
    };
    // Q6_K rows [row0, row0 + n) of a tensor `cols` wide, at dst
    auto rows6 = [&](uint8_t *dst, int64_t row0, int64_t n, int64_t cols, uint64_t tid) -> cudaError_t {
        const int64_t nb = n * (cols / QK_K);
        return launch_gen_q6k_cols(dst, nb, nb, 0, s, tid, row0 * (cols / QK_K), st);
    };
    // full-K rows [row0, row0 + n) of a tensor, at dst
    auto rows = [&](uint8_t *dst, int64_t row0, int64_t n, uint64_t tid) -> cudaError_t {
        return launch_gen_q4k_ex(dst, n * nsb_h, s, tid, row0 * nsb_h, flags, st);
    };
    auto norm = [&](float **p, int64_t n, uint64_t tid) -> cudaError_t {
        TRY(alloc(m, p, n * sizeof(float)));
        return launch_gen_norm_f32(*p, n, s, tid, st);
    };
    // the whole tied table on every rank: embedding lookups need any row;
    // the output MMVQ reads this rank's vocab rows of it
    m.mix = (c.flags & ABRA_MODEL_Q4_K_M) != 0;
    TRY(walloc(&m.embd, c.vocab, c.hidden, m.mix));
    if (m.mix)
        TRY(rows6(m.embd, 0, c.vocab, c.hidden, tensor_id(-1, 1)));
    else
        TRY(rows(m.embd, 0, c.vocab, tensor_id(-1, 1)));
    TRY(norm(&m.out_norm, c.hidden, tensor_id(-1, 2)));
    m.layers.resize(c.n_layers);
    for (int l = 0; l < c.n_layers; ++l) {
        LayerW &y = m.layers[l];
        TRY(norm(&y.attn_norm, c.hidden, tensor_id(l, 0)));
        // q|k|v rows of this rank's heads, fused: [q heads | k heads | v heads]
        // (q6 layers: q|k here, the V rows as Q6_K in wv)
        y.q6 = m.mix && q6k_layer(l, c.n_layers);
        TRY(walloc(&y.wqkv, y.q6 ? qd_l + kvd_l : qkv_l, c.hidden));
        const size_t rb = q4k_bytes(1, c.hidden);
        TRY(rows(y.wqkv, sh.q_head_lo * hd, qd_l, tensor_id(l, 1)));
        TRY(rows(y.wqkv + qd_l * rb, qd + sh.kv_head_lo * hd, kvd_l, tensor_id(l, 1)));
        if (y.q6) {
            TRY(walloc(&y.wv, kvd_l, c.hidden, true));
            TRY(rows6(y.wv, qd + kvd + sh.kv_head_lo * hd, kvd_l, c.hidden, tensor_id(l, 1)));
        } else {
            TRY(rows(y.wqkv + (qd_l + kvd_l) * rb, qd + kvd + sh.kv_head_lo * hd, kvd_l, tensor_id(l, 1)));
        }
        TRY(norm(&y.q_norm, c.head_dim, tensor_id(l, 2)));
        TRY(norm(&y.k_norm, c.head_dim, tensor_id(l, 3)));
        // o: K-shard = this rank's canonical slices = its heads' columns
        TRY(walloc(&y.wo, c.hidden, qd_l));
        TRY(launch_gen_q4k_cols(y.wo, c.hidden, nsb_o, slice_start(nsb_o, sh.sl_base),
                                slice_start(nsb_o, sh.sl_base + sh.sl_cnt), s, tensor_id(l, 4), 0,
                                flags, st));
        TRY(norm(&y.ffn_norm, c.hidden, tensor_id(l, 5)));
        TRY(walloc(&y.wgate, ffn_l, c.hidden));
        TRY(rows(y.wgate, sh.ffn_lo, ffn_l, tensor_id(l, 6)));
        TRY(walloc(&y.wup, ffn_l, c.hidden));
        TRY(rows(y.wup, sh.ffn_lo, ffn_l, tensor_id(l, 7)));
        // down: K-shard = this rank's FFN units (Q6_K only unsharded)
        TRY(walloc(&y.wdown, c.hidden, ffn_l, y.q6));
        if (y.q6)
            TRY(rows6(y.wdown, 0, c.hidden, c.ffn, tensor_id(l, 8)));
        else
            TRY(launch_gen_q4k_cols(y.wdown, c.hidden, nsb_f, sh.ffn_lo / QK_K, sh.ffn_hi / QK_K, s,
                                    tensor_id(l, 8), 0, flags, st));
    }
    const int B = m.batch;
    const size_t kv = static_cast<size_t>(B) * c.n_layers * sh.kv_heads * c.max_ctx * c.head_dim * 2;
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
    int64_t mx = c.hidden > ffn_l ? c.hidden : ffn_l;
    if (qd_l > mx) mx = qd_l;
    TRY(alloc(m, &m.h, static_cast<size_t>(B) * c.hidden * 4));
    TRY(alloc(m, &m.h2, static_cast<size_t>(B) * c.hidden * 4));
    TRY(alloc(m, &m.delta, static_cast<size_t>(B) * c.hidden * 4));
    TRY(alloc(m, &m.qkv, B * qkv_l * 4));
    TRY(alloc(m, &m.q, B * qd_l * 4));
    TRY(alloc(m, &m.att, B * qd_l * 4));
    TRY(alloc(m, &m.part_m, static_cast<size_t>(B) * sh.q_heads * m.max_chunks * 4));
    TRY(alloc(m, &m.part_l, static_cast<size_t>(B) * sh.q_heads * m.max_chunks * 4));
    TRY(alloc(m, &m.part_o, static_cast<size_t>(B) * sh.q_heads * m.max_chunks * c.head_dim * 4));
    TRY(alloc(m, &m.act, B * ffn_l * 4));
    TRY(alloc(m, &m.logits, static_cast<size_t>(B) * vocab_l * 4));
    TRY(alloc(m, &m.xq, B * (mx / QK8_1) * Q81_BYTES));
    TRY(alloc(m, &m.oq, B * (qd_l / QK8_1) * Q81_BYTES));
    TRY(alloc(m, &m.aq, B * (ffn_l / QK8_1) * Q81_BYTES));
    TRY(alloc(m, &m.tokens, static_cast<size_t>(B) * (c.max_ctx + 1) * 4));
    TRY(alloc(m, &m.picks, static_cast<size_t>(B) * (c.max_ctx + 1) * 4));
    if (B > 1) {
        TRY(alloc(m, &m.gbuf, B * ffn_l * 4));
        TRY(alloc(m, &m.ubuf, B * ffn_l * 4));
        int64_t ws = 8 * c.hidden;  // k-parts x rows of the K-split launches
        if (2 * ffn_l > ws) ws = 2 * ffn_l;
        if (2 * qkv_l > ws) ws = 2 * qkv_l;
        TRY(alloc(m, &m.tc_ws, static_cast<size_t>(B) * ws * 4));
    }
    TRY(alloc(m, &m.pos, 4));
    TRY(alloc(m, &m.nprompt, 4));
    TRY(alloc(m, &m.amax, 8));
    TRY(cudaMemsetAsync(m.amax, 0, 8, st));
    TRY(cudaMemsetAsync(m.tokens, 0, static_cast<size_t>(B) * (c.max_ctx + 1) * 4, st));
    TRY(cudaMemsetAsync(m.picks, 0, static_cast<size_t>(B) * (c.max_ctx + 1) * 4, st));
    TRY(cudaMemsetAsync(m.pos, 0, 4, st));
    TRY(cudaMemsetAsync(m.nprompt, 0, 4, st));
    if (B == 1 && sh.world == 1 && !m.mix && !(c.flags & ABRA_MODEL_KERNEL_CHAIN) &&
        persist_supported(c.hidden, c.n_heads, c.n_kv_heads, c.ffn, c.head_dim, nullptr)) {
        std::vector<PersistLayer> pl(c.n_layers);
        for (int l = 0; l < c.n_layers; ++l) {
            const LayerW &y = m.layers[l];
            pl[l] = {y.wqkv, y.wo, y.wgate, y.wup, y.wdown, y.attn_norm, y.q_norm, y.k_norm, y.ffn_norm};
        }
        if (c.n_layers > 0) {
            TRY(alloc(m, &m.players, pl.size() * sizeof(PersistLayer)));
            TRY(cudaMemcpyAsync(m.players, pl.data(), pl.size() * sizeof(PersistLayer),
                                cudaMemcpyHostToDevice, st));
        }
        const size_t sb = persist_sync_bytes(c.n_heads);
        TRY(alloc(m, reinterpret_cast<uint8_t **>(&m.psync), sb));
        TRY(cudaMemsetAsync(m.psync, 0, sb, st));
        m.persist = true;
    }
    if (sh.world > 1) {
        const size_t recv = static_cast<size_t>(2 * c.n_layers) * sh.world * B * c.hidden * 4;
        m.arena_recv = (recv + 255) / 256 * 256;
        m.arena_bytes = m.arena_recv + (static_cast<size_t>(4 * c.n_layers + 3 + B) * 8 + 255) / 256 * 256;
        TRY(cudaMalloc(&m.arena, m.arena_bytes));
        TRY(cudaMemsetAsync(m.arena, 0, m.arena_bytes, st));
        m.peer[sh.rank] = m.arena;
    }
    return cudaStreamSynchronize(st);
}

// One tensor of a GGUF file as a rank holds it: the ggml type of the slot,
// the whole tensor's N rows of K (rb bytes each), the rank's rows
// [r0, r0 + nr) and bytes [b0, b0 + nb) of each (nb == rb: whole rows), and
// where they go: buffer buf, after dst_row rows of nb bytes (the q|k|v rows
// share one buffer).  Row-split tensors (q, k, v, gate, up) keep the rank's
// heads or FFN units; K-split ones (o, down) its canonical K-slices of every
// row; the tied table and the norms are whole on every rank -- the placement
// build() gives the seeded weights.
enum : int {
    BUF_EMBD, BUF_OUT_NORM, BUF_ATTN_NORM, BUF_FFN_NORM, BUF_Q_NORM, BUF_K_NORM, BUF_WQKV, BUF_WV,
    BUF_WO, BUF_WGATE, BUF_WUP, BUF_WDOWN
};

struct TensorSlice {
    int type, buf;
    int64_t N, K, rb, r0, nr, b0, nb, dst_row;
};

static int tensor_slice(const abra_model_config &c, const abra_tp_shard &sh, bool mix, int layer,
                        int slot, TensorSlice &t) {
    const int64_t hd = c.head_dim, qd = static_cast<int64_t>(c.n_heads) * hd;
    const int64_t kvd = static_cast<int64_t>(c.n_kv_heads) * hd;
    const int64_t qd_l = sh.q_heads * hd, kvd_l = sh.kv_heads * hd;
    const int nsb_o = static_cast<int>(qd / QK_K);
    auto block = [](int type) -> int64_t { return type == ABRA_GGML_Q6_K ? 210 : Q4K_BYTES; };
    auto rows = [&](int buf, int type, int64_t n, int64_t k, int64_t lo, int64_t cnt, int64_t at) {
        t.buf = buf;
        t.type = type;
        t.N = n;
        t.K = k;
        t.rb = k / QK_K * block(type);
        t.r0 = lo;
        t.nr = cnt;
        t.b0 = 0;
        t.nb = t.rb;
        t.dst_row = at;
    };
    auto f32 = [&](int buf, int64_t n) {
        t.buf = buf;
        t.type = ABRA_GGML_F32;
        t.N = 1;
        t.K = n;
        t.rb = t.nb = n * 4;
        t.r0 = t.b0 = t.dst_row = 0;
        t.nr = 1;
    };
    if (layer == -1) {
        if (slot == ABRA_TENSOR_TOKEN_EMBD)
            rows(BUF_EMBD, mix ? ABRA_GGML_Q6_K : ABRA_GGML_Q4_K, c.vocab, c.hidden, 0, c.vocab, 0);
        else if (slot == ABRA_TENSOR_OUTPUT_NORM)
            f32(BUF_OUT_NORM, c.hidden);
        else
            return ABRA_E_INVALID;
        return ABRA_OK;
    }
    if (layer < 0 || layer >= c.n_layers) return ABRA_E_INVALID;
    const bool q6 = mix && q6k_layer(layer, c.n_layers);
    switch (slot) {
        case ABRA_TENSOR_ATTN_NORM: f32(BUF_ATTN_NORM, c.hidden); break;
        case ABRA_TENSOR_FFN_NORM: f32(BUF_FFN_NORM, c.hidden); break;
        case ABRA_TENSOR_ATTN_Q_NORM: f32(BUF_Q_NORM, hd); break;
        case ABRA_TENSOR_ATTN_K_NORM: f32(BUF_K_NORM, hd); break;
        case ABRA_TENSOR_ATTN_Q:
            rows(BUF_WQKV, ABRA_GGML_Q4_K, qd, c.hidden, sh.q_head_lo * hd, qd_l, 0);
            break;
        case ABRA_TENSOR_ATTN_K:
            rows(BUF_WQKV, ABRA_GGML_Q4_K, kvd, c.hidden, sh.kv_head_lo * hd, kvd_l, qd_l);
            break;
        case ABRA_TENSOR_ATTN_V:
            if (q6)
                rows(BUF_WV, ABRA_GGML_Q6_K, kvd, c.hidden, sh.kv_head_lo * hd, kvd_l, 0);
            else
                rows(BUF_WQKV, ABRA_GGML_Q4_K, kvd, c.hidden, sh.kv_head_lo * hd, kvd_l, qd_l + kvd_l);
            break;
        case ABRA_TENSOR_ATTN_OUTPUT:  // this rank's canonical K-slices of every row
            rows(BUF_WO, ABRA_GGML_Q4_K, c.hidden, qd, 0, c.hidden, 0);
            t.b0 = slice_start(nsb_o, sh.sl_base) * Q4K_BYTES;
            t.nb = slice_start(nsb_o, sh.sl_base + sh.sl_cnt) * Q4K_BYTES - t.b0;
            break;
        case ABRA_TENSOR_FFN_GATE:
        case ABRA_TENSOR_FFN_UP:
            rows(slot == ABRA_TENSOR_FFN_GATE ? BUF_WGATE : BUF_WUP, ABRA_GGML_Q4_K, c.ffn, c.hidden,
                 sh.ffn_lo, sh.ffn_hi - sh.ffn_lo, 0);
            break;
        case ABRA_TENSOR_FFN_DOWN: {
            const int type = q6 ? ABRA_GGML_Q6_K : ABRA_GGML_Q4_K;
            rows(BUF_WDOWN, type, c.hidden, c.ffn, 0, c.hidden, 0);
            t.b0 = sh.ffn_lo / QK_K * block(type);
            t.nb = (sh.ffn_hi - sh.ffn_lo) / QK_K * block(type);
            break;
        }
        default: return ABRA_E_INVALID;
    }
    return ABRA_OK;
}

// Local MMVQ shapes of one rank: {N, K, nmat, fused RMSNorm input}; qk is
// the q|k-only fused MMVQ of a Q6_K-V layer, v its Q6_K V rows.
struct StepShapes {
    int64_t qkv[4], o[4], gate_up[4], down[4], out[4], qk[4], v[4];
};

static StepShapes step_shapes(const abra_model_config &c, const abra_tp_shard &sh) {
    const int64_t hd = c.head_dim;
    const int64_t qkv_l = (sh.q_heads + 2 * sh.kv_heads) * hd, qd_l = sh.q_heads * hd;
    const int64_t ffn_l = sh.ffn_hi - sh.ffn_lo, vocab_l = sh.vocab_hi - sh.vocab_lo;
    const int64_t kvd_l = sh.kv_heads * hd;
    return {{qkv_l, c.hidden, 1, 1}, {c.hidden, qd_l, 1, 0}, {ffn_l, c.hidden, 2, 1},
            {c.hidden, ffn_l, 1, 0}, {vocab_l, c.hidden, 1, 1}, {qkv_l - kvd_l, c.hidden, 1, 1},
            {kvd_l, c.hidden, 1, 0}};
}

static const MmvqConfig *tuned(const int64_t sh[4]) {
    return mmvq_candidate_by_id(abra_tune_get(sh[0], sh[1], 1, static_cast<int>(sh[2])));
}

static const MmvqConfig *tuned6(const int64_t sh[4]) {
    return q6k_candidate_by_id(abra_q6k_tune_get(sh[0], sh[1], 1));
}

// The batched step (batch 32): every GEMV on the tensor cores with all
// sequences as its 32 columns; the column-wise kernels take the sequence as
// a grid dimension.  Per sequence the arithmetic is the batch-1 step's,
// kernel for kernel, so the logits are the same bits.
static cudaError_t record_step_batched(const Model &m, cudaStream_t st) {
    const abra_model_config &c = m.cfg;
    const abra_tp_shard &sh = m.sh;
    const int B = m.batch, L = c.n_layers, W = sh.world;
    const bool tp = W > 1;
    const bool pdl = (c.flags & ABRA_MODEL_NO_PDL) == 0;
    const int pf = pdl ? MMVQ_PDL : 0;
    const int64_t hd = c.head_dim;
    const int64_t qd = static_cast<int64_t>(sh.q_heads) * hd;  // this rank's q heads
    const int64_t qkv_rows = static_cast<int64_t>(sh.q_heads + 2 * sh.kv_heads) * hd;
    const int64_t ffn = sh.ffn_hi - sh.ffn_lo, vocab = sh.vocab_hi - sh.vocab_lo;
    const size_t kv_layer = static_cast<size_t>(sh.kv_heads) * c.max_ctx * c.head_dim;
    const int64_t tok_stride = c.max_ctx + 1;
    const float scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(c.head_dim)));
    SeqStrides sb;
    sb.batch = B;
    sb.qkv = qkv_rows;
    sb.q = qd;
    sb.kv = static_cast<int64_t>(L) * kv_layer;
    DeltaSet none = {}, one = {};
    one.p[0] = m.delta;
    one.G = 1;
    auto tc = [&](const void *w, const void *x, float *y, int64_t N, int64_t K, int ks) {
        return launch_mmvq_tc(w, x, y, N, K, N, ks, m.tc_ws, pf, st);
    };
    // Tensor parallel: o and down are K-sharded on canonical slices, so a
    // rank's output is the subtree over its k-parts sl_base .. sl_base +
    // sl_cnt - 1 of the 8-way split; it is pushed into slot `slot` of every
    // rank's arena, and the next residual + RMSNorm waits for all W and adds
    // them in the fixed tree (bit-identical to one GPU)
    auto kshard = [&](const void *w, const void *x, int64_t K, int nsb_full, int slot) {
        TcOpts o;
        o.nsb_sl = nsb_full;
        o.sb_base = slice_start(nsb_full, sh.sl_base);
        o.part = sh.sl_base;
        o.nparts = sh.sl_cnt;
        o.npeer = W;
        for (int q = 0; q < W; ++q) {
            o.peer_y[q] = m.recv_of(m.peer[q], sh.rank, slot);
            o.peer_cnt[q] = m.cnt_of(m.peer[q], slot);
        }
        o.cta_cnt = m.cta_cnt(slot);
        return launch_mmvq_tc(w, x, nullptr, c.hidden, K, c.hidden, 8, m.tc_ws, pf, st, &o);
    };
    auto slot_deltas = [&](int slot) {
        DeltaSet d = {};
        d.G = W;
        for (int q = 0; q < W; ++q) d.p[q] = m.recv(q, slot);
        return d;
    };
    auto resnorm = [&](const DeltaSet &ds, const float *norm, int wait_slot) {
        if (tp && wait_slot >= 0)
            return launch_residual_rmsnorm_quant(m.h, slot_deltas(wait_slot), norm, c.eps, m.xq, c.hidden, B,
                                                 pdl, st, m.cnt_of(m.arena, wait_slot), m.epoch(),
                                                 static_cast<unsigned long long>(W));
        return launch_residual_rmsnorm_quant(m.h, ds, norm, c.eps, m.xq, c.hidden, B, pdl, st);
    };
    TRY(launch_embed(m.embd, c.hidden, m.tokens, m.pos, m.h, pdl, st, B, tok_stride));
    for (int l = 0; l < L; ++l) {
        const LayerW &y = m.layers[l];
        TRY(resnorm(l == 0 ? none : one, y.attn_norm, l == 0 ? -1 : 2 * l - 1));
        TRY(tc(y.wqkv, m.xq, m.qkv, qkv_rows, c.hidden, 2));
        TRY(launch_qk_norm_rope_kv(m.qkv, y.q_norm, y.k_norm, c.eps, m.rope, m.pos, m.q,
                                   m.kc + l * kv_layer, m.vc + l * kv_layer, sh.q_heads, sh.kv_heads,
                                   c.max_ctx, pdl, st, sb));
        TRY(launch_attention(m.q, m.kc + l * kv_layer, m.vc + l * kv_layer, m.pos, scale, sh.q_heads,
                             sh.kv_heads, c.max_ctx, m.part_m, m.part_l, m.part_o, m.att, m.oq, pdl,
                             st, sb));
        if (tp)
            TRY(kshard(y.wo, m.oq, qd, static_cast<int>(c.n_heads * hd / QK_K), 2 * l));
        else
            TRY(tc(y.wo, m.oq, m.delta, c.hidden, qd, 8));
        TRY(resnorm(one, y.ffn_norm, 2 * l));
        TRY(tc(y.wgate, m.xq, m.gbuf, ffn, c.hidden, 2));
        TRY(tc(y.wup, m.xq, m.ubuf, ffn, c.hidden, 2));
        TRY(launch_swiglu_quant(m.gbuf, m.ubuf, m.aq, static_cast<int64_t>(B) * ffn, pdl, st));
        if (tp)
            TRY(kshard(y.wdown, m.aq, ffn, c.ffn / QK_K, 2 * l + 1));
        else
            TRY(tc(y.wdown, m.aq, m.delta, c.hidden, ffn, 8));
    }
    TRY(resnorm(L > 0 ? one : none, m.out_norm, L > 0 ? 2 * L - 1 : -1));
    const size_t row_h = q4k_bytes(1, c.hidden);
    TRY(tc(m.embd + static_cast<size_t>(sh.vocab_lo) * row_h, m.xq, m.logits, vocab, c.hidden, 1));
    if (!tp)
        return launch_argmax_batch(m.logits, c.vocab, c.vocab, m.tokens, m.picks, tok_stride, m.pos,
                                   m.nprompt, c.max_ctx, B, pdl, st);
    // each rank's per-sequence keys meet in every rank's key words
    TpKeyPush push = {};
    push.npeer = W;
    for (int q = 0; q < W; ++q) {
        push.key[q] = m.key_of(m.peer[q]);
        push.cnt[q] = m.cnt_of(m.peer[q], 2 * L);
    }
    push.cta_cnt = m.cta_cnt(2 * L);
    TRY(launch_argmax_keys_batch(m.logits, static_cast<int>(vocab), vocab, static_cast<int>(sh.vocab_lo), push, B,
                                 pdl, st));
    return launch_argmax_finish_batch(m.key_of(m.arena), B, m.tokens, m.picks, tok_stride, m.pos, m.nprompt,
                                      c.max_ctx, m.cnt_of(m.arena, 2 * L), m.epoch(),
                                      static_cast<unsigned long long>(W), pdl, st);
}

// Prefill: the P prompt tokens at tokens[*pos .. *pos + P) of the batch-1
// model as P columns -- every GEMV on the tensor cores (32 columns per
// launch), RoPE, the KV append and attention with column b at position
// *pos + b of the model's one KV cache (causal: column b attends to positions
// <= *pos + b, all written by the same RoPE/KV launch before the attention
// launch).  Per column the arithmetic is the decode step's, kernel for
// kernel, so the cache holds the bits token-by-token decoding writes.  No
// logits: the last prompt token goes through the decode step.
constexpr int kPrefillMax = 256;

static cudaError_t record_layers(const Model &m, int P, cudaStream_t st) {
    const abra_model_config &c = m.cfg;
    const int L = c.n_layers;
    const bool pdl = (c.flags & ABRA_MODEL_NO_PDL) == 0;
    const int pf = pdl ? MMVQ_PDL : 0;
    const int64_t hd = c.head_dim, qd = c.n_heads * hd;
    const int64_t qkv_rows = (c.n_heads + 2 * c.n_kv_heads) * hd;
    const size_t kv_layer = static_cast<size_t>(c.n_kv_heads) * c.max_ctx * c.head_dim;
    const float scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(c.head_dim)));
    SeqStrides sb;
    sb.batch = P;
    sb.qkv = qkv_rows;
    sb.q = qd;
    sb.kv = 0;
    sb.pos = 1;
    DeltaSet none = {}, one = {};
    one.p[0] = m.pdelta;
    one.G = 1;
    // y[c][n] = W x[c] for the P columns, 32 at a time
    auto tc = [&](const void *w, const uint8_t *x, float *y, int64_t N, int64_t K, int ks) -> cudaError_t {
        const int64_t xcol = K / QK8_1 * Q81_BYTES;
        for (int t = 0; t < P / 32; ++t)
            TRY(launch_mmvq_tc(w, x + t * 32 * xcol, y + t * 32 * N, N, K, N, ks, m.pws, pf, st));
        return cudaSuccess;
    };
    TRY(launch_embed(m.embd, c.hidden, m.tokens, m.pos, m.ph, pdl, st, P, 1));
    for (int l = 0; l < L; ++l) {
        const LayerW &y = m.layers[l];
        TRY(launch_residual_rmsnorm_quant(m.ph, l == 0 ? none : one, y.attn_norm, c.eps, m.pxq, c.hidden,
                                          P, pdl, st));
        TRY(tc(y.wqkv, m.pxq, m.pqkv, qkv_rows, c.hidden, 2));
        TRY(launch_qk_norm_rope_kv(m.pqkv, y.q_norm, y.k_norm, c.eps, m.rope, m.pos, m.pq,
                                   m.kc + l * kv_layer, m.vc + l * kv_layer, c.n_heads, c.n_kv_heads,
                                   c.max_ctx, pdl, st, sb));
        TRY(launch_attention(m.pq, m.kc + l * kv_layer, m.vc + l * kv_layer, m.pos, scale, c.n_heads,
                             c.n_kv_heads, c.max_ctx, m.ppart_m, m.ppart_l, m.ppart_o, nullptr, m.poq,
                             pdl, st, sb));
        TRY(tc(y.wo, m.poq, m.pdelta, c.hidden, qd, 8));
        TRY(launch_residual_rmsnorm_quant(m.ph, one, y.ffn_norm, c.eps, m.pxq, c.hidden, P, pdl, st));
        TRY(tc(y.wgate, m.pxq, m.pg, c.ffn, c.hidden, 2));
        TRY(tc(y.wup, m.pxq, m.pu, c.ffn, c.hidden, 2));
        TRY(launch_swiglu_quant(m.pg, m.pu, m.paq, static_cast<int64_t>(P) * c.ffn, pdl, st));
        TRY(tc(y.wdown, m.paq, m.pdelta, c.hidden, c.ffn, 8));
    }
    return cudaSuccess;
}

static cudaError_t record_prefill(const Model &m, int P, cudaStream_t st) {
    TRY(record_layers(m, P, st));
    return launch_pos_advance(m.pos, P, m.cfg.max_ctx, (m.cfg.flags & ABRA_MODEL_NO_PDL) == 0, st);
}

// Verification of draft tokens (prompt-lookup decoding): the 32 tokens at
// tokens[*pos .. *pos + 32) as one prefill chunk, then the final residual +
// RMSNorm + Q8_1, the tied output GEMV for all 32 columns on the tensor
// cores and each column's greedy pick into vpick.  Position and history are
// committed by the host (abra_model_verify), which knows how many drafts
// held.  Per column the logits are the decode step's bits.
static cudaError_t record_verify(const Model &m, cudaStream_t st) {
    const abra_model_config &c = m.cfg;
    const bool pdl = (c.flags & ABRA_MODEL_NO_PDL) == 0;
    TRY(record_layers(m, 32, st));
    DeltaSet none = {}, one = {};
    one.p[0] = m.pdelta;
    one.G = 1;
    TRY(launch_residual_rmsnorm_quant(m.ph, c.n_layers > 0 ? one : none, m.out_norm, c.eps, m.pxq,
                                      c.hidden, 32, pdl, st));
    TRY(launch_mmvq_tc(m.embd, m.pxq, m.plogits, c.vocab, c.hidden, c.vocab, 1, nullptr,
                       pdl ? MMVQ_PDL : 0, st));
    return launch_argmax_cols(m.plogits, c.vocab, c.vocab, m.vpick, 32, pdl, st);
}

static cudaError_t prefill_buffers(Model &m) {
    if (m.vhost) return cudaSuccess;  // the last allocation: all of them are in place
    const abra_model_config &c = m.cfg;
    const int64_t P = kPrefillMax, hd = c.head_dim, qd = c.n_heads * hd;
    const int64_t qkv_rows = (c.n_heads + 2 * c.n_kv_heads) * hd;
    int64_t mx = c.hidden > c.ffn ? c.hidden : c.ffn;
    if (qd > mx) mx = qd;
    TRY(alloc(m, &m.ph, P * c.hidden * 4));
    TRY(alloc(m, &m.pdelta, P * c.hidden * 4));
    TRY(alloc(m, &m.pqkv, P * qkv_rows * 4));
    TRY(alloc(m, &m.pq, P * qd * 4));
    TRY(alloc(m, &m.pg, P * c.ffn * 4));
    TRY(alloc(m, &m.pu, P * c.ffn * 4));
    TRY(alloc(m, &m.ppart_m, P * c.n_heads * m.max_chunks * 4));
    TRY(alloc(m, &m.ppart_l, P * c.n_heads * m.max_chunks * 4));
    TRY(alloc(m, &m.ppart_o, P * c.n_heads * m.max_chunks * c.head_dim * 4));
    TRY(alloc(m, &m.pxq, P * (mx / QK8_1) * Q81_BYTES));
    TRY(alloc(m, &m.poq, P * (qd / QK8_1) * Q81_BYTES));
    TRY(alloc(m, &m.paq, P * (c.ffn / QK8_1) * Q81_BYTES));
    int64_t ws = 8 * c.hidden;  // k-parts x rows of the K-split launches
    if (2 * c.ffn > ws) ws = 2 * c.ffn;
    if (2 * qkv_rows > ws) ws = 2 * qkv_rows;
    TRY(alloc(m, &m.pws, 32 * ws * 4));
    TRY(alloc(m, &m.plogits, static_cast<size_t>(32) * c.vocab * 4));
    TRY(alloc(m, &m.vpick, 32 * 4));
    TRY(prepare_mmvq_tc());
    return cudaHostAlloc(reinterpret_cast<void **>(&m.vhost), 64 * sizeof(int32_t), cudaHostAllocDefault);
}

// Prompt-lookup draft (the reference's draft(), tests/lookup_decode.cpp:39-51):
// the most recent earlier occurrence of the last `key` tokens of the history,
// scanning back from history.size() - 2 key, proposes the up to `limit`
// tokens that followed it.
static int lookup_draft(const int32_t *h, int n, int key, int limit, int32_t *out) {
    if (limit <= 0 || key < 1 || n < 2 * key) return 0;
    const int suffix = n - key;
    for (int pos = suffix - key; pos >= 0; --pos) {
        if (std::equal(h + pos, h + pos + key, h + suffix)) {
            const int cnt = std::min(limit, suffix - pos - key);
            for (int j = 0; j < cnt; ++j) out[j] = h[pos + key + j];
            return cnt > 0 ? cnt : 0;
        }
    }
    return 0;
}

static PersistModel persist_model(const Model &m) {
    const abra_model_config &c = m.cfg;
    PersistModel pm = {};
    pm.n_layers = c.n_layers;
    pm.hidden = c.hidden;
    pm.n_heads = c.n_heads;
    pm.n_kv = c.n_kv_heads;
    pm.ffn = c.ffn;
    pm.vocab = c.vocab;
    pm.max_ctx = c.max_ctx;
    pm.eps = c.eps;
    pm.layers = m.players;
    pm.embd = m.embd;
    pm.out_norm = m.out_norm;
    pm.h0 = m.h;
    pm.h1 = m.h2;
    pm.delta = m.delta;
    pm.qkv = m.qkv;
    pm.att = m.att;
    pm.part_m = m.part_m;
    pm.part_l = m.part_l;
    pm.part_o = m.part_o;
    pm.act = m.act;
    pm.logits = m.logits;
    pm.oq = m.oq;
    pm.kc = m.kc;
    pm.vc = m.vc;
    pm.rope = m.rope;
    pm.tokens = m.tokens;
    pm.picks = m.picks;
    pm.pos = m.pos;
    pm.nprompt = m.nprompt;
    pm.amax = m.amax;
    pm.sync = m.psync;
    return pm;
}

// The decode step for the token at tokens[*pos] (recorded into the graph).
static cudaError_t record_step(const Model &m, cudaStream_t st) {
    if (m.batch > 1) return record_step_batched(m, st);
    if (m.persist) return launch_persist_step(persist_model(m), st);
    const abra_model_config &c = m.cfg;
    const abra_tp_shard &sh = m.sh;
    const int W = sh.world;
    const bool tp = W > 1;
    const bool pdl = (c.flags & ABRA_MODEL_NO_PDL) == 0;
    const int pf = pdl ? MMVQ_PDL : 0;
    const StepShapes ss = step_shapes(c, sh);
    const size_t kv_layer = static_cast<size_t>(sh.kv_heads) * c.max_ctx * c.head_dim;
    const float scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(c.head_dim)));
    const int L = c.n_layers;
    DeltaSet none = {}, one = {};
    none.G = 0;
    one.p[0] = m.delta;
    one.G = 1;
    // K-sharded outputs (o, down) of every rank land in slot 2l / 2l+1 of
    // each rank's arena; the consumer sums them in the canonical tree
    auto slot_deltas = [&](int slot) {
        DeltaSet d = {};
        d.G = W;
        for (int q = 0; q < W; ++q) d.p[q] = m.recv(q, slot);
        return d;
    };
    MmvqOpts kshard;  // slicing of this rank's o / down K-shard
    kshard.sl_nsb = 0;
    if (tp) {
        kshard.sl_base = sh.sl_base;
        kshard.sl_cnt = sh.sl_cnt;
    }
    MmvqOpts proto_o = kshard, proto_down = kshard;
    proto_o.sl_nsb = static_cast<int>(c.n_heads * c.head_dim / QK_K);
    proto_down.sl_nsb = c.ffn / QK_K;
    // each rank's launch publishes once per step (its last CTA)
    const int64_t per_o = W, per_down = W, per_out = W;
    auto push_to = [&](MmvqOpts &t, int slot) {
        t.npeer = W;
        t.cta_cnt = m.cta_cnt(slot);
        for (int q = 0; q < W; ++q) {
            t.peer_y[q] = reinterpret_cast<float *>(m.peer[q]) +
                          (static_cast<size_t>(slot) * W + sh.rank) * c.hidden;
            t.peer_cnt[q] = m.cnt_of(m.peer[q], slot);
        }
    };
    auto wait_on = [&](MmvqOpts &t, int slot, int64_t per_step) {
        t.wait_cnt = m.cnt_of(m.arena, slot);
        t.epoch = m.epoch();
        t.wait_per_step = static_cast<unsigned long long>(per_step);
    };
    // residual stream ping-pong: every MMVQ with a fused RMSNorm prologue
    // reads h[cur] (+ the pending deltas) and CTA 0 writes the sum to h[cur^1]
    float *h[2] = {m.h, m.h2};
    int cur = 0;
    auto fused = [&](const void *w, const void *w2, const DeltaSet &ds, const float *norm,
                     float *y, const int64_t shp[4], unsigned long long *amax,
                     const MmvqOpts *t, uint8_t *x_out = nullptr) -> cudaError_t {
        const MmvqConfig *cfg = tuned(shp);
        if (!cfg) return cudaErrorInvalidValue;
        MmvqXin xin = {h[cur], h[cur ^ 1], ds, norm, c.eps, x_out};
        cur ^= 1;
        return launch_mmvq_q4k_xin(*cfg, w, w2, xin, y, shp[0], shp[1], pf, st, amax, t);
    };
    // Q6_K MMVQ (the Q4_K_M type map; unsharded)
    auto plain6 = [&](const void *w, const void *x, float *y, const int64_t shp[4],
                      unsigned long long *amax, const MmvqOpts *t) -> cudaError_t {
        const MmvqConfig *cfg = tuned6(shp);
        if (!cfg) return cudaErrorInvalidValue;
        return launch_mmvq_q6k(*cfg, w, x, y, shp[0], shp[1], 1, shp[0], pf, st, amax, t);
    };
    auto plain = [&](const void *w, const void *x, float *y, const int64_t shp[4],
                     const MmvqOpts *t) -> cudaError_t {
        const MmvqConfig *cfg = tuned(shp);
        if (!cfg) return cudaErrorInvalidValue;
        return launch_mmvq_q4k(*cfg, w, nullptr, x, y, shp[0], shp[1], 1, shp[0], pf, st, nullptr, t);
    };
    // Each MMVQ streams the next MMVQ's weights into L2 while it runs (it is
    // latency-bound, so HBM has room): q|k|v -> o -> gate, up -> down -> the
    // next layer's q|k|v (after the last layer: the head of this rank's output
    // rows; after the output: layer 0's q|k|v of the next token).
    const bool prefetch = (c.flags & ABRA_MODEL_NO_PREFETCH) == 0;
    const size_t row_h = m.mix ? q6k_bytes(1, c.hidden) : q4k_bytes(1, c.hidden);
    auto bytes_of = [&](const int64_t shp[4], bool q6 = false) {
        return static_cast<int64_t>(q6 ? q6k_bytes(shp[0], shp[1]) : q4k_bytes(shp[0], shp[1]));
    };
    const int64_t qkv_bytes0 = L > 0 ? bytes_of(m.layers[0].q6 ? ss.qk : ss.qkv) : 0;
    const uint8_t *out_w = m.embd + static_cast<size_t>(sh.vocab_lo) * row_h;
    const int64_t out_head = std::min<int64_t>(bytes_of(ss.out, m.mix), int64_t(32) << 20) / 16 * 16;
    auto next_of = [&](MmvqOpts &t, const void *a, int64_t na, const void *b = nullptr,
                       int64_t nb = 0) {
        if (!prefetch) return;
        t.pf_ptr[0] = a;
        t.pf_bytes[0] = na;
        t.pf_ptr[1] = b;
        t.pf_bytes[1] = nb;
    };
    if (m.mix)
        TRY(launch_embed_q6k(m.embd, c.hidden, m.tokens, m.pos, h[cur], pdl, st));
    else
        TRY(launch_embed(m.embd, c.hidden, m.tokens, m.pos, h[cur], pdl, st));
    for (int l = 0; l < L; ++l) {
        const LayerW &y = m.layers[l];
        // residual + RMSNorm + Q8_1 fused into the q|k|v MMVQ
        MmvqOpts tq;
        if (tp && l > 0) wait_on(tq, 2 * l - 1, per_down);
        next_of(tq, y.wo, bytes_of(ss.o));
        const DeltaSet &dq = l == 0 ? none : (tp ? slot_deltas(2 * l - 1) : one);
        if (y.q6) {  // q|k, exporting the Q8_1 activation, then the Q6_K V rows
            TRY(fused(y.wqkv, nullptr, dq, y.attn_norm, m.qkv, ss.qk, nullptr, &tq, m.xq));
            TRY(plain6(y.wv, m.xq, m.qkv + ss.qk[0], ss.v, nullptr, nullptr));
        } else {
            TRY(fused(y.wqkv, nullptr, dq, y.attn_norm, m.qkv, ss.qkv, nullptr, &tq));
        }
        TRY(launch_qk_norm_rope_kv(m.qkv, y.q_norm, y.k_norm, c.eps, m.rope, m.pos, m.q,
                                   m.kc + l * kv_layer, m.vc + l * kv_layer, sh.q_heads,
                                   sh.kv_heads, c.max_ctx, pdl, st));
        TRY(launch_attention(m.q, m.kc + l * kv_layer, m.vc + l * kv_layer, m.pos, scale,
                             sh.q_heads, sh.kv_heads, c.max_ctx, m.part_m, m.part_l, m.part_o,
                             m.att, m.oq, pdl, st));
        MmvqOpts to = tp ? proto_o : MmvqOpts();
        if (tp) push_to(to, 2 * l);
        next_of(to, y.wgate, bytes_of(ss.gate_up), y.wup, bytes_of(ss.gate_up));
        TRY(plain(y.wo, m.oq, m.delta, ss.o, &to));
        // residual + RMSNorm + Q8_1 fused into the gate/up SwiGLU MMVQ
        MmvqOpts tg;
        if (tp) wait_on(tg, 2 * l, per_o);
        next_of(tg, y.wdown, bytes_of(ss.down, y.q6));
        TRY(fused(y.wgate, y.wup, tp ? slot_deltas(2 * l) : one, y.ffn_norm, m.act, ss.gate_up,
                  nullptr, &tg));
        TRY(launch_quantize_q8_1(m.act, m.aq, ss.gate_up[0], 1, st));
        MmvqOpts td = tp ? proto_down : MmvqOpts();
        if (tp) push_to(td, 2 * l + 1);
        if (l + 1 < L)
            next_of(td, m.layers[l + 1].wqkv, bytes_of(m.layers[l + 1].q6 ? ss.qk : ss.qkv));
        else
            next_of(td, out_w, out_head);
        if (y.q6)
            TRY(plain6(y.wdown, m.aq, m.delta, ss.down, nullptr, &td));
        else
            TRY(plain(y.wdown, m.aq, m.delta, ss.down, &td));
    }
    // final residual + RMSNorm fused into the tied output MMVQ over this
    // rank's vocab rows, which also reduces the greedy argmax (ties to the
    // lowest id); with TP every rank's keys meet in every rank's key word
    if (!tp) {
        MmvqOpts t1;
        if (L > 0) next_of(t1, m.layers[0].wqkv, qkv_bytes0);
        if (m.mix) {  // Q6_K table: standalone residual + RMSNorm + Q8_1, then the MMVQ
            TRY(launch_residual_rmsnorm_quant(h[cur], L > 0 ? one : none, m.out_norm, c.eps, m.xq,
                                              c.hidden, 1, pdl, st));
            TRY(plain6(m.embd, m.xq, m.logits, ss.out, m.amax, &t1));
        } else {
            TRY(fused(m.embd, nullptr, L > 0 ? one : none, m.out_norm, m.logits, ss.out, m.amax, &t1));
        }
        return launch_argmax_finish(m.amax, m.tokens, m.picks, m.pos, m.nprompt, c.max_ctx, pdl, st);
    }
    // this rank's CTAs reduce into the local key m.amax; the last one
    // forwards it to every rank's combined key
    MmvqOpts tout;
    tout.row_offset = static_cast<int>(sh.vocab_lo);
    tout.npeer = W;
    tout.cta_cnt = m.cta_cnt(2 * L);
    for (int q = 0; q < W; ++q) {
        tout.peer_amax[q] = m.key_of(m.peer[q]);
        tout.peer_cnt[q] = m.cnt_of(m.peer[q], 2 * L);
    }
    if (L > 0) wait_on(tout, 2 * L - 1, per_down);
    if (L > 0) next_of(tout, m.layers[0].wqkv, qkv_bytes0);
    TRY(fused(out_w, nullptr, L > 0 ? slot_deltas(2 * L - 1) : none, m.out_norm, m.logits, ss.out,
              m.amax, &tout));
    return launch_argmax_finish(m.key_of(m.arena), m.tokens, m.picks, m.pos, m.nprompt, c.max_ctx,
                                pdl, st, m.cnt_of(m.arena, 2 * L), m.epoch(),
                                static_cast<unsigned long long>(per_out));
}

static cudaError_t prepare(const Model &m) {
    if (m.batch > 1) return prepare_mmvq_tc();
    if (m.persist) return persist_prepare(m.cfg.hidden, m.cfg.n_heads, m.cfg.n_kv_heads, m.cfg.ffn);
    const StepShapes ss = step_shapes(m.cfg, m.sh);
    for (const int64_t *sh : {ss.qkv, ss.o, ss.gate_up, ss.down, ss.out, ss.qk}) {
        const MmvqConfig *cfg = tuned(sh);
        if (!cfg) return cudaErrorInvalidValue;
        TRY(prepare_mmvq(*cfg, 1, static_cast<int>(sh[2]), sh[3] != 0));
    }
    if (m.mix) {
        for (const int64_t *sh : {ss.v, ss.down, ss.out}) {
            const MmvqConfig *cfg = tuned6(sh);
            if (!cfg) return cudaErrorInvalidValue;
            TRY(prepare_mmvq_q6k(*cfg, 1));
        }
    }
    return cudaSuccess;
}

static cudaError_t capture(Model &m) {
    if (m.graph) return cudaSuccess;
    TRY(prepare(m));  // kernel attributes are set outside the capture
    if ((m.cfg.flags & ABRA_MODEL_EAGER) || m.persist_eager) return cudaSuccess;
    cudaGraph_t g = nullptr;
    TRY(cudaStreamBeginCapture(m.stream, cudaStreamCaptureModeThreadLocal));
    cudaError_t e = record_step(m, m.stream);
    cudaError_t e2 = cudaStreamEndCapture(m.stream, &g);
    if (e != cudaSuccess || e2 != cudaSuccess) {
        if (g) cudaGraphDestroy(g);
        if (m.persist) {  // a cooperative launch this driver cannot capture: launch it per step
            cudaGetLastError();
            m.persist_eager = true;
            return cudaSuccess;
        }
        return e != cudaSuccess ? e : e2;
    }
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

int abra_model_path(void *model, int32_t *persistent) {
    Model *m = static_cast<Model *>(model);
    if (!m || !persistent) return model_fail(ABRA_E_INVALID, "null pointer", cudaSuccess);
    *persistent = m->persist ? 1 : 0;
    return ABRA_OK;
}

int abra_persist_plan(const abra_model_config *cfg, int32_t sms, int64_t out[9]) {
    if (!cfg || !out || sms < 1) return model_fail(ABRA_E_INVALID, "bad arguments", cudaSuccess);
    const char *why = "";
    if (cfg->n_layers < 0 || cfg->vocab < 1 ||
        !abra::persist_plan_check(cfg->n_layers, cfg->hidden, cfg->n_heads, cfg->n_kv_heads, cfg->ffn,
                                  cfg->vocab, sms, out, &why))
        return model_fail(ABRA_E_UNSUPPORTED, why, cudaSuccess);
    return ABRA_OK;
}

int abra_tp_shard_info(const abra_model_config *cfg, int32_t rank, int32_t world,
                       abra_tp_shard *out) {
    if (!cfg || !out) return model_fail(ABRA_E_INVALID, "null pointer", cudaSuccess);
    const int rc = abra::tp_shard(*cfg, rank, world, *out);
    return rc == ABRA_OK ? ABRA_OK : model_fail(rc, "no tensor-parallel split of this configuration", cudaSuccess);
}

int abra_model_create(const abra_model_config *cfg, void **out) {
    return abra_model_create_tp(cfg, 0, 1, out);
}

static int create_model(const abra_model_config *cfg, int32_t rank, int32_t world, int32_t batch,
                        void **out);

int abra_model_create_tp(const abra_model_config *cfg, int32_t rank, int32_t world, void **out) {
    return create_model(cfg, rank, world, 1, out);
}

int abra_model_create_batched(const abra_model_config *cfg, int32_t batch, void **out) {
    if (batch != 1 && batch != 32) return model_fail(ABRA_E_UNSUPPORTED, "batch must be 1 or 32", cudaSuccess);
    return create_model(cfg, 0, 1, batch, out);
}

int abra_model_create_batched_tp(const abra_model_config *cfg, int32_t batch, int32_t rank, int32_t world,
                                 void **out) {
    if (batch != 1 && batch != 32) return model_fail(ABRA_E_UNSUPPORTED, "batch must be 1 or 32", cudaSuccess);
    return create_model(cfg, rank, world, batch, out);
}

static int create_model(const abra_model_config *cfg, int32_t rank, int32_t world, int32_t batch,
                        void **out) {
    if (!cfg || !out) return model_fail(ABRA_E_INVALID, "null pointer", cudaSuccess);
    const abra_model_config &c = *cfg;
    if (c.head_dim != 128 || c.n_heads <= 0 || c.n_kv_heads <= 0 || c.n_heads % c.n_kv_heads ||
        c.n_heads / c.n_kv_heads > 8 || c.hidden % 256 || c.ffn % 256 ||
        (c.n_heads * c.head_dim) % 256 || c.vocab <= 0 || c.max_ctx <= 0 || c.n_layers < 0 ||
        c.hidden > 16384)
        return model_fail(ABRA_E_UNSUPPORTED, "unsupported model configuration", cudaSuccess);
    if ((c.flags & ABRA_MODEL_Q4_K_M) && (world > 1 || batch > 1))
        return model_fail(ABRA_E_UNSUPPORTED, "the Q4_K_M type map runs on one GPU at batch 1", cudaSuccess);
    abra_tp_shard shard = {};
    const int src = abra::tp_shard(c, rank, world, shard);
    if (src != ABRA_OK) return model_fail(src, "no tensor-parallel split of this configuration", cudaSuccess);
    Model *m = new (std::nothrow) Model();
    if (!m) return model_fail(ABRA_E_INVALID, "out of host memory", cudaSuccess);
    m->cfg = c;
    m->sh = shard;
    m->batch = batch;
    m->connected = world == 1;
    cudaError_t e = cudaGetDevice(&m->device);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking);
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
    for (cudaGraphExec_t g : m->pgraph)
        if (g) cudaGraphExecDestroy(g);
    if (m->vgraph) cudaGraphExecDestroy(m->vgraph);
    if (m->vhost) cudaFreeHost(m->vhost);
    if (m->pinned) cudaFreeHost(m->pinned);
    for (int q = 0; q < m->sh.world; ++q)
        if (m->peer[q] && m->peer[q] != m->arena) cudaIpcCloseMemHandle(m->peer[q]);
    if (m->arena) cudaFree(m->arena);
    for (void *p : m->allocs) cudaFree(p);
    if (m->stream) cudaStreamDestroy(m->stream);
    delete m;
    return ABRA_OK;
}

int abra_model_tp_handle(void *model, void *handle, int32_t size) {
    Model *m = static_cast<Model *>(model);
    if (!m || !handle || size < static_cast<int32_t>(sizeof(cudaIpcMemHandle_t)))
        return model_fail(ABRA_E_INVALID, "bad arguments", cudaSuccess);
    if (!m->arena) return model_fail(ABRA_E_INVALID, "not a tensor-parallel model", cudaSuccess);
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, m->arena);
    if (e != cudaSuccess) return model_fail(ABRA_E_CUDA, "cudaIpcGetMemHandle", e);
    std::memcpy(handle, &h, sizeof h);
    return ABRA_OK;
}

int abra_model_tp_connect(void *model, const void *handles, int32_t size_each) {
    Model *m = static_cast<Model *>(model);
    if (!m || !handles || size_each < static_cast<int32_t>(sizeof(cudaIpcMemHandle_t)))
        return model_fail(ABRA_E_INVALID, "bad arguments", cudaSuccess);
    if (!m->arena || m->connected) return model_fail(ABRA_E_INVALID, "not a fresh tensor-parallel model", cudaSuccess);
    for (int q = 0; q < m->sh.world; ++q) {
        if (q == m->sh.rank) continue;
        cudaIpcMemHandle_t h;
        std::memcpy(&h, static_cast<const uint8_t *>(handles) + static_cast<size_t>(q) * size_each, sizeof h);
        void *p = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) return model_fail(ABRA_E_CUDA, "cudaIpcOpenMemHandle", e);
        m->peer[q] = static_cast<uint8_t *>(p);
    }
    m->connected = true;
    // record the step now, so that the ranks' first steps start together
    cudaError_t e = abra::capture(*m);
    return e == cudaSuccess ? ABRA_OK : model_fail(ABRA_E_CUDA, "graph capture", e);
}

int abra_model_reset_batched(void *model, const int32_t *prompts, int32_t n_prompt) {
    Model *m = static_cast<Model *>(model);
    if (!m || !prompts || n_prompt < 1 || n_prompt > m->cfg.max_ctx)
        return model_fail(ABRA_E_INVALID, "bad prompt", cudaSuccess);
    const int B = m->batch;
    for (int64_t i = 0; i < static_cast<int64_t>(B) * n_prompt; ++i)
        if (prompts[i] < 0 || prompts[i] >= m->cfg.vocab)
            return model_fail(ABRA_E_INVALID, "token id out of range", cudaSuccess);
    const int32_t zero = 0;
    const size_t stride = static_cast<size_t>(m->cfg.max_ctx) + 1;
    cudaError_t e = cudaSuccess;
    for (int b = 0; b < B && e == cudaSuccess; ++b)
        e = cudaMemcpyAsync(m->tokens + b * stride, prompts + static_cast<size_t>(b) * n_prompt,
                            n_prompt * 4, cudaMemcpyHostToDevice, m->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(m->pos, &zero, 4, cudaMemcpyHostToDevice, m->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(m->nprompt, &n_prompt, 4, cudaMemcpyHostToDevice, m->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
    if (e == cudaSuccess) {
        m->host_pos = 0;
        m->host_nprompt = n_prompt;
    }
    return e == cudaSuccess ? ABRA_OK : model_fail(ABRA_E_CUDA, "reset", e);
}

int abra_model_read_batched(void *model, int32_t *tokens, int32_t n_tokens, float *logits) {
    Model *m = static_cast<Model *>(model);
    if (!m || n_tokens < 0 || n_tokens > m->cfg.max_ctx + 1)
        return model_fail(ABRA_E_INVALID, "bad arguments", cudaSuccess);
    const size_t stride = static_cast<size_t>(m->cfg.max_ctx) + 1;
    cudaError_t e = cudaStreamSynchronize(m->stream);
    for (int b = 0; b < m->batch && e == cudaSuccess && tokens && n_tokens; ++b)
        e = cudaMemcpy(tokens + static_cast<size_t>(b) * n_tokens, m->tokens + b * stride, n_tokens * 4,
                       cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && logits)
        e = cudaMemcpy(logits, m->logits, static_cast<size_t>(m->batch) * (m->sh.vocab_hi - m->sh.vocab_lo) * 4,
                       cudaMemcpyDeviceToHost);
    return e == cudaSuccess ? ABRA_OK : model_fail(ABRA_E_CUDA, "read", e);
}

int abra_model_reset(void *model, const int32_t *prompt, int32_t n_prompt) {
    Model *m = static_cast<Model *>(model);
    if (!m || !prompt || n_prompt < 1 || n_prompt > m->cfg.max_ctx)
        return model_fail(ABRA_E_INVALID, "bad prompt", cudaSuccess);
    if (m->batch > 1) return model_fail(ABRA_E_INVALID, "batched model: use abra_model_reset_batched", cudaSuccess);
    for (int i = 0; i < n_prompt; ++i)
        if (prompt[i] < 0 || prompt[i] >= m->cfg.vocab)
            return model_fail(ABRA_E_INVALID, "token id out of range", cudaSuccess);
    const int32_t zero = 0;
    cudaError_t e = cudaMemcpyAsync(m->tokens, prompt, n_prompt * 4, cudaMemcpyHostToDevice, m->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(m->pos, &zero, 4, cudaMemcpyHostToDevice, m->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(m->nprompt, &n_prompt, 4, cudaMemcpyHostToDevice, m->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
    if (e == cudaSuccess) {
        m->host_pos = 0;
        m->host_nprompt = n_prompt;
    }
    return e == cudaSuccess ? ABRA_OK : model_fail(ABRA_E_CUDA, "reset", e);
}

int abra_model_prefill(void *model, int32_t n_tokens) {
    Model *m = static_cast<Model *>(model);
    if (!m || n_tokens < 0 || n_tokens % 32)
        return model_fail(ABRA_E_INVALID, "n_tokens must be a multiple of 32", cudaSuccess);
    if (m->batch > 1 || m->sh.world > 1 || m->mix)
        return model_fail(ABRA_E_UNSUPPORTED, "prefill runs on a one-GPU batch-1 all-Q4_K model", cudaSuccess);
    if (static_cast<int64_t>(m->host_pos) + n_tokens > static_cast<int64_t>(m->host_nprompt) - 1)
        return model_fail(ABRA_E_INVALID, "prefill must leave the last prompt token to a decode step", cudaSuccess);
    cudaError_t e = abra::prefill_buffers(*m);
    if (e != cudaSuccess) return model_fail(ABRA_E_CUDA, "prefill buffers", e);
    for (int done = 0; done < n_tokens;) {
        const int P = std::min(n_tokens - done, abra::kPrefillMax);
        cudaGraphExec_t &g = m->pgraph[P / 32 - 1];
        if (!g && !(m->cfg.flags & ABRA_MODEL_EAGER)) {
            cudaGraph_t gr = nullptr;
            e = cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal);
            if (e != cudaSuccess) return model_fail(ABRA_E_CUDA, "prefill capture", e);
            const cudaError_t e1 = abra::record_prefill(*m, P, m->stream);
            e = cudaStreamEndCapture(m->stream, &gr);
            if (e1 == cudaSuccess && e == cudaSuccess) e = cudaGraphInstantiate(&g, gr, 0);
            if (gr) cudaGraphDestroy(gr);
            if (e1 != cudaSuccess) e = e1;
            if (e != cudaSuccess) return model_fail(ABRA_E_CUDA, "prefill capture", e);
        }
        e = g ? cudaGraphLaunch(g, m->stream) : abra::record_prefill(*m, P, m->stream);
        if (e != cudaSuccess) return model_fail(ABRA_E_CUDA, "prefill launch", e);
        m->host_pos += P;
        done += P;
    }
    return ABRA_OK;
}

int abra_model_verify(void *model, const int32_t *draft, int32_t n_draft, int32_t *picks_out,
                      int32_t *kept_out) {
    Model *m = static_cast<Model *>(model);
    if (!m || n_draft < 0 || n_draft > 31 || (n_draft > 0 && !draft))
        return model_fail(ABRA_E_INVALID, "n_draft must be in 0..31", cudaSuccess);
    if (m->batch > 1 || m->sh.world > 1 || m->mix)
        return model_fail(ABRA_E_UNSUPPORTED, "verification runs on a one-GPU batch-1 all-Q4_K model", cudaSuccess);
    const int32_t p = m->host_pos;
    if (p < m->host_nprompt)
        return model_fail(ABRA_E_INVALID, "verify after the prompt: the current token must be a pick", cudaSuccess);
    if (static_cast<int64_t>(p) + 32 > m->cfg.max_ctx)
        return model_fail(ABRA_E_INVALID, "verification needs 32 positions below max_ctx", cudaSuccess);
    for (int j = 0; j < n_draft; ++j)
        if (draft[j] < 0 || draft[j] >= m->cfg.vocab)
            return model_fail(ABRA_E_INVALID, "token id out of range", cudaSuccess);
    cudaError_t e = abra::prefill_buffers(*m);
    if (e != cudaSuccess) return model_fail(ABRA_E_CUDA, "verify buffers", e);
    if (!m->vgraph && !(m->cfg.flags & ABRA_MODEL_EAGER)) {
        cudaGraph_t gr = nullptr;
        e = cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal);
        if (e != cudaSuccess) return model_fail(ABRA_E_CUDA, "verify capture", e);
        const cudaError_t e1 = abra::record_verify(*m, m->stream);
        e = cudaStreamEndCapture(m->stream, &gr);
        if (e1 == cudaSuccess && e == cudaSuccess) e = cudaGraphInstantiate(&m->vgraph, gr, 0);
        if (gr) cudaGraphDestroy(gr);
        if (e1 != cudaSuccess) e = e1;
        if (e != cudaSuccess) return model_fail(ABRA_E_CUDA, "verify capture", e);
    }
    int32_t *hp = m->vhost;  // [0, 32) picks, [32, 64) staging
    for (int j = 0; j < n_draft; ++j) hp[32 + j] = draft[j];
    if (n_draft > 0)
        e = cudaMemcpyAsync(m->tokens + p + 1, hp + 32, n_draft * 4, cudaMemcpyHostToDevice, m->stream);
    if (e == cudaSuccess) e = m->vgraph ? cudaGraphLaunch(m->vgraph, m->stream) : abra::record_verify(*m, m->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(hp, m->vpick, 32 * 4, cudaMemcpyDeviceToHost, m->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
    if (e != cudaSuccess) return model_fail(ABRA_E_CUDA, "verify", e);
    // keep the current token and every draft that equals the pick before it
    int kept = 1;
    while (kept - 1 < n_draft && hp[kept - 1] == draft[kept - 1]) ++kept;
    if (picks_out)
        for (int j = 0; j <= n_draft; ++j) picks_out[j] = hp[j];
    // commit as kept decode steps would: picks[p + j], the next token, *pos
    hp[32] = hp[kept - 1];
    hp[33] = p + kept;
    e = cudaMemcpyAsync(m->picks + p, hp, kept * 4, cudaMemcpyHostToDevice, m->stream);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(m->tokens + p + kept, hp + 32, 4, cudaMemcpyHostToDevice, m->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(m->pos, hp + 33, 4, cudaMemcpyHostToDevice, m->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
    if (e != cudaSuccess) return model_fail(ABRA_E_CUDA, "verify commit", e);
    m->host_pos = p + kept;
    if (kept_out) *kept_out = kept;
    return ABRA_OK;
}

int abra_lookup_draft(const int32_t *history, int32_t n, int32_t key, int32_t limit, int32_t *out) {
    if ((n > 0 && !history) || n < 0 || (limit > 0 && !out)) return ABRA_E_INVALID;
    return abra::lookup_draft(history, n, key, limit, out);
}

int abra_model_generate_lookup(void *model, const int32_t *prompt, int32_t n_prompt, int32_t n_gen,
                               int32_t key, int32_t draft_max, int32_t *out, int32_t *stats) {
    Model *m = static_cast<Model *>(model);
    if (!m || !prompt || !out || n_prompt < 1 || n_gen < 1 || key < 1 || draft_max < 0 || draft_max > 31 ||
        static_cast<int64_t>(n_prompt) + n_gen > m->cfg.max_ctx + 1)
        return model_fail(ABRA_E_INVALID, "bad arguments", cudaSuccess);
    if (m->batch > 1 || m->sh.world > 1 || m->mix)
        return model_fail(ABRA_E_UNSUPPORTED, "lookup decoding runs on a one-GPU batch-1 all-Q4_K model", cudaSuccess);
    int rc = abra_model_reset(model, prompt, n_prompt);
    const int n_pf = (n_prompt - 1) / 32 * 32;
    if (!rc && n_pf) rc = abra_model_prefill(model, n_pf);
    if (!rc) rc = abra_model_step(model, n_prompt - n_pf);
    if (rc) return rc;
    // the pick at the model's position, after the queued work on its stream
    auto read_current = [&](int32_t *v) {
        cudaError_t e = cudaMemcpyAsync(m->vhost ? m->vhost + 63 : v, m->tokens + m->host_pos, 4,
                                        cudaMemcpyDeviceToHost, m->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
        if (e == cudaSuccess && m->vhost) *v = m->vhost[63];
        return e;
    };
    int32_t current = 0;
    cudaError_t e = abra::prefill_buffers(*m);  // also the pinned staging words
    if (e == cudaSuccess) e = read_current(&current);
    if (e != cudaSuccess) return model_fail(ABRA_E_CUDA, "read pick", e);
    std::vector<int32_t> history(prompt, prompt + n_prompt), gen;
    int32_t cand[32], proposed = 0, accepted = 0, blocks = 0;
    while (static_cast<int>(gen.size()) < n_gen) {
        if (static_cast<int>(gen.size()) == n_gen - 1) {  // the last token is already picked
            gen.push_back(current);
            break;
        }
        history.push_back(current);
        const int limit = std::min(draft_max, n_gen - static_cast<int>(gen.size()) - 1);
        const int nc = abra::lookup_draft(history.data(), static_cast<int>(history.size()), key, limit, cand);
        ++blocks;
        if (nc == 0 || static_cast<int64_t>(m->host_pos) + 32 > m->cfg.max_ctx) {
            rc = abra_model_step(model, 1);  // no draft: one decode step
            if (rc) return rc;
            gen.push_back(current);
            e = read_current(&current);
            if (e != cudaSuccess) return model_fail(ABRA_E_CUDA, "read pick", e);
            continue;
        }
        int32_t picks[32], kept = 0;
        rc = abra_model_verify(model, cand, nc, picks, &kept);
        if (rc) return rc;
        proposed += nc;
        accepted += kept - 1;
        gen.push_back(current);
        for (int j = 0; j + 1 < kept; ++j) {
            gen.push_back(cand[j]);
            history.push_back(cand[j]);
        }
        current = picks[kept - 1];
    }
    std::copy(gen.begin(), gen.begin() + n_gen, out);
    if (stats) {
        stats[0] = proposed;
        stats[1] = accepted;
        stats[2] = blocks;
    }
    return ABRA_OK;
}

int abra_model_step(void *model, int32_t n_steps) {
    Model *m = static_cast<Model *>(model);
    if (!m || n_steps < 0) return model_fail(ABRA_E_INVALID, "bad arguments", cudaSuccess);
    if (static_cast<int64_t>(m->host_pos) + n_steps > m->cfg.max_ctx)
        return model_fail(ABRA_E_INVALID, "steps would pass max_ctx", cudaSuccess);
    if (!m->connected) return model_fail(ABRA_E_INVALID, "tensor-parallel model not connected", cudaSuccess);
    m->host_pos += n_steps;
    cudaError_t e = abra::capture(*m);
    if (e != cudaSuccess) return model_fail(ABRA_E_CUDA, "graph capture", e);
    for (int i = 0; i < n_steps; ++i) {
        e = m->graph ? cudaGraphLaunch(m->graph, m->stream) : abra::record_step(*m, m->stream);
        if (e != cudaSuccess) return model_fail(ABRA_E_CUDA, "step", e);
    }
    return ABRA_OK;
}

int abra_model_invalidate(void *model) {
    Model *m = static_cast<Model *>(model);
    if (!m) return model_fail(ABRA_E_INVALID, "bad arguments", cudaSuccess);
    cudaError_t e = cudaStreamSynchronize(m->stream);
    if (e != cudaSuccess) return model_fail(ABRA_E_CUDA, "sync", e);
    if (m->graph) cudaGraphExecDestroy(m->graph);
    m->graph = nullptr;
    return ABRA_OK;
}

// After a synchronize: a kernel's bounded wait that gave up, or an
// out-of-range token id it refused to index with (the device error word,
// left set), fails the call instead of passing its garbage on.
static int device_waits_ok() {
    unsigned v = 0;
    cudaError_t e = abra::read_error_words(&v, false);
    if (e != cudaSuccess) return model_fail(ABRA_E_CUDA, "device error word", e);
    if (v) {
        snprintf(g_model_err, sizeof g_model_err, "%s (device error word 0x%x)",
                 v == 0x10u ? "a kernel met an out-of-range token id" : "a kernel's bounded wait gave up", v);
        return ABRA_E_CUDA;
    }
    return ABRA_OK;
}

int abra_model_sync(void *model) {
    Model *m = static_cast<Model *>(model);
    if (!m) return ABRA_E_INVALID;
    cudaError_t e = cudaStreamSynchronize(m->stream);
    return e == cudaSuccess ? device_waits_ok() : model_fail(ABRA_E_CUDA, "sync", e);
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
        e = cudaMemcpy(logits, m->logits, static_cast<size_t>(m->sh.vocab_hi - m->sh.vocab_lo) * 4,
                       cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && pos) e = cudaMemcpy(pos, m->pos, 4, cudaMemcpyDeviceToHost);
    return e == cudaSuccess ? device_waits_ok() : model_fail(ABRA_E_CUDA, "read", e);
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
    if (m->batch > 1) return model_fail(ABRA_E_UNSUPPORTED, "streaming is for batch 1", cudaSuccess);
    if (static_cast<int64_t>(m->host_pos) + n > m->cfg.max_ctx)
        return model_fail(ABRA_E_INVALID, "steps would pass max_ctx", cudaSuccess);
    if (!m->connected) return model_fail(ABRA_E_INVALID, "tensor-parallel model not connected", cudaSuccess);
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

// One tensor of a GGUF file (ggml layout: rows of K/256 blocks, row-major)
// into the model's buffers: whole tensors on one GPU; on a tensor-parallel
// rank, its rows (q, k, v, gate, up) or its canonical K-slices of every row
// (o, down).  The tied table is whole on every rank.
int abra_model_load_tensor(void *model, int32_t layer, int32_t slot, int32_t ggml_type,
                           const void *host, uint64_t bytes) {
    Model *m = static_cast<Model *>(model);
    if (!m || !host) return model_fail(ABRA_E_INVALID, "null pointer", cudaSuccess);
    if (m->batch > 1) return model_fail(ABRA_E_UNSUPPORTED, "load into a batch-1 model", cudaSuccess);
    abra::TensorSlice t;
    if (abra::tensor_slice(m->cfg, m->sh, m->mix, layer, slot, t) != ABRA_OK)
        return model_fail(ABRA_E_INVALID, "unknown tensor (layer, slot)", cudaSuccess);
    if (ggml_type != t.type)
        return model_fail(ABRA_E_INVALID, "tensor type differs from the model's type for this slot", cudaSuccess);
    if (bytes != static_cast<uint64_t>(t.N * t.rb))
        return model_fail(ABRA_E_INVALID, "tensor size differs from the model's shape", cudaSuccess);
    uint8_t *dst = nullptr;
    if (layer == -1) {
        dst = t.buf == abra::BUF_EMBD ? m->embd : reinterpret_cast<uint8_t *>(m->out_norm);
    } else {
        abra::LayerW &y = m->layers[layer];
        switch (t.buf) {
            case abra::BUF_ATTN_NORM: dst = reinterpret_cast<uint8_t *>(y.attn_norm); break;
            case abra::BUF_FFN_NORM: dst = reinterpret_cast<uint8_t *>(y.ffn_norm); break;
            case abra::BUF_Q_NORM: dst = reinterpret_cast<uint8_t *>(y.q_norm); break;
            case abra::BUF_K_NORM: dst = reinterpret_cast<uint8_t *>(y.k_norm); break;
            case abra::BUF_WQKV: dst = y.wqkv; break;
            case abra::BUF_WV: dst = y.wv; break;
            case abra::BUF_WO: dst = y.wo; break;
            case abra::BUF_WGATE: dst = y.wgate; break;
            case abra::BUF_WUP: dst = y.wup; break;
            case abra::BUF_WDOWN: dst = y.wdown; break;
            default: return model_fail(ABRA_E_INVALID, "unknown tensor slot", cudaSuccess);
        }
    }
    dst += t.dst_row * t.nb;  // the rank's rows of the slot sit after dst_row others
    const uint8_t *src = static_cast<const uint8_t *>(host) + t.r0 * t.rb + t.b0;
    cudaError_t e = cudaMemcpy2DAsync(dst, t.nb, src, t.rb, t.nb, t.nr, cudaMemcpyHostToDevice, m->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
    return e == cudaSuccess ? ABRA_OK : model_fail(ABRA_E_CUDA, "tensor upload", e);
}

int abra_tp_tensor_slice(const abra_model_config *cfg, int32_t rank, int32_t world, int32_t layer,
                         int32_t slot, int64_t *out) {
    if (!cfg || !out) return model_fail(ABRA_E_INVALID, "null pointer", cudaSuccess);
    abra_tp_shard sh = {};
    const int rc = abra::tp_shard(*cfg, rank, world, sh);
    if (rc != ABRA_OK) return model_fail(rc, "no tensor-parallel split of this configuration", cudaSuccess);
    abra::TensorSlice t;
    if (abra::tensor_slice(*cfg, sh, (cfg->flags & ABRA_MODEL_Q4_K_M) != 0, layer, slot, t) != ABRA_OK)
        return model_fail(ABRA_E_INVALID, "unknown tensor (layer, slot)", cudaSuccess);
    const int64_t v[8] = {t.type, t.N, t.K, t.rb, t.r0, t.nr, t.b0, t.nb};
    std::memcpy(out, v, sizeof v);
    return ABRA_OK;
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
