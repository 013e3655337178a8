// decode.cuh -- launchers of the decode-step kernels (decode_kernels.cu) and
// the generator options used by the model runtime (model.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace abra {

// Per-sequence element strides of a batch of sequences sharing one position
// (batch 1: all zero).
struct SeqStrides {
    int batch = 1;
    int64_t qkv = 0, q = 0, kv = 0;
    // position step per sequence: 0 when every sequence is at *pos (batched
    // decode), 1 for a prefill chunk, whose column b is the token at *pos + b
    // of one sequence (kv = 0: the columns share one cache)
    int pos = 0;
};

cudaError_t launch_embed(const void *E, int hidden, const int32_t *tokens, const int32_t *pos,
                         float *h, bool pdl, cudaStream_t s, int batch = 1, int64_t tok_stride = 0);
// The same lookup from a Q6_K table (210-byte blocks).
cudaError_t launch_embed_q6k(const void *E, int hidden, const int32_t *tokens, const int32_t *pos,
                             float *h, bool pdl, cudaStream_t s, int batch = 1,
                             int64_t tok_stride = 0);
// With wait_cnt (tensor parallel): first wait, bounded, until *wait_cnt >=
// (*epoch + 1) * per_step -- every rank's partial sums of the step have arrived.
cudaError_t launch_residual_rmsnorm_quant(float *h, const DeltaSet &ds, const float *w,
                                          float eps, void *y, int K, int ncols, bool pdl,
                                          cudaStream_t s, const unsigned long long *wait_cnt = nullptr,
                                          const unsigned long long *epoch = nullptr,
                                          unsigned long long per_step = 0);
cudaError_t launch_qk_norm_rope_kv(const float *qkv, const float *q_norm, const float *k_norm,
                                   float eps, const float *rope, const int32_t *pos, float *q_out,
                                   void *kc, void *vc, int n_heads, int n_kv, int max_ctx,
                                   bool pdl, cudaStream_t s, const SeqStrides &b = SeqStrides());
cudaError_t launch_attention(const float *q, const void *kc, const void *vc, const int32_t *pos,
                             float scale, int n_heads, int n_kv, int max_ctx, float *part_m,
                             float *part_l, float *part_o, float *out_f32, void *out_q8,
                             bool pdl, cudaStream_t s, const SeqStrides &b = SeqStrides());
// Reads the argmax key left by the output MMVQ, resets it, appends the pick.
// Tensor parallel (epoch != nullptr): first waits until *wait_cnt >=
// (*epoch + 1) * per_step (every rank's keys have arrived), then advances
// *epoch.
cudaError_t launch_argmax_finish(unsigned long long *key, int32_t *tokens, int32_t *picks,
                                 int32_t *pos, const int32_t *n_prompt, int max_ctx, bool pdl,
                                 cudaStream_t s, const unsigned long long *wait_cnt = nullptr,
                                 unsigned long long *epoch = nullptr,
                                 unsigned long long per_step = 0);
// Greedy picks of a batch of sequences (logits rows ldl apart, token rows
// tok_stride apart), then one advance of the shared position.
cudaError_t launch_argmax_batch(const float *logits, int n, int64_t ldl, int32_t *tokens,
                                int32_t *picks, int64_t tok_stride, int32_t *pos,
                                const int32_t *n_prompt, int max_ctx, int batch, bool pdl,
                                cudaStream_t s);
// Tensor parallel, batch: where each rank's per-sequence argmax keys go.
struct TpKeyPush {
    int npeer;
    unsigned long long *key[8];  // rank q's key words [batch]
    unsigned long long *cnt[8];  // rank q's arrival counter of the output
    unsigned long long *cta_cnt; // this rank's CTA count of the launch
};
// Each sequence's key over this rank's vocab rows (logits rows ldl apart,
// row ids offset by row_offset), merged into every rank's key words.
cudaError_t launch_argmax_keys_batch(const float *logits, int n, int64_t ldl, int row_offset,
                                     const TpKeyPush &push, int batch, bool pdl, cudaStream_t s);
// Waits for every rank's keys, writes the picks and next tokens of the batch,
// resets the keys, advances the epoch and the shared position.
cudaError_t launch_argmax_finish_batch(unsigned long long *keys, int batch, int32_t *tokens, int32_t *picks,
                                       int64_t tok_stride, int32_t *pos, const int32_t *n_prompt, int max_ctx,
                                       const unsigned long long *wait_cnt, unsigned long long *epoch,
                                       unsigned long long per_step, bool pdl, cudaStream_t s);
// out[c] = argmax of column c of logits (ldl floats apart), c < ncols.
cudaError_t launch_argmax_cols(const float *logits, int n, int64_t ldl, int32_t *out, int ncols,
                               bool pdl, cudaStream_t s);
// *pos = min(*pos + n, max_ctx).
cudaError_t launch_pos_advance(int32_t *pos, int n, int max_ctx, bool pdl, cudaStream_t s);
// y = Q8_1 of up * silu(gate), n values (a multiple of 32).
cudaError_t launch_swiglu_quant(const float *g, const float *u, void *y, int64_t n, bool pdl,
                                cudaStream_t s);

// ------------------------------------------------ persistent decode step ---
// One batch-1 decode token of the all-Q4_K model as one cooperative kernel
// (decode_persistent.cu); bit-identical to the kernel chain.
struct PersistLayer {
    const uint8_t *wqkv, *wo, *wgate, *wup, *wdown;
    const float *attn_norm, *q_norm, *k_norm, *ffn_norm;
};
struct PersistModel {
    int n_layers, hidden, n_heads, n_kv, ffn, vocab, max_ctx;
    float eps;
    const PersistLayer *layers;  // device array of n_layers entries
    const uint8_t *embd;
    const float *out_norm;
    float *h0, *h1, *delta, *qkv, *att, *part_m, *part_l, *part_o, *act, *logits;
    uint8_t *oq;
    void *kc, *vc;  // fp16 caches [layer][kv head][max_ctx][128]
    const float *rope;
    int32_t *tokens, *picks, *pos;
    const int32_t *nprompt;
    unsigned long long *amax;
    void *sync;  // persist_sync_bytes() zeroed bytes: barrier and arrival counters
};
size_t persist_sync_bytes(int n_heads);
// False (with a reason) when the shape does not fit the kernel's ring and
// shared-memory plan; the model then runs the kernel chain.
bool persist_supported(int hidden, int n_heads, int n_kv, int ffn, int head_dim, const char **why);
// Kernel attributes and the co-residency check (outside stream capture).
cudaError_t persist_prepare(int hidden, int n_heads, int n_kv, int ffn);
cudaError_t launch_persist_step(const PersistModel &pm, cudaStream_t st);
// Host-side walk of every weight copy the kernel would issue on `sms` SMs.
bool persist_plan_check(int n_layers, int hidden, int n_heads, int n_kv, int ffn, int vocab, int sms,
                        int64_t out[9], const char **why);

// Generator variants (gen_quant.cu).
cudaError_t launch_gen_q4k_ex(void *dst, int64_t nblocks, uint64_t seed, uint64_t tensor_id,
                              int64_t block_offset, int flags, cudaStream_t stream);
cudaError_t launch_gen_norm_f32(float *dst, int64_t n, uint64_t seed, uint64_t tensor_id,
                                cudaStream_t stream);
// Rows [row0, row0 + rows) x superblock columns [sb_lo, sb_hi) of a Q4_K
// tensor with rows of nsb_g superblocks (a K-shard), bytes identical to the
// same blocks of the whole tensor.
cudaError_t launch_gen_q4k_cols(void *dst, int64_t rows, int64_t nsb_g, int64_t sb_lo,
                                int64_t sb_hi, uint64_t seed, uint64_t tensor_id, int64_t row0,
                                int flags, cudaStream_t stream);
// Q6_K blocks: local block i is global block block_offset + (i / width) *
// gstride + i % width of the tensor's stream (width = nblocks, gstride = 0:
// a contiguous run), bytes identical to abra_gen_q6k's.
cudaError_t launch_gen_q6k_cols(void *dst, int64_t nblocks, int64_t width, int64_t gstride,
                                uint64_t seed, uint64_t tensor_id, int64_t block_offset,
                                cudaStream_t stream);

}  // namespace abra
