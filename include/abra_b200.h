/*
 * abra_b200.h -- C ABI of libabra_b200.so, the sm_100a Q4_K x Q8_1 decode
 * path.
 *
 * Conventions (all entry points):
 *   - Pointers are device pointers on the calling thread's current CUDA
 *     device unless stated otherwise; `stream` is a cudaStream_t (NULL = the
 *     legacy default stream).  Work is stream-ordered and asynchronous.
 *   - Return 0 on success, a negative ABRA_E* code on error; the message is
 *     available from abra_last_error() (thread-local).  No exception crosses
 *     the ABI.  The reference throws std::invalid_argument for the same
 *     conditions (kernels/q4k/q4k_q8_mmvq.cu:266-268,302,312-314;
 *     kernels/q4k/q4k_family.cu:200-202,279).
 *   - Layouts are ggml's: Q4_K rows of K/256 superblocks of 144 B, row-major;
 *     Q8_1 activation columns of K/32 blocks of 36 B, column after column;
 *     fp32 outputs y[c * ldy + r].  Weight and activation buffers must be
 *     16-byte aligned.
 *   - The library allocates no device memory in these calls.
 */
#ifndef ABRA_B200_H
#define ABRA_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ABRA_OK 0
#define ABRA_E_INVALID (-1)     /* bad shape, alignment, id or pointer */
#define ABRA_E_CUDA (-2)        /* a CUDA runtime call failed */
#define ABRA_E_UNSUPPORTED (-3) /* shape/batch outside what the kernels cover */

/* Flags for abra_q4k_mmvq_ex. */
#define ABRA_MMVQ_PDL 1 /* programmatic dependent launch: weights are
                           prefetched before the previous kernel in the
                           stream completes, so the weights must not be
                           written by that kernel */

/* ---------------------------------------------------------- library ---- */
const char *abra_version(void);
const char *abra_last_error(void);
/* Device error word set by kernels whose bounded waits gave up (bit 0: an
 * mbarrier wait, bit 1: a cross-rank flag wait, bit 2: a wait for a free
 * ring stage, bit 3: a grid barrier of the persistent decode step) or that
 * met a token id outside the vocabulary and read row 0 instead (bit 4).
 * clear != 0 resets it.  Synchronises the current device. */
int abra_device_error(uint32_t *out, int32_t clear);
/* Failure detection without a fault: waits on a device counter that nothing
 * increments with the bounded cross-rank wait of the tensor-parallel kernels;
 * returns the error bits it raised (bit 1: a flag wait gave up; then cleared)
 * and how long the wait ran (about one second).  The context stays usable.
 * Synchronous; allocates 16 bytes of device memory. */
int abra_test_flag_timeout(uint32_t *error_bits, uint64_t *waited_ns);

/* ------------------------------------------------------------- MMVQ ---- */
/* y = W x for Q4_K W (N x K) and ncols Q8_1 columns, 1 <= ncols <= 8,
 * K % 256 == 0, K <= 65536 (configurations whose staging does not fit in
 * shared memory return ABRA_E_CUDA).  Picks the tuned candidate for (N, K, ncols).
 * Replaces launch_q4k_autotuned (kernels/q4k/q4k_family.cuh:89-97) and the
 * mul_mat_vec_q hook abra_dispatch_mmvq (kernels/q4k/abra-mmvq.cuh:209-220). */
int abra_q4k_mmvq(const void *w_q4k, const void *x_q8_1, float *y, int64_t N, int64_t K,
                  int32_t ncols, void *stream);

/* One named candidate of the family (ids from abra_candidate_info).
 * Replaces launch_q4k_candidate (kernels/q4k/q4k_family.cuh:63-71). */
int abra_q4k_mmvq_candidate(int32_t candidate, const void *w_q4k, const void *x_q8_1,
                            float *y, int64_t N, int64_t K, int32_t ncols, void *stream);

/* Combined pipeline: quantize ncols fp32 columns x (K each) to Q8_1 in the
 * caller's scratch x_q8_1_scratch (ncols * K/32 * 36 bytes, 16-byte
 * aligned), then y = W x with the named candidate (0 = tuned).  Replaces
 * launch_q4k_candidate_combined_pipeline / launch_q4k_autotuned_combined_pipeline
 * (kernels/q4k/q4k_family.cuh:73-82,99-108; q4k_family.cu:283-295,451-463). */
int abra_q4k_mmvq_combined(int32_t candidate, const void *w_q4k, const float *x,
                           void *x_q8_1_scratch, float *y, int64_t N, int64_t K, int32_t ncols,
                           void *stream);

/* The same combined pipeline with no caller scratch and no allocation: the
 * Q8_1 blocks go to a static device array of 147,456 bytes (K * ncols <=
 * 131,072; larger requests return ABRA_E_UNSUPPORTED).  For callers that may
 * not allocate device memory where they multiply.  The first call on each
 * device resolves that device's scratch address; make it before any stream
 * capture.  That address is kept for the life of the process: after
 * cudaDeviceReset on a device, do not call this entry point on it again.
 * Nothing in the scratch needs to start at zero.  Calls that can overlap on
 * one device (different streams or threads) race on the scratch.  This entry
 * point has no counterpart in the reference. */
int abra_q4k_mmvq_combined_static(int32_t candidate, const void *w_q4k, const float *x,
                                  float *y, int64_t N, int64_t K, int32_t ncols, void *stream);

/* Row-parallel (K-sharded) MMVQ: w holds columns [k0, k0 + K) of an
 * N x K_full matrix, where [k0, k0 + K) are the canonical K-slices
 * [sl_base, sl_base + sl_cnt), sl_cnt in {1, 2, 4, 8}, of K_full (slice i of a row of n = K_full/256
 * superblocks starts at superblock i*(n/8) + min(i, n%8)); x holds the same
 * K activations.  y gets this shard's partial sums, each a subtree of the
 * unsharded sum, so adding the shards' partials in the fixed tree
 * (2: p0+p1; 4: (p0+p1)+(p2+p3); 8: three levels) reproduces the unsharded
 * y bit for bit.  The reference's tensor split sums its shards with an
 * NCCL all-reduce instead (docs/research/1080ti-speed-results.md:76-81). */
int abra_q4k_mmvq_kshard(const void *w_q4k, const void *x_q8_1, float *y, int64_t N, int64_t K,
                         int32_t ncols, int64_t K_full, int32_t sl_base, int32_t sl_cnt,
                         int32_t candidate, int32_t flags, void *stream);

/* Batch-32 MMVQ on the 5th-generation tensor cores (tcgen05.mma kind::i8,
 * TMEM accumulators): y = W x for ncols = 32 Q8_1 columns, bit-identical
 * to abra_q4k_mmvq (the exact int32 sub-block dots come from the tensor
 * core, the fp32 scaling follows the same canonical order).  ks in
 * {1, 2, 4, 8} splits K over CTAs along the canonical slices; ks > 1 needs
 * workspace = ks * 32 * N floats (one more launch combines the parts).  The
 * reference has no tensor-core path: its batched decode runs its MMVQ
 * family per column group (kernels/q4k/q4k_family.cu:12-110). */
int abra_q4k_mmvq_tc(const void *w_q4k, const void *x_q8_1, float *y, int64_t N, int64_t K,
                     int32_t ncols, int64_t ldy, int32_t ks, float *workspace, int32_t flags,
                     void *stream);

/* Full form: explicit output column stride ldy >= N, candidate (0 = tuned)
 * and ABRA_MMVQ_* flags. */
int abra_q4k_mmvq_ex(const void *w_q4k, const void *x_q8_1, float *y, int64_t N, int64_t K,
                     int32_t ncols, int64_t ldy, int32_t candidate, int32_t flags,
                     void *stream);

/* Fused gate/up with SwiGLU, one pass over the shared activation:
 * y = (W_up x) * silu(W_gate x), silu(g) = g / (1 + exp(-g)).  W_gate and
 * W_up are N x K Q4_K each.  Replaces the reference's GATE kernel
 * (kernels/q4k/abra-mmvq.cuh:118-143,175-186) with GGML_GLU_OP_SWIGLU. */
int abra_q4k_mmvq_swiglu(const void *w_gate, const void *w_up, const void *x_q8_1, float *y,
                         int64_t N, int64_t K, int32_t ncols, int64_t ldy, int32_t candidate,
                         int32_t flags, void *stream);

/* Debug form of the same kernel: also stores the exact int32 sub-block dot
 * products P[c][r][b][s] (ncols*N*(K/256)*8) and activation sums
 * M[c][b][s] (ncols*(K/256)*8).  ks selects the k-split (1, 2 or 4);
 * ncols in {1, 2, 4, 8}.  The reference computes the same integers inside
 * vec_dot_q4_K_q8_1_impl_vmmq (kernels/q4k/q4k_vecdot.cuh:35-36). */
int abra_q4k_mmvq_partials(const void *w_q4k, const void *x_q8_1, float *y, int32_t *P,
                           int32_t *M, int64_t N, int64_t K, int32_t ncols, int32_t ks,
                           void *stream);

/* Drop-in for the reference's C shim of the same name and signature
 * (kernels/q4k/upstream_adapter.cuh:12-19): one Q8_1 column. */
void launch_pinned_upstream_mmvq(const void *d_w_q4, const void *d_x_q8, float *d_y,
                                 int64_t N, int64_t K, void *stream);

/* Drop-ins for the two host functions of the same shim
 * (kernels/q4k/upstream_adapter.cuh:28-38), which the reference forwards to
 * llama.cpp's quantize_row_q4_K_ref / dequantize_row_q4_K.  CPU only, no
 * GPU needed.  x: k floats (k % 256 == 0) -> k/256 Q4_K blocks of 144 bytes
 * (the reference declares y as block_q4_K *; the bytes are the same), by the
 * published Q4_K algorithm (a weighted affine fit per 32-value sub-block, then
 * 6-bit scale and min multipliers of fp16 superblock scales).  Dequantize:
 * y = (d * sc) * q - dmin * m per value.  A k that is not a multiple of 256
 * writes nothing and records the error for abra_last_error (the reference
 * asserts). */
void quantize_row_q4_K_upstream_cpu(const float *x, void *y, int64_t k);
void dequantize_row_q4_K_upstream_cpu(const void *x, float *y, int64_t k);

/* The reference's opt-in 148-byte prepack of Q4_K weights
 * (kernels/q4k/abra-packed-q4.cuh:3-31; made by abra_prepare_q4 when
 * ABRA_PREPACK=1, tools/prepare-packed-weights.py:49-69): per superblock fp16
 * d and dmin, the eight 6-bit scales and mins unpacked to bytes
 * [sc_2j, sc_2j+1, m_2j, m_2j+1] for each pair j, then the 128 nibble bytes.
 * nblocks superblocks of 144 bytes in, of 148 out (both 16-byte aligned). */
int abra_q4k_pack(const void *w_q4k, void *w_packed, int64_t nblocks, void *stream);
/* y = W x at batch 1 over packed weights (N rows of K/256 packed
 * superblocks): the lane-mapped MMVQ reading the unpacked scale bytes; y is
 * bit-identical to abra_q4k_mmvq on the unpacked weights.  ABRA_E_UNSUPPORTED
 * when no unit size keeps the packed rows' copies 16-byte aligned. */
int abra_q4k_mmvq_packed(const void *w_packed, const void *x_q8_1, float *y, int64_t N, int64_t K,
                         int32_t flags, void *stream);

/* --------------------------------------------------------- Q8_1 -------- */
/* x: ncols columns of K fp32 (K % 32 == 0) -> ncols x K/32 Q8_1 blocks.
 * Replaces launch_quantize_f32_to_q8_1 / launch_custom_reference_q8_1_quantizer
 * (kernels/q4k/q4k_q8_mmvq.cuh:91-103; semantics q4k_q8_mmvq.cu:223-255). */
int abra_quantize_q8_1(const float *x, void *x_q8_1, int64_t K, int32_t ncols, void *stream);

/* Drop-in for kernels/q4k/upstream_adapter.cuh:21-26 (one column). */
void launch_pinned_upstream_q8_1_quantize(const float *d_x_f32, void *d_x_q8, int64_t K,
                                          void *stream);

/* Fused RMSNorm -> Q8_1, quantize once: xn = (x * r) * w with
 * r = 1/sqrt(mean(x^2) + eps); xn is quantized to Q8_1 (and also written to
 * xn_out when it is not NULL).  K % 32 == 0, K <= 16384.  Replaces the
 * RMSNorm + per-consumer quantize pair that the reference's Q8 reuse cache
 * de-duplicates (kernels/q4k/abra-q8-reuse.cuh:3-71). */
int abra_rmsnorm_quantize_q8_1(const float *x, const float *w, float eps, void *x_q8_1,
                               float *xn_out, int64_t K, int32_t ncols, void *stream);

/* RMSNorm -> Q8_1 -> MMVQ in one kernel, batch 1: every CTA normalizes the
 * fp32 input x (K values) with the norm weights and quantizes it to Q8_1 in
 * its own shared memory, in the order of abra_rmsnorm_quantize_q8_1, then
 * runs the MMVQ on it, so the activation never makes a round trip through
 * HBM and the result is bit-identical to abra_rmsnorm_quantize_q8_1 followed
 * by abra_q4k_mmvq (w_up == NULL) or abra_q4k_mmvq_swiglu (w_up != NULL: y =
 * (W_up xq) * silu(W_gate xq) with W_gate = w).  x_q8_out, when not NULL,
 * receives the K/32 Q8_1 blocks (written by one CTA) for another consumer of
 * the same activation.  This is the decode runtime's form of the reference's
 * quantize-once reuse (kernels/q4k/abra-q8-reuse.cuh:3-71), where the
 * consumers of one normalized activation share a single Q8_1 copy.
 * w, w_up and norm_w 16-byte aligned; x, y, x_q8_out 4-byte aligned;
 * candidate 0 = tuned; flags ABRA_MMVQ_PDL. */
int abra_q4k_mmvq_rmsnorm(const void *w_q4k, const void *w_up, const float *x,
                          const float *norm_w, float eps, float *y, void *x_q8_out, int64_t N,
                          int64_t K, int32_t candidate, int32_t flags, void *stream);

/* ------------------------------------------------------- generators ---- */
/* Seeded synthetic Q4_K superblocks [block_offset, block_offset+nblocks) of
 * tensor tensor_id: d, dmin ~ U(0.001, 0.02) fp16, scales/mins ~ U{0..63},
 * nibbles ~ U{0..15}.  dst 8-byte aligned. */
int abra_gen_q4k(void *dst, int64_t nblocks, uint64_t seed, uint64_t tensor_id,
                 int64_t block_offset, void *stream);
/* dst[i] = fmaf(u_i, scale, offset), u_i ~ U[0,1) on a 2^-24 grid. */
int abra_gen_uniform_f32(float *dst, int64_t n, uint64_t seed, uint64_t tensor_id,
                         int64_t offset_index, float scale, float offset, void *stream);

/* --------------------------------------------------------- autotuner --- */
/* Candidate enumeration: index 0..abra_candidate_count()-1 -> id, feed mode
 * (0 TMA per-row bulk copies, 1 TMA whole-unit copy, 2 direct 128-bit loads),
 * k-split, consumer warps, CTAs per SM, stage budget (KiB).  Replaces
 * get_all_candidate_ids / get_candidate_spec (kernels/q4k/q4k_family.cuh:59-61). */
int abra_candidate_count(void);
int abra_candidate_info(int32_t index, int32_t *id, int32_t *mode, int32_t *ks, int32_t *ncw,
                        int32_t *ctas_per_sm, int32_t *stage_kb);
/* Tuning table keyed by (N, K, ncols, nmat), nmat = 1 for MMVQ and 2 for the
 * fused gate/up form.  Replaces register_autotuned_table_entry /
 * get_autotuned_candidate_for_shape (kernels/q4k/q4k_family.cuh:86-87). */
int abra_tune_set(int64_t N, int64_t K, int32_t ncols, int32_t nmat, int32_t candidate);
int abra_tune_get(int64_t N, int64_t K, int32_t ncols, int32_t nmat); /* candidate id */
int abra_tune_clear(void); /* clears the Q4_K and the Q6_K tables */

/* ------------------------------------------------------------ Q6_K ----- */
/* y[c][r] = sum_k W[r][k] x[c][k] for N x K Q6_K rows W (ggml's block_q6_K,
 * 210 bytes per 256 weights: ql[128], qh[64], int8 scales[16], fp16 d;
 * w = d * scales[e/16] * (q - 32)) and ncols (1..8) Q8_1 columns x.  The
 * Q6_K leg of the reference's dispatch, abra_dispatch_mmvq<GGML_TYPE_Q6_K>
 * (kernels/q4k/abra-mmvq.cuh:209-221, which runs ggml's vec_dot_q6_K_q8_1
 * at :138-141; the reference's f64 oracle for it is
 * tests/runtime_kernel_test.cu:82-106).  Exact int32 16-weight dots, fp32
 * scaling in a fixed order, the canonical eight K-slices of the Q4_K path.
 * w 16-byte aligned; x 16-byte aligned; ldy >= N; candidate 0 = tuned. */
int abra_q6k_mmvq(const void *w_q6k, const void *x_q8_1, float *y, int64_t N, int64_t K,
                  int32_t ncols, void *stream);
int abra_q6k_mmvq_ex(const void *w_q6k, const void *x_q8_1, float *y, int64_t N, int64_t K,
                     int32_t ncols, int64_t ldy, int32_t candidate, int32_t flags,
                     void *stream);
/* K-shard form (row-parallel tensor parallelism), as abra_q4k_mmvq_kshard:
 * w holds canonical slices [sl_base, sl_base + sl_cnt) of rows K_full wide;
 * y is that shard's subtree of the unsharded result. */
int abra_q6k_mmvq_kshard(const void *w_q6k, const void *x_q8_1, float *y, int64_t N, int64_t K,
                         int32_t ncols, int64_t K_full, int32_t sl_base, int32_t sl_cnt,
                         int32_t candidate, int32_t flags, void *stream);
/* Debug form: also stores the exact int32 dots P[c][r][b][j] of the 16
 * sub-blocks j (16 weights each) of every superblock b. */
int abra_q6k_mmvq_partials(const void *w_q6k, const void *x_q8_1, float *y, int32_t *P,
                           int64_t N, int64_t K, int32_t ncols, void *stream);
/* Seeded synthetic Q6_K blocks [block_offset, block_offset + nblocks) of
 * tensor tensor_id: ql, qh, scales uniform over byte values, d ~
 * U(0.0001, 0.002) fp16.  dst 2-byte aligned. */
int abra_gen_q6k(void *dst, int64_t nblocks, uint64_t seed, uint64_t tensor_id,
                 int64_t block_offset, void *stream);
/* Q6_K candidates (index 0..count-1 -> id, feed mode 0 per-row bulk copies,
 * 1 whole-unit copy, 2 direct loads; k-split; CTAs per SM; stage KiB) and
 * their tuning table keyed by (N, K, ncols). */
int abra_q6k_candidate_count(void);
int abra_q6k_candidate_info(int32_t index, int32_t *id, int32_t *mode, int32_t *ks,
                            int32_t *ctas_per_sm, int32_t *stage_kb);
int abra_q6k_tune_set(int64_t N, int64_t K, int32_t ncols, int32_t candidate);
int abra_q6k_tune_get(int64_t N, int64_t K, int32_t ncols);

/* Launch plan of one MMVQ call, computed on the host exactly as the dispatch
 * computes it, for a GPU with sm_count SMs (0: the current device's): no
 * device call when sm_count > 0.  ggml_type ABRA_GGML_Q4_K (nmat 1, or 2 for
 * the fused gate/up form; xin 1 for the fused RMSNorm prologue of the decode
 * runtime, batch 1) or ABRA_GGML_Q6_K (nmat 1, xin 0); candidate 0 = tuned;
 * K_full > 0 names a K-shard as in the _kshard calls.  out[8] = grid, threads
 * per CTA, ring depth, per-row stage pitch, bytes per stage, dynamic shared
 * memory, row groups of 8, offset of the stage ring in shared memory: what a
 * host-side check needs to follow every address the kernel's copies form.
 * The reference has no counterpart (its launch geometry is fixed per
 * candidate, kernels/q4k/q4k_family.cu:12-110). */
int abra_mmvq_plan_info(int32_t ggml_type, int32_t candidate, int64_t N, int64_t K, int32_t ncols,
                        int32_t nmat, int32_t xin, int64_t K_full, int32_t sl_base, int32_t sl_cnt,
                        int32_t sm_count, int64_t *out);

/* ------------------------------------------------------ decode model --- */
/* Qwen3-4B-shaped decode with every linear layer Q4_K:
 * the native runtime that the reference delegates to llama.cpp.  Weights
 * are generated on the device from a seed (the same counter-based generator
 * as abra_gen_q4k; tensor ids: 1 embedding/output (tied), 2 output norm,
 * 100 + 16 l + {0 attn_norm, 1 q|k|v, 2 q_norm, 3 k_norm, 4 o, 5 ffn_norm,
 * 6 gate, 7 up, 8 down}); norm weights are +-U(0.8, 1.2) with random sign.
 * Unlike the kernel entry points above, the model allocates (weights, fp16
 * KV cache for max_ctx positions, activations) and owns a CUDA stream. */
typedef struct {
    int32_t n_layers, hidden, n_heads, n_kv_heads, head_dim, ffn, vocab, max_ctx;
    float rope_theta, eps;
    uint64_t seed;
    int32_t centered; /* 1: centred Q4_K variant (zero-mean sub-blocks) */
    int32_t flags;    /* ABRA_MODEL_* */
} abra_model_config;

#define ABRA_MODEL_EAGER 1  /* launch kernels per step instead of a CUDA graph */
#define ABRA_MODEL_NO_PDL 2 /* no programmatic dependent launch */
#define ABRA_MODEL_NO_PREFETCH 4 /* no L2 prefetch of the next kernel's weights */
/* The real Qwen3-4B-Q4_K_M type map instead of all-Q4_K: the tied
 * embedding/output is Q6_K, and attn_v and ffn_down are Q6_K in layers l
 * with l < n/8, l >= 7n/8 or (l - n/8) % 3 == 2 (layers 0-3, 6, 9, ..., 30,
 * 31-35 of 36, the reference's census bench/results/m3/qwen3-q4k-tensor-map.json);
 * Q6_K tensors are generated like abra_gen_q6k from the same tensor ids (V
 * rows keep their row index in tensor 1).  One GPU, batch 1. */
#define ABRA_MODEL_Q4_K_M 8
/* Run the batch-1 step as the chain of per-operation kernels (one CUDA graph
 * of ~290 launches) instead of the persistent decode kernel.  The persistent
 * kernel is the default wherever it applies: batch 1, one GPU, all-Q4_K
 * weights, q heads per kv head in {1, 2, 4, 8}; both give bit-identical
 * logits and tokens. */
#define ABRA_MODEL_KERNEL_CHAIN 16

int abra_model_default_config(abra_model_config *cfg); /* Qwen3-4B, max_ctx 4096 */
/* *persistent = 1 when each decode step of this model is one launch of the
 * persistent decode kernel (the reference's per-token decode loop,
 * tests/runtime_logits.cpp:59-108, as one cooperative kernel: a CTA per SM
 * streams its share of every layer's weights through a shared-memory ring
 * ahead of grid-wide phase barriers), 0 when it is the kernel chain. */
int abra_model_path(void *model, int32_t *persistent);
/* Host-only check of the persistent kernel's plan for a model shape on a GPU
 * with `sms` SMs: walks every weight copy of every CTA's token and checks it
 * against its ring slot and its tensor.  out = {dynamic shared memory, ring
 * bytes (16 or 8 slots), weight units of the busiest CTA, copies checked,
 * rows per unit of the q|k|v, o, gate/up, down and output GEMVs}.
 * ABRA_E_UNSUPPORTED when the shape does not fit the kernel (the model then
 * runs the kernel chain). */
int abra_persist_plan(const abra_model_config *cfg, int32_t sms, int64_t out[9]);
int abra_model_create(const abra_model_config *cfg, void **model);
int abra_model_destroy(void *model);
/* Load a prompt (token ids) and rewind to position 0 (synchronous). */
int abra_model_reset(void *model, const int32_t *prompt, int32_t n_prompt);
/* Run n decode steps (asynchronous on the model's stream): each consumes
 * tokens[pos], appends the greedy pick once past the prompt, pos += 1. */
int abra_model_step(void *model, int32_t n_steps);
/* Prompt processing: the next n_tokens prompt tokens (a multiple of 32) in
 * chunks of up to 256 tokens, each chunk one pass of the layers with the
 * tokens as the 32-column tiles of the tcgen05 GEMVs and causal attention
 * over the shared KV cache.  It writes the KV cache bit-identically to
 * n_tokens decode steps, without logits; at least the last prompt token is
 * left to abra_model_step.  Asynchronous on the model's stream; one GPU,
 * batch 1, all-Q4_K models.  Counterpart of llama.cpp's batched prompt
 * evaluation, which the reference measures as pp512
 * (docs/research/1080ti-speed-results.md:84-91). */
int abra_model_prefill(void *model, int32_t n_tokens);
/* Prompt-lookup speculative decoding (the reference's tests/lookup_decode.cpp:
 * draft :39-51, verification and rollback :107-131).
 * abra_lookup_draft: the most recent earlier occurrence of the last `key`
 * tokens of history[0, n) proposes the up to `limit` tokens that followed
 * it; returns their count (written to out).  Host only.
 * abra_model_verify: after the prompt, with the current token (the last
 * pick) at the model's position p, evaluates [current, draft[0..n_draft))
 * (n_draft <= 31) as one 32-column pass with logits -- the same bits as
 * decode steps -- keeps the current token and every draft that equals the
 * greedy pick before it (*kept_out = 1 + accepted), and commits: the picks,
 * the next token at p + kept and the position p + kept (the KV rows past it
 * are rewritten before they are read).  picks_out receives the n_draft + 1
 * greedy picks.  Needs p + 32 <= max_ctx.  abra_model_read's logits stay
 * those of the last decode step.
 * abra_model_generate_lookup: the reference's loop -- prompt (prefill and a
 * decode step), then per block a draft from the history and its
 * verification (a plain decode step when there is no draft); the n_gen
 * tokens equal greedy decoding's.  stats (optional): proposed, accepted,
 * blocks.  One GPU, batch 1, all-Q4_K models. */
int abra_lookup_draft(const int32_t *history, int32_t n, int32_t key, int32_t limit, int32_t *out);
int abra_model_verify(void *model, const int32_t *draft, int32_t n_draft, int32_t *picks_out,
                      int32_t *kept_out);
int abra_model_generate_lookup(void *model, const int32_t *prompt, int32_t n_prompt, int32_t n_gen,
                               int32_t key, int32_t draft_max, int32_t *out, int32_t *stats);
int abra_model_sync(void *model);
/* Drop the recorded step (after abra_tune_set, for example); the next step
 * records it again.  Not for tensor-parallel models, whose ranks record
 * together at connect. */
int abra_model_invalidate(void *model);
/* Synchronises, then copies tokens[0..n_tokens) (prompt then picks), the
 * last step's logits (vocab floats) and the position; NULL skips an item. */
int abra_model_read(void *model, int32_t *tokens, int32_t n_tokens, float *logits,
                    int32_t *pos);
/* reset + (n_prompt + n_gen - 1) steps; out receives the n_gen picks. */
int abra_model_generate(void *model, const int32_t *prompt, int32_t n_prompt, int32_t n_gen,
                        int32_t *out);
/* Serving loop from the current position: per token, copy the token to
 * feed from pinned host memory to the device, run one step, copy the pick
 * back and wait for it (the host sees every token as it is produced). */
int abra_model_decode_streaming(void *model, int32_t n, int32_t *out);
int abra_model_info(void *model, void **stream, uint64_t *weight_bytes, uint64_t *kv_bytes);

/* Weights from a GGUF file.  Slots of layer -1: token_embd (1, tied with
 * the output), output_norm (2); of layer l: the GGUF names blk.l.<name>. */
#define ABRA_TENSOR_ATTN_NORM 0
#define ABRA_TENSOR_ATTN_Q 1
#define ABRA_TENSOR_ATTN_Q_NORM 2
#define ABRA_TENSOR_ATTN_K_NORM 3
#define ABRA_TENSOR_ATTN_OUTPUT 4
#define ABRA_TENSOR_FFN_NORM 5
#define ABRA_TENSOR_FFN_GATE 6
#define ABRA_TENSOR_FFN_UP 7
#define ABRA_TENSOR_FFN_DOWN 8
#define ABRA_TENSOR_ATTN_K 9
#define ABRA_TENSOR_ATTN_V 10
#define ABRA_TENSOR_TOKEN_EMBD 1  /* layer -1 */
#define ABRA_TENSOR_OUTPUT_NORM 2 /* layer -1 */
/* ggml tensor types a slot can hold */
#define ABRA_GGML_F32 0
#define ABRA_GGML_Q4_K 12
#define ABRA_GGML_Q6_K 14
/* Copy one tensor's data, as stored in a GGUF file (ggml layout: N rows of
 * K/256 blocks for a [K, N] weight; fp32 vectors for norms), from host
 * memory into the model, overwriting the seeded weights.  ggml_type and
 * bytes must match the model's slot exactly (whole, unsharded tensor); a
 * tensor-parallel rank keeps its own rows or canonical K-slices.  The
 * reference reads these files through llama.cpp; its census of the real
 * Qwen3-4B-Q4_K_M tensors is bench/results/m3/qwen3-q4k-tensor-map.json
 * (parser: tools/extract-qwen3-tensor-map.py:15-141).  Batch-1 models. */
int abra_model_load_tensor(void *model, int32_t layer, int32_t slot, int32_t ggml_type,
                           const void *host, uint64_t bytes);
/* What rank `rank` of `world` keeps of a slot's tensor (host only):
 * out[8] = {ggml type, N rows, K, bytes per row, first row, rows, first byte
 * of each row, bytes of each row} -- whole rows of its heads / FFN units, or
 * its canonical K-slices of every row (o, down). */
int abra_tp_tensor_slice(const abra_model_config *cfg, int32_t rank, int32_t world, int32_t layer,
                         int32_t slot, int64_t *out);
const char *abra_model_last_error(void);

/* ------------------------------------------------- batched decode --- */
/* batch = 32 sequences decoded in lockstep at one shared position, every
 * GEMV on the tcgen05 tensor cores (abra_q4k_mmvq_tc) with the sequences as
 * its 32 columns; the per-sequence logits and tokens are bit-identical to
 * the batch-1 model's.  batch = 1 is abra_model_create.  Prompts of the
 * batch share one length; tokens and logits are read per sequence. */
int abra_model_create_batched(const abra_model_config *cfg, int32_t batch, void **model);
/* prompts: batch x n_prompt token ids, sequence after sequence. */
int abra_model_reset_batched(void *model, const int32_t *prompts, int32_t n_prompt);
/* tokens: batch x n_tokens (prompt then picks), logits: batch x vocab. */
int abra_model_read_batched(void *model, int32_t *tokens, int32_t n_tokens, float *logits);

/* ------------------------------------------- tensor-parallel decode --- */
/* The same model split over world = 2, 4 or 8 GPUs of one node, one process
 * (or thread) per GPU.  Replaces the reference's llama.cpp tensor split with
 * an fp32 all-reduce after attn_output and ffn_down and its tied-output vocab
 * split (tools/prepare-output-split.py:8-32, runtime argmax
 * tests/runtime_logits.cpp:101).  Heads, FFN units and vocab rows are split;
 * o and down are K-sharded on canonical K-slice boundaries and each rank
 * pushes its fp32 partial sums straight from the MMVQ epilogue into every
 * rank's exchange arena over NVLink (peer stores, then a release counter);
 * the next kernel waits (bounded) for all ranks and adds the partials in the
 * fixed slice tree, so logits and greedy tokens are bit-identical to the
 * single-GPU model for every world size.  The argmax keys meet the same way.
 * Every rank must run the same sequence of calls; destroy only after all
 * ranks have finished stepping (a barrier), since peers write into each
 * other's arenas. */
typedef struct {
    int32_t rank, world;
    int32_t q_head_lo, q_heads, kv_head_lo, kv_heads; /* this rank's heads */
    int32_t ffn_lo, ffn_hi;    /* rows of gate/up and columns of down */
    int32_t sl_base, sl_cnt;   /* canonical K-slices of o and down held here */
    int64_t vocab_lo, vocab_hi; /* rows of the tied output (logits held here) */
} abra_tp_shard;

/* The split a rank would hold (no GPU needed); ABRA_E_UNSUPPORTED when the
 * configuration has no split at this world size. */
int abra_tp_shard_info(const abra_model_config *cfg, int32_t rank, int32_t world,
                       abra_tp_shard *out);
/* Build this rank's shard on the current device (world == 1 is
 * abra_model_create). */
int abra_model_create_tp(const abra_model_config *cfg, int32_t rank, int32_t world,
                         void **model);
/* The 64-byte CUDA IPC handle of this rank's exchange arena. */
int abra_model_tp_handle(void *model, void *handle, int32_t size);
/* Map every other rank's arena (handles: world entries of size_each bytes,
 * indexed by rank).  Required before the first step. */
int abra_model_tp_connect(void *model, const void *handles, int32_t size_each);
/* This rank's shard of the batch-32 model (abra_model_create_batched split
 * the same way): every GEMV on the tensor cores over the rank's rows or
 * K-slices; the o and down partial sums are pushed from the tcgen05 MMVQ's
 * epilogue into every rank's arena and each sequence's argmax keys meet on
 * every rank, so the tokens equal the one-GPU batch-32 model's.  Connect
 * with abra_model_tp_handle / abra_model_tp_connect as above. */
int abra_model_create_batched_tp(const abra_model_config *cfg, int32_t batch, int32_t rank,
                                 int32_t world, void **model);

#ifdef __cplusplus
}
#endif
#endif /* ABRA_B200_H */
