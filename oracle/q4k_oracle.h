/*
 * q4k_oracle.h -- CPU oracle for the Q4_K x Q8_1 decode path.
 *
 * TEST INFRASTRUCTURE ONLY.  This is the test oracle: tests/, the smoke entry
 * and the CPU-baseline leg of bench.py call it; the product library never
 * links or calls it.  It restates, in plain C, the arithmetic of the
 * reference (talystalys/abra):
 *   - block layouts            kernels/q4k/q4k_q8_mmvq.cuh:42-57
 *   - 6-bit scale/min unpack   tests/q4k_q8_test.cu:44-52
 *   - nibble layout + f64 dot  tests/q4k_q8_test.cu:54-107
 *   - vec_dot_q4_K_q8_1        kernels/q4k/q4k_vecdot.cuh:23-87
 *   - F32 -> Q8_1 quantizer    kernels/q4k/q4k_q8_mmvq.cu:223-255
 * and defines the canonical fp32 evaluation order that every CUDA kernel of
 * abra_b200 reproduces bit for bit (exact int32 sub-block partials, fixed
 * per-superblock tree, eight fixed K-slices).
 */
#ifndef ABRA_Q4K_ORACLE_H
#define ABRA_Q4K_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- fp16 helpers (IEEE binary16, round-to-nearest-even) ---------------- */
uint16_t orc_f32_to_f16(float f);
float    orc_f16_to_f32(uint16_t h);

/* ---- seeded synthetic generators (counter-based, splitmix64) ------------ */
/* Word i of the stream of (seed, tensor_id): the i-th splitmix64 output
 * from key = orc_stream_key(seed, tensor_id). */
uint64_t orc_stream_key(uint64_t seed, uint64_t tensor_id);
uint64_t orc_stream_word(uint64_t key, uint64_t i);
/* Q4_K superblocks [block_offset, block_offset + nblocks) of tensor
 * `tensor_id`: d, dmin ~ U(0.001, 0.02) as fp16, 12 scale bytes (= sixteen
 * 6-bit sc/m values ~ U{0..63}) and 128 nibble bytes (nibbles ~ U{0..15}). */
void orc_gen_q4k(uint8_t *dst, int64_t nblocks, uint64_t seed, uint64_t tensor_id,
                 int64_t block_offset);
/* flags bit 0: centred variant -- same d, scales and nibbles, but
 * dmin = 7.5 d max(sc) / 63 and m_s = round(63 sc_s / max(sc)), so each
 * sub-block's weights have mean ~0. */
void orc_gen_q4k_ex(uint8_t *dst, int64_t nblocks, uint64_t seed, uint64_t tensor_id,
                    int64_t block_offset, int32_t flags);
/* fp32 values fmaf(u, scale, offset) with u ~ U[0,1) on a 2^-24 grid. */
void orc_gen_uniform_f32(float *dst, int64_t n, uint64_t seed, uint64_t tensor_id,
                         int64_t offset_index, float scale, float offset);

/* Synthetic-model norm weights: +-U(0.8, 1.2), random sign (bit 0). */
void orc_gen_norm_f32(float *dst, int64_t n, uint64_t seed, uint64_t tensor_id);

/* ---- Q8_1 quantizer (reference semantics, q4k_q8_mmvq.cu:223-255) ------- */
/* x: ncols x K fp32 (column-contiguous); y: ncols x (K/32) blocks of 36 B. */
void orc_quantize_q8_1(const float *x, uint8_t *y, int64_t K, int32_t ncols);

/* Fused RMSNorm -> Q8_1: xn = (x * r) * w with r = 1/sqrt(mean(x^2) + eps),
 * sum of squares in the canonical 256-thread order.  xn_out may be NULL. */
void orc_rmsnorm_quantize_q8_1(const float *x, const float *w, float eps, uint8_t *y,
                               float *xn_out, int64_t K, int32_t ncols);
float orc_rms_scale(const float *x, float eps, int64_t K);

/* ---- elementwise math (same op sequence as the CUDA kernels) ----------- */
float orc_expf(float x);
float orc_silu(float g);
void orc_swiglu(const float *gate, const float *up, float *y, int64_t n);

/* ---- MMVQ ---------------------------------------------------------------- */
/* Exact int32 partials.  P[c][r][b][s] = sum_{l<32} q4 * q8 over sub-block s
 * of superblock b of row r against column c; M[c][b][s] = sum_{l<32} q8. */
void orc_q4k_partials(const uint8_t *w, const uint8_t *xq, int32_t *P, int32_t *M,
                      int64_t N, int64_t K, int32_t ncols);
/* Canonical fp32 GEMV, y[c][r].  nthreads > 1 uses OpenMP over rows. */
/* llama.cpp's CPU Q4_K path restated (the timed CPU baseline, not a parity
 * target): Q8_K activation blocks (fp32 d, 256 int8, 16 int16 sums; 292 B)
 * and the Q4_K x Q8_K dot; nthreads > 1 uses OpenMP over rows. */
void orc_quantize_q8_K(const float *x, uint8_t *y, int64_t K, int32_t ncols);
void orc_q4k_q8k_gemv(const uint8_t *w, const uint8_t *yq, float *y, int64_t N, int64_t K,
                      int32_t ncols, int32_t nthreads);
void orc_q4k_gemv(const uint8_t *w, const uint8_t *xq, float *y, int64_t N, int64_t K,
                  int32_t ncols, int32_t nthreads);
/* Canonical per-slice values v[c][r][8] (the eight K-slice sums before the
 * final tree), used to check split-K and tensor-parallel partitions. */
void orc_q4k_gemv_slices(const uint8_t *w, const uint8_t *xq, float *v, int64_t N,
                         int64_t K, int32_t ncols);
/* Independent double-precision oracle (tests/q4k_q8_test.cu:54-107). */
void orc_q4k_gemv_f64(const uint8_t *w, const uint8_t *xq, double *y, int64_t N,
                      int64_t K, int32_t ncols);
/* Per-row tolerance scale: sum_k |w_k| * |x_k| in double. */
void orc_q4k_absdot_f64(const uint8_t *w, const uint8_t *xq, double *s, int64_t N,
                        int64_t K, int32_t ncols);
/* Dequantize Q4_K rows to fp32 (w = fmaf(d*sc, q, -(dmin*m))). */
void orc_dequant_q4k(const uint8_t *w, float *out, int64_t nblocks);

/* Canonical K-slice layout for nsb superblocks: start[0..8]. */
void orc_slice_starts(int32_t nsb, int32_t *start9);

int32_t orc_max_threads(void);

/* Integer-dot implementation of the GEMVs: 0 scalar, 1 AVX2, 2 AVX-512 VNNI
 * (the best the host has, unless lowered; the results are the same bits). */
int32_t orc_simd_level(void);
void orc_set_simd_level(int32_t level); /* < 0: the best again */

#ifdef __cplusplus
}
#endif
#endif
