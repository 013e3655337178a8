/*
 * q6k_oracle.h -- CPU oracle for the Q6_K x Q8_1 MMVQ.
 *
 * TEST INFRASTRUCTURE ONLY: tests/ and bench.py's CPU leg call it as the
 * reference result; the product library never links or calls it.  Restates the
 * reference (talystalys/abra):
 *   - Q6_K leg of the MMVQ dispatch   kernels/q4k/abra-mmvq.cuh:138-141
 *   - f64 Q6_K oracle                 tests/runtime_kernel_test.cu:82-106
 * and defines the canonical fp32 order the CUDA Q6_K kernel reproduces bit
 * for bit: exact int32 16-weight sub-block dots, per-Q8_1-block scaling,
 * a fixed per-superblock tree and the same eight K-slices as Q4_K.
 */
#ifndef ABRA_Q6K_ORACLE_H
#define ABRA_Q6K_ORACLE_H

#include <stdint.h>

#include "q4k_oracle.h"

#ifdef __cplusplus
extern "C" {
#endif

#define Q6K_BYTES 210

/* Q6_K superblocks [block_offset, block_offset + nblocks) of tensor
 * `tensor_id`: ql, qh and the 16 int8 scales uniform over all byte values
 * (27 stream words per block, the first 26 give bytes 0..207), d ~
 * U(0.0001, 0.002) as fp16 from word 26. */
void orc_gen_q6k(uint8_t *dst, int64_t nblocks, uint64_t seed, uint64_t tensor_id,
                 int64_t block_offset);

/* Exact int32 sub-block dots P[c][r][b][16]. */
void orc_q6k_partials(const uint8_t *w, const uint8_t *xq, int32_t *P, int64_t N, int64_t K,
                      int32_t ncols);
/* Canonical fp32 GEMV y[c][r]; nthreads > 1 uses OpenMP over rows. */
void orc_q6k_gemv(const uint8_t *w, const uint8_t *xq, float *y, int64_t N, int64_t K,
                  int32_t ncols, int32_t nthreads);
/* The eight canonical K-slice sums v[c][r][8] before the final tree. */
void orc_q6k_gemv_slices(const uint8_t *w, const uint8_t *xq, float *v, int64_t N, int64_t K,
                         int32_t ncols);
/* The reference's double-precision oracle, loop for loop. */
void orc_q6k_gemv_f64(const uint8_t *w, const uint8_t *xq, double *y, int64_t N, int64_t K,
                      int32_t ncols);
/* Per-row tolerance scale sum_k |w_k| |x_k| in double. */
void orc_q6k_absdot_f64(const uint8_t *w, const uint8_t *xq, double *s, int64_t N, int64_t K,
                        int32_t ncols);
/* w = (d * sc) * (q - 32) per element, fp32. */
void orc_dequant_q6k(const uint8_t *w, float *out, int64_t nblocks);

#ifdef __cplusplus
}
#endif
#endif
