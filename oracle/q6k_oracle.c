/*
 * q6k_oracle.c -- CPU oracle for the Q6_K x Q8_1 MMVQ (the second weight
 * type of the reference's MMVQ dispatch).
 *
 * TEST INFRASTRUCTURE ONLY (see q6k_oracle.h).  Compiled with
 * -ffp-contract=off so that every fp32 operation rounds once, in the order
 * written; the CUDA kernel (abra_b200/csrc/mmvq_q6k.cu) performs the same
 * operations in the same order.
 *
 * Reference formulas restated here (paths inside talystalys/abra):
 *   Q6_K dispatch ........... kernels/q4k/abra-mmvq.cuh:138-141 (calls ggml's
 *                             vec_dot_q6_K_q8_1, llama.cpp commit 169e4a7f,
 *                             pinned by tools/setup-llama-cpp.sh:11-12)
 *   f64 Q6_K oracle ......... tests/runtime_kernel_test.cu:82-106
 *   test shapes and inputs .. tests/runtime_kernel_test.cu:119-123
 * The block is ggml's block_q6_K (210 bytes): ql[128] low 4 bits, qh[64]
 * high 2 bits, int8 scales[16] (one per 16 weights), fp16 d; weight
 * w = d * scales[e/16] * (q - 32) with q the 6-bit code of element e.
 */
#include "q6k_oracle.h"

#include <math.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define QK_K 256
#define QK8_1 32
#define Q81_BYTES 36

static inline float half_at(const uint8_t *p) {
    uint16_t h;
    memcpy(&h, p, 2);
    return orc_f16_to_f32(h);
}

/* 6-bit code of element e (0..255) of a block, in the element order of the
 * reference's f64 oracle (tests/runtime_kernel_test.cu:91-97): e = half*128 +
 * group*32 + lane; the low 4 bits are the low nibble of ql[half*64 + lane +
 * (group%2)*32] for group < 2 and its high nibble otherwise; the high 2 bits
 * are bits 2*group.. of qh[half*32 + lane]. */
static inline int q6_code(const uint8_t *blk, int e) {
    const int half = e >> 7, r = e & 127, group = r >> 5, lane = r & 31;
    const int qlb = blk[half * 64 + lane + (group & 1) * 32];
    const int low = group < 2 ? (qlb & 15) : (qlb >> 4);
    const int hi = (blk[128 + half * 32 + lane] >> (2 * group)) & 3;
    return low | (hi << 4);
}

void orc_gen_q6k(uint8_t *dst, int64_t nblocks, uint64_t seed, uint64_t tensor_id,
                 int64_t block_offset) {
    const uint64_t key = orc_stream_key(seed, tensor_id);
    for (int64_t i = 0; i < nblocks; ++i) {
        const uint64_t gb = (uint64_t)(block_offset + i);
        uint8_t *blk = dst + i * Q6K_BYTES;
        for (int w = 0; w < 26; ++w) { /* ql, qh, scales: bytes 0..207 */
            const uint64_t h = orc_stream_word(key, gb * 27u + (uint64_t)w);
            memcpy(blk + 8 * w, &h, 8); /* little-endian host */
        }
        const uint64_t h = orc_stream_word(key, gb * 27u + 26u);
        const float d = fmaf((float)(uint32_t)(h >> 40) * 5.9604644775390625e-08f, 0.0019f, 0.0001f);
        const uint16_t hd = orc_f32_to_f16(d);
        memcpy(blk + 208, &hd, 2);
    }
}

/* Exact int32 sub-block dots of one superblock: P[j] = sum over the 16
 * elements e of sub-block j of (q6(e) - 32) * q8(e). */
static inline void sb_partials(const uint8_t *blk, const uint8_t *xb, int32_t P[16]) {
    for (int j = 0; j < 16; ++j) {
        const int8_t *q8 = (const int8_t *)(xb + (j >> 1) * Q81_BYTES + 4) + 16 * (j & 1);
        int32_t acc = 0;
        for (int l = 0; l < 16; ++l) acc += (q6_code(blk, 16 * j + l) - 32) * q8[l];
        P[j] = acc;
    }
}

/* Canonical fp32 value of one superblock:
 *   I_b = P_2b * sc_2b + P_2b+1 * sc_2b+1        (exact int32, b = 0..7)
 *   t_b = d8_b * float(I_b)
 *   S   = ((t_0 + t_1) + (t_2 + t_3)) + ((t_4 + t_5) + (t_6 + t_7))
 *   value = d * S */
static inline float sb_value(const uint8_t *blk, const uint8_t *xb, const int32_t P[16]) {
    const int8_t *sc = (const int8_t *)(blk + 192);
    float t[8];
    for (int b = 0; b < 8; ++b) {
        const int32_t I = P[2 * b] * sc[2 * b] + P[2 * b + 1] * sc[2 * b + 1];
        t[b] = half_at(xb + b * Q81_BYTES) * (float)I;
    }
    const float S = ((t[0] + t[1]) + (t[2] + t[3])) + ((t[4] + t[5]) + (t[6] + t[7]));
    return half_at(blk + 208) * S;
}

static inline float tree8(const float v[8]) {
    return ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
}

static void row_slices(const uint8_t *wrow, const uint8_t *xcol, const int32_t start9[9],
                       float v[8]) {
    for (int i = 0; i < 8; ++i) {
        float acc = 0.0f;
        for (int b = start9[i]; b < start9[i + 1]; ++b) {
            int32_t P[16];
            const uint8_t *blk = wrow + (int64_t)b * Q6K_BYTES;
            const uint8_t *xb = xcol + (int64_t)b * 8 * Q81_BYTES;
            sb_partials(blk, xb, P);
            const float c = sb_value(blk, xb, P);
            acc = (b == start9[i]) ? c : acc + c;
        }
        v[i] = acc;
    }
}

void orc_q6k_partials(const uint8_t *w, const uint8_t *xq, int32_t *P, int64_t N, int64_t K,
                      int32_t ncols) {
    const int64_t nsb = K / QK_K;
    for (int32_t c = 0; c < ncols; ++c) {
        const uint8_t *xcol = xq + (int64_t)c * (K / QK8_1) * Q81_BYTES;
        for (int64_t r = 0; r < N; ++r)
            for (int64_t b = 0; b < nsb; ++b)
                sb_partials(w + (r * nsb + b) * Q6K_BYTES, xcol + b * 8 * Q81_BYTES,
                            P + ((c * N + r) * nsb + b) * 16);
    }
}

void orc_q6k_gemv(const uint8_t *w, const uint8_t *xq, float *y, int64_t N, int64_t K,
                  int32_t ncols, int32_t nthreads) {
    const int32_t nsb = (int32_t)(K / QK_K);
    int32_t start9[9];
    orc_slice_starts(nsb, start9);
    if (nthreads < 1) nthreads = 1;
#pragma omp parallel for num_threads(nthreads) schedule(static)
    for (int64_t r = 0; r < N; ++r) {
        for (int32_t c = 0; c < ncols; ++c) {
            float v[8];
            row_slices(w + r * nsb * Q6K_BYTES, xq + (int64_t)c * (K / QK8_1) * Q81_BYTES, start9, v);
            y[(int64_t)c * N + r] = tree8(v);
        }
    }
}

void orc_q6k_gemv_slices(const uint8_t *w, const uint8_t *xq, float *v, int64_t N, int64_t K,
                         int32_t ncols) {
    const int32_t nsb = (int32_t)(K / QK_K);
    int32_t start9[9];
    orc_slice_starts(nsb, start9);
    for (int32_t c = 0; c < ncols; ++c)
        for (int64_t r = 0; r < N; ++r)
            row_slices(w + r * nsb * Q6K_BYTES, xq + (int64_t)c * (K / QK8_1) * Q81_BYTES, start9,
                       v + ((int64_t)c * N + r) * 8);
}

/* Restates the reference's q6_oracle (tests/runtime_kernel_test.cu:82-106)
 * loop for loop: double accumulation over half, lane, group. */
void orc_q6k_gemv_f64(const uint8_t *w, const uint8_t *xq, double *y, int64_t N, int64_t K,
                      int32_t ncols) {
    const int64_t nsb = K / QK_K;
    for (int32_t c = 0; c < ncols; ++c) {
        const uint8_t *x = xq + (int64_t)c * (K / QK8_1) * Q81_BYTES;
        for (int64_t row = 0; row < N; ++row) {
            double total = 0;
            for (int64_t b = 0; b < nsb; ++b) {
                const uint8_t *block = w + (row * nsb + b) * Q6K_BYTES;
                const double d = half_at(block + 208);
                for (int half = 0; half < 2; ++half) {
                    const uint8_t *ql = block + half * 64;
                    const uint8_t *qh = block + 128 + half * 32;
                    const int8_t *scales = (const int8_t *)(block + 192) + half * 8;
                    for (int lane = 0; lane < 32; ++lane) {
                        for (int group = 0; group < 4; ++group) {
                            const int low = group < 2 ? ql[lane + (group % 2) * 32] & 15
                                                      : ql[lane + (group % 2) * 32] >> 4;
                            const int quant = (low | (((qh[lane] >> (group * 2)) & 3) << 4)) - 32;
                            const int index = half * 128 + group * 32 + lane;
                            const uint8_t *act = x + (b * 8 + index / 32) * Q81_BYTES;
                            total += d * scales[lane / 16 + group * 2] * quant *
                                     (double)half_at(act) * ((const int8_t *)(act + 4))[index % 32];
                        }
                    }
                }
            }
            y[(int64_t)c * N + row] = total;
        }
    }
}

void orc_q6k_absdot_f64(const uint8_t *w, const uint8_t *xq, double *s, int64_t N, int64_t K,
                        int32_t ncols) {
    const int64_t nsb = K / QK_K;
    for (int32_t c = 0; c < ncols; ++c) {
        const uint8_t *x = xq + (int64_t)c * (K / QK8_1) * Q81_BYTES;
        for (int64_t r = 0; r < N; ++r) {
            double acc = 0.0;
            for (int64_t b = 0; b < nsb; ++b) {
                const uint8_t *blk = w + (r * nsb + b) * Q6K_BYTES;
                const int8_t *sc = (const int8_t *)(blk + 192);
                const double d = half_at(blk + 208);
                for (int e = 0; e < QK_K; ++e) {
                    const uint8_t *act = x + (b * 8 + e / 32) * Q81_BYTES;
                    acc += fabs(d * sc[e / 16] * (q6_code(blk, e) - 32)) *
                           fabs((double)half_at(act) * ((const int8_t *)(act + 4))[e % 32]);
                }
            }
            s[(int64_t)c * N + r] = acc;
        }
    }
}

void orc_dequant_q6k(const uint8_t *w, float *out, int64_t nblocks) {
    for (int64_t i = 0; i < nblocks; ++i) {
        const uint8_t *blk = w + i * Q6K_BYTES;
        const int8_t *sc = (const int8_t *)(blk + 192);
        const float d = half_at(blk + 208);
        for (int e = 0; e < QK_K; ++e)
            out[i * QK_K + e] = (d * (float)sc[e / 16]) * (float)(q6_code(blk, e) - 32);
    }
}
