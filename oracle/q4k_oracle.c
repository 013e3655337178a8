/*
 * q4k_oracle.c -- CPU oracle for the Q4_K x Q8_1 decode path.
 *
 * TEST INFRASTRUCTURE ONLY (see q4k_oracle.h).  Compiled with
 * -ffp-contract=off so that every fp32 operation below rounds exactly once,
 * in the order written; the CUDA kernels use __fmul_rn/__fadd_rn/__fmaf_rn in
 * the same order, which is what makes the two bit-identical.
 *
 * Reference formulas restated here (paths inside talystalys/abra):
 *   block_q4_K / block_q8_1 ........ kernels/q4k/q4k_q8_mmvq.cuh:42-57
 *   get_scale_min_k4 ............... tests/q4k_q8_test.cu:44-52
 *   f64 oracle ..................... tests/q4k_q8_test.cu:54-107
 *   vec_dot_q4_K_q8_1 .............. kernels/q4k/q4k_vecdot.cuh:23-87
 *   Q8_1 quantizer ................. kernels/q4k/q4k_q8_mmvq.cu:223-255
 */
#include "q4k_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define QK_K 256
#define QK8_1 32
#define Q4K_BYTES 144
#define Q81_BYTES 36

/* ------------------------------------------------------------------------ */
/* fp16 <-> fp32, IEEE binary16 with round-to-nearest-even                  */
/* ------------------------------------------------------------------------ */
float orc_f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h >> 15) << 31;
    const uint32_t exp = (h >> 10) & 0x1f;
    const uint32_t man = h & 0x3ff;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else { /* subnormal: value = man * 2^-24, exact in fp32 */
            float v = (float)man * 5.9604644775390625e-08f;
            memcpy(&bits, &v, 4);
            bits |= sign;
        }
    } else if (exp == 0x1f) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((exp + 112u) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

uint16_t orc_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    const uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) { /* inf or nan */
        return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
    }
    if (ax >= 0x477ff000u) { /* rounds to >= 65520 -> inf */
        return (uint16_t)(sign | 0x7c00u);
    }
    if (ax < 0x38800000u) { /* below 2^-14: subnormal half (or zero) */
        /* value / 2^-24, rounded to nearest even, as an integer 0..1024 */
        const uint32_t e = ax >> 23;
        if (e < 102) return sign; /* < 2^-25: rounds to 0 */
        const uint32_t m = (ax & 0x7fffffu) | 0x800000u;
        const uint32_t shift = 126 - e; /* 14 + (126-14-e) ... */
        /* value = m * 2^(e-150); in units of 2^-24 -> m * 2^(e-126) */
        const uint32_t q = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1u);
        const uint32_t half = 1u << (shift - 1);
        uint32_t r = q;
        if (rem > half || (rem == half && (q & 1u))) r++;
        return (uint16_t)(sign | r);
    }
    /* normal half */
    uint32_t r = ((ax >> 13) - (112u << 10));
    const uint32_t rem = ax & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) r++;
    return (uint16_t)(sign | r);
}

/* ------------------------------------------------------------------------ */
/* Counter-based generator: word i of a stream is the splitmix64 finaliser   */
/* applied to key + (i+1) * golden-gamma, i.e. the i-th splitmix64 output.   */
/* ------------------------------------------------------------------------ */
static inline uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
static inline uint64_t stream_key(uint64_t seed, uint64_t tensor_id) {
    return mix64(seed + 0x9E3779B97F4A7C15ull) ^ mix64(tensor_id * 0xD1B54A32D192ED03ull + 1ull);
}
static inline uint64_t stream_word(uint64_t key, uint64_t i) {
    return mix64(key + (i + 1ull) * 0x9E3779B97F4A7C15ull);
}
uint64_t orc_stream_key(uint64_t seed, uint64_t tensor_id) { return stream_key(seed, tensor_id); }
uint64_t orc_stream_word(uint64_t key, uint64_t i) { return stream_word(key, i); }
static inline float unit24(uint64_t bits24) { /* exact: 24-bit int * 2^-24 */
    return (float)(uint32_t)bits24 * 5.9604644775390625e-08f;
}

/* 12 packed scale bytes <-> eight 6-bit scales and mins (the packing that
 * get_scale_min_k4, tests/q4k_q8_test.cu:44-52, reads). */
static void unpack_scales(const uint8_t *q, int sc[8], int m[8]) {
    for (int j = 0; j < 4; ++j) {
        sc[j] = q[j] & 63;
        m[j] = q[j + 4] & 63;
        sc[j + 4] = (q[j + 8] & 0xF) | ((q[j] >> 6) << 4);
        m[j + 4] = (q[j + 8] >> 4) | ((q[j + 4] >> 6) << 4);
    }
}
static void pack_scales(const int sc[8], const int m[8], uint8_t *q) {
    for (int j = 0; j < 4; ++j) {
        q[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
        q[j + 4] = (uint8_t)((m[j] & 63) | ((m[j + 4] >> 4) << 6));
        q[j + 8] = (uint8_t)((sc[j + 4] & 15) | ((m[j + 4] & 15) << 4));
    }
}

void orc_gen_q4k_ex(uint8_t *dst, int64_t nblocks, uint64_t seed, uint64_t tensor_id,
                    int64_t block_offset, int32_t flags) {
    const uint64_t key = stream_key(seed, tensor_id);
    for (int64_t i = 0; i < nblocks; ++i) {
        const uint64_t gb = (uint64_t)(block_offset + i);
        uint8_t *blk = dst + i * Q4K_BYTES;
        for (int w = 0; w < 18; ++w) {
            const uint64_t h = stream_word(key, gb * 18u + (uint64_t)w);
            memcpy(blk + 8 * w, &h, 8); /* little-endian host */
        }
        const uint64_t h0 = stream_word(key, gb * 18u);
        const float d = fmaf(unit24(h0 >> 40), 0.019f, 0.001f);
        const float dmin = fmaf(unit24((h0 >> 16) & 0xffffffu), 0.019f, 0.001f);
        const uint16_t hd = orc_f32_to_f16(d);
        uint16_t hm = orc_f32_to_f16(dmin);
        if (flags & 1) {
            /* centred: dmin * m_s ~= 7.5 * d * sc_s, so every sub-block of
             * d*sc*q - dmin*m has mean ~0 over nibbles ~ U{0..15} */
            int sc[8], m[8], mx = 0;
            unpack_scales(blk + 4, sc, m);
            for (int s = 0; s < 8; ++s) mx = sc[s] > mx ? sc[s] : mx;
            if (mx == 0) {
                hm = 0;
                for (int s = 0; s < 8; ++s) m[s] = 0;
            } else {
                const float df = orc_f16_to_f32(hd);
                hm = orc_f32_to_f16(((7.5f * df) * (float)mx) / 63.0f);
                for (int s = 0; s < 8; ++s) m[s] = (63 * sc[s] + mx / 2) / mx;
            }
            pack_scales(sc, m, blk + 4);
        }
        memcpy(blk + 0, &hd, 2);
        memcpy(blk + 2, &hm, 2);
    }
}

void orc_gen_q4k(uint8_t *dst, int64_t nblocks, uint64_t seed, uint64_t tensor_id,
                 int64_t block_offset) {
    orc_gen_q4k_ex(dst, nblocks, seed, tensor_id, block_offset, 0);
}

void orc_gen_uniform_f32(float *dst, int64_t n, uint64_t seed, uint64_t tensor_id,
                         int64_t offset_index, float scale, float offset) {
    const uint64_t key = stream_key(seed, tensor_id);
    for (int64_t i = 0; i < n; ++i) {
        const uint64_t h = stream_word(key, (uint64_t)(offset_index + i));
        dst[i] = fmaf(unit24(h >> 40), scale, offset);
    }
}

/* Norm weights of the synthetic model: magnitude fmaf(u, 0.4, 0.8) ~ U(0.8,
 * 1.2) from bits 63..40 of the stream word, sign from bit 0. */
void orc_gen_norm_f32(float *dst, int64_t n, uint64_t seed, uint64_t tensor_id) {
    const uint64_t key = stream_key(seed, tensor_id);
    for (int64_t i = 0; i < n; ++i) {
        const uint64_t h = stream_word(key, (uint64_t)i);
        const float v = fmaf(unit24(h >> 40), 0.4f, 0.8f);
        dst[i] = (h & 1u) ? -v : v;
    }
}

/* ------------------------------------------------------------------------ */
/* Q8_1 quantizer.  Restates kernels/q4k/q4k_q8_mmvq.cu:223-255: amax over   */
/* 32, d = amax/127, id = d>0 ? 1/d : 0, q = (int8)roundf(x*id), s = d*sum.  */
/* ------------------------------------------------------------------------ */
static void quantize_block(const float *x, uint8_t *out) {
    float amax = 0.0f;
    for (int j = 0; j < QK8_1; ++j) {
        const float v = fabsf(x[j]);
        if (v > amax) amax = v;
    }
    const float d = amax / 127.0f;
    const float id = d > 0.0f ? 1.0f / d : 0.0f;
    int sum = 0;
    int8_t *qs = (int8_t *)(out + 4);
    for (int j = 0; j < QK8_1; ++j) {
        const int8_t q = (int8_t)roundf(x[j] * id);
        qs[j] = q;
        sum += q;
    }
    const uint16_t hd = orc_f32_to_f16(d);
    const uint16_t hs = orc_f32_to_f16(d * (float)sum);
    memcpy(out + 0, &hd, 2);
    memcpy(out + 2, &hs, 2);
}

void orc_quantize_q8_1(const float *x, uint8_t *y, int64_t K, int32_t ncols) {
    const int64_t nb = K / QK8_1;
    for (int32_t c = 0; c < ncols; ++c)
        for (int64_t i = 0; i < nb; ++i)
            quantize_block(x + c * K + i * QK8_1, y + (c * nb + i) * Q81_BYTES);
}

/* Canonical sum of squares: 256 threads; thread t accumulates x[t + 256 i]
 * with fmaf in increasing i; each 32-lane warp reduces with an xor butterfly
 * (masks 16, 8, 4, 2, 1); the eight warp sums are added in warp order. */
static float canonical_sumsq(const float *x, int64_t K) {
    float lane[256];
    for (int t = 0; t < 256; ++t) {
        float acc = 0.0f;
        for (int64_t i = t; i < K; i += 256) acc = fmaf(x[i], x[i], acc);
        lane[t] = acc;
    }
    float warp[8];
    for (int w = 0; w < 8; ++w) {
        float v[32], tmp[32];
        for (int l = 0; l < 32; ++l) v[l] = lane[w * 32 + l];
        for (int m = 16; m >= 1; m >>= 1) {
            for (int l = 0; l < 32; ++l) tmp[l] = v[l] + v[l ^ m];
            memcpy(v, tmp, sizeof v);
        }
        warp[w] = v[0];
    }
    float total = warp[0];
    for (int w = 1; w < 8; ++w) total = total + warp[w];
    return total;
}

float orc_rms_scale(const float *x, float eps, int64_t K) {
    const float mean = canonical_sumsq(x, K) / (float)K;
    return 1.0f / sqrtf(mean + eps);
}

void orc_rmsnorm_quantize_q8_1(const float *x, const float *w, float eps, uint8_t *y,
                               float *xn_out, int64_t K, int32_t ncols) {
    float *tmp = (float *)malloc((size_t)K * sizeof(float));
    for (int32_t c = 0; c < ncols; ++c) {
        const float *xc = x + c * K;
        const float r = orc_rms_scale(xc, eps, K);
        for (int64_t i = 0; i < K; ++i) tmp[i] = (xc[i] * r) * w[i];
        if (xn_out) memcpy(xn_out + c * K, tmp, (size_t)K * sizeof(float));
        orc_quantize_q8_1(tmp, y + c * (K / QK8_1) * Q81_BYTES, K, 1);
    }
    free(tmp);
}

/* ------------------------------------------------------------------------ */
/* exp: Cody & Waite range reduction x = k ln2 + r (ln2 split into a 16-bit  */
/* head and a tail), e^r by the degree-7 Taylor polynomial in Horner form,   */
/* then scaling by 2^k.  Every step is an IEEE fp32 operation (fmaf, *), so  */
/* the CUDA copy in abra_b200/csrc/common.cuh returns the same bits.          */
/* Error about 2 ulp against the exact exponential.                           */
/* ------------------------------------------------------------------------ */
static inline float pow2i(int k) { /* 2^k for -126 <= k <= 127 */
    const uint32_t bits = (uint32_t)(k + 127) << 23;
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

float orc_expf(float x) {
    if (x != x) return x;
    if (x > 88.75f) return INFINITY;
    if (x < -104.0f) return 0.0f;
    const float kf = rintf(x * 0x1.715476p+0f);        /* x * log2(e) */
    float r = fmaf(kf, -0x1.62e400p-1f, x);            /* - k * ln2 (head) */
    r = fmaf(kf, -0x1.7f7d1cp-20f, r);                 /* - k * ln2 (tail) */
    float p = 0x1.a01a02p-13f;                         /* 1/5040 */
    p = fmaf(p, r, 0x1.6c16c2p-10f);                   /* 1/720 */
    p = fmaf(p, r, 0x1.111112p-7f);                    /* 1/120 */
    p = fmaf(p, r, 0x1.555556p-5f);                    /* 1/24 */
    p = fmaf(p, r, 0x1.555556p-3f);                    /* 1/6 */
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    const int k = (int)kf;
    if (k > 127) return (p * pow2i(127)) * pow2i(k - 127);
    if (k < -126) return (p * pow2i(k + 64)) * pow2i(-64);
    return p * pow2i(k);
}

/* silu(g) = g / (1 + exp(-g)) (ggml's ggml_cuda_op_silu_single formula). */
float orc_silu(float g) { return g / (1.0f + orc_expf(-g)); }

/* y = up * silu(gate), the GLU epilogue of the fused gate/up kernel
 * (reference: kernels/q4k/abra-mmvq.cuh:175-186, GGML_GLU_OP_SWIGLU). */
void orc_swiglu(const float *gate, const float *up, float *y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) y[i] = up[i] * orc_silu(gate[i]);
}

/* ------------------------------------------------------------------------ */
/* Q4_K helpers                                                             */
/* ------------------------------------------------------------------------ */
/* 6-bit scale and min of sub-block j (tests/q4k_q8_test.cu:44-52). */
static inline void scale_min(const uint8_t *q, int j, int *sc, int *m) {
    if (j < 4) {
        *sc = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        *m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}
static inline float half_at(const uint8_t *p) {
    uint16_t h;
    memcpy(&h, p, 2);
    return orc_f16_to_f32(h);
}

/* Exact int32 partials of one superblock against one column's 8 Q8_1 blocks.
 * Sub-block 2p uses the low nibbles of qs[32p..32p+31], sub-block 2p+1 the
 * high nibbles of the same bytes (tests/q4k_q8_test.cu:76-102). */
static inline void sb_partials(const uint8_t *blk, const uint8_t *xb, int32_t P[8],
                               int32_t M[8]) {
    const uint8_t *qs = blk + 16;
    for (int p = 0; p < 4; ++p) {
        const int8_t *q8lo = (const int8_t *)(xb + (2 * p) * Q81_BYTES + 4);
        const int8_t *q8hi = (const int8_t *)(xb + (2 * p + 1) * Q81_BYTES + 4);
        int32_t plo = 0, phi = 0, mlo = 0, mhi = 0;
        for (int l = 0; l < 32; ++l) {
            const int byte = qs[32 * p + l];
            plo += (byte & 0xF) * q8lo[l];
            phi += (byte >> 4) * q8hi[l];
            mlo += q8lo[l];
            mhi += q8hi[l];
        }
        P[2 * p] = plo;
        P[2 * p + 1] = phi;
        M[2 * p] = mlo;
        M[2 * p + 1] = mhi;
    }
}

/* Canonical fp32 value of one superblock (the order the kernels follow):
 *   t_s = d8_s * float(P_s * sc_s)      u_s = (d8_s * float(M_s)) * float(m_s)
 *   tp_p = t_2p + t_2p+1                 up_p = u_2p + u_2p+1
 *   Sd = (tp_0 + tp_1) + (tp_2 + tp_3)   Sm likewise
 *   value = fmaf(d, Sd, -(dmin * Sm))
 * d8_s*float(M_s) and P_s*sc_s are exact, so each t_s/u_s rounds once. */
static inline float sb_value(const uint8_t *blk, const uint8_t *xb, const int32_t P[8],
                             const int32_t M[8]) {
    const float d = half_at(blk), dmin = half_at(blk + 2);
    float tp[4], up[4];
    for (int p = 0; p < 4; ++p) {
        float t[2], u[2];
        for (int i = 0; i < 2; ++i) {
            const int s = 2 * p + i;
            int sc, m;
            scale_min(blk + 4, s, &sc, &m);
            const float d8 = half_at(xb + s * Q81_BYTES);
            t[i] = d8 * (float)(P[s] * sc);
            const float A = d8 * (float)M[s];
            u[i] = A * (float)m;
        }
        tp[p] = t[0] + t[1];
        up[p] = u[0] + u[1];
    }
    const float Sd = (tp[0] + tp[1]) + (tp[2] + tp[3]);
    const float Sm = (up[0] + up[1]) + (up[2] + up[3]);
    return fmaf(d, Sd, -(dmin * Sm));
}

void orc_slice_starts(int32_t nsb, int32_t *start9) {
    start9[0] = 0;
    for (int i = 0; i < 8; ++i) start9[i + 1] = start9[i] + nsb / 8 + (i < nsb % 8 ? 1 : 0);
}

static inline float tree8(const float v[8]) {
    return ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
}

/* ---- the integer sub-block dots, vectorised ------------------------------
 * P[s] = sum_l q4 * q8 over sub-block s is an exact integer in any order, so
 * the GEMVs compute it with the widest integer dot the host has (AVX-512
 * VNNI vpdpbusd, AVX2 vpmaddubsw + vpmaddwd, or the scalar loop of
 * sb_partials) on activations staged once per column as contiguous int8;
 * the fp32 part (sb_value) is unchanged.  Sub-block 2p is the low nibbles of
 * qs[32p..32p+31] against x[64p..64p+31], sub-block 2p+1 the high nibbles
 * against x[64p+32..64p+63], so one 64-byte step covers a pair. */
typedef void (*sb_dots_fn)(const uint8_t *qs, const int8_t *x, int32_t P[8]);

static void sb_dots_scalar(const uint8_t *qs, const int8_t *x, int32_t P[8]) {
    for (int p = 0; p < 4; ++p) {
        int32_t lo = 0, hi = 0;
        for (int l = 0; l < 32; ++l) {
            lo += (qs[32 * p + l] & 0xF) * x[64 * p + l];
            hi += (qs[32 * p + l] >> 4) * x[64 * p + 32 + l];
        }
        P[2 * p] = lo;
        P[2 * p + 1] = hi;
    }
}

#if defined(__x86_64__) && defined(__GNUC__)
#include <immintrin.h>

__attribute__((target("avx2"))) static inline int32_t hsum8_avx2(__m256i v) {
    __m128i s = _mm_add_epi32(_mm256_castsi256_si128(v), _mm256_extracti128_si256(v, 1));
    s = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0x4E));
    s = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0xB1));
    return _mm_cvtsi128_si32(s);
}

__attribute__((target("avx2"))) static void sb_dots_avx2(const uint8_t *qs, const int8_t *x,
                                                        int32_t P[8]) {
    const __m256i m4 = _mm256_set1_epi8(0x0F), ones = _mm256_set1_epi16(1);
    for (int p = 0; p < 4; ++p) {
        const __m256i b = _mm256_loadu_si256((const __m256i *)(qs + 32 * p));
        const __m256i lo = _mm256_and_si256(b, m4);
        const __m256i hi = _mm256_and_si256(_mm256_srli_epi16(b, 4), m4);
        const __m256i xl = _mm256_loadu_si256((const __m256i *)(x + 64 * p));
        const __m256i xh = _mm256_loadu_si256((const __m256i *)(x + 64 * p + 32));
        /* u4 x s8 pair sums stay within int16 (|15 * 127 * 2| < 2^15) */
        P[2 * p] = hsum8_avx2(_mm256_madd_epi16(_mm256_maddubs_epi16(lo, xl), ones));
        P[2 * p + 1] = hsum8_avx2(_mm256_madd_epi16(_mm256_maddubs_epi16(hi, xh), ones));
    }
}

__attribute__((target("avx512f,avx512bw,avx512vnni,avx2"))) static void sb_dots_vnni(
    const uint8_t *qs, const int8_t *x, int32_t P[8]) {
    const __m256i m4 = _mm256_set1_epi8(0x0F);
    for (int p = 0; p < 4; ++p) {
        const __m256i b = _mm256_loadu_si256((const __m256i *)(qs + 32 * p));
        const __m256i lo = _mm256_and_si256(b, m4);
        const __m256i hi = _mm256_and_si256(_mm256_srli_epi16(b, 4), m4);
        const __m512i wv = _mm512_inserti64x4(_mm512_castsi256_si512(lo), hi, 1);
        const __m512i xv = _mm512_loadu_si512((const void *)(x + 64 * p));
        const __m512i acc = _mm512_dpbusd_epi32(_mm512_setzero_si512(), wv, xv);
        P[2 * p] = hsum8_avx2(_mm512_castsi512_si256(acc));
        P[2 * p + 1] = hsum8_avx2(_mm512_extracti64x4_epi64(acc, 1));
    }
}
#endif

static int32_t g_simd = -1; /* -1: not chosen yet; 0 scalar, 1 AVX2, 2 AVX-512 VNNI */

int32_t orc_simd_level(void) {
    if (g_simd < 0) {
        g_simd = 0;
#if defined(__x86_64__) && defined(__GNUC__)
        __builtin_cpu_init();
        if (__builtin_cpu_supports("avx2")) g_simd = 1;
        if (__builtin_cpu_supports("avx512f") && __builtin_cpu_supports("avx512bw") &&
            __builtin_cpu_supports("avx512vnni"))
            g_simd = 2;
#endif
    }
    return g_simd;
}

void orc_set_simd_level(int32_t level) {
    const int32_t best = (g_simd = -1, orc_simd_level());
    g_simd = level < 0 ? best : (level < best ? level : best);
}

static sb_dots_fn sb_dots(void) {
#if defined(__x86_64__) && defined(__GNUC__)
    switch (orc_simd_level()) {
        case 2: return sb_dots_vnni;
        case 1: return sb_dots_avx2;
        default: break;
    }
#endif
    return sb_dots_scalar;
}

/* One activation column staged for the vectorised dots: the K int8 values
 * contiguous and M[s] = sum of each 32-block. */
typedef struct {
    int8_t *x8;
    int32_t *M;
    float *d8; /* the blocks' fp16 scales as fp32 (the values half_at gives) */
} xstage;

static xstage stage_column(const uint8_t *xcol, int64_t K) {
    xstage st;
    st.x8 = (int8_t *)malloc((size_t)K);
    st.M = (int32_t *)malloc((size_t)(K / QK8_1) * sizeof(int32_t));
    st.d8 = (float *)malloc((size_t)(K / QK8_1) * sizeof(float));
    for (int64_t i = 0; i < K / QK8_1; ++i) {
        const int8_t *q = (const int8_t *)(xcol + i * Q81_BYTES + 4);
        int32_t m = 0;
        for (int l = 0; l < QK8_1; ++l) {
            st.x8[i * QK8_1 + l] = q[l];
            m += q[l];
        }
        st.M[i] = m;
        st.d8[i] = half_at(xcol + i * Q81_BYTES);
    }
    return st;
}

static void free_stage(xstage *st) {
    free(st->x8);
    free(st->M);
    free(st->d8);
}

/* sb_value with the column's staged d8: the same operations on the same
 * values, so the same bits. */
static inline float sb_value_staged(const uint8_t *blk, const float *d8, const int32_t P[8],
                                    const int32_t M[8]) {
    const float d = half_at(blk), dmin = half_at(blk + 2);
    float tp[4], up[4];
    for (int p = 0; p < 4; ++p) {
        float t[2], u[2];
        for (int i = 0; i < 2; ++i) {
            const int s = 2 * p + i;
            int sc, m;
            scale_min(blk + 4, s, &sc, &m);
            t[i] = d8[s] * (float)(P[s] * sc);
            const float A = d8[s] * (float)M[s];
            u[i] = A * (float)m;
        }
        tp[p] = t[0] + t[1];
        up[p] = u[0] + u[1];
    }
    const float Sd = (tp[0] + tp[1]) + (tp[2] + tp[3]);
    const float Sm = (up[0] + up[1]) + (up[2] + up[3]);
    return fmaf(d, Sd, -(dmin * Sm));
}

/* Slice sums of one row against one column: sequential within a slice,
 * +0.0f for an empty slice. */
static void row_slices(const uint8_t *wrow, const xstage *st, sb_dots_fn dots,
                       const int32_t start9[9], float v[8]) {
    for (int i = 0; i < 8; ++i) {
        float acc = 0.0f;
        for (int b = start9[i]; b < start9[i + 1]; ++b) {
            int32_t P[8];
            const uint8_t *blk = wrow + (int64_t)b * Q4K_BYTES;
            dots(blk + 16, st->x8 + (int64_t)b * QK_K, P);
            const float c = sb_value_staged(blk, st->d8 + (int64_t)b * 8, P, st->M + (int64_t)b * 8);
            acc = (b == start9[i]) ? c : acc + c;
        }
        v[i] = acc;
    }
}

void orc_q4k_partials(const uint8_t *w, const uint8_t *xq, int32_t *P, int32_t *M,
                      int64_t N, int64_t K, int32_t ncols) {
    const int64_t nsb = K / QK_K;
    for (int32_t c = 0; c < ncols; ++c) {
        const uint8_t *xcol = xq + (int64_t)c * (K / QK8_1) * Q81_BYTES;
        for (int64_t r = 0; r < N; ++r)
            for (int64_t b = 0; b < nsb; ++b) {
                int32_t p8[8], m8[8];
                sb_partials(w + (r * nsb + b) * Q4K_BYTES, xcol + b * 8 * Q81_BYTES, p8, m8);
                memcpy(P + ((c * N + r) * nsb + b) * 8, p8, sizeof p8);
                if (r == 0) memcpy(M + (c * nsb + b) * 8, m8, sizeof m8);
            }
    }
}

void orc_q4k_gemv(const uint8_t *w, const uint8_t *xq, float *y, int64_t N, int64_t K,
                  int32_t ncols, int32_t nthreads) {
    const int32_t nsb = (int32_t)(K / QK_K);
    int32_t start9[9];
    orc_slice_starts(nsb, start9);
    if (nthreads < 1) nthreads = 1;
    const sb_dots_fn dots = sb_dots();
    xstage *st = (xstage *)malloc((size_t)ncols * sizeof(xstage));
    for (int32_t c = 0; c < ncols; ++c) st[c] = stage_column(xq + (int64_t)c * (K / QK8_1) * Q81_BYTES, K);
#pragma omp parallel for num_threads(nthreads) schedule(static)
    for (int64_t r = 0; r < N; ++r) {
        for (int32_t c = 0; c < ncols; ++c) {
            float v[8];
            row_slices(w + r * nsb * Q4K_BYTES, &st[c], dots, start9, v);
            y[(int64_t)c * N + r] = tree8(v);
        }
    }
    for (int32_t c = 0; c < ncols; ++c) free_stage(&st[c]);
    free(st);
}

/* ------------------------------------------------------------------------ */
/* llama.cpp's CPU Q4_K path, restated: the timed CPU baseline              */
/* ------------------------------------------------------------------------ */
/* On the CPU, ggml multiplies Q4_K rows by activations quantized to Q8_K
 * rather than Q8_1: blocks of 256 int8 values with one fp32 scale and the
 * sixteen sums of 16 values (block_q8_K: float d; int8 qs[256];
 * int16 bsums[16], 292 bytes).  Restated here from the published algorithm
 * of ggml's quantize_row_q8_K and generic vec_dot_q4_K_q8_K (llama.cpp
 * commit 169e4a7f, which the reference pins in tools/setup-llama-cpp.sh),
 * with the integer dots on the same vectorised helpers as above.  It times
 * the CPU path the reference itself runs on the host; it is not a parity
 * target. */
#define Q8K_BYTES 292

void orc_quantize_q8_K(const float *x, uint8_t *y, int64_t K, int32_t ncols) {
    const int64_t nb = K / QK_K;
    for (int32_t c = 0; c < ncols; ++c)
        for (int64_t b = 0; b < nb; ++b) {
            const float *xb = x + (int64_t)c * K + b * QK_K;
            uint8_t *out = y + ((int64_t)c * nb + b) * Q8K_BYTES;
            float amax = 0.0f, mx = 0.0f; /* the value of largest magnitude, with its sign */
            for (int j = 0; j < QK_K; ++j)
                if (fabsf(xb[j]) > amax) {
                    amax = fabsf(xb[j]);
                    mx = xb[j];
                }
            int8_t q[QK_K];
            int16_t bs[16];
            float d = 0.0f;
            if (amax == 0.0f) {
                memset(q, 0, sizeof q);
            } else {
                /* that value maps to -127; the far side may reach +128,
                 * which is clipped to 127 */
                const float iscale = -127.0f / mx;
                for (int j = 0; j < QK_K; ++j) {
                    const int v = (int)nearbyintf(iscale * xb[j]);
                    q[j] = (int8_t)(v < 127 ? v : 127);
                }
                d = 1.0f / iscale;
            }
            for (int g = 0; g < 16; ++g) {
                int s = 0;
                for (int l = 0; l < 16; ++l) s += q[16 * g + l];
                bs[g] = (int16_t)s;
            }
            memcpy(out, &d, 4);
            memcpy(out + 4, q, QK_K);
            memcpy(out + 4 + QK_K, bs, sizeof bs);
        }
}

/* y[c][r] = sum over superblocks of d_x d_y sum_s sc_s P_s
 *                                 - dmin_x d_y sum_s m_s (bsums_2s + bsums_2s+1),
 * with P_s the exact int32 dot of sub-block s (ggml's vec_dot_q4_K_q8_K). */
void orc_q4k_q8k_gemv(const uint8_t *w, const uint8_t *yq, float *y, int64_t N, int64_t K,
                      int32_t ncols, int32_t nthreads) {
    const int64_t nsb = K / QK_K;
    if (nthreads < 1) nthreads = 1;
    const sb_dots_fn dots = sb_dots();
#pragma omp parallel for num_threads(nthreads) schedule(static)
    for (int64_t r = 0; r < N; ++r) {
        for (int32_t c = 0; c < ncols; ++c) {
            const uint8_t *ycol = yq + (int64_t)c * nsb * Q8K_BYTES;
            float sumf = 0.0f;
            for (int64_t b = 0; b < nsb; ++b) {
                const uint8_t *blk = w + (r * nsb + b) * Q4K_BYTES;
                const uint8_t *yb = ycol + b * Q8K_BYTES;
                float yd;
                int16_t bs[16];
                memcpy(&yd, yb, 4);
                memcpy(bs, yb + 4 + QK_K, sizeof bs);
                int32_t P[8];
                dots(blk + 16, (const int8_t *)(yb + 4), P);
                int32_t sumi = 0, summ = 0;
                for (int s = 0; s < 8; ++s) {
                    int sc, m;
                    scale_min(blk + 4, s, &sc, &m);
                    sumi += P[s] * sc;
                    summ += (bs[2 * s] + bs[2 * s + 1]) * m;
                }
                sumf += (half_at(blk) * yd) * (float)sumi - (half_at(blk + 2) * yd) * (float)summ;
            }
            y[(int64_t)c * N + r] = sumf;
        }
    }
}

void orc_q4k_gemv_slices(const uint8_t *w, const uint8_t *xq, float *v, int64_t N,
                         int64_t K, int32_t ncols) {
    const int32_t nsb = (int32_t)(K / QK_K);
    int32_t start9[9];
    orc_slice_starts(nsb, start9);
    const sb_dots_fn dots = sb_dots();
    for (int32_t c = 0; c < ncols; ++c) {
        xstage st = stage_column(xq + (int64_t)c * (K / QK8_1) * Q81_BYTES, K);
        for (int64_t r = 0; r < N; ++r)
            row_slices(w + r * nsb * Q4K_BYTES, &st, dots, start9, v + ((int64_t)c * N + r) * 8);
        free_stage(&st);
    }
}

/* Independent f64 oracle, restating tests/q4k_q8_test.cu:54-107. */
void orc_q4k_gemv_f64(const uint8_t *w, const uint8_t *xq, double *y, int64_t N,
                      int64_t K, int32_t ncols) {
    const int64_t nsb = K / QK_K;
    for (int32_t c = 0; c < ncols; ++c) {
        const uint8_t *xcol = xq + (int64_t)c * (K / QK8_1) * Q81_BYTES;
        for (int64_t r = 0; r < N; ++r) {
            double acc = 0.0;
            for (int64_t b = 0; b < nsb; ++b) {
                const uint8_t *blk = w + (r * nsb + b) * Q4K_BYTES;
                const double d = half_at(blk), dmin = half_at(blk + 2);
                for (int p = 0; p < 4; ++p) {
                    int sc0, m0, sc1, m1;
                    scale_min(blk + 4, 2 * p, &sc0, &m0);
                    scale_min(blk + 4, 2 * p + 1, &sc1, &m1);
                    const uint8_t *x0 = xcol + (b * 8 + 2 * p) * Q81_BYTES;
                    const uint8_t *x1 = xcol + (b * 8 + 2 * p + 1) * Q81_BYTES;
                    const double d80 = half_at(x0), d81 = half_at(x1);
                    for (int l = 0; l < 32; ++l) {
                        const int byte = blk[16 + 32 * p + l];
                        const double w0 = d * sc0 * (byte & 0xF) - dmin * m0;
                        const double w1 = d * sc1 * (byte >> 4) - dmin * m1;
                        acc += w0 * (d80 * ((const int8_t *)(x0 + 4))[l]) +
                               w1 * (d81 * ((const int8_t *)(x1 + 4))[l]);
                    }
                }
            }
            y[(int64_t)c * N + r] = acc;
        }
    }
}

void orc_q4k_absdot_f64(const uint8_t *w, const uint8_t *xq, double *s, int64_t N,
                        int64_t K, int32_t ncols) {
    const int64_t nsb = K / QK_K;
    for (int32_t c = 0; c < ncols; ++c) {
        const uint8_t *xcol = xq + (int64_t)c * (K / QK8_1) * Q81_BYTES;
        for (int64_t r = 0; r < N; ++r) {
            double acc = 0.0;
            for (int64_t b = 0; b < nsb; ++b) {
                const uint8_t *blk = w + (r * nsb + b) * Q4K_BYTES;
                const double d = half_at(blk), dmin = half_at(blk + 2);
                for (int p = 0; p < 4; ++p)
                    for (int i = 0; i < 2; ++i) {
                        int sc, m;
                        scale_min(blk + 4, 2 * p + i, &sc, &m);
                        const uint8_t *xb = xcol + (b * 8 + 2 * p + i) * Q81_BYTES;
                        const double d8 = half_at(xb);
                        for (int l = 0; l < 32; ++l) {
                            const int byte = blk[16 + 32 * p + l];
                            const int q = i ? (byte >> 4) : (byte & 0xF);
                            acc += fabs(d * sc * q - dmin * m) *
                                   fabs(d8 * ((const int8_t *)(xb + 4))[l]);
                        }
                    }
            }
            s[(int64_t)c * N + r] = acc;
        }
    }
}

void orc_dequant_q4k(const uint8_t *w, float *out, int64_t nblocks) {
    for (int64_t i = 0; i < nblocks; ++i) {
        const uint8_t *blk = w + i * Q4K_BYTES;
        const float d = half_at(blk), dmin = half_at(blk + 2);
        for (int p = 0; p < 4; ++p)
            for (int h = 0; h < 2; ++h) {
                int sc, m;
                scale_min(blk + 4, 2 * p + h, &sc, &m);
                const float a = d * (float)sc;
                const float bm = dmin * (float)m;
                for (int l = 0; l < 32; ++l) {
                    const int byte = blk[16 + 32 * p + l];
                    const int q = h ? (byte >> 4) : (byte & 0xF);
                    out[i * QK_K + 64 * p + 32 * h + l] = fmaf(a, (float)q, -bm);
                }
            }
    }
}

int32_t orc_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
