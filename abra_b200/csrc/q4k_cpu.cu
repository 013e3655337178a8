// q4k_cpu.cu -- host-side Q4_K row quantization and dequantization, the two
// CPU functions of the reference's adapter ABI
// (kernels/q4k/upstream_adapter.cuh:28-38).  The reference forwards them to
// llama.cpp's quantize_row_q4_K_ref / dequantize_row_q4_K (pinned commit
// 169e4a7ff201e666c2325bcd35afb64573e39d09, upstream_adapter.cu:106-120); its
// test and benchmark harnesses make their Q4_K weights with the first
// (tests/q4k_q8_test.cu:357,430,506,589, bench/micro/q4k_q8_bench.cu:287).
//
// The quantizer restates the published Q4_K algorithm of llama.cpp's
// k-quants (ggml-quants.c, the "make_qkx2_quants" search; the format is the
// one in kernels/q4k/q4k_q8_mmvq.cuh:42-47):
//   1. each 32-value sub-block j gets importance weights w_l = rms(x_j) + |x_l|
//      and a weighted least-squares affine fit x ~ s_j * q + m_j (m_j <= 0,
//      codes q in 0..15): start from the min/max fit, then try 21 inverse
//      scales (15 + (-1 + 0.1 i)) / (max - min), refit scale and offset in
//      closed form on each candidate's codes, keep the lowest weighted
//      squared error;
//   2. the superblock scale d = max_j s_j / 63 and dmin = max_j (-m_j) / 63
//      (fp16), the 6-bit per-sub-block multipliers round(63 s_j / max s) and
//      round(63 (-m_j) / max(-m)), packed in the 12-byte layout;
//   3. final codes q = clamp(round((x + dmin * m6) / (d * sc6)), 0, 15) with
//      the decoded fp16 scales, packed low nibble / high nibble per 64 values.
// Every rounding to an integer is to nearest, ties to even.  Operations are
// kept in the order of that algorithm so that the same inputs give the same
// codes; bit-equality with llama.cpp itself cannot be checked without it.
//
// Dequantization is the format's definition: y = (d * sc) * q - (dmin * m),
// two separately rounded fp32 products and one subtraction.
#include <cuda_fp16.h>

#include <cmath>
#include <cstdint>
#include <cstring>

#include "abra_b200.h"
#include "common.cuh"
#include "kernels.cuh"

namespace abra {
namespace {

constexpr int kSub = 32;        // values per sub-block
constexpr int kCodeMax = 15;    // 4-bit codes
constexpr int kSixBitMax = 63;  // 6-bit scale multipliers

inline int round_even(float v) { return static_cast<int>(std::nearbyint(v)); }
inline int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

// Weighted squared error of the affine reconstruction s * q + m.
float affine_error(const float *x, const float *w, const uint8_t *q, float s, float m) {
    float err = 0.0f;
    for (int i = 0; i < kSub; ++i) {
        const float diff = s * q[i] + m - x[i];
        err += w[i] * (diff * diff);
    }
    return err;
}

// Step 1 for one sub-block: codes into q, returns the scale s (>= 0) and
// stores the offset magnitude -m (>= 0) into *neg_offset.
float fit_sub_block(const float *x, const float *w, uint8_t *q, float *neg_offset) {
    float lo = x[0], hi = x[0];
    float wsum = w[0];
    float wx = wsum * x[0];
    for (int i = 1; i < kSub; ++i) {
        lo = x[i] < lo ? x[i] : lo;
        hi = x[i] > hi ? x[i] : hi;
        wsum += w[i];
        wx += w[i] * x[i];
    }
    if (lo > 0.0f) lo = 0.0f;
    if (hi == lo) {  // constant non-positive sub-block
        std::memset(q, 0, kSub);
        *neg_offset = -lo;
        return 0.0f;
    }
    // the plain min/max fit
    float inv = kCodeMax / (hi - lo);
    float scale = 1.0f / inv;
    float offset = lo;
    for (int i = 0; i < kSub; ++i) q[i] = static_cast<uint8_t>(clampi(round_even(inv * (x[i] - lo)), 0, kCodeMax));
    float best = affine_error(x, w, q, scale, offset);
    // candidates around it, refit in closed form on their codes
    uint8_t cand[kSub];
    for (int step = 0; step <= 20; ++step) {
        inv = (-1.0f + 0.1f * step + kCodeMax) / (hi - lo);
        float sl = 0.0f, sl2 = 0.0f, sxl = 0.0f;
        for (int i = 0; i < kSub; ++i) {
            const int c = clampi(round_even(inv * (x[i] - lo)), 0, kCodeMax);
            cand[i] = static_cast<uint8_t>(c);
            sl += w[i] * c;
            sl2 += w[i] * c * c;
            sxl += w[i] * c * x[i];
        }
        const float det = wsum * sl2 - sl * sl;
        if (!(det > 0.0f)) continue;
        float s = (wsum * sxl - wx * sl) / det;
        float m = (sl2 * wx - sl * sxl) / det;
        if (m > 0.0f) {  // the offset must not be positive: refit the scale alone
            m = 0.0f;
            s = sxl / sl2;
        }
        const float err = affine_error(x, w, cand, s, m);
        if (err < best) {
            std::memcpy(q, cand, kSub);
            best = err;
            scale = s;
            offset = m;
        }
    }
    *neg_offset = -offset;
    return scale;
}

void quantize_superblock(const float *x, uint8_t *blk) {
    uint8_t codes[QK_K];
    float scale[8], neg_off[8];
    float wts[kSub];
    float max_scale = 0.0f, max_off = 0.0f;
    for (int j = 0; j < 8; ++j) {
        const float *xj = x + kSub * j;
        float ss = 0.0f;
        for (int l = 0; l < kSub; ++l) ss += xj[l] * xj[l];
        const float rms = std::sqrt(ss / kSub);
        for (int l = 0; l < kSub; ++l) wts[l] = rms + std::fabs(xj[l]);
        scale[j] = fit_sub_block(xj, wts, codes + kSub * j, &neg_off[j]);
        if (scale[j] > max_scale) max_scale = scale[j];
        if (neg_off[j] > max_off) max_off = neg_off[j];
    }
    const float inv_scale = max_scale > 0.0f ? kSixBitMax / max_scale : 0.0f;
    const float inv_off = max_off > 0.0f ? kSixBitMax / max_off : 0.0f;
    uint8_t *sc12 = blk + 4;
    std::memset(sc12, 0, 12);
    for (int j = 0; j < 8; ++j) {
        uint8_t ls = static_cast<uint8_t>(round_even(inv_scale * scale[j]));
        uint8_t lm = static_cast<uint8_t>(round_even(inv_off * neg_off[j]));
        if (ls > kSixBitMax) ls = kSixBitMax;
        if (lm > kSixBitMax) lm = kSixBitMax;
        if (j < 4) {
            sc12[j] = ls;
            sc12[j + 4] = lm;
        } else {
            sc12[j + 4] = static_cast<uint8_t>((ls & 0xF) | ((lm & 0xF) << 4));
            sc12[j - 4] |= static_cast<uint8_t>((ls >> 4) << 6);
            sc12[j] |= static_cast<uint8_t>((lm >> 4) << 6);
        }
    }
    const __half hd = __float2half_rn(max_scale / kSixBitMax);
    const __half hm = __float2half_rn(max_off / kSixBitMax);
    std::memcpy(blk, &hd, 2);
    std::memcpy(blk + 2, &hm, 2);
    const float d = __half2float(hd), dmin = __half2float(hm);
    for (int j = 0; j < 8; ++j) {
        int sc, m;
        scale_min_one(sc12, j, sc, m);
        const float dj = d * sc;
        if (dj == 0.0f) continue;  // keep the fit's codes
        const float mj = dmin * m;
        for (int l = 0; l < kSub; ++l)
            codes[kSub * j + l] = static_cast<uint8_t>(clampi(round_even((x[kSub * j + l] + mj) / dj), 0, kCodeMax));
    }
    uint8_t *qs = blk + 16;
    for (int p = 0; p < 4; ++p)
        for (int l = 0; l < kSub; ++l)
            qs[32 * p + l] = static_cast<uint8_t>(codes[64 * p + l] | (codes[64 * p + 32 + l] << 4));
}

void dequantize_superblock(const uint8_t *blk, float *y) {
    __half hd, hm;
    std::memcpy(&hd, blk, 2);
    std::memcpy(&hm, blk + 2, 2);
    const float d = __half2float(hd), dmin = __half2float(hm);
    const uint8_t *qs = blk + 16;
    for (int j = 0; j < 8; ++j) {
        int sc, m;
        scale_min_one(blk + 4, j, sc, m);
        const float a = d * static_cast<float>(sc);
        const float b = dmin * static_cast<float>(m);
        const int p = j >> 1, shift = 4 * (j & 1);
        for (int l = 0; l < kSub; ++l) {
            const float q = static_cast<float>((qs[32 * p + l] >> shift) & 0xF);
            const float prod = a * q;
            y[kSub * j + l] = prod - b;
        }
    }
}

}  // namespace
}  // namespace abra

extern "C" {

void quantize_row_q4_K_upstream_cpu(const float *x, void *y, int64_t k) {
    if (!x || !y || k < 0 || k % abra::QK_K) {
        abra::record_failure(ABRA_E_INVALID, "quantize_row_q4_K_upstream_cpu: k must be a multiple of 256");
        return;
    }
    uint8_t *out = static_cast<uint8_t *>(y);
    for (int64_t b = 0; b < k / abra::QK_K; ++b)
        abra::quantize_superblock(x + b * abra::QK_K, out + b * abra::Q4K_BYTES);
}

void dequantize_row_q4_K_upstream_cpu(const void *x, float *y, int64_t k) {
    if (!x || !y || k < 0 || k % abra::QK_K) {
        abra::record_failure(ABRA_E_INVALID, "dequantize_row_q4_K_upstream_cpu: k must be a multiple of 256");
        return;
    }
    const uint8_t *in = static_cast<const uint8_t *>(x);
    for (int64_t b = 0; b < k / abra::QK_K; ++b)
        abra::dequantize_superblock(in + b * abra::Q4K_BYTES, y + b * abra::QK_K);
}

}  // extern "C"
