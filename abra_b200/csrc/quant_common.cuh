// quant_common.cuh -- device helpers shared by the quantizer, the fused
// RMSNorm kernels and the decode kernels: the warp-level Q8_1 block quantizer
// and the canonical 256-thread sum of squares.  Both follow the operation
// order of the CPU oracle (orc_quantize_q8_1, canonical_sumsq).
#pragma once

#include "common.cuh"

namespace abra {

// One warp quantizes one 32-element block; lane j owns element j.
__device__ __forceinline__ void quantize_block_warp(float x, block_q8_1 *out, int lane) {
    float amax = fmaxf(0.0f, fabsf(x));
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, m));
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d > 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    const int q = static_cast<int>(static_cast<int8_t>(static_cast<int>(roundf(__fmul_rn(x, id)))));
    int sum = q;
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, m);
    // gather four bytes per word: lane k (k < 8) assembles qs[4k .. 4k+3]
    const uint32_t qb = static_cast<uint32_t>(q) & 0xffu;
    const int src = (lane & 7) * 4;
    const uint32_t b0 = __shfl_sync(0xffffffffu, qb, src + 0);
    const uint32_t b1 = __shfl_sync(0xffffffffu, qb, src + 1);
    const uint32_t b2 = __shfl_sync(0xffffffffu, qb, src + 2);
    const uint32_t b3 = __shfl_sync(0xffffffffu, qb, src + 3);
    uint32_t *o = reinterpret_cast<uint32_t *>(out);
    if (lane < 8) o[1 + lane] = b0 | (b1 << 8) | (b2 << 16) | (b3 << 24);
    if (lane == 8) {
        const uint32_t hd = __half_as_ushort(__float2half_rn(d));
        const uint32_t hs = __half_as_ushort(__float2half_rn(__fmul_rn(d, static_cast<float>(sum))));
        o[0] = hd | (hs << 16);
    }
}

// Canonical sum of squares over K values with a 256-thread CTA: thread t
// accumulates x[t + 256 i] with fmaf, each warp reduces with an xor butterfly
// (masks 16..1), the eight warp sums are added in warp order.
constexpr int RMS_THREADS = 256;

__device__ __forceinline__ float block_sumsq_canonical(const float *x, int K, float *red) {
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    float acc = 0.0f;
    for (int i = t; i < K; i += RMS_THREADS) acc = __fmaf_rn(x[i], x[i], acc);
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, m));
    if (lane == 0) red[warp] = acc;
    __syncthreads();
    float total = red[0];
#pragma unroll
    for (int w = 1; w < RMS_THREADS / 32; ++w) total = __fadd_rn(total, red[w]);
    __syncthreads();
    return total;
}


}  // namespace abra
