// gen_quant.cu -- seeded weight generator, F32 -> Q8_1 quantizer and the
// fused RMSNorm -> Q8_1 kernel.
//
// Quantizer semantics follow the reference's in-tree quantizer
// (kernels/q4k/q4k_q8_mmvq.cu:223-255): amax over 32, d = amax/127,
// id = d > 0 ? 1/d : 0, q = (int8)roundf(x*id), s = d * sum(q).  Every fp32
// operation is written with an explicit-rounding intrinsic so that nvcc does
// not contract it; the CPU oracle performs the same operations in the same
// order, so the Q8_1 bytes agree bit for bit.
#include "common.cuh"
#include "kernels.cuh"

namespace abra {

// ------------------------------------------------------------ generator ---
// One thread per 8-byte word of the superblock array.  Word 0 of each block
// carries d and dmin ~ U(0.001, 0.02) in its low four bytes.
__global__ void gen_q4k_kernel(uint64_t *__restrict__ dst, int64_t nblocks, uint64_t key,
                               int64_t block_offset) {
    const int64_t nwords = nblocks * 18;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nwords;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t blk = i / 18;
        const int w = static_cast<int>(i - blk * 18);
        const uint64_t gword = static_cast<uint64_t>(block_offset + blk) * 18u + w;
        uint64_t h = stream_word(key, gword);
        if (w == 0) {
            const float d = __fmaf_rn(unit24(h >> 40), 0.019f, 0.001f);
            const float dmin = __fmaf_rn(unit24((h >> 16) & 0xffffffu), 0.019f, 0.001f);
            const uint64_t hd = __half_as_ushort(__float2half_rn(d));
            const uint64_t hm = __half_as_ushort(__float2half_rn(dmin));
            h = (h & 0xffffffff00000000ull) | hd | (hm << 16);
        }
        dst[i] = h;
    }
}

__global__ void gen_uniform_f32_kernel(float *__restrict__ dst, int64_t n, uint64_t key,
                                       int64_t offset_index, float scale, float offset) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const uint64_t h = stream_word(key, static_cast<uint64_t>(offset_index + i));
        dst[i] = __fmaf_rn(unit24(h >> 40), scale, offset);
    }
}

cudaError_t launch_gen_q4k(void *dst, int64_t nblocks, uint64_t seed, uint64_t tensor_id,
                           int64_t block_offset, cudaStream_t stream) {
    if (nblocks <= 0) return cudaSuccess;
    const int64_t nwords = nblocks * 18;
    const int threads = 256;
    const int64_t want = (nwords + threads - 1) / threads;
    const int grid = static_cast<int>(want < 148 * 32 ? want : 148 * 32);
    gen_q4k_kernel<<<grid, threads, 0, stream>>>(static_cast<uint64_t *>(dst), nblocks,
                                                 stream_key(seed, tensor_id), block_offset);
    return cudaGetLastError();
}

cudaError_t launch_gen_uniform_f32(float *dst, int64_t n, uint64_t seed, uint64_t tensor_id,
                                   int64_t offset_index, float scale, float offset,
                                   cudaStream_t stream) {
    if (n <= 0) return cudaSuccess;
    const int threads = 256;
    const int64_t want = (n + threads - 1) / threads;
    const int grid = static_cast<int>(want < 148 * 32 ? want : 148 * 32);
    gen_uniform_f32_kernel<<<grid, threads, 0, stream>>>(dst, n, stream_key(seed, tensor_id),
                                                         offset_index, scale, offset);
    return cudaGetLastError();
}

// ------------------------------------------------------------ quantizer ---
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

__global__ void quantize_q8_1_kernel(const float *__restrict__ x, block_q8_1 *__restrict__ y,
                                     int64_t nblocks_total) {
    const int lane = threadIdx.x & 31;
    const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    pdl_wait();
    pdl_launch_dependents();
    if (warp >= nblocks_total) return;
    quantize_block_warp(x[warp * QK8_1 + lane], y + warp, lane);
}

cudaError_t launch_quantize_q8_1(const float *x, void *y, int64_t K, int ncols,
                                 cudaStream_t stream) {
    const int64_t nb = (K / QK8_1) * ncols;
    if (nb <= 0) return cudaSuccess;
    const int threads = 256;
    const int64_t grid = (nb * 32 + threads - 1) / threads;
    quantize_q8_1_kernel<<<static_cast<unsigned>(grid), threads, 0, stream>>>(
        x, static_cast<block_q8_1 *>(y), nb);
    return cudaGetLastError();
}

// ------------------------------------------------ fused RMSNorm -> Q8_1 ---
// One 256-thread CTA per column.  Sum of squares in the canonical order:
// thread t accumulates x[t + 256 i] with fmaf, each warp reduces with an xor
// butterfly (masks 16..1), the eight warp sums are added in warp order.
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

__global__ void __launch_bounds__(RMS_THREADS)
    rmsnorm_quantize_q8_1_kernel(const float *__restrict__ x, const float *__restrict__ w,
                                 float eps, block_q8_1 *__restrict__ y, float *__restrict__ xn_out,
                                 int K) {
    extern __shared__ float s_xn[];  // K floats
    __shared__ float red[RMS_THREADS / 32];
    const int c = blockIdx.x;
    const float *xc = x + static_cast<int64_t>(c) * K;
    pdl_wait();
    pdl_launch_dependents();
    const float total = block_sumsq_canonical(xc, K, red);
    const float r =
        __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(total, static_cast<float>(K)), eps)));
    for (int i = threadIdx.x; i < K; i += RMS_THREADS) {
        const float v = __fmul_rn(__fmul_rn(xc[i], r), w[i]);
        s_xn[i] = v;
        if (xn_out) xn_out[static_cast<int64_t>(c) * K + i] = v;
    }
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nb = K / QK8_1;
    block_q8_1 *yc = y + static_cast<int64_t>(c) * nb;
    for (int b = warp; b < nb; b += RMS_THREADS / 32) quantize_block_warp(s_xn[b * QK8_1 + lane], yc + b, lane);
}

cudaError_t launch_rmsnorm_quantize_q8_1(const float *x, const float *w, float eps, void *y,
                                         float *xn_out, int64_t K, int ncols,
                                         cudaStream_t stream) {
    if (ncols <= 0) return cudaSuccess;
    const size_t smem = static_cast<size_t>(K) * sizeof(float);
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(rmsnorm_quantize_q8_1_kernel,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem));
        if (e != cudaSuccess) return e;
    }
    rmsnorm_quantize_q8_1_kernel<<<ncols, RMS_THREADS, smem, stream>>>(
        x, w, eps, static_cast<block_q8_1 *>(y), xn_out, static_cast<int>(K));
    return cudaGetLastError();
}

}  // namespace abra

ABRA_ERROR_WORD_ACCESSOR(error_word_gen_quant)
