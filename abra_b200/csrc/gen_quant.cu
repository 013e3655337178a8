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
#include "quant_common.cuh"

namespace abra {

// ------------------------------------------------------------ generator ---
// One thread per 8-byte word of the superblock array.  Word 0 of each block
// carries d and dmin ~ U(0.001, 0.02) in its low four bytes.
// Centred variant (flags bit 0): keep d, the scales and the nibbles, set
// dmin = 7.5 d max(sc) / 63 and m_s = round(63 sc_s / max(sc)) so each
// sub-block's weights have mean ~0.  Words 0 and 1 (bytes 0..15: d, dmin,
// the 12 scale bytes) are then written together by the word-0 thread.
__device__ void centre_header(uint64_t &w0, uint64_t &w1) {
    uint8_t b[16];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        b[i] = static_cast<uint8_t>(w0 >> (8 * i));
        b[8 + i] = static_cast<uint8_t>(w1 >> (8 * i));
    }
    const uint8_t *q = b + 4;
    int sc[8], m[8], mx = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        sc[j] = q[j] & 63;
        sc[j + 4] = (q[j + 8] & 0xF) | ((q[j] >> 6) << 4);
    }
#pragma unroll
    for (int s = 0; s < 8; ++s) mx = sc[s] > mx ? sc[s] : mx;
    uint16_t hm = 0;
    if (mx == 0) {
#pragma unroll
        for (int s = 0; s < 8; ++s) m[s] = 0;
    } else {
        const float df = __half2float(__ushort_as_half(static_cast<unsigned short>(b[0] | (b[1] << 8))));
        hm = __half_as_ushort(__float2half_rn(
            __fdiv_rn(__fmul_rn(__fmul_rn(7.5f, df), static_cast<float>(mx)), 63.0f)));
#pragma unroll
        for (int s = 0; s < 8; ++s) m[s] = (63 * sc[s] + mx / 2) / mx;
    }
    uint8_t o[16];
    o[0] = b[0];
    o[1] = b[1];
    o[2] = static_cast<uint8_t>(hm & 0xff);
    o[3] = static_cast<uint8_t>(hm >> 8);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        o[4 + j] = static_cast<uint8_t>((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
        o[8 + j] = static_cast<uint8_t>((m[j] & 63) | ((m[j + 4] >> 4) << 6));
        o[12 + j] = static_cast<uint8_t>((sc[j + 4] & 15) | ((m[j + 4] & 15) << 4));
    }
    w0 = 0;
    w1 = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        w0 |= static_cast<uint64_t>(o[i]) << (8 * i);
        w1 |= static_cast<uint64_t>(o[8 + i]) << (8 * i);
    }
}

// Local block blk is global block block_offset + (blk / width) * gstride +
// blk % width: a contiguous run when width >= nblocks, or a column range of
// width superblocks out of rows of gstride (a K-shard).
__global__ void gen_q4k_kernel(uint64_t *__restrict__ dst, int64_t nblocks, uint64_t key,
                               int64_t block_offset, int64_t width, int64_t gstride, int flags) {
    const int64_t nwords = nblocks * 18;
    const bool centred = (flags & 1) != 0;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nwords;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t blk = i / 18;
        const int w = static_cast<int>(i - blk * 18);
        if (centred && w == 1) continue;  // written by the word-0 thread
        const int64_t gblk = block_offset + (blk / width) * gstride + blk % width;
        const uint64_t gword = static_cast<uint64_t>(gblk) * 18u + w;
        uint64_t h = stream_word(key, gword);
        if (w == 0) {
            const float d = __fmaf_rn(unit24(h >> 40), 0.019f, 0.001f);
            const float dmin = __fmaf_rn(unit24((h >> 16) & 0xffffffu), 0.019f, 0.001f);
            const uint64_t hd = __half_as_ushort(__float2half_rn(d));
            const uint64_t hm = __half_as_ushort(__float2half_rn(dmin));
            h = (h & 0xffffffff00000000ull) | hd | (hm << 16);
            if (centred) {
                uint64_t h1 = stream_word(key, gword + 1);
                centre_header(h, h1);
                dst[i + 1] = h1;
            }
        }
        dst[i] = h;
    }
}

// Norm weights of the synthetic model: +-U(0.8, 1.2), sign from bit 0.
__global__ void gen_norm_f32_kernel(float *__restrict__ dst, int64_t n, uint64_t key) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const uint64_t h = stream_word(key, static_cast<uint64_t>(i));
        const float v = __fmaf_rn(unit24(h >> 40), 0.4f, 0.8f);
        dst[i] = (h & 1u) ? -v : v;
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

cudaError_t launch_gen_q4k_ex(void *dst, int64_t nblocks, uint64_t seed, uint64_t tensor_id,
                              int64_t block_offset, int flags, cudaStream_t stream) {
    if (nblocks <= 0) return cudaSuccess;
    const int64_t nwords = nblocks * 18;
    const int threads = 256;
    const int64_t want = (nwords + threads - 1) / threads;
    const int grid = static_cast<int>(want < 148 * 32 ? want : 148 * 32);
    gen_q4k_kernel<<<grid, threads, 0, stream>>>(static_cast<uint64_t *>(dst), nblocks,
                                                 stream_key(seed, tensor_id), block_offset,
                                                 nblocks, 0, flags);
    return cudaGetLastError();
}

cudaError_t launch_gen_q4k_cols(void *dst, int64_t rows, int64_t nsb_g, int64_t sb_lo,
                                int64_t sb_hi, uint64_t seed, uint64_t tensor_id, int64_t row0,
                                int flags, cudaStream_t stream) {
    const int64_t width = sb_hi - sb_lo, nblocks = rows * width;
    if (nblocks <= 0) return cudaSuccess;
    const int64_t nwords = nblocks * 18;
    const int threads = 256;
    const int64_t want = (nwords + threads - 1) / threads;
    const int grid = static_cast<int>(want < 148 * 32 ? want : 148 * 32);
    gen_q4k_kernel<<<grid, threads, 0, stream>>>(static_cast<uint64_t *>(dst), nblocks,
                                                 stream_key(seed, tensor_id), row0 * nsb_g + sb_lo,
                                                 width, nsb_g, flags);
    return cudaGetLastError();
}

cudaError_t launch_gen_q4k(void *dst, int64_t nblocks, uint64_t seed, uint64_t tensor_id,
                           int64_t block_offset, cudaStream_t stream) {
    return launch_gen_q4k_ex(dst, nblocks, seed, tensor_id, block_offset, 0, stream);
}

// Q6_K blocks (210 bytes): thread i writes word w = i % 27 of local block
// i / 27 -- words 0..25 are bytes 8w..8w+7 (ql, qh, scales), word 26 gives
// d ~ U(0.0001, 0.002) as fp16 at byte 208.  Stores are 16-bit: a block is
// only 2-byte aligned.  Local block blk is global block block_offset +
// (blk / width) * gstride + blk % width, as for Q4_K.
__global__ void gen_q6k_kernel(uint16_t *__restrict__ dst, int64_t nblocks, uint64_t key,
                               int64_t block_offset, int64_t width, int64_t gstride) {
    const int64_t nwords = nblocks * 27;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nwords;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t blk = i / 27;
        const int w = static_cast<int>(i - blk * 27);
        const int64_t row = blk / width;
        const int64_t gb = block_offset + row * gstride + (blk - row * width);
        const uint64_t h = stream_word(key, static_cast<uint64_t>(gb) * 27u + static_cast<uint64_t>(w));
        uint16_t *b = dst + blk * 105;  // 210 bytes = 105 halfwords
        if (w < 26) {
#pragma unroll
            for (int k = 0; k < 4; ++k) b[4 * w + k] = static_cast<uint16_t>(h >> (16 * k));
        } else {
            const float d = __fmaf_rn(unit24(h >> 40), 0.0019f, 0.0001f);
            b[104] = __half_as_ushort(__float2half_rn(d));
        }
    }
}

cudaError_t launch_gen_q6k_cols(void *dst, int64_t nblocks, int64_t width, int64_t gstride,
                                uint64_t seed, uint64_t tensor_id, int64_t block_offset,
                                cudaStream_t stream) {
    if (nblocks <= 0) return cudaSuccess;
    if (reinterpret_cast<uintptr_t>(dst) & 1) return cudaErrorInvalidValue;
    const int64_t nwords = nblocks * 27;
    const int threads = 256;
    const int64_t want = (nwords + threads - 1) / threads;
    const int grid = static_cast<int>(want < 148 * 32 ? want : 148 * 32);
    gen_q6k_kernel<<<grid, threads, 0, stream>>>(static_cast<uint16_t *>(dst), nblocks,
                                                 stream_key(seed, tensor_id), block_offset, width,
                                                 gstride);
    return cudaGetLastError();
}

cudaError_t launch_gen_q6k(void *dst, int64_t nblocks, uint64_t seed, uint64_t tensor_id,
                           int64_t block_offset, cudaStream_t stream) {
    return launch_gen_q6k_cols(dst, nblocks, nblocks, 0, seed, tensor_id, block_offset, stream);
}

cudaError_t launch_gen_norm_f32(float *dst, int64_t n, uint64_t seed, uint64_t tensor_id,
                                cudaStream_t stream) {
    if (n <= 0) return cudaSuccess;
    const int threads = 256;
    const int64_t want = (n + threads - 1) / threads;
    const int grid = static_cast<int>(want < 148 * 32 ? want : 148 * 32);
    gen_norm_f32_kernel<<<grid, threads, 0, stream>>>(dst, n, stream_key(seed, tensor_id));
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
