// decode_kernels.cu -- the non-GEMV kernels of the Qwen3-4B-shaped decode
// step: tied-embedding dequantization, residual add + RMSNorm + Q8_1,
// QK-RMSNorm + NEOX RoPE + fp16 KV append, chunked attention with a fixed
// log-sum-exp merge (+ Q8_1 of the result), and greedy argmax.
//
// Every fp32 operation uses an explicit-rounding intrinsic in the order the
// CPU oracle (oracle/model_oracle.c) performs it, so the decode step is
// bit-identical to the oracle.  Positions and tokens are read from device
// memory so one captured CUDA graph serves every step.
#include "common.cuh"
#include "decode.cuh"
#include "quant_common.cuh"

namespace abra {

// ---------------------------------------------------------------- embed ---
// h = dequant(E[tokens[*pos]]): w = fmaf(d * sc, q, -(dmin * m)).  Sequence
// blockIdx.y of a batch reads tokens + y * tok_stride and writes h + y * hidden.
__global__ void embed_kernel(const uint8_t *__restrict__ E, int hidden,
                             const int32_t *__restrict__ tokens, const int32_t *__restrict__ pos,
                             float *__restrict__ h, int64_t tok_stride) {
    pdl_wait();
    pdl_launch_dependents();
    tokens += blockIdx.y * tok_stride;
    h += static_cast<int64_t>(blockIdx.y) * hidden;
    const int tok = tokens[*pos];
    const uint8_t *row = E + static_cast<int64_t>(tok) * (hidden / QK_K) * Q4K_BYTES;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < hidden; i += blockDim.x * gridDim.x) {
        const int b = i >> 8, r = i & 255, p = r >> 6, hh = (r >> 5) & 1, l = r & 31;
        const uint8_t *blk = row + b * Q4K_BYTES;
        const float d = __half2float(*reinterpret_cast<const __half *>(blk));
        const float dmin = __half2float(*reinterpret_cast<const __half *>(blk + 2));
        int sc, m;
        scale_min_one(blk + 4, 2 * p + hh, sc, m);
        const int byte = blk[16 + 32 * p + l];
        const int q = hh ? (byte >> 4) : (byte & 15);
        const float a = __fmul_rn(d, static_cast<float>(sc));
        const float bm = __fmul_rn(dmin, static_cast<float>(m));
        h[i] = __fmaf_rn(a, static_cast<float>(q), -bm);
    }
}

// Q6_K rows of the tied table (the Q4_K_M type map): element e of a 256-block
// is (d * scales[e / 16]) * (q - 32), q the 6-bit code in ggml's block_q6_K
// order (low nibble of ql[64 half + lane + 32 (group % 2)] for groups 0, 1,
// high nibble for 2, 3; bits 2 group of qh[32 half + lane]).
__global__ void embed_q6k_kernel(const uint8_t *__restrict__ E, int hidden,
                                 const int32_t *__restrict__ tokens, const int32_t *__restrict__ pos,
                                 float *__restrict__ h, int64_t tok_stride) {
    pdl_wait();
    pdl_launch_dependents();
    tokens += blockIdx.y * tok_stride;
    h += static_cast<int64_t>(blockIdx.y) * hidden;
    const int tok = tokens[*pos];
    const uint8_t *row = E + static_cast<int64_t>(tok) * (hidden / QK_K) * 210;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < hidden; i += blockDim.x * gridDim.x) {
        const int e = i & 255, half = e >> 7, group = (e >> 5) & 3, lane = e & 31;
        const uint8_t *blk = row + static_cast<int64_t>(i >> 8) * 210;
        const int qlb = blk[half * 64 + lane + (group & 1) * 32];
        const int low = group < 2 ? (qlb & 15) : (qlb >> 4);
        const int q = low | (((blk[128 + half * 32 + lane] >> (2 * group)) & 3) << 4);
        const int sc = static_cast<int8_t>(blk[192 + (e >> 4)]);
        const float d = __half2float(*reinterpret_cast<const __half *>(blk + 208));
        h[i] = __fmul_rn(__fmul_rn(d, static_cast<float>(sc)), static_cast<float>(q - 32));
    }
}

// ------------------------------------------ residual + RMSNorm + Q8_1 ---
// h = h + D (D = fixed-order tree of G partial deltas, G in {0,1,2,4,8}),
// then Q8_1 of (h * r) * w, r = 1/sqrt(mean(h^2) + eps).  One CTA per column.
// 1024 threads: the canonical 256-lane sum of squares runs on threads
// 0..255 (same order as block_sumsq_canonical), every thread takes part in
// the residual add, the scaling and (as 32 warps) the Q8_1 blocks.
constexpr int RES_THREADS = 1024;

__global__ void __launch_bounds__(RES_THREADS)
    residual_rmsnorm_quant_kernel(float *__restrict__ h, const DeltaSet ds,
                                  const float *__restrict__ w, float eps,
                                  block_q8_1 *__restrict__ y, int K,
                                  const unsigned long long *wait_cnt, const unsigned long long *epoch,
                                  unsigned long long per_step) {
    extern __shared__ float s_x[];
    __shared__ float red[RMS_THREADS / 32];
    __shared__ float s_r;
    pdl_wait();
    pdl_launch_dependents();
    const int c = blockIdx.x, t = threadIdx.x;
    if (wait_cnt) {  // tensor parallel: every rank's partial sums have arrived (bounded)
        if (t == 0) wait_count(wait_cnt, (__ldcg(epoch) + 1ull) * per_step);
        __syncthreads();
    }
    float *hc = h + static_cast<int64_t>(c) * K;
    for (int i = t; i < K; i += RES_THREADS) {
        float v = hc[i];
        if (ds.G > 0) {
            v = __fadd_rn(v, delta_tree(ds, static_cast<int64_t>(c) * K + i));
            hc[i] = v;
        }
        s_x[i] = v;
    }
    __syncthreads();
    if (t < RMS_THREADS) {
        float acc = 0.0f;
        for (int i = t; i < K; i += RMS_THREADS) acc = __fmaf_rn(s_x[i], s_x[i], acc);
#pragma unroll
        for (int m = 16; m >= 1; m >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, m));
        if ((t & 31) == 0) red[t >> 5] = acc;
    }
    __syncthreads();
    if (t == 0) {
        float total = red[0];
#pragma unroll
        for (int k = 1; k < RMS_THREADS / 32; ++k) total = __fadd_rn(total, red[k]);
        s_r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(total, static_cast<float>(K)), eps)));
    }
    __syncthreads();
    const float r = s_r;
    for (int i = t; i < K; i += RES_THREADS) s_x[i] = __fmul_rn(__fmul_rn(s_x[i], r), w[i]);
    __syncthreads();
    const int lane = t & 31, warp = t >> 5;
    block_q8_1 *yc = y + static_cast<int64_t>(c) * (K / QK8_1);
    for (int b = warp; b < K / QK8_1; b += RES_THREADS / 32)
        quantize_block_warp(s_x[b * QK8_1 + lane], yc + b, lane);
}

// ------------------------------------------- QK-norm + RoPE + KV append ---
// One warp per head of qkv = [q heads | k heads | v heads] x 128.  Lane t
// holds elements 4t..4t+3.  q/k: RMSNorm over the head (fmaf over the lane's
// four, xor butterfly 16..1), times the norm weight, then NEOX RoPE pairs
// (i, i+64) with the host cos/sin table row of this position.  q stays fp32;
// k and v are stored fp16 at kv[head][pos][128].
// Sequence blockIdx.y of a batch: qkv, q_out and the KV cache advance by
// their per-sequence strides, the position by pos_stride (a prefill chunk:
// column b is position *pos + b of one cache).
__global__ void __launch_bounds__(256)
    qk_norm_rope_kv_kernel(const float *__restrict__ qkv, const float *__restrict__ q_norm,
                           const float *__restrict__ k_norm, float eps,
                           const float *__restrict__ rope, const int32_t *__restrict__ pos_p,
                           float *__restrict__ q_out, __half *__restrict__ kc,
                           __half *__restrict__ vc, int n_heads, int n_kv, int max_ctx,
                           int64_t qkv_stride, int64_t q_stride, int64_t kv_stride,
                           int pos_stride) {
    pdl_wait();
    pdl_launch_dependents();
    qkv += blockIdx.y * qkv_stride;
    q_out += blockIdx.y * q_stride;
    kc += blockIdx.y * kv_stride;
    vc += blockIdx.y * kv_stride;
    const int lane = threadIdx.x & 31;
    const int hw = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (hw >= n_heads + 2 * n_kv) return;
    const int pos = *pos_p + static_cast<int>(blockIdx.y) * pos_stride;
    if (pos >= max_ctx) return;  // the host never steps past max_ctx; no write out of range
    const float4 xv = *reinterpret_cast<const float4 *>(qkv + static_cast<int64_t>(hw) * 128 + 4 * lane);
    const float x[4] = {xv.x, xv.y, xv.z, xv.w};
    if (hw >= n_heads + n_kv) {  // v head: store fp16 as is
        const int g = hw - n_heads - n_kv;
        __half *dst = vc + (static_cast<int64_t>(g) * max_ctx + pos) * 128 + 4 * lane;
#pragma unroll
        for (int k = 0; k < 4; ++k) dst[k] = __float2half_rn(x[k]);
        return;
    }
    const float *nw = hw < n_heads ? q_norm : k_norm;
    float acc = 0.0f;
#pragma unroll
    for (int k = 0; k < 4; ++k) acc = __fmaf_rn(x[k], x[k], acc);
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, m));
    const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(acc, 128.0f), eps)));
    float y[4], o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) y[k] = __fmul_rn(__fmul_rn(x[k], r), nw[4 * lane + k]);
    const float *cs = rope + static_cast<int64_t>(pos) * 128;  // [64][2]
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const float partner = __shfl_xor_sync(0xffffffffu, y[k], 16);
        const int i = 4 * (lane & 15) + k;
        const float c = cs[2 * i], s = cs[2 * i + 1];
        if (lane < 16)
            o[k] = __fmaf_rn(y[k], c, -__fmul_rn(partner, s));  // x0 = y, x1 = partner
        else
            o[k] = __fmaf_rn(partner, s, __fmul_rn(y[k], c));   // x0 = partner, x1 = y
    }
    if (hw < n_heads) {
        *reinterpret_cast<float4 *>(q_out + static_cast<int64_t>(hw) * 128 + 4 * lane) =
            make_float4(o[0], o[1], o[2], o[3]);
    } else {
        const int g = hw - n_heads;
        __half *dst = kc + (static_cast<int64_t>(g) * max_ctx + pos) * 128 + 4 * lane;
#pragma unroll
        for (int k = 0; k < 4; ++k) dst[k] = __float2half_rn(o[k]);
    }
}

// ------------------------------------------------------------ attention ---
// Partials of one (kv head g, chunk c of 256 positions) for its GQA group of
// q heads.  Thread t owns slot t (position c*256 + t): scores by a
// sequential fmaf over d = 0..127, times scale.  m = chunk max, e = exp(s -
// m) (0 past L), l = per-warp xor butterfly then warps in order.  PV: warp w
// walks its 32 slots in order, lane l owns dims 4l..4l+3 (fmaf chain);
// warps are added in order.
constexpr int ATT_CHUNK = 256;
constexpr int ATT_MAXG = 8;  // q heads per kv head supported

// Sequence blockIdx.z of a batch: q and the KV cache advance by their strides,
// the partials by (kv heads * GQ) * max_chunks per sequence.
template <int GQ>
__global__ void __launch_bounds__(256)
    attention_chunk_kernel(const float *__restrict__ q, const __half *__restrict__ kc,
                           const __half *__restrict__ vc, const int32_t *__restrict__ pos_p,
                           float scale, int max_ctx, int max_chunks,
                           float *__restrict__ part_m, float *__restrict__ part_l,
                           float *__restrict__ part_o, int64_t q_stride, int64_t kv_stride,
                           int pos_stride) {
    {
        const int64_t z = blockIdx.z;
        const int64_t pstride = static_cast<int64_t>(gridDim.x) * GQ * max_chunks;
        q += z * q_stride;
        kc += z * kv_stride;
        vc += z * kv_stride;
        part_m += z * pstride;
        part_l += z * pstride;
        part_o += z * pstride * 128;
    }
    __shared__ __align__(16) float s_q[GQ][128];
    __shared__ float s_e[GQ][ATT_CHUNK];
    __shared__ float s_red[GQ][8];
    __shared__ __align__(16) float s_o[8][GQ][128];
    pdl_wait();
    pdl_launch_dependents();
    const int L = min(*pos_p + static_cast<int>(blockIdx.z) * pos_stride + 1, max_ctx);
    const int c = blockIdx.y, g = blockIdx.x;
    if (c * ATT_CHUNK >= L) return;
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    for (int i = t; i < GQ * 128; i += 256) s_q[i / 128][i % 128] = q[static_cast<int64_t>(g * GQ) * 128 + i];
    __syncthreads();
    const int j = c * ATT_CHUNK + t;
    const bool valid = j < L;
    // scores: sequential fmaf over d = 0..127 (all 16 row loads issued first)
    float s[GQ];
#pragma unroll
    for (int h = 0; h < GQ; ++h) s[h] = 0.0f;
    if (valid) {
        const uint4 *krow = reinterpret_cast<const uint4 *>(kc + (static_cast<int64_t>(g) * max_ctx + j) * 128);
        uint4 kv[16];
#pragma unroll
        for (int d8 = 0; d8 < 16; ++d8) kv[d8] = __ldg(krow + d8);
#pragma unroll
        for (int d8 = 0; d8 < 16; ++d8) {
            const __half2 *k2 = reinterpret_cast<const __half2 *>(&kv[d8]);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float2 kf = __half22float2(k2[e]);
#pragma unroll
                for (int h = 0; h < GQ; ++h) {
                    const float2 qv = *reinterpret_cast<const float2 *>(&s_q[h][d8 * 8 + 2 * e]);
                    s[h] = __fmaf_rn(qv.x, kf.x, s[h]);
                    s[h] = __fmaf_rn(qv.y, kf.y, s[h]);
                }
            }
        }
    }
    // chunk max per head, e = exp(s - m), per-warp butterfly sums
#pragma unroll
    for (int h = 0; h < GQ; ++h) {
        const float sv = valid ? __fmul_rn(s[h], scale) : -INFINITY;
        float mx = sv;
#pragma unroll
        for (int m = 16; m >= 1; m >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, m));
        if (lane == 0) s_red[h][warp] = mx;
        s[h] = sv;
    }
    __syncthreads();
    float ev[GQ];
#pragma unroll
    for (int h = 0; h < GQ; ++h) {
        float mx = s_red[h][0];
#pragma unroll
        for (int w = 1; w < 8; ++w) mx = fmaxf(mx, s_red[h][w]);
        ev[h] = valid ? abra_expf(__fsub_rn(s[h], mx)) : 0.0f;
        s_e[h][t] = ev[h];
        if (t == 0) part_m[static_cast<int64_t>(g * GQ + h) * max_chunks + c] = mx;
    }
    __syncthreads();  // s_red is reused for the sums
#pragma unroll
    for (int h = 0; h < GQ; ++h) {
        float v = ev[h];
#pragma unroll
        for (int m = 16; m >= 1; m >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, m));
        if (lane == 0) s_red[h][warp] = v;
    }
    __syncwarp();
    // PV: this warp's 32 slots in order, V segments fetched 8 slots at a time
    float acc[GQ][4];
#pragma unroll
    for (int h = 0; h < GQ; ++h)
#pragma unroll
        for (int k = 0; k < 4; ++k) acc[h][k] = 0.0f;
    const int j0 = c * ATT_CHUNK + warp * 32;
    const int nv = max(0, min(32, L - j0));
    const __half *vbase = vc + (static_cast<int64_t>(g) * max_ctx + j0) * 128 + 4 * lane;
#pragma unroll
    for (int g8 = 0; g8 < 4; ++g8) {
        if (g8 * 8 >= nv) break;
        uint2 vv[8];
#pragma unroll
        for (int u = 0; u < 8; ++u)
            if (g8 * 8 + u < nv) vv[u] = __ldg(reinterpret_cast<const uint2 *>(vbase + (g8 * 8 + u) * 128));
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            if (g8 * 8 + u < nv) {
                const float2 v01 = __half22float2(*reinterpret_cast<const __half2 *>(&vv[u].x));
                const float2 v23 = __half22float2(*reinterpret_cast<const __half2 *>(&vv[u].y));
                const float vf[4] = {v01.x, v01.y, v23.x, v23.y};
#pragma unroll
                for (int h = 0; h < GQ; ++h) {
                    const float e = s_e[h][warp * 32 + g8 * 8 + u];
#pragma unroll
                    for (int k = 0; k < 4; ++k) acc[h][k] = __fmaf_rn(e, vf[k], acc[h][k]);
                }
            }
        }
    }
#pragma unroll
    for (int h = 0; h < GQ; ++h)
        *reinterpret_cast<float4 *>(&s_o[warp][h][4 * lane]) = make_float4(acc[h][0], acc[h][1], acc[h][2], acc[h][3]);
    __syncthreads();
    for (int i = t; i < GQ * 128; i += 256) {
        const int h = i / 128, d = i % 128;
        float o = s_o[0][h][d];
#pragma unroll
        for (int w = 1; w < 8; ++w) o = __fadd_rn(o, s_o[w][h][d]);
        part_o[(static_cast<int64_t>(g * GQ + h) * max_chunks + c) * 128 + d] = o;
    }
    if (t < GQ) {
        float l = s_red[t][0];
#pragma unroll
        for (int w = 1; w < 8; ++w) l = __fadd_rn(l, s_red[t][w]);
        part_l[static_cast<int64_t>(g * GQ + t) * max_chunks + c] = l;
    }
}

// Merge the chunk partials of one q head (one warp per head, lane owns dims
// 4l..4l+3): M = max m_c, w_c = exp(m_c - M), L = fmaf(l_c, w_c, L),
// O = fmaf(o_c, w_c, O) over chunks in order, out = O / L; then Q8_1 of the
// head's 128 values (4 blocks of 32, 8 lanes per block).
__global__ void __launch_bounds__(256)
    attention_merge_quant_kernel(const float *__restrict__ part_m,
                                 const float *__restrict__ part_l,
                                 const float *__restrict__ part_o,
                                 const int32_t *__restrict__ pos_p, int n_heads, int max_chunks,
                                 float *__restrict__ out_f32, block_q8_1 *__restrict__ out_q8,
                                 int pos_stride) {
    pdl_wait();
    pdl_launch_dependents();
    {  // sequence blockIdx.y of a batch
        const int64_t y = blockIdx.y, pstride = static_cast<int64_t>(n_heads) * max_chunks;
        part_m += y * pstride;
        part_l += y * pstride;
        part_o += y * pstride * 128;
        if (out_f32) out_f32 += y * n_heads * 128;
        out_q8 += y * n_heads * 4;
    }
    const int lane = threadIdx.x & 31;
    const int hq = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (hq >= n_heads) return;
    const int L = min(*pos_p + static_cast<int>(blockIdx.y) * pos_stride + 1, max_chunks * ATT_CHUNK);
    const int nch = (L + ATT_CHUNK - 1) / ATT_CHUNK;
    const float *pm = part_m + static_cast<int64_t>(hq) * max_chunks;
    const float *pl = part_l + static_cast<int64_t>(hq) * max_chunks;
    float M = pm[0];
    for (int c = 1; c < nch; ++c) M = fmaxf(M, pm[c]);
    float Ls = 0.0f, O[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int c = 0; c < nch; ++c) {
        const float wc = abra_expf(__fsub_rn(pm[c], M));
        Ls = __fmaf_rn(pl[c], wc, Ls);
        const float4 o = *reinterpret_cast<const float4 *>(part_o + (static_cast<int64_t>(hq) * max_chunks + c) * 128 + 4 * lane);
        O[0] = __fmaf_rn(o.x, wc, O[0]);
        O[1] = __fmaf_rn(o.y, wc, O[1]);
        O[2] = __fmaf_rn(o.z, wc, O[2]);
        O[3] = __fmaf_rn(o.w, wc, O[3]);
    }
    float x[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) x[k] = __fdiv_rn(O[k], Ls);
    if (out_f32)
        *reinterpret_cast<float4 *>(out_f32 + static_cast<int64_t>(hq) * 128 + 4 * lane) = make_float4(x[0], x[1], x[2], x[3]);
    // Q8_1 (reference semantics): 8 lanes x 4 values per 32-block
    float amax = fmaxf(fmaxf(fabsf(x[0]), fabsf(x[1])), fmaxf(fabsf(x[2]), fabsf(x[3])));
    amax = fmaxf(0.0f, amax);
#pragma unroll
    for (int m = 4; m >= 1; m >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, m));
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d > 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    int qv[4], sum = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        qv[k] = static_cast<int>(static_cast<int8_t>(static_cast<int>(roundf(__fmul_rn(x[k], id)))));
        sum += qv[k];
    }
#pragma unroll
    for (int m = 4; m >= 1; m >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, m);
    block_q8_1 *blk = out_q8 + static_cast<int64_t>(hq) * 4 + (lane >> 3);
    uint32_t *o32 = reinterpret_cast<uint32_t *>(blk);
    o32[1 + (lane & 7)] = (static_cast<uint32_t>(qv[0]) & 0xffu) | ((static_cast<uint32_t>(qv[1]) & 0xffu) << 8) |
                          ((static_cast<uint32_t>(qv[2]) & 0xffu) << 16) | ((static_cast<uint32_t>(qv[3]) & 0xffu) << 24);
    if ((lane & 7) == 0) {
        const uint32_t hd = __half_as_ushort(__float2half_rn(d));
        const uint32_t hs = __half_as_ushort(__float2half_rn(__fmul_rn(d, static_cast<float>(sum))));
        o32[0] = hd | (hs << 16);
    }
}

// --------------------------------------------------------------- argmax ---
// Finish of the argmax fused into the output MMVQ: decode the winning key
// (ties already resolved to the lowest row), reset it for the next step,
// record the pick, append it past the prompt, advance *pos.
__global__ void argmax_finish_kernel(unsigned long long *__restrict__ key,
                                     int32_t *__restrict__ tokens, int32_t *__restrict__ picks,
                                     int32_t *__restrict__ pos_p,
                                     const int32_t *__restrict__ n_prompt_p, int max_ctx,
                                     const unsigned long long *wait_cnt,
                                     unsigned long long *epoch, unsigned long long per_step) {
    pdl_wait();
    pdl_launch_dependents();
    if (threadIdx.x != 0) return;
    if (epoch) {  // tensor parallel: every rank's keys have arrived
        const unsigned long long e = __ldcg(epoch);
        if (wait_cnt) wait_count(wait_cnt, (e + 1ull) * per_step);
        *epoch = e + 1ull;
    }
    const unsigned long long k = __ldcg(key);
    *key = 0ull;
    const int bi = static_cast<int>(0xFFFFFFFFu - static_cast<unsigned>(k & 0xFFFFFFFFull));
    const int p = *pos_p;
    if (p < max_ctx) {  // the host never steps past max_ctx
        picks[p] = bi;
        if (p + 1 >= *n_prompt_p) tokens[p + 1] = bi;
        *pos_p = p + 1;
    }
}

// ------------------------------------------------------ batched decode ---
// Greedy pick of sequence blockIdx.x of a batch: largest of its n logits
// (row stride ldl), ties to the lowest index; records picks[seq][*pos] and,
// past the prompt, tokens[seq][*pos + 1].  The shared position advances in
// pos_advance_kernel once every sequence has read it.
__global__ void __launch_bounds__(1024)
    argmax_batch_kernel(const float *__restrict__ x, int n, int64_t ldl,
                        int32_t *__restrict__ tokens, int32_t *__restrict__ picks,
                        int64_t tok_stride, const int32_t *__restrict__ pos_p,
                        const int32_t *__restrict__ n_prompt_p, int max_ctx) {
    __shared__ float sv[32];
    __shared__ int si[32];
    pdl_wait();
    pdl_launch_dependents();
    x += blockIdx.x * ldl;
    tokens += blockIdx.x * tok_stride;
    picks += blockIdx.x * tok_stride;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = x[i];
        if (v > bv) {
            bv = v;
            bi = i;
        }
    }
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, m);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, m);
        if (ov > bv || (ov == bv && oi < bi)) {
            bv = ov;
            bi = oi;
        }
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) {
        sv[warp] = bv;
        si[warp] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w)
            if (sv[w] > bv || (sv[w] == bv && si[w] < bi)) {
                bv = sv[w];
                bi = si[w];
            }
        const int p = *pos_p;
        if (bi == 0x7fffffff) bi = 0;
        if (p < max_ctx) {  // the host never steps past max_ctx
            picks[p] = bi;
            if (p + 1 >= *n_prompt_p) tokens[p + 1] = bi;
        }
    }
}

// Tensor parallel, batch: the key of each sequence's largest logit among
// this rank's vocab rows (argmax_key of (value, row_offset + row): ties to
// the lowest id), merged into that sequence's key word on every rank; each
// CTA then counts itself on cta_cnt and the launch's last CTA adds 1 to every
// rank's counter with release semantics at system scope.  One CTA of 1024
// threads per sequence.
__global__ void __launch_bounds__(1024)
    argmax_keys_batch_kernel(const float *__restrict__ x, int n, int64_t ldl, int row_offset,
                             const TpKeyPush push) {
    __shared__ unsigned long long sk[32];
    pdl_wait();
    pdl_launch_dependents();
    x += blockIdx.x * ldl;
    unsigned long long best = 0ull;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const unsigned long long k = argmax_key(x[i], row_offset + i);
        best = k > best ? k : best;
    }
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) {
        const unsigned long long o = __shfl_xor_sync(0xffffffffu, best, m);
        best = o > best ? o : best;
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) sk[warp] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w) best = sk[w] > best ? sk[w] : best;
        for (int q = 0; q < push.npeer; ++q) atomicMax_system(push.key[q] + blockIdx.x, best);
        const unsigned long long old = atom_add_acq_rel_gpu(push.cta_cnt, 1ull);
        if ((old + 1ull) % gridDim.x == 0ull)
            for (int q = 0; q < push.npeer; ++q) red_release_sys_add(push.cnt[q], 1ull);
    }
}

// Tensor parallel, batch: once every rank's keys have arrived (bounded wait
// on wait_cnt), each sequence's pick from its key word (then reset), the
// picks and, past the prompt, the next tokens; then the step's epoch and the
// shared position advance.
__global__ void argmax_finish_batch_kernel(unsigned long long *__restrict__ keys, int batch,
                                           int32_t *__restrict__ tokens, int32_t *__restrict__ picks,
                                           int64_t tok_stride, int32_t *__restrict__ pos_p,
                                           const int32_t *__restrict__ n_prompt_p, int max_ctx,
                                           const unsigned long long *wait_cnt, unsigned long long *epoch,
                                           unsigned long long per_step) {
    __shared__ int s_pos;
    __shared__ unsigned long long s_e;
    pdl_wait();
    pdl_launch_dependents();
    const int t = threadIdx.x;
    if (t == 0) {
        s_e = __ldcg(epoch);
        wait_count(wait_cnt, (s_e + 1ull) * per_step);
        s_pos = *pos_p;
    }
    __syncthreads();
    const int p = s_pos;
    for (int b = t; b < batch; b += blockDim.x) {
        const unsigned long long k = __ldcg(keys + b);
        keys[b] = 0ull;
        const int bi = static_cast<int>(0xFFFFFFFFu - static_cast<unsigned>(k & 0xFFFFFFFFull));
        if (p < max_ctx) {  // the host never steps past max_ctx
            picks[b * tok_stride + p] = bi;
            if (p + 1 >= *n_prompt_p) tokens[b * tok_stride + p + 1] = bi;
        }
    }
    __syncthreads();
    if (t == 0) {
        *epoch = s_e + 1ull;
        if (p < max_ctx) *pos_p = p + 1;
    }
}

// out[c] = argmax of logits column c (ties to the lowest index, the order of
// argmax_batch_kernel); one CTA of 1024 threads per column.
__global__ void argmax_cols_kernel(const float *__restrict__ x, int n, int64_t ldl,
                                   int32_t *__restrict__ out) {
    __shared__ float sv[32];
    __shared__ int si[32];
    pdl_wait();
    pdl_launch_dependents();
    x += blockIdx.x * ldl;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = x[i];
        if (v > bv) {
            bv = v;
            bi = i;
        }
    }
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, m);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, m);
        if (ov > bv || (ov == bv && oi < bi)) {
            bv = ov;
            bi = oi;
        }
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) {
        sv[warp] = bv;
        si[warp] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w)
            if (sv[w] > bv || (sv[w] == bv && si[w] < bi)) {
                bv = sv[w];
                bi = si[w];
            }
        out[blockIdx.x] = bi == 0x7fffffff ? 0 : bi;
    }
}

__global__ void pos_advance_kernel(int32_t *__restrict__ pos_p, int n, int max_ctx) {
    pdl_wait();
    pdl_launch_dependents();
    if (threadIdx.x == 0) *pos_p = min(*pos_p + n, max_ctx);
}

// act = up * silu(gate) (the fused gate/up MMVQ's epilogue, elementwise),
// then its Q8_1 blocks; one warp per 32-block.
__global__ void __launch_bounds__(256)
    swiglu_quant_kernel(const float *__restrict__ g, const float *__restrict__ u,
                        block_q8_1 *__restrict__ y, int64_t nblocks_total) {
    const int lane = threadIdx.x & 31;
    const int64_t warp = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
    pdl_wait();
    pdl_launch_dependents();
    if (warp >= nblocks_total) return;
    const int64_t i = warp * QK8_1 + lane;
    quantize_block_warp(__fmul_rn(u[i], abra_silu(g[i])), y + warp, lane);
}

// ----------------------------------------------------------- launchers ---
static cudaLaunchAttribute pdl_attr() {
    cudaLaunchAttribute a;
    a.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    a.val.programmaticStreamSerializationAllowed = 1;
    return a;
}

template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t stream, bool pdl, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1] = {pdl_attr()};
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k, static_cast<KArgs>(args)...);
}

cudaError_t launch_embed(const void *E, int hidden, const int32_t *tokens, const int32_t *pos,
                         float *h, bool pdl, cudaStream_t s, int batch, int64_t tok_stride) {
    return launch_pdl(embed_kernel, dim3((hidden + 255) / 256, batch), dim3(256), 0, s, pdl,
                      static_cast<const uint8_t *>(E), hidden, tokens, pos, h, tok_stride);
}

cudaError_t launch_embed_q6k(const void *E, int hidden, const int32_t *tokens, const int32_t *pos,
                             float *h, bool pdl, cudaStream_t s, int batch, int64_t tok_stride) {
    return launch_pdl(embed_q6k_kernel, dim3((hidden + 255) / 256, batch), dim3(256), 0, s, pdl,
                      static_cast<const uint8_t *>(E), hidden, tokens, pos, h, tok_stride);
}

cudaError_t launch_residual_rmsnorm_quant(float *h, const DeltaSet &ds, const float *w,
                                          float eps, void *y, int K, int ncols, bool pdl,
                                          cudaStream_t s, const unsigned long long *wait_cnt,
                                          const unsigned long long *epoch, unsigned long long per_step) {
    const size_t smem = static_cast<size_t>(K) * sizeof(float);
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(residual_rmsnorm_quant_kernel,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem));
        if (e != cudaSuccess) return e;
    }
    return launch_pdl(residual_rmsnorm_quant_kernel, dim3(ncols), dim3(RES_THREADS), smem, s, pdl,
                      h, ds, w, eps, static_cast<block_q8_1 *>(y), K, wait_cnt, epoch, per_step);
}

cudaError_t launch_qk_norm_rope_kv(const float *qkv, const float *q_norm, const float *k_norm,
                                   float eps, const float *rope, const int32_t *pos, float *q_out,
                                   void *kc, void *vc, int n_heads, int n_kv, int max_ctx,
                                   bool pdl, cudaStream_t s, const SeqStrides &b) {
    const int heads = n_heads + 2 * n_kv;
    return launch_pdl(qk_norm_rope_kv_kernel, dim3((heads + 7) / 8, b.batch), dim3(256), 0, s, pdl,
                      qkv, q_norm, k_norm, eps, rope, pos, q_out, static_cast<__half *>(kc),
                      static_cast<__half *>(vc), n_heads, n_kv, max_ctx, b.qkv, b.q, b.kv, b.pos);
}

cudaError_t launch_attention(const float *q, const void *kc, const void *vc, const int32_t *pos,
                             float scale, int n_heads, int n_kv, int max_ctx, float *part_m,
                             float *part_l, float *part_o, float *out_f32, void *out_q8,
                             bool pdl, cudaStream_t s, const SeqStrides &b) {
    const int gq = n_heads / n_kv;
    if (gq > ATT_MAXG || n_heads % n_kv) return cudaErrorInvalidValue;
    const int max_chunks = (max_ctx + ATT_CHUNK - 1) / ATT_CHUNK;
    const dim3 grid(n_kv, max_chunks, b.batch);
    const __half *k = static_cast<const __half *>(kc);
    const __half *v = static_cast<const __half *>(vc);
    cudaError_t e;
#define ABRA_ATT(G)                                                                                  \
    launch_pdl(attention_chunk_kernel<G>, grid, dim3(256), 0, s, pdl, q, k, v, pos, scale, max_ctx, \
               max_chunks, part_m, part_l, part_o, b.q, b.kv, b.pos)
    switch (gq) {
        case 1: e = ABRA_ATT(1); break;
        case 2: e = ABRA_ATT(2); break;
        case 4: e = ABRA_ATT(4); break;
        case 8: e = ABRA_ATT(8); break;
        default: return cudaErrorInvalidValue;
    }
#undef ABRA_ATT
    if (e != cudaSuccess) return e;
    return launch_pdl(attention_merge_quant_kernel, dim3((n_heads + 7) / 8, b.batch), dim3(256), 0, s,
                      pdl, static_cast<const float *>(part_m), static_cast<const float *>(part_l),
                      static_cast<const float *>(part_o), pos, n_heads, max_chunks, out_f32,
                      static_cast<block_q8_1 *>(out_q8), b.pos);
}

cudaError_t launch_argmax_batch(const float *logits, int n, int64_t ldl, int32_t *tokens,
                                int32_t *picks, int64_t tok_stride, int32_t *pos,
                                const int32_t *n_prompt, int max_ctx, int batch, bool pdl,
                                cudaStream_t s) {
    cudaError_t e = launch_pdl(argmax_batch_kernel, dim3(batch), dim3(1024), 0, s, pdl, logits, n,
                               ldl, tokens, picks, tok_stride, static_cast<const int32_t *>(pos),
                               n_prompt, max_ctx);
    if (e != cudaSuccess) return e;
    return launch_pdl(pos_advance_kernel, dim3(1), dim3(32), 0, s, pdl, pos, 1, max_ctx);
}

cudaError_t launch_argmax_keys_batch(const float *logits, int n, int64_t ldl, int row_offset,
                                     const TpKeyPush &push, int batch, bool pdl, cudaStream_t s) {
    if (push.npeer < 1 || push.npeer > 8 || !push.cta_cnt) return cudaErrorInvalidValue;
    return launch_pdl(argmax_keys_batch_kernel, dim3(batch), dim3(1024), 0, s, pdl, logits, n, ldl, row_offset,
                      push);
}

cudaError_t launch_argmax_finish_batch(unsigned long long *keys, int batch, int32_t *tokens, int32_t *picks,
                                       int64_t tok_stride, int32_t *pos, const int32_t *n_prompt, int max_ctx,
                                       const unsigned long long *wait_cnt, unsigned long long *epoch,
                                       unsigned long long per_step, bool pdl, cudaStream_t s) {
    if (!wait_cnt || !epoch) return cudaErrorInvalidValue;
    return launch_pdl(argmax_finish_batch_kernel, dim3(1), dim3(64), 0, s, pdl, keys, batch, tokens, picks,
                      tok_stride, pos, n_prompt, max_ctx, wait_cnt, epoch, per_step);
}

cudaError_t launch_argmax_cols(const float *logits, int n, int64_t ldl, int32_t *out, int ncols,
                               bool pdl, cudaStream_t s) {
    return launch_pdl(argmax_cols_kernel, dim3(ncols), dim3(1024), 0, s, pdl, logits, n, ldl, out);
}

cudaError_t launch_pos_advance(int32_t *pos, int n, int max_ctx, bool pdl, cudaStream_t s) {
    return launch_pdl(pos_advance_kernel, dim3(1), dim3(32), 0, s, pdl, pos, n, max_ctx);
}

cudaError_t launch_swiglu_quant(const float *g, const float *u, void *y, int64_t n, bool pdl,
                                cudaStream_t s) {
    const int64_t nb = n / QK8_1;
    const int64_t grid = (nb * 32 + 255) / 256;
    return launch_pdl(swiglu_quant_kernel, dim3(static_cast<unsigned>(grid)), dim3(256), 0, s, pdl, g, u,
                      static_cast<block_q8_1 *>(y), nb);
}

cudaError_t launch_argmax_finish(unsigned long long *key, int32_t *tokens, int32_t *picks,
                                 int32_t *pos, const int32_t *n_prompt, int max_ctx, bool pdl,
                                 cudaStream_t s, const unsigned long long *wait_cnt,
                                 unsigned long long *epoch, unsigned long long per_step) {
    return launch_pdl(argmax_finish_kernel, dim3(1), dim3(32), 0, s, pdl, key, tokens, picks, pos,
                      n_prompt, max_ctx, wait_cnt, epoch, per_step);
}

}  // namespace abra

ABRA_ERROR_WORD_ACCESSOR(error_word_decode)
