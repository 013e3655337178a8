// mmvq_q6k_impl.cuh -- the Q6_K x Q8_1 MMVQ kernel template (sm_100a).
//
// y[c][r] = sum_k w[r][k] * x[c][k] for Q6_K rows w (ggml's block_q6_K,
// 210 bytes per 256 weights: ql[128], qh[64], int8 scales[16], fp16 d) and
// Q8_1 activation columns x: the Q6_K leg of the reference's MMVQ dispatch
// (kernels/q4k/abra-mmvq.cuh:138-141, ggml's vec_dot_q6_K_q8_1), whose
// element order the reference's f64 oracle spells out
// (tests/runtime_kernel_test.cu:82-106).
//
// A 210-byte superblock is only 2-byte aligned, so every weight read is an
// aligned 32-bit word pair joined by a funnel shift.  Three ways to feed a
// unit of 8 rows x one k-part, as for Q4_K:
//   Q6_ROWS    a producer warp copies each row's byte range of the part with
//              one cp.async.bulk (start rounded down, end rounded up to 16
//              bytes, never past the last 16-byte boundary of the weights;
//              the last few bytes of the tensor, if any, by plain loads);
//   Q6_WHOLE   one bulk copy per unit (KS == 1): 8 whole rows are contiguous
//              and start on a 16-byte boundary (8 * 210 * nsb = 1680 nsb);
//   Q6_DIRECT  no producer: lanes load their words with ld.global.nc, one
//              superblock ahead.
// No copy uses cluster multicast.
//
// Consumer lane (p = lane/8 = 2h + s, g = lane%8): row g of the unit, half h
// of the superblock, ql bytes [64h + 32s, +32) -- the low nibbles are Q8_1
// block 4h+s (group s), the high nibbles block 4h+s+2 (group s+2) -- with the
// qh bytes [32h, +32) that both lanes of the half share.  Each lane forms the
// four exact int32 16-weight dots of its two blocks by dp4a on the unsigned
// 6-bit codes, less 32 x the block-half sums of the activation.
//
// Canonical fp32 order (shared with the CPU oracle, bit for bit):
//   I_b = P_2b sc_2b + P_2b+1 sc_2b+1 (exact),  t_b = d8_b * float(I_b)
//   S = ((t_0 + t_1) + (t_2 + t_3)) + ((t_4 + t_5) + (t_6 + t_7))
//       [xor 8 gives t_4h+s + t_4h+s^1 in either order, xor 16 the halves]
//   value(superblock) = d * S; the eight K-slices and their tree as Q4_K.
#pragma once

#include "mmvq_impl.cuh"

namespace abra {

constexpr int Q6K_BYTES = 210;

enum Q6Mode : int { Q6_ROWS = 0, Q6_WHOLE = 1, Q6_DIRECT = 2 };

struct Q6Params {
    const uint8_t *W;  // N rows of nsb blocks, 16-byte aligned
    const uint8_t *X;  // Q8_1 columns
    float *Y;
    int N, nsb;
    int64_t ldy;
    int64_t w_bytes;  // N * nsb * 210
    int rg_total, nstage, pitch, stage_bytes;
    int32_t *P;                // debug partials (EMIT_P): [c][r][b][16]
    unsigned long long *amax;  // optional per-column argmax keys
    int row_offset;            // added to row ids in argmax keys
    int sl_nsb, sl_base, sl_shift;  // K-shard slicing, as MmvqParams
    const uint8_t *pf_ptr[2];        // L2 prefetch of the next kernels' weights
    int64_t pf_bytes[2];
};

struct Q6Layout {
    int off_full, off_empty, off_red, off_qs, off_d8, off_m, off_stage, bytes;
};

__host__ __device__ __forceinline__ Q6Layout q6_layout(int ncols, int ks, int ncw, int nsb,
                                                       int nstage, int stage_bytes, bool staged) {
    Q6Layout L;
    L.off_full = 0;
    L.off_empty = 8 * nstage;
    int o = staged ? 16 * nstage : 0;
    L.off_red = align_up(o, 16);
    o = L.off_red + (ks > 1 ? 2 * ncw * 8 * ncols * 4 : 0);
    L.off_qs = align_up(o, 128);
    o = L.off_qs + ncols * nsb * 256;
    L.off_d8 = align_up(o, 16);
    o = L.off_d8 + ncols * nsb * 8 * 4;
    L.off_m = align_up(o, 16);
    o = L.off_m + ncols * nsb * 16 * 4;
    L.off_stage = align_up(o, 128);
    L.bytes = L.off_stage + (staged ? nstage * stage_bytes : 0);
    return L;
}

// n words starting at byte address p (any even address): aligned words
// joined by a funnel shift; reads the n+1 aligned words covering the run.
template <int NW, bool GLOBAL>
__device__ __forceinline__ void q6_words(const uint8_t *p, uint32_t (&out)[NW]) {
    const uint32_t *a = reinterpret_cast<const uint32_t *>(reinterpret_cast<uintptr_t>(p) & ~uintptr_t(3));
    const uint32_t sh = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(p) & 3u) * 8u;
    uint32_t w[NW + 1];
#pragma unroll
    for (int k = 0; k <= NW; ++k) w[k] = GLOBAL ? __ldg(a + k) : a[k];
#pragma unroll
    for (int k = 0; k < NW; ++k) out[k] = __funnelshift_r(w[k], w[k + 1], sh);
}

template <bool GLOBAL>
__device__ __forceinline__ uint32_t q6_u16(const uint8_t *p) {
    const uint16_t *a = reinterpret_cast<const uint16_t *>(p);
    return GLOBAL ? static_cast<uint32_t>(__ldg(a)) : static_cast<uint32_t>(*a);
}

// Raw bytes of one superblock that lane (h, s) needs: 32 ql bytes, 32 qh
// bytes, the scale pairs of its two groups and d.  Every read stays inside
// the block: the ql and qh runs end at least 4 bytes before its end, the
// scales and d are 16-bit loads.
struct Q6Raw {
    uint32_t ql[8], qh[8], scA, scB, d;
};

template <bool GLOBAL>
__device__ __forceinline__ void q6_fetch(const uint8_t *blk, int h, int s, Q6Raw &r) {
    q6_words<8, GLOBAL>(blk + 64 * h + 32 * s, r.ql);
    q6_words<8, GLOBAL>(blk + 128 + 32 * h, r.qh);
    r.scA = q6_u16<GLOBAL>(blk + 192 + 8 * h + 2 * s);
    r.scB = q6_u16<GLOBAL>(blk + 196 + 8 * h + 2 * s);
    r.d = q6_u16<GLOBAL>(blk + 208);
}

// Signed byte k (0, 1) of a 16-bit pair.
__device__ __forceinline__ int q6_sbyte(uint32_t pair, int k) {
    return static_cast<int>(static_cast<int8_t>((pair >> (8 * k)) & 0xffu));
}

// Values of one superblock for every column (lane (h, s) of row g), the
// int32 dots of its four sub-blocks in P[c][0..3] (sub-blocks 8h+2s, +1 of
// group s, 8h+2s+4, +5 of group s+2).
template <int NCOLS>
__device__ __forceinline__ void q6_values(const Q6Raw &r, int h, int s, const uint8_t *aq,
                                          const float *ad8, const int *am, int nsb, int b,
                                          float (&v)[NCOLS], int (&P)[NCOLS][4]) {
    uint32_t va[8], vb[8];
    const int shA = 4 - 2 * s, shB = 2 * s;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        va[k] = (r.ql[k] & 0x0F0F0F0Fu) | ((r.qh[k] << shA) & 0x30303030u);
        vb[k] = ((r.ql[k] >> 4) & 0x0F0F0F0Fu) | ((r.qh[k] >> shB) & 0x30303030u);
    }
    const int scA0 = q6_sbyte(r.scA, 0), scA1 = q6_sbyte(r.scA, 1);
    const int scB0 = q6_sbyte(r.scB, 0), scB1 = q6_sbyte(r.scB, 1);
    const float d = half_lo(r.d);
    const int bA = 4 * h + s, bB = bA + 2;
#pragma unroll
    for (int c = 0; c < NCOLS; ++c) {
        const int base = (c * nsb + b) * 8;
        const uint4 *xa = reinterpret_cast<const uint4 *>(aq + static_cast<int64_t>(base + bA) * 32);
        const uint4 *xb = reinterpret_cast<const uint4 *>(aq + static_cast<int64_t>(base + bB) * 32);
        const uint4 a0 = xa[0], a1 = xa[1], b0 = xb[0], b1 = xb[1];
        const int2 mA = *reinterpret_cast<const int2 *>(am + (base + bA) * 2);
        const int2 mB = *reinterpret_cast<const int2 *>(am + (base + bB) * 2);
        int pA0 = 0, pA1 = 0, pB0 = 0, pB1 = 0;
        pA0 = dp4a_us(va[0], a0.x, pA0);
        pA0 = dp4a_us(va[1], a0.y, pA0);
        pA0 = dp4a_us(va[2], a0.z, pA0);
        pA0 = dp4a_us(va[3], a0.w, pA0);
        pA1 = dp4a_us(va[4], a1.x, pA1);
        pA1 = dp4a_us(va[5], a1.y, pA1);
        pA1 = dp4a_us(va[6], a1.z, pA1);
        pA1 = dp4a_us(va[7], a1.w, pA1);
        pB0 = dp4a_us(vb[0], b0.x, pB0);
        pB0 = dp4a_us(vb[1], b0.y, pB0);
        pB0 = dp4a_us(vb[2], b0.z, pB0);
        pB0 = dp4a_us(vb[3], b0.w, pB0);
        pB1 = dp4a_us(vb[4], b1.x, pB1);
        pB1 = dp4a_us(vb[5], b1.y, pB1);
        pB1 = dp4a_us(vb[6], b1.z, pB1);
        pB1 = dp4a_us(vb[7], b1.w, pB1);
        pA0 -= 32 * mA.x;  // (q - 32) . x = q . x - 32 sum(x), exact
        pA1 -= 32 * mA.y;
        pB0 -= 32 * mB.x;
        pB1 -= 32 * mB.y;
        P[c][0] = pA0;
        P[c][1] = pA1;
        P[c][2] = pB0;
        P[c][3] = pB1;
        const float tA = __fmul_rn(ad8[base + bA], __int2float_rn(pA0 * scA0 + pA1 * scA1));
        const float tB = __fmul_rn(ad8[base + bB], __int2float_rn(pB0 * scB0 + pB1 * scB1));
        const float xA = __fadd_rn(tA, __shfl_xor_sync(0xffffffffu, tA, 8));
        const float xB = __fadd_rn(tB, __shfl_xor_sync(0xffffffffu, tB, 8));
        float q = __fadd_rn(xA, xB);
        q = __fadd_rn(q, __shfl_xor_sync(0xffffffffu, q, 16));
        v[c] = __fmul_rn(d, q);
    }
}

// Producer: bytes [start, end) of the weights into dst, where dst holds the
// 16-byte-aligned run from start & ~15.  Bulk-copies up to the last 16-byte
// boundary of the tensor and plain-copies what lies past it.  Returns the
// bulk bytes (for the stage's expected transaction count).
__device__ __forceinline__ uint32_t q6_tail_copy(uint8_t *dst, const uint8_t *W, int64_t start,
                                                 int64_t end, int64_t w_bytes) {
    const int64_t a = start & ~int64_t(15);
    const int64_t lim = w_bytes & ~int64_t(15);
    int64_t b = (end + 15) & ~int64_t(15);
    if (b > lim) b = lim;
    if (b < a) b = a;
    for (int64_t t = b; t < end; ++t) dst[t - a] = W[t];
    return static_cast<uint32_t>(b - a);
}

// Debug store of a lane's four sub-block dots (rows < N only).
template <int NCOLS>
__device__ __forceinline__ void q6_emit_p(int32_t *P, int N, int nsb, int row, int b, int h, int s,
                                          const int (&v)[NCOLS][4]) {
    if (row >= N) return;
    const int jA = 8 * h + 2 * s;
#pragma unroll
    for (int c = 0; c < NCOLS; ++c) {
        int32_t *dst = P + ((static_cast<int64_t>(c) * N + row) * nsb + b) * 16;
        dst[jA] = v[c][0];
        dst[jA + 1] = v[c][1];
        dst[jA + 4] = v[c][2];
        dst[jA + 5] = v[c][3];
    }
}

template <int NCOLS, int KS, int NCW, int MODE, bool EMIT_P>
__global__ void __launch_bounds__((NCW + (MODE == Q6_DIRECT ? 0 : 1)) * 32, MODE == Q6_DIRECT && NCOLS <= 4 ? 2 : 1)
    mmvq_q6k_kernel(const Q6Params prm) {
    constexpr int NSL = 8 / KS;
    constexpr int NGRP = NCW / KS;
    constexpr bool STAGED = MODE != Q6_DIRECT;
    static_assert(NCW % KS == 0, "consumer warps must be a multiple of KS");
    static_assert(MODE != Q6_WHOLE || KS == 1, "whole-unit copies need KS == 1");
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ unsigned long long s_amax[NCOLS];
    const int N = prm.N, nsb = prm.nsb, nstage = prm.nstage, pitch = prm.pitch;
    const Q6Layout L = q6_layout(NCOLS, KS, NCW, nsb, nstage, prm.stage_bytes, STAGED);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L.off_full);
    uint64_t *empty = reinterpret_cast<uint64_t *>(smem + L.off_empty);
    float *red = reinterpret_cast<float *>(smem + L.off_red);
    uint8_t *aq = smem + L.off_qs;
    float *ad8 = reinterpret_cast<float *>(smem + L.off_d8);
    int *am = reinterpret_cast<int *>(smem + L.off_m);
    uint8_t *stage = smem + L.off_stage;
    const int64_t RB = static_cast<int64_t>(nsb) * Q6K_BYTES;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = gridDim.x;
    const int rg_begin = static_cast<int>(static_cast<int64_t>(blockIdx.x) * prm.rg_total / G);
    const int rg_end = static_cast<int>(static_cast<int64_t>(blockIdx.x + 1) * prm.rg_total / G);
    const int nrg = rg_end - rg_begin;

    if constexpr (STAGED) {
        if (threadIdx.x == 0) {
            for (int s = 0; s < nstage; ++s) {
                mbar_init(&full[s], 1);
                mbar_init(&empty[s], 1);
            }
            fence_mbar_init();
        }
        __syncthreads();
    }
    pdl_launch_dependents();

    if constexpr (STAGED) {
        if (warp == NCW) {
            // ------------------------------------------------ producer ---
            const uint64_t pol = policy_evict_first();
            const int U = nrg * KS;
            for (int u = 0; u < U; ++u) {
                if (u == nstage) prefetch_regions(prm.pf_ptr, prm.pf_bytes, lane);  // after the first ring fill
                const int s = u % nstage, k = u / nstage;
                if (k > 0 && !mbar_wait(&empty[s], (k - 1) & 1, ERR_WAIT_EMPTY)) break;
                const int rg = rg_begin + u / KS, j = u % KS;
                const int sb_lo = shard_slice(prm.sl_nsb, prm.sl_base, prm.sl_shift, j * NSL);
                const int sb_hi = shard_slice(prm.sl_nsb, prm.sl_base, prm.sl_shift, (j + 1) * NSL);
                const int row0 = rg * 8;
                const int nvalid = min(8, N - row0);
                uint8_t *dst = stage + s * prm.stage_bytes;
                int64_t start = 0, end = 0;
                uint32_t bulk = 0;
                if (sb_hi > sb_lo) {
                    if constexpr (MODE == Q6_WHOLE) {
                        start = row0 * RB;
                        end = (row0 + nvalid) * RB;
                        if (lane == 0) bulk = q6_tail_copy(dst, prm.W, start, end, prm.w_bytes);
                    } else if (lane < nvalid) {
                        start = (row0 + lane) * RB + static_cast<int64_t>(sb_lo) * Q6K_BYTES;
                        end = (row0 + lane) * RB + static_cast<int64_t>(sb_hi) * Q6K_BYTES;
                        bulk = q6_tail_copy(dst + lane * pitch, prm.W, start, end, prm.w_bytes);
                    }
                }
                uint32_t total = bulk;
#pragma unroll
                for (int m = 16; m >= 1; m >>= 1) total += __shfl_xor_sync(0xffffffffu, total, m);
                __syncwarp();  // the plain tail stores precede the arrival
                if (lane == 0) mbar_arrive_expect_tx(&full[s], total);
                __syncwarp();
                if (bulk > 0) {
                    uint8_t *d = MODE == Q6_WHOLE ? dst : dst + lane * pitch;
                    bulk_g2s(d, prm.W + (start & ~int64_t(15)), bulk, &full[s], pol);
                }
            }
            if (U <= nstage) prefetch_regions(prm.pf_ptr, prm.pf_bytes, lane);
            return;
        }
    }

    // -------------------------------------------------------- consumers ---
    pdl_wait();  // x is produced by the preceding kernel
    const int nblk = nsb * 8;
    for (int i = threadIdx.x; i < NCOLS * nblk; i += NCW * 32) {
        const uint32_t *src = reinterpret_cast<const uint32_t *>(prm.X + static_cast<int64_t>(i) * Q81_BYTES);
        const uint32_t hw = __ldg(src);
        uint32_t q[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) q[k] = __ldg(src + 1 + k);
        uint4 *dst = reinterpret_cast<uint4 *>(aq + static_cast<int64_t>(i) * 32);
        dst[0] = make_uint4(q[0], q[1], q[2], q[3]);
        dst[1] = make_uint4(q[4], q[5], q[6], q[7]);
        int m0 = 0, m1 = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            m0 = dp4a_ss(0x01010101, static_cast<int>(q[k]), m0);
            m1 = dp4a_ss(0x01010101, static_cast<int>(q[k + 4]), m1);
        }
        ad8[i] = half_lo(hw);
        *reinterpret_cast<int2 *>(am + 2 * i) = make_int2(m0, m1);
    }
    if (threadIdx.x < NCOLS) s_amax[threadIdx.x] = 0ull;
    named_bar_sync(1, NCW * 32);
    if constexpr (!STAGED) {
        if (warp == NCW - 1) prefetch_regions(prm.pf_ptr, prm.pf_bytes, lane);
    }

    const int grp = warp / KS, j = warp % KS;
    const int p = lane >> 3, g = lane & 7, h = p >> 1, s = p & 1;
    int bnd[NSL + 1];
#pragma unroll
    for (int i = 0; i <= NSL; ++i) bnd[i] = shard_slice(prm.sl_nsb, prm.sl_base, prm.sl_shift, j * NSL + i);
    const int sb_part = bnd[0];
    const int sb_part_end = bnd[NSL];
    bool poisoned = false;
    int round = 0;
    for (int r = grp; r < nrg; r += NGRP, ++round) {
        const int u = r * KS + j;
        const int st = u % nstage, k = u / nstage;
        const int row = (rg_begin + r) * 8 + g;
        const uint8_t *base;
        if constexpr (STAGED) {
            if (!poisoned && !mbar_wait(&full[st], k & 1)) poisoned = true;
            const int row0 = (rg_begin + r) * 8;
            if constexpr (MODE == Q6_WHOLE) {
                base = stage + st * prm.stage_bytes + static_cast<int64_t>(g) * RB;
            } else {
                const int64_t start = (row0 + g) * RB + static_cast<int64_t>(sb_part) * Q6K_BYTES;
                base = stage + st * prm.stage_bytes + g * pitch + (start & 15);
            }
            if constexpr (MODE == Q6_WHOLE) base += static_cast<int64_t>(sb_part) * Q6K_BYTES;
        } else {
            const int64_t rr = row < N ? row : N - 1;  // clamp: a tail lane reads a valid row
            base = prm.W + rr * RB + static_cast<int64_t>(sb_part) * Q6K_BYTES;
        }
        float acc[NCOLS][NSL];
        Q6Raw nxt;
        if constexpr (!STAGED) {
            if (sb_part < sb_part_end) q6_fetch<true>(base, h, s, nxt);
        }
#pragma unroll
        for (int i = 0; i < NSL; ++i) {
            const int b0 = bnd[i], b1 = bnd[i + 1];
#pragma unroll
            for (int c = 0; c < NCOLS; ++c) acc[c][i] = 0.0f;
            for (int b = b0; b < b1; ++b) {
                Q6Raw cur;
                if constexpr (STAGED) {
                    // rows past N read stage bytes nobody copied; their
                    // values are dropped below
                    q6_fetch<false>(base + (b - sb_part) * Q6K_BYTES, h, s, cur);
                } else {  // the next superblock loads while this one is valued
                    cur = nxt;
                    if (b + 1 < sb_part_end) q6_fetch<true>(base + (b + 1 - sb_part) * Q6K_BYTES, h, s, nxt);
                }
                float v[NCOLS];
                int P[NCOLS][4];
                q6_values<NCOLS>(cur, h, s, aq, ad8, am, nsb, b, v, P);
#pragma unroll
                for (int c = 0; c < NCOLS; ++c) acc[c][i] = (b == b0) ? v[c] : __fadd_rn(acc[c][i], v[c]);
                if constexpr (EMIT_P) q6_emit_p<NCOLS>(prm.P, N, nsb, row, b, h, s, P);
            }
        }
        if constexpr (STAGED) {
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[st]);
        }
        float sub[NCOLS];
#pragma unroll
        for (int c = 0; c < NCOLS; ++c) sub[c] = tree_sum<NSL>(acc[c]);
        if constexpr (KS > 1) {
            float *slot = red + ((round & 1) * NCW + warp) * 8 * NCOLS;
            if (p == 0) {
#pragma unroll
                for (int c = 0; c < NCOLS; ++c) slot[g * NCOLS + c] = sub[c];
            }
            named_bar_sync(2 + grp, KS * 32);
            if (j == 0 && p == 0) {
#pragma unroll
                for (int c = 0; c < NCOLS; ++c) {
                    float parts[KS];
#pragma unroll
                    for (int jj = 0; jj < KS; ++jj)
                        parts[jj] = red[((round & 1) * NCW + grp * KS + jj) * 8 * NCOLS + g * NCOLS + c];
                    sub[c] = tree_sum<KS>(parts);
                }
            }
        }
        if (j == 0 && p == 0) {
#pragma unroll
            for (int c = 0; c < NCOLS; ++c) {
                const float yv = sub[c];
                if (row < N) prm.Y[c * prm.ldy + row] = yv;
                if (prm.amax) {  // lanes 0..7 hold the unit's eight rows
                    unsigned long long key = row < N ? argmax_key(yv, row + prm.row_offset) : 0ull;
#pragma unroll
                    for (int m = 1; m < 8; m <<= 1) {
                        const unsigned long long o = __shfl_xor_sync(0x000000ffu, key, m);
                        key = o > key ? o : key;
                    }
                    if (g == 0) atomicMax(&s_amax[c], key);
                }
            }
        }
    }
    if (prm.amax) {
        named_bar_sync(1, NCW * 32);
        if (threadIdx.x < NCOLS) atomicMax(&prm.amax[threadIdx.x], s_amax[threadIdx.x]);
    }
}

using Q6Fn = void (*)(const Q6Params);

// [mode][ks index] for one batch width (whole: ks index 0 only), plus the
// EMIT_P variant (rows, KS 1).
struct Q6Table {
    Q6Fn fn[3][4];
    Q6Fn partials;
};

#define ABRA_Q6_NCW 8

template <int NC>
Q6Table make_q6_table() {
    Q6Table t = {};
    constexpr int W = ABRA_Q6_NCW;
    t.fn[Q6_ROWS][0] = mmvq_q6k_kernel<NC, 1, W, Q6_ROWS, false>;
    t.fn[Q6_ROWS][1] = mmvq_q6k_kernel<NC, 2, W, Q6_ROWS, false>;
    t.fn[Q6_ROWS][2] = mmvq_q6k_kernel<NC, 4, W, Q6_ROWS, false>;
    t.fn[Q6_ROWS][3] = mmvq_q6k_kernel<NC, 8, W, Q6_ROWS, false>;
    t.fn[Q6_WHOLE][0] = mmvq_q6k_kernel<NC, 1, W, Q6_WHOLE, false>;
    t.fn[Q6_DIRECT][0] = mmvq_q6k_kernel<NC, 1, W, Q6_DIRECT, false>;
    t.fn[Q6_DIRECT][1] = mmvq_q6k_kernel<NC, 2, W, Q6_DIRECT, false>;
    t.fn[Q6_DIRECT][2] = mmvq_q6k_kernel<NC, 4, W, Q6_DIRECT, false>;
    t.fn[Q6_DIRECT][3] = mmvq_q6k_kernel<NC, 8, W, Q6_DIRECT, false>;
    t.partials = mmvq_q6k_kernel<NC, 1, W, Q6_ROWS, true>;
    return t;
}

const Q6Table &q6_table_c1();
const Q6Table &q6_table_c2();
const Q6Table &q6_table_c3();
const Q6Table &q6_table_c4();
const Q6Table &q6_table_c5();
const Q6Table &q6_table_c6();
const Q6Table &q6_table_c7();
const Q6Table &q6_table_c8();

}  // namespace abra
