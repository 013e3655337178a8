// mmvq_impl.cuh -- the Q4_K x Q8_1 MMVQ kernel template (sm_100a).
//
// Computes y[c][r] = sum_k w[r][k] * x[c][k] for Q4_K rows w and Q8_1
// activation columns x -- the operation of the reference's
// vec_dot_q4_K_q8_1 / mul_mat_vec_q family (kernels/q4k/q4k_vecdot.cuh:23-87,
// kernels/q4k/q4k_family.cu:12-90) -- and, with NMAT == 2, the fused gate/up
// form y = (W_up x) * silu(W_gate x) of the reference's GATE kernel
// (kernels/q4k/abra-mmvq.cuh:118-143,175-186).
//
// Work unit: 8 rows x one k-part (KS k-parts per row).  Three ways to feed it:
//   MODE_TMA_ROWS   a producer warp fetches each unit with one cp.async.bulk per
//                   row into a ring of shared-memory stages (mbarrier-guarded);
//                   the row pitch is padded to an odd number of 16-byte chunks so
//                   eight rows' 128-bit loads hit eight distinct bank groups;
//   MODE_TMA_WHOLE  same ring, one bulk copy per unit (8 consecutive rows are
//                   contiguous in HBM when KS == 1), unpadded pitch;
//   MODE_DIRECT     no producer: consumer lanes load their superblock bytes
//                   with 128-bit ld.global.nc, one superblock ahead.
// No copy uses cluster multicast.
//
// Consumer lane (p = lane/8, g = lane%8) owns row g of the unit and nibble
// pair p (sub-blocks 2p, 2p+1): two exact int32 sub-block dot products by
// dp4a (the high nibbles as unsigned bytes masked in place, 16x the product).
// The eight lanes of a quarter warp share p, so activation loads broadcast.
//
// Canonical fp32 order (shared with the CPU oracle, bit for bit):
//   t_s = d8_s * float(P_s * sc_s),  u_s = (d8_s * float(M_s)) * float(m_s)
//   S   = ((t_0 + t_1) + (t_2 + t_3)) + ((t_4 + t_5) + (t_6 + t_7))  [xor 8, 16]
//   value(superblock) = fmaf(d, S_d, -(dmin * S_m))
//   eight canonical K-slices, sequential within a slice, then a fixed tree;
// k-parts are subtrees of that tree, so every candidate gives the same bits,
// and so does any split of K across GPUs along slice boundaries.
#pragma once

#include "common.cuh"

namespace abra {

// MODE_LANE (3) is the lane-mapped batch-1 kernel of mmvq_lane.cu, not this
// template; at other batch widths, and with a fused input or tensor-parallel
// options, its candidates run a plan of this template (mmvq_classic).
enum MmvqMode : int { MODE_TMA_ROWS = 0, MODE_TMA_WHOLE = 1, MODE_DIRECT = 2, MODE_LANE = 3 };

struct MmvqParams {
    const uint8_t *W[2];  // matrix 0 (gate when NMAT == 2), matrix 1 (up)
    const uint8_t *X;     // Q8_1 columns
    float *Y;
    int N, nsb;
    int64_t ldy;
    int rg_total, nstage, pitch;
    int32_t *P, *M;              // debug partials (EMIT_P)
    unsigned long long *amax;    // optional per-column argmax keys (argmax_key)
    // fp32 input with the residual add + RMSNorm + Q8_1 fused in (XIN):
    // x = h_in + tree(deltas), written to h_out by CTA 0; every CTA quantizes
    // (x * r) * norm_w in its own shared memory.
    const float *h_in;
    float *h_out;
    DeltaSet deltas;
    const float *norm_w;
    float eps;
    // K-shard slicing (sl_cnt in 1, 2, 4, 8): the shard holds global canonical
    // slices [sl_base, sl_base + sl_cnt) of rows of sl_nsb superblocks; they
    // sit at local slices 0, s, 2s, .. (stride s = 8 / sl_cnt) and the other
    // local slices are empty (+0.0), so the local tree is the shard's subtree
    // of the unsharded tree and every k-part gets real work (sl_nsb == nsb,
    // sl_base == 0, sl_cnt == 8 when K is not sharded).
    int sl_nsb, sl_base, sl_shift;  // sl_shift = log2(8 / sl_cnt)
    int row_offset;  // added to row ids in argmax keys (vocab shards)
    // Tensor-parallel push (npeer > 0): output rows go to peer_y[q] for every
    // rank q; each CTA then counts itself on cta_cnt (GPU scope, acq_rel), and
    // the launch's last CTA forwards this rank's argmax keys (amax, read and
    // reset) to peer_amax[q] and adds 1 to peer_cnt[q] with release
    // semantics at system scope.
    int npeer;
    float *peer_y[8];
    unsigned long long *peer_amax[8];
    unsigned long long *peer_cnt[8];
    unsigned long long *cta_cnt;
    // Tensor-parallel wait (fused input only): before reading the deltas,
    // *wait_cnt >= (*epoch + 1) * wait_per_step, bounded in time.
    const unsigned long long *wait_cnt;
    const unsigned long long *epoch;
    unsigned long long wait_per_step;
    // L2 prefetch of the next kernels' weights, split evenly over the CTAs
    const uint8_t *pf_ptr[2];
    int64_t pf_bytes[2];
    // fused input only: CTA 0 also stores the Q8_1 blocks it built (the
    // bytes the standalone quantizer would write), for a later MMVQ of
    // another weight type on the same activation
    uint8_t *x_out;
};

// This CTA's share of up to two L2 prefetch regions, issued by one warp in
// 16 KB pieces.
__device__ __forceinline__ void prefetch_regions(const uint8_t *const (&ptr)[2],
                                                 const int64_t (&bytes)[2], int lane) {
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int64_t units = bytes[r] >> 4;  // 16-byte units
        if (units <= 0) continue;
        const int64_t u0 = units * blockIdx.x / gridDim.x;
        const int64_t u1 = units * (blockIdx.x + 1) / gridDim.x;
        constexpr int64_t PIECE = 1024;  // 16 KB
        for (int64_t u = u0 + lane * PIECE; u < u1; u += 32 * PIECE) {
            const int64_t n = u1 - u < PIECE ? u1 - u : PIECE;
            prefetch_l2_bulk(ptr[r] + (u << 4), static_cast<uint32_t>(n << 4));
        }
    }
}

__device__ __forceinline__ void prefetch_share(const MmvqParams &prm, int lane) {
    prefetch_regions(prm.pf_ptr, prm.pf_bytes, lane);
}

// First superblock (relative to the shard) of local canonical slice i
// (0 <= i <= 8): the real slices before it are those at multiples of the
// stride 2^sl_shift below i.
__host__ __device__ __forceinline__ int shard_slice(int sl_nsb, int sl_base, int sl_shift, int i) {
    return slice_start(sl_nsb, sl_base + ((i + (1 << sl_shift) - 1) >> sl_shift)) -
           slice_start(sl_nsb, sl_base);
}

__host__ __device__ __forceinline__ int align_up(int v, int a) { return (v + a - 1) / a * a; }

struct MmvqLayout {
    int off_full, off_empty, off_red, off_qs, off_d8, off_A, off_x, off_stage, bytes;
};

__host__ __device__ __forceinline__ MmvqLayout mmvq_layout(int ncols, int ks, int ncw, int nsb,
                                                           int nstage, int pitch, int nmat,
                                                           bool staged, bool xin = false) {
    MmvqLayout L;
    L.off_full = 0;
    L.off_empty = 8 * nstage;
    int o = staged ? 16 * nstage : 0;
    L.off_red = align_up(o, 16);
    o = L.off_red + (ks > 1 ? 2 * ncw * 8 * ncols * nmat * 4 : 0);
    L.off_qs = align_up(o, 128);
    o = L.off_qs + ncols * nsb * 256;
    L.off_d8 = align_up(o, 16);
    o = L.off_d8 + ncols * nsb * 8 * 4;
    L.off_A = o;
    o += ncols * nsb * 8 * 4;
    L.off_x = align_up(o, 16);
    o = L.off_x + (xin ? 2 * nsb * 256 * 4 : 0);  // x and the norm weights (batch 1)
    L.off_stage = align_up(o, 128);
    L.bytes = L.off_stage + (staged ? nstage * 8 * nmat * pitch : 0);
    return L;
}

// Weight side of one superblock for lane pair p: scales, mins, nibbles.
struct SbWeights {
    float d, dmin, fm0, fm1;
    int sc0, sc1;
    uint32_t lo[8], hi[8];
};

struct SbRaw {
    uint4 hdr, qa, qb;
};

__device__ __forceinline__ void fetch_sb_smem(const uint8_t *sbp, int p, SbRaw &r) {
    r.hdr = *reinterpret_cast<const uint4 *>(sbp);
    r.qa = *reinterpret_cast<const uint4 *>(sbp + 16 + 32 * p);
    r.qb = *reinterpret_cast<const uint4 *>(sbp + 32 + 32 * p);
}

__device__ __forceinline__ uint4 ldg_nc_v4(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ void fetch_sb_global(const uint8_t *sbp, int p, SbRaw &r) {
    r.hdr = ldg_nc_v4(sbp);
    r.qa = ldg_nc_v4(sbp + 16 + 32 * p);
    r.qb = ldg_nc_v4(sbp + 32 + 32 * p);
}

__device__ __forceinline__ void decode_sb(const SbRaw &r, int p, SbWeights &w) {
    int m0, m1;
    scale_min_pair(r.hdr.y, r.hdr.z, r.hdr.w, p, w.sc0, m0, w.sc1, m1);
    w.d = half_lo(r.hdr.x);
    w.dmin = half_hi(r.hdr.x);
    w.fm0 = static_cast<float>(m0);
    w.fm1 = static_cast<float>(m1);
    const uint32_t qw[8] = {r.qa.x, r.qa.y, r.qa.z, r.qa.w, r.qb.x, r.qb.y, r.qb.z, r.qb.w};
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        w.lo[k] = qw[k] & 0x0F0F0F0Fu;
        w.hi[k] = qw[k] & 0xF0F0F0F0u;
    }
}

// Values of one superblock for every column and each of NMAT matrices that
// share the activation; aq/ad8/aA point at the staged activation.
template <int NCOLS, int NMAT>
__device__ __forceinline__ void sb_values(const SbWeights (&w)[NMAT], int p, const uint8_t *aq,
                                          const float *ad8, const float *aA, int nsb, int b,
                                          float (&v)[NMAT][NCOLS], int (&P0)[NCOLS],
                                          int (&P1)[NCOLS]) {
#pragma unroll
    for (int c = 0; c < NCOLS; ++c) {
        const uint4 *a = reinterpret_cast<const uint4 *>(aq + (c * nsb + b) * 256 + 64 * p);
        const uint4 a0 = a[0], a1 = a[1], a2 = a[2], a3 = a[3];
        const float2 d8 = *reinterpret_cast<const float2 *>(ad8 + (c * nsb + b) * 8 + 2 * p);
        const float2 A = *reinterpret_cast<const float2 *>(aA + (c * nsb + b) * 8 + 2 * p);
#pragma unroll
        for (int m = 0; m < NMAT; ++m) {
            const uint32_t *lo = w[m].lo, *hi = w[m].hi;
            int s0 = 0, s1 = 0;
            s0 = dp4a_ss(lo[0], a0.x, s0);
            s0 = dp4a_ss(lo[1], a0.y, s0);
            s0 = dp4a_ss(lo[2], a0.z, s0);
            s0 = dp4a_ss(lo[3], a0.w, s0);
            s0 = dp4a_ss(lo[4], a1.x, s0);
            s0 = dp4a_ss(lo[5], a1.y, s0);
            s0 = dp4a_ss(lo[6], a1.z, s0);
            s0 = dp4a_ss(lo[7], a1.w, s0);
            s1 = dp4a_us(hi[0], a2.x, s1);
            s1 = dp4a_us(hi[1], a2.y, s1);
            s1 = dp4a_us(hi[2], a2.z, s1);
            s1 = dp4a_us(hi[3], a2.w, s1);
            s1 = dp4a_us(hi[4], a3.x, s1);
            s1 = dp4a_us(hi[5], a3.y, s1);
            s1 = dp4a_us(hi[6], a3.z, s1);
            s1 = dp4a_us(hi[7], a3.w, s1);
            s1 >>= 4;  // exact: the masked high nibbles carry a factor of 16
            if (m == 0) {
                P0[c] = s0;
                P1[c] = s1;
            }
            const float t0 = __fmul_rn(d8.x, __int2float_rn(s0 * w[m].sc0));
            const float t1 = __fmul_rn(d8.y, __int2float_rn(s1 * w[m].sc1));
            float tp = __fadd_rn(t0, t1);
            float up = __fadd_rn(__fmul_rn(A.x, w[m].fm0), __fmul_rn(A.y, w[m].fm1));
            tp = __fadd_rn(tp, __shfl_xor_sync(0xffffffffu, tp, 8));
            up = __fadd_rn(up, __shfl_xor_sync(0xffffffffu, up, 8));
            tp = __fadd_rn(tp, __shfl_xor_sync(0xffffffffu, tp, 16));
            up = __fadd_rn(up, __shfl_xor_sync(0xffffffffu, up, 16));
            v[m][c] = __fmaf_rn(w[m].d, tp, -__fmul_rn(w[m].dmin, up));
        }
    }
}

template <int N>
__device__ __forceinline__ float tree_sum(const float *a) {
    if constexpr (N == 1) {
        return a[0];
    } else if constexpr (N == 2) {
        return __fadd_rn(a[0], a[1]);
    } else if constexpr (N == 4) {
        return __fadd_rn(__fadd_rn(a[0], a[1]), __fadd_rn(a[2], a[3]));
    } else {
        return __fadd_rn(__fadd_rn(__fadd_rn(a[0], a[1]), __fadd_rn(a[2], a[3])),
                         __fadd_rn(__fadd_rn(a[4], a[5]), __fadd_rn(a[6], a[7])));
    }
}

template <int NCOLS, int KS, int NCW, int MODE, int NMAT, bool EMIT_P, bool XIN = false>
__global__ void __launch_bounds__((NCW + (MODE == MODE_DIRECT ? 0 : 1)) * 32, MODE == MODE_DIRECT ? 2 : 1)
    mmvq_q4k_kernel(const MmvqParams prm) {
    constexpr int NSL = 8 / KS;     // canonical slices per k-part
    constexpr int NGRP = NCW / KS;  // warp groups, one row group each at a time
    constexpr bool STAGED = MODE != MODE_DIRECT;
    static_assert(NCW % KS == 0, "consumer warps must be a multiple of KS");
    static_assert(MODE != MODE_TMA_WHOLE || KS == 1, "whole-unit copies need KS == 1");
    static_assert(!XIN || NCW * 32 == 256, "the fused RMSNorm uses the canonical 256 lanes");
    static_assert(!XIN || NCOLS == 1, "the fused RMSNorm input is batch 1");
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ unsigned long long s_amax[NCOLS];
    __shared__ float s_nred[1][8];
    const int N = prm.N, nsb = prm.nsb, nstage = prm.nstage, pitch = prm.pitch;
    const MmvqLayout L = mmvq_layout(NCOLS, KS, NCW, nsb, nstage, pitch, NMAT, STAGED, XIN);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L.off_full);
    uint64_t *empty = reinterpret_cast<uint64_t *>(smem + L.off_empty);
    float *red = reinterpret_cast<float *>(smem + L.off_red);
    uint8_t *aq = smem + L.off_qs;
    float *ad8 = reinterpret_cast<float *>(smem + L.off_d8);
    float *aA = reinterpret_cast<float *>(smem + L.off_A);
    uint8_t *stage = smem + L.off_stage;

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
                if (u == nstage) prefetch_share(prm, lane);  // after the first ring fill
                const int s = u % nstage, k = u / nstage;
                if (k > 0 && !mbar_wait(&empty[s], (k - 1) & 1, ERR_WAIT_EMPTY)) break;
                const int rg = rg_begin + u / KS, j = u % KS;
                const int sb_lo = shard_slice(prm.sl_nsb, prm.sl_base, prm.sl_shift, j * NSL);
                const int sb_hi = shard_slice(prm.sl_nsb, prm.sl_base, prm.sl_shift, (j + 1) * NSL);
                const uint32_t part_bytes = static_cast<uint32_t>(sb_hi - sb_lo) * Q4K_BYTES;
                const int row0 = rg * 8;
                const int nvalid = min(8, N - row0);
                if (lane == 0) mbar_arrive_expect_tx(&full[s], NMAT * nvalid * part_bytes);
                __syncwarp();
                if (part_bytes > 0) {
#pragma unroll
                    for (int m = 0; m < NMAT; ++m) {
                        uint8_t *dst = stage + (s * NMAT + m) * 8 * pitch;
                        if constexpr (MODE == MODE_TMA_WHOLE) {
                            if (lane == 0)
                                bulk_g2s(dst, prm.W[m] + static_cast<int64_t>(row0) * nsb * Q4K_BYTES,
                                         nvalid * part_bytes, &full[s], pol);
                        } else {
                            if (lane < nvalid)
                                bulk_g2s(dst + lane * pitch,
                                         prm.W[m] + (static_cast<int64_t>(row0 + lane) * nsb + sb_lo) *
                                                        Q4K_BYTES,
                                         part_bytes, &full[s], pol);
                        }
                    }
                }
            }
            if (U <= nstage) prefetch_share(prm, lane);
            return;
        }
    }

    // -------------------------------------------------------- consumers ---
    const int nblk = nsb * 8;
    if constexpr (XIN) {
        // the norm weights are immutable: stage them before waiting on the
        // kernel that produced the residual stream
        const int K = nsb * QK_K;
        float *s_w = reinterpret_cast<float *>(smem + L.off_x) + K;
        for (int i = threadIdx.x * 4; i < K; i += NCW * 32 * 4)
            *reinterpret_cast<float4 *>(s_w + i) = __ldg(reinterpret_cast<const float4 *>(prm.norm_w + i));
    }
    pdl_wait();  // x is produced by the preceding kernel
    if constexpr (XIN) {
        if (prm.wait_cnt) {  // the other ranks' partial sums have arrived
            if (threadIdx.x == 0)
                wait_count(prm.wait_cnt, (__ldcg(prm.epoch) + 1ull) * prm.wait_per_step);
            named_bar_sync(1, NCW * 32);
        }
    }
    if constexpr (XIN) {
        // residual add + RMSNorm + Q8_1 of the fp32 input, in this CTA's shared
        // memory, in the canonical order: thread t sums x[t + 256 k]^2 with
        // fmaf in k order, xor butterfly 16..1, the eight warp sums in order;
        // r = 1 / sqrt(sum / K + eps); then (x * r) * w and the reference Q8_1
        // rounding per 32-block.  Loads are issued eight at a time.
        const int K = nsb * QK_K;
        float *s_x = reinterpret_cast<float *>(smem + L.off_x);
        const float *s_w = s_x + K;
        const int t = threadIdx.x;
        float acc = 0.0f;
        for (int i0 = t; i0 < K; i0 += 256 * 8) {
            float v[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const int i = i0 + k * 256;
                v[k] = i < K ? prm.h_in[i] : 0.0f;
            }
            if (prm.deltas.G > 0) {
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const int i = i0 + k * 256;
                    if (i < K) v[k] = __fadd_rn(v[k], delta_tree(prm.deltas, i));
                }
            }
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const int i = i0 + k * 256;
                if (i < K) {
                    if (blockIdx.x == 0 && prm.h_out) prm.h_out[i] = v[k];
                    s_x[i] = v[k];
                    acc = __fmaf_rn(v[k], v[k], acc);
                }
            }
        }
#pragma unroll
        for (int m = 16; m >= 1; m >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, m));
        if (lane == 0) s_nred[0][warp] = acc;
        named_bar_sync(1, NCW * 32);
        float total = s_nred[0][0];
#pragma unroll
        for (int w = 1; w < 8; ++w) total = __fadd_rn(total, s_nred[0][w]);
        const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(total, static_cast<float>(K)), prm.eps)));
        // eight lanes per 32-block, four elements each; a warp covers four
        // consecutive blocks (nblk is a multiple of 8, so all four exist)
        const int sub = lane & 7;
        for (int b0 = warp * 4; b0 < nblk; b0 += NCW * 4) {
            const int i = b0 + (lane >> 3);
            const float4 xv = *reinterpret_cast<const float4 *>(s_x + i * QK8_1 + sub * 4);
            const float4 wv = *reinterpret_cast<const float4 *>(s_w + i * QK8_1 + sub * 4);
            const float x0 = __fmul_rn(__fmul_rn(xv.x, r), wv.x);
            const float x1 = __fmul_rn(__fmul_rn(xv.y, r), wv.y);
            const float x2 = __fmul_rn(__fmul_rn(xv.z, r), wv.z);
            const float x3 = __fmul_rn(__fmul_rn(xv.w, r), wv.w);
            float amax = fmaxf(fmaxf(fabsf(x0), fabsf(x1)), fmaxf(fabsf(x2), fabsf(x3)));
            amax = fmaxf(0.0f, amax);
#pragma unroll
            for (int m = 4; m >= 1; m >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, m));
            const float d = __fdiv_rn(amax, 127.0f);
            const float id = d > 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
            const int q0 = static_cast<int>(static_cast<int8_t>(static_cast<int>(roundf(__fmul_rn(x0, id)))));
            const int q1 = static_cast<int>(static_cast<int8_t>(static_cast<int>(roundf(__fmul_rn(x1, id)))));
            const int q2 = static_cast<int>(static_cast<int8_t>(static_cast<int>(roundf(__fmul_rn(x2, id)))));
            const int q3 = static_cast<int>(static_cast<int8_t>(static_cast<int>(roundf(__fmul_rn(x3, id)))));
            int sum = (q0 + q1) + (q2 + q3);
#pragma unroll
            for (int m = 4; m >= 1; m >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, m);
            const uint32_t packed = (static_cast<uint32_t>(q0) & 0xffu) |
                                    ((static_cast<uint32_t>(q1) & 0xffu) << 8) |
                                    ((static_cast<uint32_t>(q2) & 0xffu) << 16) |
                                    (static_cast<uint32_t>(q3) << 24);
            *reinterpret_cast<uint32_t *>(aq + i * 32 + sub * 4) = packed;
            if (sub == 0) {
                const float d8 = __half2float(__float2half_rn(d));
                ad8[i] = d8;
                aA[i] = __fmul_rn(d8, __int2float_rn(sum));
            }
            if (blockIdx.x == 0 && prm.x_out) {  // d, s = d * sum as fp16, then the 32 int8
                uint8_t *blk = prm.x_out + static_cast<int64_t>(i) * Q81_BYTES;
                *reinterpret_cast<uint32_t *>(blk + 4 + sub * 4) = packed;
                if (sub == 0)
                    *reinterpret_cast<uint32_t *>(blk) =
                        static_cast<uint32_t>(__half_as_ushort(__float2half_rn(d))) |
                        (static_cast<uint32_t>(__half_as_ushort(
                             __float2half_rn(__fmul_rn(d, __int2float_rn(sum))))) << 16);
            }
        }
    }
    for (int i = threadIdx.x; i < (XIN ? 0 : NCOLS * nblk); i += NCW * 32) {
        const int c = i / nblk, blk = i - c * nblk;
        const uint32_t *src = reinterpret_cast<const uint32_t *>(
            prm.X + (static_cast<int64_t>(c) * nblk + blk) * Q81_BYTES);
        const uint32_t h = __ldg(src);
        uint32_t q[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) q[k] = __ldg(src + 1 + k);
        uint4 *dst = reinterpret_cast<uint4 *>(aq + static_cast<int64_t>(i) * 32);
        dst[0] = make_uint4(q[0], q[1], q[2], q[3]);
        dst[1] = make_uint4(q[4], q[5], q[6], q[7]);
        int msum = 0;
#pragma unroll
        for (int k = 0; k < 8; ++k) msum = dp4a_ss(0x01010101, static_cast<int>(q[k]), msum);
        const float d8 = half_lo(h);
        ad8[i] = d8;
        aA[i] = __fmul_rn(d8, __int2float_rn(msum));  // exact: 11 x 12 bits
        if constexpr (EMIT_P) {
            if (blockIdx.x == 0) prm.M[i] = msum;
        }
    }
    if (threadIdx.x < NCOLS) s_amax[threadIdx.x] = 0ull;
    named_bar_sync(1, NCW * 32);
    if constexpr (!STAGED) {
        if (warp == NCW - 1) prefetch_share(prm, lane);
    }

    const int grp = warp / KS, j = warp % KS;
    const int p = lane >> 3, g = lane & 7;
    // this warp's slice bounds, once: superblocks [bnd[i], bnd[i+1]) of local
    // slice j*NSL + i, relative to the row (or shard) start
    int bnd[NSL + 1];
#pragma unroll
    for (int i = 0; i <= NSL; ++i) bnd[i] = shard_slice(prm.sl_nsb, prm.sl_base, prm.sl_shift, j * NSL + i);
    const int sb_part = bnd[0];
    const int sb_part_end = bnd[NSL];
    bool poisoned = false;
    int round = 0;
    for (int r = grp; r < nrg; r += NGRP, ++round) {
        const int u = r * KS + j;
        const int s = u % nstage, k = u / nstage;
        const int row = (rg_begin + r) * 8 + g;
        const uint8_t *base[NMAT];
        if constexpr (STAGED) {
            if (!poisoned && !mbar_wait(&full[s], k & 1)) poisoned = true;
#pragma unroll
            for (int m = 0; m < NMAT; ++m) base[m] = stage + ((s * NMAT + m) * 8 + g) * pitch;
        } else {
            const int64_t rr = row < N ? row : N - 1;  // clamp: a tail lane reads a valid row
#pragma unroll
            for (int m = 0; m < NMAT; ++m) base[m] = prm.W[m] + (rr * nsb + sb_part) * Q4K_BYTES;
        }
        float acc[NMAT][NCOLS][NSL];
        SbRaw nxt[NMAT];
        if constexpr (!STAGED) {
            if (sb_part < sb_part_end) {
#pragma unroll
                for (int m = 0; m < NMAT; ++m) fetch_sb_global(base[m], p, nxt[m]);
            }
        }
#pragma unroll
        for (int i = 0; i < NSL; ++i) {
            const int b0 = bnd[i], b1 = bnd[i + 1];
#pragma unroll
            for (int m = 0; m < NMAT; ++m)
#pragma unroll
                for (int c = 0; c < NCOLS; ++c) acc[m][c][i] = 0.0f;
            for (int b = b0; b < b1; ++b) {
                SbWeights w[NMAT];
                if constexpr (STAGED) {
#pragma unroll
                    for (int m = 0; m < NMAT; ++m) {
                        SbRaw raw;
                        fetch_sb_smem(base[m] + (b - sb_part) * Q4K_BYTES, p, raw);
                        decode_sb(raw, p, w[m]);
                    }
                } else {
                    SbRaw cur[NMAT];
#pragma unroll
                    for (int m = 0; m < NMAT; ++m) cur[m] = nxt[m];
                    if (b + 1 < sb_part_end) {
#pragma unroll
                        for (int m = 0; m < NMAT; ++m)
                            fetch_sb_global(base[m] + (b + 1 - sb_part) * Q4K_BYTES, p, nxt[m]);
                    }
#pragma unroll
                    for (int m = 0; m < NMAT; ++m) decode_sb(cur[m], p, w[m]);
                }
                float v[NMAT][NCOLS];
                int P0[NCOLS], P1[NCOLS];
                sb_values<NCOLS, NMAT>(w, p, aq, ad8, aA, nsb, b, v, P0, P1);
#pragma unroll
                for (int m = 0; m < NMAT; ++m)
#pragma unroll
                    for (int c = 0; c < NCOLS; ++c)
                        acc[m][c][i] = (b == b0) ? v[m][c] : __fadd_rn(acc[m][c][i], v[m][c]);
                if constexpr (EMIT_P) {
                    if (row < N) {
#pragma unroll
                        for (int c = 0; c < NCOLS; ++c) {
                            int32_t *dst = prm.P + ((static_cast<int64_t>(c) * N + row) * nsb + b) * 8 + 2 * p;
                            dst[0] = P0[c];
                            dst[1] = P1[c];
                        }
                    }
                }
            }
        }
        if constexpr (STAGED) {
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        float sub[NMAT][NCOLS];
#pragma unroll
        for (int m = 0; m < NMAT; ++m)
#pragma unroll
            for (int c = 0; c < NCOLS; ++c) sub[m][c] = tree_sum<NSL>(acc[m][c]);
        if constexpr (KS > 1) {
            float *slot = red + ((round & 1) * NCW + warp) * 8 * NCOLS * NMAT;
            if (p == 0) {
#pragma unroll
                for (int m = 0; m < NMAT; ++m)
#pragma unroll
                    for (int c = 0; c < NCOLS; ++c) slot[(g * NMAT + m) * NCOLS + c] = sub[m][c];
            }
            named_bar_sync(2 + grp, KS * 32);
            if (j == 0 && p == 0) {
#pragma unroll
                for (int m = 0; m < NMAT; ++m)
#pragma unroll
                    for (int c = 0; c < NCOLS; ++c) {
                        float parts[KS];
#pragma unroll
                        for (int jj = 0; jj < KS; ++jj)
                            parts[jj] = red[((round & 1) * NCW + grp * KS + jj) * 8 * NCOLS * NMAT +
                                            (g * NMAT + m) * NCOLS + c];
                        sub[m][c] = tree_sum<KS>(parts);
                    }
            }
        }
        if (j == 0 && p == 0) {
#pragma unroll
            for (int c = 0; c < NCOLS; ++c) {
                float yv = sub[0][c];
                if constexpr (NMAT == 2) yv = __fmul_rn(sub[1][c], abra_silu(sub[0][c]));
                if (row < N) {
                    if (prm.npeer > 0 && prm.peer_y[0]) {  // push the partial to every rank
                        for (int q = 0; q < prm.npeer; ++q) prm.peer_y[q][c * prm.ldy + row] = yv;
                    } else {
                        prm.Y[c * prm.ldy + row] = yv;
                    }
                }
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
    if (prm.npeer > 0) {
        // every consumer's stores are done: count this CTA on this GPU; the
        // last CTA of the launch publishes the whole launch to each rank
        named_bar_sync(1, NCW * 32);
        if (threadIdx.x == 0) {
            if (prm.amax)
                for (int c = 0; c < NCOLS; ++c) atomicMax(&prm.amax[c], s_amax[c]);
            const unsigned long long old = atom_add_acq_rel_gpu(prm.cta_cnt, 1ull);
            if ((old + 1ull) % gridDim.x == 0ull) {
                if (prm.amax && prm.peer_amax[0]) {
                    for (int c = 0; c < NCOLS; ++c) {
                        const unsigned long long key = atomicExch(&prm.amax[c], 0ull);
                        for (int q = 0; q < prm.npeer; ++q) atomicMax_system(prm.peer_amax[q] + c, key);
                    }
                }
                // release at system scope: every store this launch made
                // (ordered before this point by the acq_rel count) is visible
                // to a rank that acquires the arrival
                for (int q = 0; q < prm.npeer; ++q) red_release_sys_add(prm.peer_cnt[q], 1ull);
            }
        }
    } else if (prm.amax) {
        named_bar_sync(1, NCW * 32);
        if (threadIdx.x < NCOLS) atomicMax(&prm.amax[threadIdx.x], s_amax[threadIdx.x]);
    }
}

using MmvqFn = void (*)(const MmvqParams);

// Kernel table for one batch width: index [mode][ks index][nmat-1].
// ks index: 0 -> 1, 1 -> 2, 2 -> 4, 3 -> 8.
struct MmvqTable {
    MmvqFn fn[3][4][2];
    MmvqFn partials[3];  // MODE_TMA_ROWS, NMAT 1, KS 1/2/4, EMIT_P
    MmvqFn xin[3][4][2]; // fused residual + RMSNorm + Q8_1 input (batch 1 only)
};

#define ABRA_MMVQ_NCW 8

template <int NC>
MmvqTable make_mmvq_table() {
    MmvqTable t = {};
    constexpr int W = ABRA_MMVQ_NCW;
    t.fn[MODE_TMA_ROWS][0][0] = mmvq_q4k_kernel<NC, 1, W, MODE_TMA_ROWS, 1, false>;
    t.fn[MODE_TMA_ROWS][1][0] = mmvq_q4k_kernel<NC, 2, W, MODE_TMA_ROWS, 1, false>;
    t.fn[MODE_TMA_ROWS][2][0] = mmvq_q4k_kernel<NC, 4, W, MODE_TMA_ROWS, 1, false>;
    t.fn[MODE_TMA_ROWS][3][0] = mmvq_q4k_kernel<NC, 8, W, MODE_TMA_ROWS, 1, false>;
    t.fn[MODE_TMA_ROWS][0][1] = mmvq_q4k_kernel<NC, 1, W, MODE_TMA_ROWS, 2, false>;
    t.fn[MODE_TMA_ROWS][1][1] = mmvq_q4k_kernel<NC, 2, W, MODE_TMA_ROWS, 2, false>;
    t.fn[MODE_TMA_ROWS][2][1] = mmvq_q4k_kernel<NC, 4, W, MODE_TMA_ROWS, 2, false>;
    t.fn[MODE_TMA_ROWS][3][1] = mmvq_q4k_kernel<NC, 8, W, MODE_TMA_ROWS, 2, false>;
    t.fn[MODE_TMA_WHOLE][0][0] = mmvq_q4k_kernel<NC, 1, W, MODE_TMA_WHOLE, 1, false>;
    t.fn[MODE_TMA_WHOLE][0][1] = mmvq_q4k_kernel<NC, 1, W, MODE_TMA_WHOLE, 2, false>;
    t.fn[MODE_DIRECT][0][0] = mmvq_q4k_kernel<NC, 1, W, MODE_DIRECT, 1, false>;
    t.fn[MODE_DIRECT][1][0] = mmvq_q4k_kernel<NC, 2, W, MODE_DIRECT, 1, false>;
    t.fn[MODE_DIRECT][2][0] = mmvq_q4k_kernel<NC, 4, W, MODE_DIRECT, 1, false>;
    t.fn[MODE_DIRECT][3][0] = mmvq_q4k_kernel<NC, 8, W, MODE_DIRECT, 1, false>;
    t.fn[MODE_DIRECT][0][1] = mmvq_q4k_kernel<NC, 1, W, MODE_DIRECT, 2, false>;
    t.fn[MODE_DIRECT][1][1] = mmvq_q4k_kernel<NC, 2, W, MODE_DIRECT, 2, false>;
    t.fn[MODE_DIRECT][2][1] = mmvq_q4k_kernel<NC, 4, W, MODE_DIRECT, 2, false>;
    t.fn[MODE_DIRECT][3][1] = mmvq_q4k_kernel<NC, 8, W, MODE_DIRECT, 2, false>;
    if constexpr (NC == 1 || NC == 2 || NC == 4 || NC == 8) {
        t.partials[0] = mmvq_q4k_kernel<NC, 1, W, MODE_TMA_ROWS, 1, true>;
        t.partials[1] = mmvq_q4k_kernel<NC, 2, W, MODE_TMA_ROWS, 1, true>;
        t.partials[2] = mmvq_q4k_kernel<NC, 4, W, MODE_TMA_ROWS, 1, true>;
    }
    if constexpr (NC == 1) {
        t.xin[MODE_TMA_ROWS][0][0] = mmvq_q4k_kernel<NC, 1, W, MODE_TMA_ROWS, 1, false, true>;
        t.xin[MODE_TMA_ROWS][1][0] = mmvq_q4k_kernel<NC, 2, W, MODE_TMA_ROWS, 1, false, true>;
        t.xin[MODE_TMA_ROWS][2][0] = mmvq_q4k_kernel<NC, 4, W, MODE_TMA_ROWS, 1, false, true>;
        t.xin[MODE_TMA_ROWS][3][0] = mmvq_q4k_kernel<NC, 8, W, MODE_TMA_ROWS, 1, false, true>;
        t.xin[MODE_TMA_ROWS][0][1] = mmvq_q4k_kernel<NC, 1, W, MODE_TMA_ROWS, 2, false, true>;
        t.xin[MODE_TMA_ROWS][1][1] = mmvq_q4k_kernel<NC, 2, W, MODE_TMA_ROWS, 2, false, true>;
        t.xin[MODE_TMA_ROWS][2][1] = mmvq_q4k_kernel<NC, 4, W, MODE_TMA_ROWS, 2, false, true>;
        t.xin[MODE_TMA_ROWS][3][1] = mmvq_q4k_kernel<NC, 8, W, MODE_TMA_ROWS, 2, false, true>;
        t.xin[MODE_TMA_WHOLE][0][0] = mmvq_q4k_kernel<NC, 1, W, MODE_TMA_WHOLE, 1, false, true>;
        t.xin[MODE_TMA_WHOLE][0][1] = mmvq_q4k_kernel<NC, 1, W, MODE_TMA_WHOLE, 2, false, true>;
        t.xin[MODE_DIRECT][0][0] = mmvq_q4k_kernel<NC, 1, W, MODE_DIRECT, 1, false, true>;
        t.xin[MODE_DIRECT][1][0] = mmvq_q4k_kernel<NC, 2, W, MODE_DIRECT, 1, false, true>;
        t.xin[MODE_DIRECT][2][0] = mmvq_q4k_kernel<NC, 4, W, MODE_DIRECT, 1, false, true>;
        t.xin[MODE_DIRECT][3][0] = mmvq_q4k_kernel<NC, 8, W, MODE_DIRECT, 1, false, true>;
        t.xin[MODE_DIRECT][0][1] = mmvq_q4k_kernel<NC, 1, W, MODE_DIRECT, 2, false, true>;
        t.xin[MODE_DIRECT][1][1] = mmvq_q4k_kernel<NC, 2, W, MODE_DIRECT, 2, false, true>;
        t.xin[MODE_DIRECT][2][1] = mmvq_q4k_kernel<NC, 4, W, MODE_DIRECT, 2, false, true>;
        t.xin[MODE_DIRECT][3][1] = mmvq_q4k_kernel<NC, 8, W, MODE_DIRECT, 2, false, true>;
    }
    return t;
}

// Defined in mmvq_c<N>.cu, one translation unit per batch width.
const MmvqTable &mmvq_table_c1();
const MmvqTable &mmvq_table_c2();
const MmvqTable &mmvq_table_c3();
const MmvqTable &mmvq_table_c4();
const MmvqTable &mmvq_table_c5();
const MmvqTable &mmvq_table_c6();
const MmvqTable &mmvq_table_c7();
const MmvqTable &mmvq_table_c8();

}  // namespace abra
