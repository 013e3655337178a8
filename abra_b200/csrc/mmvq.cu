// mmvq.cu -- Q4_K x Q8_1 matrix-vector product (MMVQ) for sm_100a.
//
// Computes y[c][r] = sum_k w[r][k] * x[c][k] for Q4_K rows w and Q8_1
// activation columns x, the operation of the reference's
// vec_dot_q4_K_q8_1 / mul_mat_vec_q family (kernels/q4k/q4k_vecdot.cuh:23-87,
// kernels/q4k/q4k_family.cu:12-90).
//
// Design (B200):
//   * Weights stream through shared memory.  Rows of one superblock row are
//     contiguous in HBM, so a unit of work -- 8 rows x one k-part -- is fetched
//     with eight cp.async.bulk copies (no multicast) issued by a producer warp
//     into a ring of stages, each guarded by an mbarrier with a byte count.
//     The row pitch in shared memory is padded to an odd number of 16-byte
//     chunks, so the 128-bit loads of eight rows hit eight distinct bank groups.
//   * Consumer lane (p = lane/8, g = lane%8) owns row g of the unit and nibble
//     pair p (sub-blocks 2p and 2p+1) of each superblock: it loads 32 nibble
//     bytes and 64 activation bytes and forms the two exact int32 sub-block
//     dot products with dp4a (the high nibbles as unsigned bytes masked in
//     place, giving 16x the product).  The eight lanes of a quarter warp share
//     p, so every activation load is a broadcast.
//   * fp32 evaluation follows one canonical order, shared with the CPU oracle:
//       t_s = d8_s * float(P_s * sc_s),  u_s = (d8_s * float(M_s)) * float(m_s)
//       S   = ((t_0 + t_1) + (t_2 + t_3)) + ((t_4 + t_5) + (t_6 + t_7))   [xor 8, xor 16]
//       value(superblock) = fmaf(d, S_d, -(dmin * S_m))
//       eight canonical K-slices, sequential within a slice, then a fixed tree.
//     k-parts (KS of them) are subtrees of that tree, so any KS gives the same
//     bits; so does any split of K across GPUs along slice boundaries.
//   * Activations are staged once per CTA into shared memory together with
//     d8 and d8*M per sub-block (M = sum of the 32 int8, computed once per
//     activation, never per row).
//   * Programmatic dependent launch (optional): the producer prefetches
//     weights before griddepcontrol.wait; consumers wait before reading x.
#include <cstdio>
#include <mutex>

#include "common.cuh"
#include "kernels.cuh"

namespace abra {

__host__ __device__ __forceinline__ int align_up(int v, int a) { return (v + a - 1) / a * a; }

struct MmvqLayout {
    int off_full, off_empty, off_red, off_qs, off_d8, off_A, off_stage, bytes;
};

__host__ __device__ __forceinline__ MmvqLayout mmvq_layout(int ncols, int ks, int ncw, int nsb,
                                                           int nstage, int pitch) {
    MmvqLayout L;
    L.off_full = 0;
    L.off_empty = 8 * nstage;
    int o = 16 * nstage;
    L.off_red = align_up(o, 16);
    o = L.off_red + (ks > 1 ? 2 * ncw * 8 * ncols * 4 : 0);
    L.off_qs = align_up(o, 128);
    o = L.off_qs + ncols * nsb * 256;
    L.off_d8 = align_up(o, 16);
    o = L.off_d8 + ncols * nsb * 8 * 4;
    L.off_A = o;
    o += ncols * nsb * 8 * 4;
    L.off_stage = align_up(o, 128);
    L.bytes = L.off_stage + nstage * 8 * pitch;
    return L;
}

// Values of one superblock for every column.  sbp points at the superblock
// in shared memory; aq/ad8/aA at the staged activation of column 0.
template <int NCOLS>
__device__ __forceinline__ void sb_values(const uint8_t *sbp, int p, const uint8_t *aq,
                                          const float *ad8, const float *aA, int nsb, int b,
                                          float (&v)[NCOLS], int (&P0)[NCOLS],
                                          int (&P1)[NCOLS]) {
    const uint4 hdr = *reinterpret_cast<const uint4 *>(sbp);
    const uint4 qa = *reinterpret_cast<const uint4 *>(sbp + 16 + 32 * p);
    const uint4 qb = *reinterpret_cast<const uint4 *>(sbp + 32 + 32 * p);
    int sc0, m0, sc1, m1;
    scale_min_pair(hdr.y, hdr.z, hdr.w, p, sc0, m0, sc1, m1);
    const float d = half_lo(hdr.x), dmin = half_hi(hdr.x);
    const float fm0 = static_cast<float>(m0), fm1 = static_cast<float>(m1);
    const uint32_t qw[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
    uint32_t lo[8], hi[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        lo[k] = qw[k] & 0x0F0F0F0Fu;
        hi[k] = qw[k] & 0xF0F0F0F0u;
    }
#pragma unroll
    for (int c = 0; c < NCOLS; ++c) {
        const uint4 *a = reinterpret_cast<const uint4 *>(aq + (c * nsb + b) * 256 + 64 * p);
        const uint4 a0 = a[0], a1 = a[1], a2 = a[2], a3 = a[3];
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
        P0[c] = s0;
        P1[c] = s1;
        const float2 d8 = *reinterpret_cast<const float2 *>(ad8 + (c * nsb + b) * 8 + 2 * p);
        const float2 A = *reinterpret_cast<const float2 *>(aA + (c * nsb + b) * 8 + 2 * p);
        const float t0 = __fmul_rn(d8.x, __int2float_rn(s0 * sc0));
        const float t1 = __fmul_rn(d8.y, __int2float_rn(s1 * sc1));
        float tp = __fadd_rn(t0, t1);
        float up = __fadd_rn(__fmul_rn(A.x, fm0), __fmul_rn(A.y, fm1));
        tp = __fadd_rn(tp, __shfl_xor_sync(0xffffffffu, tp, 8));
        up = __fadd_rn(up, __shfl_xor_sync(0xffffffffu, up, 8));
        tp = __fadd_rn(tp, __shfl_xor_sync(0xffffffffu, tp, 16));
        up = __fadd_rn(up, __shfl_xor_sync(0xffffffffu, up, 16));
        v[c] = __fmaf_rn(d, tp, -__fmul_rn(dmin, up));
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

template <int NCOLS, int KS, int NCW, bool EMIT_P>
__global__ void __launch_bounds__((NCW + 1) * 32, 1)
    mmvq_q4k_kernel(const uint8_t *__restrict__ W, const uint8_t *__restrict__ X,
                    float *__restrict__ Y, int N, int nsb, int64_t ldy, int rg_total,
                    int nstage, int pitch, int32_t *__restrict__ Pout,
                    int32_t *__restrict__ Mout) {
    constexpr int NSL = 8 / KS;     // canonical slices per k-part
    constexpr int NGRP = NCW / KS;  // warp groups, one row group each at a time
    static_assert(NCW % KS == 0, "consumer warps must be a multiple of KS");
    extern __shared__ __align__(128) uint8_t smem[];
    const MmvqLayout L = mmvq_layout(NCOLS, KS, NCW, nsb, nstage, pitch);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L.off_full);
    uint64_t *empty = reinterpret_cast<uint64_t *>(smem + L.off_empty);
    float *red = reinterpret_cast<float *>(smem + L.off_red);
    uint8_t *aq = smem + L.off_qs;
    float *ad8 = reinterpret_cast<float *>(smem + L.off_d8);
    float *aA = reinterpret_cast<float *>(smem + L.off_A);
    uint8_t *stage = smem + L.off_stage;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = gridDim.x;
    const int rg_begin = static_cast<int>(static_cast<int64_t>(blockIdx.x) * rg_total / G);
    const int rg_end = static_cast<int>(static_cast<int64_t>(blockIdx.x + 1) * rg_total / G);
    const int nrg = rg_end - rg_begin;
    const int U = nrg * KS;

    if (threadIdx.x == 0) {
        for (int s = 0; s < nstage; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        fence_mbar_init();
    }
    __syncthreads();
    pdl_launch_dependents();

    if (warp == NCW) {
        // ---------------------------------------------------- producer ---
        const uint64_t pol = policy_evict_first();
        for (int u = 0; u < U; ++u) {
            const int s = u % nstage, k = u / nstage;
            if (k > 0 && !mbar_wait(&empty[s], (k - 1) & 1)) break;
            const int rg = rg_begin + u / KS, j = u % KS;
            const int sb_lo = slice_start(nsb, j * NSL), sb_hi = slice_start(nsb, (j + 1) * NSL);
            const uint32_t part_bytes = static_cast<uint32_t>(sb_hi - sb_lo) * Q4K_BYTES;
            const int row0 = rg * 8;
            const int nvalid = min(8, N - row0);
            if (lane == 0) mbar_arrive_expect_tx(&full[s], nvalid * part_bytes);
            __syncwarp();
            if (lane < nvalid && part_bytes > 0)
                bulk_g2s(stage + (s * 8 + lane) * pitch,
                         W + (static_cast<int64_t>(row0 + lane) * nsb + sb_lo) * Q4K_BYTES,
                         part_bytes, &full[s], pol);
        }
        return;
    }

    // -------------------------------------------------------- consumers ---
    pdl_wait();  // x is produced by the preceding kernel
    const int nblk = nsb * 8;
    for (int i = threadIdx.x; i < NCOLS * nblk; i += NCW * 32) {
        const int c = i / nblk, blk = i - c * nblk;
        const uint32_t *src = reinterpret_cast<const uint32_t *>(
            X + (static_cast<int64_t>(c) * nblk + blk) * Q81_BYTES);
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
            if (blockIdx.x == 0) Mout[i] = msum;
        }
    }
    named_bar_sync(1, NCW * 32);

    const int grp = warp / KS, j = warp % KS;
    const int p = lane >> 3, g = lane & 7;
    const int sb_part = slice_start(nsb, j * NSL);
    bool poisoned = false;
    int round = 0;
    for (int r = grp; r < nrg; r += NGRP, ++round) {
        const int u = r * KS + j;
        const int s = u % nstage, k = u / nstage;
        if (!poisoned && !mbar_wait(&full[s], k & 1)) poisoned = true;
        const uint8_t *st = stage + (s * 8 + g) * pitch;
        const int row = (rg_begin + r) * 8 + g;
        float acc[NCOLS][NSL];
#pragma unroll
        for (int i = 0; i < NSL; ++i) {
            const int b0 = slice_start(nsb, j * NSL + i), b1 = slice_start(nsb, j * NSL + i + 1);
#pragma unroll
            for (int c = 0; c < NCOLS; ++c) acc[c][i] = 0.0f;
            for (int b = b0; b < b1; ++b) {
                float v[NCOLS];
                int P0[NCOLS], P1[NCOLS];
                sb_values<NCOLS>(st + (b - sb_part) * Q4K_BYTES, p, aq, ad8, aA, nsb, b, v, P0, P1);
#pragma unroll
                for (int c = 0; c < NCOLS; ++c) acc[c][i] = (b == b0) ? v[c] : __fadd_rn(acc[c][i], v[c]);
                if constexpr (EMIT_P) {
                    if (row < N) {
#pragma unroll
                        for (int c = 0; c < NCOLS; ++c) {
                            int32_t *dst = Pout + ((static_cast<int64_t>(c) * N + row) * nsb + b) * 8 + 2 * p;
                            dst[0] = P0[c];
                            dst[1] = P1[c];
                        }
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        float sub[NCOLS];
#pragma unroll
        for (int c = 0; c < NCOLS; ++c) sub[c] = tree_sum<NSL>(acc[c]);
        if constexpr (KS == 1) {
            if (p == 0 && row < N) {
#pragma unroll
                for (int c = 0; c < NCOLS; ++c) Y[c * ldy + row] = sub[c];
            }
        } else {
            float *slot = red + ((round & 1) * NCW + warp) * 8 * NCOLS;
            if (p == 0) {
#pragma unroll
                for (int c = 0; c < NCOLS; ++c) slot[g * NCOLS + c] = sub[c];
            }
            named_bar_sync(2 + grp, KS * 32);
            if (j == 0 && p == 0 && row < N) {
#pragma unroll
                for (int c = 0; c < NCOLS; ++c) {
                    float parts[KS];
#pragma unroll
                    for (int jj = 0; jj < KS; ++jj)
                        parts[jj] = red[((round & 1) * NCW + grp * KS + jj) * 8 * NCOLS + g * NCOLS + c];
                    Y[c * ldy + row] = tree_sum<KS>(parts);
                }
            }
        }
    }
}

// ------------------------------------------------------------- host side ---
static const MmvqConfig kCandidates[] = {
    // id, ks, ncw, ctas_per_sm, stage_kb
    {101, 1, 4, 1, 200}, {102, 1, 8, 1, 200}, {103, 1, 4, 2, 100}, {104, 1, 8, 2, 100},
    {201, 2, 4, 1, 200}, {202, 2, 8, 1, 200}, {203, 2, 4, 2, 100}, {204, 2, 8, 2, 100},
    {401, 4, 4, 1, 200}, {402, 4, 8, 1, 200}, {403, 4, 4, 2, 100}, {404, 4, 8, 2, 100},
    {802, 8, 8, 1, 200}, {804, 8, 8, 2, 100},
};

const MmvqConfig *mmvq_candidates(int *count) {
    *count = static_cast<int>(sizeof(kCandidates) / sizeof(kCandidates[0]));
    return kCandidates;
}
const MmvqConfig *mmvq_candidate_by_id(int id) {
    int n = 0;
    const MmvqConfig *c = mmvq_candidates(&n);
    for (int i = 0; i < n; ++i)
        if (c[i].id == id) return &c[i];
    return nullptr;
}

int device_sm_count() {
    static int cached[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return 148;
    if (cached[dev] == 0) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        cached[dev] = n > 0 ? n : 148;
    }
    return cached[dev];
}

using MmvqFn = void (*)(const uint8_t *, const uint8_t *, float *, int, int, int64_t, int, int,
                        int, int32_t *, int32_t *);

template <int NCOLS, int KS, int NCW, bool EMIT_P>
static MmvqFn mmvq_fn() {
    return mmvq_q4k_kernel<NCOLS, KS, NCW, EMIT_P>;
}

template <int KS, int NCW>
static MmvqFn pick_ncols(int ncols) {
    switch (ncols) {
        case 1: return mmvq_fn<1, KS, NCW, false>();
        case 2: return mmvq_fn<2, KS, NCW, false>();
        case 3: return mmvq_fn<3, KS, NCW, false>();
        case 4: return mmvq_fn<4, KS, NCW, false>();
        case 5: return mmvq_fn<5, KS, NCW, false>();
        case 6: return mmvq_fn<6, KS, NCW, false>();
        case 7: return mmvq_fn<7, KS, NCW, false>();
        case 8: return mmvq_fn<8, KS, NCW, false>();
        default: return nullptr;
    }
}

static MmvqFn pick_fn(int ks, int ncw, int ncols) {
    if (ncw == 4) {
        switch (ks) {
            case 1: return pick_ncols<1, 4>(ncols);
            case 2: return pick_ncols<2, 4>(ncols);
            case 4: return pick_ncols<4, 4>(ncols);
            default: return nullptr;
        }
    }
    if (ncw == 8) {
        switch (ks) {
            case 1: return pick_ncols<1, 8>(ncols);
            case 2: return pick_ncols<2, 8>(ncols);
            case 4: return pick_ncols<4, 8>(ncols);
            case 8: return pick_ncols<8, 8>(ncols);
            default: return nullptr;
        }
    }
    return nullptr;
}

constexpr int kMaxSmem = 227 * 1024;

static cudaError_t ensure_smem_attr(MmvqFn fn) {
    // Raise the dynamic shared-memory limit once per (kernel, device).
    static std::mutex mu;
    static const void *done[512];
    static int done_dev[512];
    static int ndone = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    for (int i = 0; i < ndone; ++i)
        if (done[i] == reinterpret_cast<const void *>(fn) && done_dev[i] == dev) return cudaSuccess;
    cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void *>(fn),
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
    if (e != cudaSuccess) return e;
    if (ndone < 512) {
        done[ndone] = reinterpret_cast<const void *>(fn);
        done_dev[ndone] = dev;
        ++ndone;
    }
    return cudaSuccess;
}

struct MmvqPlan {
    int grid, nstage, pitch, smem, rg_total;
};

static bool plan_mmvq(int ks, int ncw, int ctas_per_sm, int stage_kb, int64_t N, int nsb,
                      int ncols, MmvqPlan &pl) {
    const int nsl = 8 / ks;
    const int max_part = slice_start(nsb, nsl) * Q4K_BYTES;
    int pitch = max_part;
    if (((pitch / 16) & 1) == 0) pitch += 16;
    pl.pitch = pitch;
    pl.rg_total = static_cast<int>((N + 7) / 8);
    const int sms = device_sm_count();
    pl.grid = pl.rg_total < sms * ctas_per_sm ? pl.rg_total : sms * ctas_per_sm;
    const int rg_per_cta = (pl.rg_total + pl.grid - 1) / pl.grid;
    const int units = rg_per_cta * ks;
    const int stage_bytes = 8 * pitch;
    int nstage = (stage_kb * 1024) / stage_bytes;
    if (nstage < 2) nstage = 2;
    if (nstage > units) nstage = units;
    if (nstage < 1) nstage = 1;
    for (;;) {
        const MmvqLayout L = mmvq_layout(ncols, ks, ncw, nsb, nstage, pitch);
        if (L.bytes <= kMaxSmem) {
            pl.nstage = nstage;
            pl.smem = L.bytes;
            return true;
        }
        if (nstage == 1) return false;
        --nstage;
    }
}

static cudaError_t launch_plan(MmvqFn fn, const MmvqPlan &pl, int ncw, bool pdl,
                               const void *w, const void *x, float *y, int64_t N, int nsb,
                               int64_t ldy, int32_t *P, int32_t *M, cudaStream_t stream) {
    cudaError_t e = ensure_smem_attr(fn);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(pl.grid);
    cfg.blockDim = dim3((ncw + 1) * 32);
    cfg.dynamicSmemBytes = pl.smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, fn, static_cast<const uint8_t *>(w),
                              static_cast<const uint8_t *>(x), y, static_cast<int>(N), nsb, ldy,
                              pl.rg_total, pl.nstage, pl.pitch, P, M);
}

cudaError_t launch_mmvq_q4k(const MmvqConfig &cfg, const void *w, const void *x_q8, float *y,
                            int64_t N, int64_t K, int ncols, int64_t ldy, int flags,
                            cudaStream_t stream) {
    const int nsb = static_cast<int>(K / QK_K);
    MmvqFn fn = pick_fn(cfg.ks, cfg.ncw, ncols);
    if (!fn) return cudaErrorInvalidValue;
    MmvqPlan pl;
    if (!plan_mmvq(cfg.ks, cfg.ncw, cfg.ctas_per_sm, cfg.stage_kb, N, nsb, ncols, pl))
        return cudaErrorInvalidConfiguration;
    return launch_plan(fn, pl, cfg.ncw, (flags & MMVQ_PDL) != 0, w, x_q8, y, N, nsb, ldy,
                       nullptr, nullptr, stream);
}

template <int KS>
static MmvqFn pick_partials(int ncols) {
    switch (ncols) {
        case 1: return mmvq_fn<1, KS, 4, true>();
        case 2: return mmvq_fn<2, KS, 4, true>();
        case 4: return mmvq_fn<4, KS, 4, true>();
        case 8: return mmvq_fn<8, KS, 4, true>();
        default: return nullptr;
    }
}

cudaError_t launch_mmvq_q4k_partials(const void *w, const void *x_q8, float *y, int32_t *P,
                                     int32_t *M, int64_t N, int64_t K, int ncols, int ks,
                                     cudaStream_t stream) {
    const int nsb = static_cast<int>(K / QK_K);
    MmvqFn fn = nullptr;
    if (ks == 1) fn = pick_partials<1>(ncols);
    else if (ks == 2) fn = pick_partials<2>(ncols);
    else if (ks == 4) fn = pick_partials<4>(ncols);
    if (!fn) return cudaErrorInvalidValue;
    MmvqPlan pl;
    if (!plan_mmvq(ks, 4, 1, 200, N, nsb, ncols, pl)) return cudaErrorInvalidConfiguration;
    return launch_plan(fn, pl, 4, false, w, x_q8, y, N, nsb, N, P, M, stream);
}

}  // namespace abra

ABRA_ERROR_WORD_ACCESSOR(error_word_mmvq)
