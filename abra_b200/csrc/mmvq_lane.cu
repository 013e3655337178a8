// mmvq_lane.cu -- the lane-mapped Q4_K x Q8_1 MMVQ at batch 1 (candidate
// mode MODE_LANE).
//
// The same operation as mmvq_q4k_kernel (y = W x, or the fused gate/up
// SwiGLU with NMAT == 2; the reference's vec_dot_q4_K_q8_1 / mul_mat_vec_q,
// kernels/q4k/q4k_vecdot.cuh:23-87, kernels/q4k/q4k_family.cu:12-90), with
// the work split of the persistent decode kernel: a unit is R consecutive
// rows (R = 8, 4, 2 or 1), contiguous in HBM and so staged by ONE bulk copy
// per matrix into a ring slot; within a warp a lane owns whole superblocks
// (all eight sub-blocks: lane_gemv.cuh), so a unit is a handful of
// independent superblock dots per lane instead of a ten-step chain; eight
// lanes per row then form the canonical K-slice sums and their tree.  The
// fp32 order is the canonical one, so the bits equal every other candidate's.
//
// The CTA's units are a contiguous range; its producer warp streams them
// into the ring from the launch's first instruction (weights do not depend
// on the previous kernel), and the consumers wait for the previous kernel
// (programmatic dependent launch) only to stage the Q8_1 activation.  Every
// wait is bounded; no copy uses cluster multicast.
#include "kernels.cuh"
#include "lane_gemv.cuh"
#include "mmvq_impl.cuh"

namespace abra {

namespace {

constexpr int LN_NCW = 8;    // consumer warps
constexpr int LN_VMAX = 80;  // superblock values staged per warp (rows x matrices x superblocks)

struct LaneParams {
    const uint8_t *W[2];
    const uint8_t *X;  // Q8_1 blocks of the activation
    float *Y;
    unsigned long long *amax;  // optional argmax keys (argmax_key)
    int N, nsb, lr, nslot, slot_bytes;
    int off_vbuf, off_arec, off_ring;
};

template <int NMAT, int MINB, bool PACKED>
__global__ void __launch_bounds__((LN_NCW + 1) * 32, MINB) mmvq_lane_kernel(const LaneParams prm) {
    constexpr int SB = PACKED ? LG_PACKED_BYTES : Q4K_BYTES;  // bytes per superblock
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ unsigned long long s_amax;
    const int nslot = prm.nslot, nsb = prm.nsb, lr = prm.lr, R = 1 << lr, N = prm.N;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + nslot;
    uint8_t *ring = smem + prm.off_ring;
    const int row_bytes = nsb * SB;
    const int total = (N + R - 1) >> lr;
    const int u_begin = static_cast<int>(static_cast<int64_t>(blockIdx.x) * total / gridDim.x);
    const int nu = static_cast<int>(static_cast<int64_t>(blockIdx.x + 1) * total / gridDim.x) - u_begin;
    if (threadIdx.x == 0) {
        for (int s = 0; s < nslot; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        fence_mbar_init();
        s_amax = 0ull;
    }
    __syncthreads();
    pdl_launch_dependents();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (warp == LN_NCW) {
        // ---------------------------------------------------- producer ---
        const uint64_t pol = policy_evict_first();
        int issued = 0;
        for (int u = 0; u < nu; ++u) {
            const int s = u % nslot, k = u / nslot;
            if (k > 0 && !mbar_wait(&empty[s], (k - 1) & 1, ERR_WAIT_EMPTY)) break;
            const int row0 = (u_begin + u) << lr, nvalid = min(R, N - row0);
            const uint32_t bytes = static_cast<uint32_t>(nvalid) * row_bytes;
            if (lane == 0) mbar_arrive_expect_tx(&full[s], NMAT * bytes);
            __syncwarp();
            if (lane < NMAT)
                bulk_g2s(ring + s * prm.slot_bytes + lane * R * row_bytes,
                         prm.W[lane] + static_cast<int64_t>(row0) * row_bytes, bytes, &full[s], pol);
            issued = u + 1;
        }
        // every copy this warp issued has landed before the CTA can exit
        if (lane == 0)
            for (int u = issued > nslot ? issued - nslot : 0; u < issued; ++u)
                mbar_wait(&full[u % nslot], (u / nslot) & 1);
        __syncwarp();
        return;
    }

    // -------------------------------------------------------- consumers ---
    uint8_t *arec = smem + prm.off_arec;
    pdl_wait();  // the activation is produced by the preceding kernel
    for (int i = threadIdx.x; i < nsb * 8; i += LN_NCW * 32) {
        const uint32_t *src = reinterpret_cast<const uint32_t *>(prm.X + static_cast<int64_t>(i) * Q81_BYTES);
        uint32_t q[9];
#pragma unroll
        for (int k = 0; k < 9; ++k) q[k] = __ldcg(src + k);
        int msum = 0;
#pragma unroll
        for (int k = 1; k < 9; ++k) msum = dp4a_ss(0x01010101, static_cast<int>(q[k]), msum);
        uint8_t *rec = arec + (i >> 3) * LG_AREC;
        const int s = i & 7;
        uint4 *dst = reinterpret_cast<uint4 *>(rec + 32 * s);
        dst[0] = make_uint4(q[1], q[2], q[3], q[4]);
        dst[1] = make_uint4(q[5], q[6], q[7], q[8]);
        const float d8 = half_lo(q[0]);
        reinterpret_cast<float *>(rec + 256)[s] = d8;
        reinterpret_cast<float *>(rec + 288)[s] = __fmul_rn(d8, __int2float_rn(msum));
    }
    named_bar_sync(1, LN_NCW * 32);

    float *vbuf = reinterpret_cast<float *>(smem + prm.off_vbuf) + warp * LN_VMAX;
    const int P = 32 >> lr;
    // lane -> (row r, first superblock p); P >= 8: a quarter warp is one row
    // and eight consecutive superblocks; P == 4 (eight rows): a quarter warp
    // is four rows x two superblocks (distinct bank groups for the 2560-wide
    // matrices, whose rows are 9 * 10 chunks of 16 bytes)
    int r, p;
    if (P >= 8) {
        r = lane / P;
        p = lane % P;
    } else {
        const int q4 = lane >> 3, w8 = lane & 7;
        r = (w8 >> 1) + 4 * (q4 & 1);
        p = (w8 & 1) + 2 * (q4 >> 1);
    }
    bool poisoned = false;
    unsigned long long key = 0ull;
    for (int u = warp; u < nu; u += LN_NCW) {
        const int s = u % nslot;
        if (!poisoned && !mbar_wait(&full[s], (u / nslot) & 1)) poisoned = true;
        const uint8_t *wrow[NMAT];
#pragma unroll
        for (int m = 0; m < NMAT; ++m) wrow[m] = ring + s * prm.slot_bytes + (m * R + r) * row_bytes;
        for (int b = p; b < nsb; b += P) {
            const uint8_t *wsb[NMAT];
#pragma unroll
            for (int m = 0; m < NMAT; ++m) wsb[m] = wrow[m] + b * SB;
            float v[NMAT];
            if constexpr (PACKED)
                pk_sb_value_packed<NMAT>(wsb, arec + b * LG_AREC, v);
            else
                pk_sb_value<NMAT>(wsb, arec + b * LG_AREC, v);
#pragma unroll
            for (int m = 0; m < NMAT; ++m) vbuf[(m * R + r) * nsb + b] = v[m];
        }
        __syncwarp();
        // the slot is consumed: lane 31 stores nothing to global memory, so
        // its release does not wait for this warp's output stores
        if (lane == 31) mbar_arrive(&empty[s]);
        // row sums: lane 8g + i forms slice i of rows g, g + 4 of the unit;
        // lane 8g stores the row
        const int i = lane & 7, g = lane >> 3;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            const int rr = g + 4 * half;
            if (half == 1 && R <= 4) break;  // warp-uniform
            const int row = ((u_begin + u) << lr) + rr;
            const bool live = rr < R;
            float yv = pk_slice_tree(live ? pk_slice_sum(vbuf + rr * nsb, nsb, i) : 0.0f);
            if constexpr (NMAT == 2) {
                const float up = pk_slice_tree(live ? pk_slice_sum(vbuf + (R + rr) * nsb, nsb, i) : 0.0f);
                yv = __fmul_rn(up, abra_silu(yv));
            }
            if (i == 0 && live && row < N) {
                prm.Y[row] = yv;
                const unsigned long long k2 = argmax_key(yv, row);
                key = k2 > key ? k2 : key;
            }
        }
        __syncwarp();  // the staging buffer is reused by the next unit
    }
    if (prm.amax) {
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) {
            const unsigned long long k2 = __shfl_xor_sync(0xffffffffu, key, o);
            key = k2 > key ? k2 : key;
        }
        if (lane == 0 && key) atomicMax(&s_amax, key);
        named_bar_sync(1, LN_NCW * 32);
        if (threadIdx.x == 0 && s_amax) atomicMax(prm.amax, s_amax);
    }
}

using LaneFn = void (*)(const LaneParams);

LaneFn lane_kernel(int nmat, int minb, bool packed = false) {
    if (packed) return nmat == 1 ? mmvq_lane_kernel<1, 2, true> : nullptr;
    if (nmat == 1) return minb == 2 ? mmvq_lane_kernel<1, 2, false> : mmvq_lane_kernel<1, 1, false>;
    return minb == 2 ? mmvq_lane_kernel<2, 2, false> : mmvq_lane_kernel<2, 1, false>;
}

// The reference's prepack of one Q4_K superblock into its 148-byte form
// (kernels/q4k/abra-packed-q4.cuh:10-27): d and dmin, the eight 6-bit scales
// and mins as bytes [sc_2j, sc_2j+1, m_2j, m_2j+1] per pair j, the nibbles.
__global__ void q4k_pack_kernel(const uint8_t *__restrict__ in, uint8_t *__restrict__ out, int64_t nblocks) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= nblocks) return;
    const uint8_t *b = in + i * Q4K_BYTES;
    uint32_t *o = reinterpret_cast<uint32_t *>(out + i * LG_PACKED_BYTES);
    const uint32_t *b32 = reinterpret_cast<const uint32_t *>(b);
    o[0] = b32[0];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        int sc0, m0, sc1, m1;
        scale_min_one(b + 4, 2 * j, sc0, m0);
        scale_min_one(b + 4, 2 * j + 1, sc1, m1);
        o[1 + j] = static_cast<uint32_t>(sc0) | (static_cast<uint32_t>(sc1) << 8) | (static_cast<uint32_t>(m0) << 16) |
                   (static_cast<uint32_t>(m1) << 24);
    }
#pragma unroll 8
    for (int k = 0; k < 32; ++k) o[5 + k] = b32[4 + k];
}

}  // namespace

bool mmvq_lane_plan(const MmvqConfig &cfg, int64_t N, int nsb, int nmat, int sms, int64_t out[8],
                    bool packed) {
    if (cfg.mode != MODE_LANE || nsb <= 0 || N <= 0 || (nmat != 1 && nmat != 2)) return false;
    int R = cfg.ks;  // the candidate's largest rows per unit
    while (R > 1 && R * nmat * nsb > LN_VMAX) R >>= 1;
    if (R * nmat * nsb > LN_VMAX) return false;
    // packed rows (148 bytes per superblock) are 4-byte aligned: a unit's
    // copy needs R * nsb * 148 to be a multiple of 16 bytes
    if (packed && (R * nsb) % 4 != 0) return false;
    int lr = 0;
    while ((1 << lr) < R) ++lr;
    const int64_t row_bytes = static_cast<int64_t>(nsb) * (packed ? LG_PACKED_BYTES : Q4K_BYTES);
    const int slot_bytes = static_cast<int>(R * nmat * row_bytes);
    const int64_t total = (N + R - 1) / R;
    if (sms <= 0) sms = device_sm_count();
    const int64_t grid = total < static_cast<int64_t>(sms) * cfg.ctas_per_sm ? total : sms * cfg.ctas_per_sm;
    const int64_t units = (total + grid - 1) / grid;
    const int budget = cfg.stage_kb * 1024 / slot_bytes;
    // a slot is reused only by the warp that consumed it (nslot a multiple
    // of the consumer warps) or never (one slot per unit)
    int nslot = units <= budget ? static_cast<int>(units) : budget / LN_NCW * LN_NCW;
    if (nslot < 1) return false;
    const int off_vbuf = align_up(16 * nslot, 16);
    const int off_arec = align_up(off_vbuf + LN_NCW * LN_VMAX * 4, 128);
    const int off_ring = align_up(off_arec + nsb * LG_AREC, 128);
    const int64_t smem = off_ring + static_cast<int64_t>(nslot) * slot_bytes;
    if (smem > kMmvqMaxSmem) return false;
    const int64_t v[8] = {grid, (LN_NCW + 1) * 32, nslot, slot_bytes, smem, lr, off_arec, off_ring};
    for (int i = 0; i < 8; ++i) out[i] = v[i];
    return true;
}

cudaError_t prepare_mmvq_lane(const MmvqConfig &cfg, int nmat) {
    if (cfg.mode != MODE_LANE || (nmat != 1 && nmat != 2)) return cudaErrorInvalidValue;
    return ensure_smem_attr_ptr(reinterpret_cast<const void *>(lane_kernel(nmat, cfg.ctas_per_sm >= 2 ? 2 : 1)));
}

cudaError_t launch_q4k_pack(const void *w, void *w_packed, int64_t nblocks, cudaStream_t stream) {
    if (nblocks <= 0) return cudaErrorInvalidValue;
    q4k_pack_kernel<<<static_cast<unsigned>((nblocks + 255) / 256), 256, 0, stream>>>(
        static_cast<const uint8_t *>(w), static_cast<uint8_t *>(w_packed), nblocks);
    return cudaGetLastError();
}

cudaError_t launch_mmvq_lane(const MmvqConfig &cfg, const void *w, const void *w2, const void *x_q8, float *y,
                             int64_t N, int64_t K, int flags, cudaStream_t stream, unsigned long long *amax,
                             bool packed) {
    const int nsb = static_cast<int>(K / QK_K), nmat = w2 ? 2 : 1;
    int64_t pl[8];
    if (!mmvq_lane_plan(cfg, N, nsb, nmat, 0, pl, packed)) return cudaErrorInvalidConfiguration;
    LaneFn fn = lane_kernel(nmat, cfg.ctas_per_sm >= 2 ? 2 : 1, packed);
    if (!fn) return cudaErrorInvalidConfiguration;
    cudaError_t e = ensure_smem_attr_ptr(reinterpret_cast<const void *>(fn));
    if (e != cudaSuccess) return e;
    LaneParams prm = {};
    prm.W[0] = static_cast<const uint8_t *>(w);
    prm.W[1] = static_cast<const uint8_t *>(w2);
    prm.X = static_cast<const uint8_t *>(x_q8);
    prm.Y = y;
    prm.amax = amax;
    prm.N = static_cast<int>(N);
    prm.nsb = nsb;
    prm.lr = static_cast<int>(pl[5]);
    prm.nslot = static_cast<int>(pl[2]);
    prm.slot_bytes = static_cast<int>(pl[3]);
    prm.off_vbuf = align_up(16 * prm.nslot, 16);
    prm.off_arec = static_cast<int>(pl[6]);
    prm.off_ring = static_cast<int>(pl[7]);
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3(static_cast<unsigned>(pl[0]));
    lc.blockDim = dim3(static_cast<unsigned>(pl[1]));
    lc.dynamicSmemBytes = static_cast<size_t>(pl[4]);
    lc.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    lc.attrs = attr;
    lc.numAttrs = (flags & MMVQ_PDL) ? 1 : 0;
    return cudaLaunchKernelEx(&lc, fn, prm);
}

}  // namespace abra
