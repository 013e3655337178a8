// mmvq_tc.cu -- Q4_K x Q8_1 for a batch of 32 activation columns on the 5th
// generation tensor cores (tcgen05, kind::i8).
//
// The integer part of vec_dot_q4_K_q8_1 (kernels/q4k/q4k_vecdot.cuh:23-45:
// P_s = sum of q4 * q8 over sub-block s, exact in int32) is a matrix product
// per sub-block: for a tile of 128 weight rows and all 32 columns,
// P_s[n][c] = sum_k A_s[n][k] B_s[c][k] with A_s the sub-block's nibbles
// (u8 0..15) and B_s the Q8_1 quants (s8), K = 32 = one tcgen05.mma of shape
// M128 x N32 x K32.  A superblock is eight such MMAs into eight TMEM
// accumulators (8 x 32 columns).  The fp32 scaling then follows the same
// canonical order as the dp4a kernels and the CPU oracle, so the outputs are
// bit-identical to them:
//   t_s = d8_s * float(P_s * sc_s), u_s = A_s * float(m_s) (A_s = d8_s *
//   float(sum q8_s)), S = ((t0+t1)+(t2+t3))+((t4+t5)+(t6+t7)),
//   value = fmaf(d, S_t, -(dmin * S_u)); superblocks summed in order within a
//   canonical K-slice, slices combined by the fixed tree; a k-part (KS > 1)
//   is a subtree and the parts are combined by tree in a second kernel.
//
// CTA: 16 warps.  Thread 0 streams the tile's packed superblocks through a
// 4-stage mbarrier ring, one 2-D TMA tile copy (144 B x 128 rows, rows past
// N zero-filled; no multicast) per stage, three superblocks ahead.  Per superblock the
// consumers expand the nibbles to the MMA's K-major no-swizzle layout
// (8-row x 16-byte core matrices), stage the 32 columns' int8 quants the
// same way, one thread issues the eight MMAs and commits them to an
// mbarrier, and every consumer thread reads its row's eight accumulators
// for its 8 columns from TMEM (warp w: lanes 32 (w % 4).., columns
// 8 (w / 4)..).  Every wait is bounded; TMEM is always freed.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "../../include/abra_b200.h"
#include "common.cuh"
#include "kernels.cuh"
#include "tc_common.cuh"

namespace abra {
namespace {

constexpr int TC_M = 128;          // weight rows per tile (MMA M)
constexpr int TC_N = 32;           // activation columns (MMA N)
constexpr int TC_CONS = 512;       // consumer threads (16 warps)
constexpr int TC_THREADS = TC_CONS;  // thread 0 also issues the weight copies
constexpr int TC_STAGES = 4;
constexpr int TC_STAGE = TC_M * Q4K_BYTES;  // 18,432 B
constexpr uint32_t TC_TMEM_COLS = 512;      // 2 buffers x 8 sub-blocks x 32 columns
constexpr uint32_t TC_IDESC = tc_idesc_i8(TC_M, TC_N, false, true);  // u8 x s8 -> s32

// Two of each per-superblock buffer (A, B, row headers, d8, A-sums, TMEM
// accumulators): superblock u uses set u % 2, so its MMAs run while the
// next superblock is expanded and the previous one's epilogue runs.
struct TcLayout {
    int full, empty, mma, holder, stage, a, b, hdr, d8, am, bytes;
};
__host__ __device__ constexpr TcLayout tc_layout() {
    TcLayout L{};
    L.full = 0;
    L.empty = 8 * TC_STAGES;
    L.mma = 16 * TC_STAGES;                // 2 barriers
    L.holder = L.mma + 16;
    L.stage = 1024;
    L.a = L.stage + TC_STAGES * TC_STAGE;  // 2 x 8 x 4096 (1024-aligned)
    L.b = L.a + 2 * 8 * 4096;              // 2 x 8 x 1024
    L.hdr = L.b + 2 * 8 * 1024;            // 2 x 128 x 16
    L.d8 = L.hdr + 2 * TC_M * 16;          // 2 x 8 x 32 floats
    L.am = L.d8 + 2 * 8 * TC_N * 4;        // 2 x 8 x 32 floats
    L.bytes = L.am + 2 * 8 * TC_N * 4;
    return L;
}
static_assert(tc_layout().a % 1024 == 0, "operand tiles must be aligned");

struct TcParams {
    const uint8_t *W;  // N x nsb superblocks
    const uint8_t *X;  // 32 columns x nsb*8 Q8_1 blocks
    float *Y;          // y[c * ldy + n] (KS == 1)
    float *part;       // KS > 1: [KS][32][N]
    int N, nsb;
    int64_t ldy;
    // K-shard: slice bounds come from the whole K's nsb_sl superblocks;
    // local superblock = whole-K superblock - sb_base; k-part = j_base +
    // blockIdx.y; direct: the single k-part's tree top goes to Y
    int nsb_sl, sb_base, j_base, direct;
    // tensor-parallel push (npeer > 0): rows go to peer_y[q] instead of Y;
    // each CTA then counts itself on cta_cnt and the launch's last CTA adds
    // 1 to every peer_cnt[q] with release semantics at system scope
    int npeer;
    float *peer_y[8];
    unsigned long long *peer_cnt[8];
    unsigned long long *cta_cnt;
};

// Exact tree over a power-of-two number of slices, fed left to right: the
// slice sums combine like a binary counter, giving ((s0+s1)+(s2+s3))+...
template <int NSL>
struct SliceTree {
    float lv[4][8];
    __device__ __forceinline__ void push(int i, const float (&v)[8]) {
        float x[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) x[c] = v[c];
        int k = i, level = 0;
#pragma unroll
        for (int l = 0; l < 3; ++l) {
            if (k & 1) {
#pragma unroll
                for (int c = 0; c < 8; ++c) x[c] = __fadd_rn(lv[l][c], x[c]);
                k >>= 1;
                level = l + 1;
            } else {
                break;
            }
        }
#pragma unroll
        for (int l = 0; l < 4; ++l)
            if (l == level)
#pragma unroll
                for (int c = 0; c < 8; ++c) lv[l][c] = x[c];
    }
};

// Exact int32 -> fp32 for |x| < 2^22 on the full-rate pipes (the magic-
// number conversion): x added to the bits of 1.5 * 2^23 lands in the low
// mantissa bits of a float of exponent 23, and subtracting 1.5 * 2^23 leaves
// x exactly -- the value __int2float_rn gives, without the conversion unit,
// whose lower throughput bounds this epilogue (64 conversions per thread per
// superblock).  |P_s * sc_s| <= 32 * 15 * 127 * 63 < 2^22.
__device__ __forceinline__ float i2f_small(int x) {
    return __fsub_rn(__int_as_float(0x4B400000 + x), 12582912.0f);
}

// One 2-D tiled TMA load of box (x bytes, y rows) into this CTA's shared memory.
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y,
                                            uint64_t *bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

template <int KS>
__global__ void __launch_bounds__(TC_THREADS, 1)
    mmvq_tc_kernel(const TcParams prm, const __grid_constant__ CUtensorMap wmap) {
    constexpr int NSL = 8 / KS;
    constexpr TcLayout L = tc_layout();
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L.full);
    uint64_t *mma_bar = reinterpret_cast<uint64_t *>(smem + L.mma);
    uint32_t *holder = reinterpret_cast<uint32_t *>(smem + L.holder);
    uint8_t *stage = smem + L.stage;
    uint8_t *A = smem + L.a;
    uint8_t *B = smem + L.b;
    uint8_t *hdr = smem + L.hdr;
    float *sd8 = reinterpret_cast<float *>(smem + L.d8);
    float *sam = reinterpret_cast<float *>(smem + L.am);

    const int N = prm.N, nsb = prm.nsb, nblk = nsb * 8;
    const int row0 = blockIdx.x * TC_M, j = prm.j_base + blockIdx.y;
    const int nvalid = min(TC_M, N - row0);
    // canonical slice i of the whole K, in this launch's local superblocks
    auto sl = [&](int i) { return slice_start(prm.nsb_sl, i) - prm.sb_base; };
    const int sb_lo = sl(j * NSL), sb_hi = sl((j + 1) * NSL);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < TC_STAGES; ++s) mbar_init(&full[s], 1);
        mbar_init(&mma_bar[0], 1);
        mbar_init(&mma_bar[1], 1);
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(holder, TC_TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *holder;
    pdl_launch_dependents();

    // weight stream: superblock u of this part lands in stage u % TC_STAGES;
    // the copy for u is issued while superblock u - TC_STAGES + 1 is expanded,
    // so its stage (that of u - TC_STAGES) has been copied out already
    const uint64_t pol = policy_evict_normal();  // neighbouring boxes share edge lines
    const int nsbp = sb_hi - sb_lo;
    auto fetch = [&](int u) {
        if (u < nsbp) {
            const int s = u % TC_STAGES;
            mbar_arrive_expect_tx(&full[s], TC_STAGE);  // the whole box, zero-filled past N
            tma_load_2d(stage + s * TC_STAGE, &wmap, (sb_lo + u) * Q4K_BYTES, row0, &full[s], pol);
        }
    };
    if (threadIdx.x == 0)
        for (int u = 0; u < TC_STAGES - 1; ++u) fetch(u);  // weights are immutable: before the wait

    // -------------------------------------------------------- consumers ---
    pdl_wait();  // the activations come from the preceding kernel
    const int t = threadIdx.x;
    const int q = warp & 3, cg = warp >> 2;  // TMEM lane quarter, column group
    const int rloc = 32 * q + lane;          // this thread's row of the tile
    bool poisoned = false;
    // activation staging: threads 0..255, one (sub-block bs8, column bc)
    // each, the column fastest so eight threads fill one 128-byte core matrix
    const bool bstager = t < 256;
    const int bc = t & 31, bs8 = (t >> 5) & 7;
    uint32_t bw[9] = {};
    auto load_b = [&](int u) {  // issue the loads of superblock u's quants
        if (!bstager) return;
        const uint32_t *blk = reinterpret_cast<const uint32_t *>(
            prm.X + (static_cast<int64_t>(bc) * nblk + (sb_lo + u) * 8 + bs8) * Q81_BYTES);
#pragma unroll
        for (int k = 0; k < 9; ++k) bw[k] = __ldg(blk + k);
    };
    auto store_b = [&](int buf) {  // B in the MMA layout, d8 and A = d8 * float(sum q8)
        if (!bstager) return;
        uint8_t *Bb = B + buf * 8192 + bs8 * 1024 + (bc >> 3) * 256 + (bc & 7) * 16;
        *reinterpret_cast<uint4 *>(Bb) = make_uint4(bw[1], bw[2], bw[3], bw[4]);
        *reinterpret_cast<uint4 *>(Bb + 128) = make_uint4(bw[5], bw[6], bw[7], bw[8]);
        int ms = 0;
#pragma unroll
        for (int k = 1; k < 9; ++k) ms = dp4a_ss(0x01010101, static_cast<int>(bw[k]), ms);
        const float d8 = half_lo(bw[0]);
        sd8[buf * 256 + bs8 * TC_N + bc] = d8;
        sam[buf * 256 + bs8 * TC_N + bc] = __fmul_rn(d8, __int2float_rn(ms));
    };
    // A: the nibbles of each sub-block as u8 in K-major core matrices: row r,
    // half kk of sub-block 2p (+1 for the high nibbles) at
    // (r/8)*256 + kk*128 + (r%8)*16; consecutive threads take consecutive rows
    auto expand_a = [&](int u, int buf) {
        if (t == 0) fetch(u + TC_STAGES - 1);
        const int s = u % TC_STAGES;
        if (!poisoned && !mbar_wait(&full[s], (u / TC_STAGES) & 1)) poisoned = true;
        const uint8_t *st = stage + s * TC_STAGE;
        uint8_t *Ab = A + buf * 32768;
        for (int ci = t; ci < TC_M * 8; ci += TC_CONS) {
            const int r = ci & (TC_M - 1), pc = ci >> 7, p = pc >> 1, kk = pc & 1;
            const uint4 v = *reinterpret_cast<const uint4 *>(st + r * Q4K_BYTES + 16 + 32 * p + 16 * kk);
            const uint4 lo = make_uint4(v.x & 0x0F0F0F0Fu, v.y & 0x0F0F0F0Fu, v.z & 0x0F0F0F0Fu, v.w & 0x0F0F0F0Fu);
            const uint4 hi = make_uint4((v.x >> 4) & 0x0F0F0F0Fu, (v.y >> 4) & 0x0F0F0F0Fu,
                                        (v.z >> 4) & 0x0F0F0F0Fu, (v.w >> 4) & 0x0F0F0F0Fu);
            const int off = (r >> 3) * 256 + kk * 128 + (r & 7) * 16;
            *reinterpret_cast<uint4 *>(Ab + (2 * p) * 4096 + off) = lo;
            *reinterpret_cast<uint4 *>(Ab + (2 * p + 1) * 4096 + off) = hi;
            if (pc == 0)
                *reinterpret_cast<uint4 *>(hdr + buf * 2048 + r * 16) =
                    *reinterpret_cast<const uint4 *>(st + r * Q4K_BYTES);
        }
    };
    auto issue_mma = [&](int buf) {  // one thread, after the barrier
        tc_fence_after();
#pragma unroll
        for (int s8 = 0; s8 < 8; ++s8)
            tc_mma_i8(tmem + buf * 256 + s8 * TC_N, tc_smem_desc(A + buf * 32768 + s8 * 4096, 128, 256),
                      tc_smem_desc(B + buf * 8192 + s8 * 1024, 128, 256), TC_IDESC, 0u);
        tc_commit(&mma_bar[buf]);
    };
    // epilogue bookkeeping: canonical slice of the superblock being finished
    SliceTree<NSL> tree;
    float acc[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) acc[c] = 0.0f;
    int e_slice = 0;
    int e_lo = sb_lo, e_hi = sl(j * NSL + 1);
    auto next_slices = [&](int b) {  // push finished (and empty) slices until b lies in e_slice
        while (b >= e_hi && e_slice < NSL) {
            tree.push(e_slice, acc);
#pragma unroll
            for (int c = 0; c < 8; ++c) acc[c] = 0.0f;
            ++e_slice;
            e_lo = e_hi;
            e_hi = sl(j * NSL + e_slice + 1);
        }
    };
    auto epilogue = [&](int u, int buf) {
        const int b = sb_lo + u;
        next_slices(b);
        if (!poisoned && !mbar_wait(&mma_bar[buf], (u >> 1) & 1)) poisoned = true;
        tc_fence_after();
        const uint4 h = *reinterpret_cast<const uint4 *>(hdr + buf * 2048 + rloc * 16);
        const float d = half_lo(h.x), dmin = half_hi(h.x);
        const float *d8b = sd8 + buf * 256, *amb = sam + buf * 256;
        float tph[2][8], uph[2][8];
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            int32_t P[4][8];
#pragma unroll
            for (int s4 = 0; s4 < 4; ++s4)
                tmem_ld_x8(tmem + (static_cast<uint32_t>(32 * q) << 16) + buf * 256 + (4 * half + s4) * TC_N + 8 * cg,
                           P[s4]);
            tmem_wait_ld();
#pragma unroll
            for (int pp = 0; pp < 2; ++pp) {
                const int p = 2 * half + pp;
                int sc0, m0, sc1, m1;
                scale_min_pair(h.y, h.z, h.w, p, sc0, m0, sc1, m1);
                const float fm0 = static_cast<float>(m0), fm1 = static_cast<float>(m1);
                // this thread's 8 columns of d8 and A for sub-blocks 2p, 2p+1
                const float4 *d0 = reinterpret_cast<const float4 *>(d8b + (2 * p) * TC_N + 8 * cg);
                const float4 *d1 = reinterpret_cast<const float4 *>(d8b + (2 * p + 1) * TC_N + 8 * cg);
                const float4 *a0 = reinterpret_cast<const float4 *>(amb + (2 * p) * TC_N + 8 * cg);
                const float4 *a1 = reinterpret_cast<const float4 *>(amb + (2 * p + 1) * TC_N + 8 * cg);
                const float4 d0a = d0[0], d0b = d0[1], d1a = d1[0], d1b = d1[1];
                const float4 a0a = a0[0], a0b = a0[1], a1a = a1[0], a1b = a1[1];
                const float vd0[8] = {d0a.x, d0a.y, d0a.z, d0a.w, d0b.x, d0b.y, d0b.z, d0b.w};
                const float vd1[8] = {d1a.x, d1a.y, d1a.z, d1a.w, d1b.x, d1b.y, d1b.z, d1b.w};
                const float va0[8] = {a0a.x, a0a.y, a0a.z, a0a.w, a0b.x, a0b.y, a0b.z, a0b.w};
                const float va1[8] = {a1a.x, a1a.y, a1a.z, a1a.w, a1b.x, a1b.y, a1b.z, a1b.w};
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    const float t0 = __fmul_rn(vd0[c], i2f_small(P[2 * pp][c] * sc0));
                    const float t1 = __fmul_rn(vd1[c], i2f_small(P[2 * pp + 1][c] * sc1));
                    const float tp = __fadd_rn(t0, t1);
                    const float up = __fadd_rn(__fmul_rn(va0[c], fm0), __fmul_rn(va1[c], fm1));
                    tph[half][c] = pp == 0 ? tp : __fadd_rn(tph[half][c], tp);
                    uph[half][c] = pp == 0 ? up : __fadd_rn(uph[half][c], up);
                }
            }
        }
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            const float st_ = __fadd_rn(tph[0][c], tph[1][c]);
            const float su = __fadd_rn(uph[0][c], uph[1][c]);
            const float v = __fmaf_rn(d, st_, -__fmul_rn(dmin, su));
            acc[c] = b == e_lo ? v : __fadd_rn(acc[c], v);
        }
    };
    // pipeline: MMA(u) runs while superblock u+1 is expanded and staged and
    // superblock u's accumulators wait for the epilogue
    if (nsbp > 0) {
        load_b(0);
        expand_a(0, 0);
        store_b(0);
        fence_proxy_async_smem();
        named_bar_sync(1, TC_CONS);
        if (t == 0) issue_mma(0);
    }
    for (int u = 1; u <= nsbp; ++u) {
        const int buf = u & 1;
        if (u < nsbp) {
            load_b(u);
            expand_a(u, buf);
        }
        epilogue(u - 1, buf ^ 1);
        if (u < nsbp) store_b(buf);
        fence_proxy_async_smem();
        tc_fence_before();
        named_bar_sync(1, TC_CONS);  // buffers of u ready; TMEM set u-1 read out
        if (u < nsbp && t == 0) issue_mma(buf);
    }
    next_slices(sb_hi);  // the last slice (and any empty ones)
    constexpr int TOP = NSL == 8 ? 3 : NSL == 4 ? 2 : NSL == 2 ? 1 : 0;
    if (rloc < nvalid) {
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            const int col = 8 * cg + c;
            const float v = tree.lv[TOP][c];
            if (KS == 1 || prm.direct) {
                const int64_t at = col * prm.ldy + row0 + rloc;
                if (prm.npeer > 0)
                    for (int q = 0; q < prm.npeer; ++q) prm.peer_y[q][at] = v;
                else
                    prm.Y[at] = v;
            } else {
                prm.part[(static_cast<int64_t>(j - prm.j_base) * TC_N + col) * N + row0 + rloc] = v;
            }
        }
    }
    tc_fence_before();
    named_bar_sync(1, TC_CONS);
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, TC_TMEM_COLS);
    }
    if (prm.npeer > 0 && threadIdx.x == 0) {
        // every consumer's stores are done (the barrier above): count this
        // CTA; the launch's last CTA publishes the launch to every rank
        const unsigned long long old = atom_add_acq_rel_gpu(prm.cta_cnt, 1ull);
        if ((old + 1ull) % (static_cast<unsigned long long>(gridDim.x) * gridDim.y) == 0ull)
            for (int q = 0; q < prm.npeer; ++q) red_release_sys_add(prm.peer_cnt[q], 1ull);
    }
}

// Where a combine kernel sends its rows (tensor parallel), as TcParams.
struct TcPush {
    int npeer;
    float *peer_y[8];
    unsigned long long *peer_cnt[8];
    unsigned long long *cta_cnt;
};

// y[c][n] = tree over the KS k-part partials (the top of the slice tree, or
// of a K-shard's subtree); with push.npeer > 0 the rows go to every
// peer_y[q] instead and the launch's last CTA publishes to every rank.
template <int KS>
__global__ void __launch_bounds__(256) mmvq_tc_combine_kernel(const float *__restrict__ part, float *__restrict__ Y,
                                                              int N, int64_t ldy, const TcPush push) {
    pdl_wait();
    pdl_launch_dependents();
    const int64_t total = static_cast<int64_t>(TC_N) * N;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int c = static_cast<int>(i / N), n = static_cast<int>(i % N);
        float a[KS];
#pragma unroll
        for (int k = 0; k < KS; ++k) a[k] = part[(static_cast<int64_t>(k) * TC_N + c) * N + n];
        float y;
        if constexpr (KS == 2) {
            y = __fadd_rn(a[0], a[1]);
        } else if constexpr (KS == 4) {
            y = __fadd_rn(__fadd_rn(a[0], a[1]), __fadd_rn(a[2], a[3]));
        } else {
            y = __fadd_rn(__fadd_rn(__fadd_rn(a[0], a[1]), __fadd_rn(a[2], a[3])),
                          __fadd_rn(__fadd_rn(a[4], a[5]), __fadd_rn(a[6], a[7])));
        }
        if (push.npeer > 0)
            for (int q = 0; q < push.npeer; ++q) push.peer_y[q][c * ldy + n] = y;
        else
            Y[c * ldy + n] = y;
    }
    if (push.npeer > 0) {
        __syncthreads();
        if (threadIdx.x == 0) {
            const unsigned long long old = atom_add_acq_rel_gpu(push.cta_cnt, 1ull);
            if ((old + 1ull) % gridDim.x == 0ull)
                for (int q = 0; q < push.npeer; ++q) red_release_sys_add(push.peer_cnt[q], 1ull);
        }
    }
}

}  // namespace

// cuTensorMapEncodeTiled from the driver, resolved once through the runtime.
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

cudaError_t prepare_mmvq_tc() {
    constexpr int smem = tc_layout().bytes;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    void (*fns[4])(const TcParams, const CUtensorMap) = {mmvq_tc_kernel<1>, mmvq_tc_kernel<2>,
                                                         mmvq_tc_kernel<4>, mmvq_tc_kernel<8>};
    for (int ki = 0; ki < 4; ++ki) {
        e = cudaFuncSetAttribute(fns[ki], cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
    }
    return tensor_map_encoder() ? cudaSuccess : cudaErrorNotSupported;
}

cudaError_t launch_mmvq_tc(const void *w, const void *x_q8, float *y, int64_t N, int64_t K,
                           int64_t ldy, int ks, float *part, int flags, cudaStream_t stream,
                           const TcOpts *opt) {
    const bool shard = opt && opt->part >= 0;          // k-parts [part, part + nparts) of a ks-way split
    const int nparts = shard ? opt->nparts : ks;
    const bool single = shard && nparts == 1;          // one k-part, straight to y
    if (K % QK_K || K <= 0 || N <= 0 || ldy < N || !(ks == 1 || ks == 2 || ks == 4 || ks == 8) ||
        !(nparts == 1 || nparts == 2 || nparts == 4 || nparts == 8) || (nparts > 1 && !part) ||
        (opt && (opt->npeer < 0 || opt->npeer > 8)) || (opt && opt->npeer > 0 && !opt->cta_cnt))
        return cudaErrorInvalidValue;
    TcParams prm = {};
    const int nsb_local = static_cast<int>(K / QK_K);
    prm.nsb_sl = opt && opt->nsb_sl > 0 ? opt->nsb_sl : nsb_local;
    prm.sb_base = opt ? opt->sb_base : 0;
    prm.j_base = shard ? opt->part : 0;
    prm.direct = single ? 1 : 0;
    if (shard && (opt->part + nparts > ks || slice_start(prm.nsb_sl, opt->part * (8 / ks)) != prm.sb_base ||
                  slice_start(prm.nsb_sl, (opt->part + nparts) * (8 / ks)) - prm.sb_base != nsb_local))
        return cudaErrorInvalidValue;  // the shard must be exactly its k-parts' slices
    if (!shard && prm.nsb_sl != nsb_local) return cudaErrorInvalidValue;
    TcPush push = {};
    if (opt && opt->npeer > 0) {
        if (ks > 1 && !shard) return cudaErrorInvalidValue;
        push.npeer = opt->npeer;
        for (int q = 0; q < opt->npeer; ++q) {
            if (!opt->peer_y[q] || !opt->peer_cnt[q]) return cudaErrorInvalidValue;
            push.peer_y[q] = opt->peer_y[q];
            push.peer_cnt[q] = opt->peer_cnt[q];
        }
        push.cta_cnt = opt->cta_cnt;
        if (single || ks == 1) {  // the MMVQ's own epilogue pushes
            prm.npeer = push.npeer;
            for (int q = 0; q < push.npeer; ++q) {
                prm.peer_y[q] = push.peer_y[q];
                prm.peer_cnt[q] = push.peer_cnt[q];
            }
            prm.cta_cnt = push.cta_cnt;
        }
    }
    prm.W = static_cast<const uint8_t *>(w);
    prm.X = static_cast<const uint8_t *>(x_q8);
    prm.Y = y;
    prm.part = part;
    prm.N = static_cast<int>(N);
    prm.nsb = static_cast<int>(K / QK_K);
    prm.ldy = ldy;
    // the weights as a 2-D byte tensor: rows of nsb * 144 bytes, N rows;
    // box = one superblock column (144 B) x 128 rows
    PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
    if (!encode) return cudaErrorNotSupported;
    CUtensorMap wmap;
    const cuuint64_t gdim[2] = {static_cast<cuuint64_t>(K / QK_K) * Q4K_BYTES, static_cast<cuuint64_t>(N)};
    const cuuint64_t gstride[1] = {static_cast<cuuint64_t>(K / QK_K) * Q4K_BYTES};
    const cuuint32_t box[2] = {Q4K_BYTES, TC_M};
    const cuuint32_t estride[2] = {1, 1};
    if (encode(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(w), gdim, gstride, box, estride,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return cudaErrorInvalidValue;
    void (*fn)(const TcParams, const CUtensorMap) = ks == 1 ? mmvq_tc_kernel<1>
                                 : ks == 2 ? mmvq_tc_kernel<2>
                                 : ks == 4 ? mmvq_tc_kernel<4>
                                           : mmvq_tc_kernel<8>;
    constexpr int smem = tc_layout().bytes;
    // the shared-memory opt-in, once per device and k-split (also keeps the
    // call out of any later stream capture)
    static bool attr_set[64][4] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const int ki = ks == 1 ? 0 : ks == 2 ? 1 : ks == 4 ? 2 : 3;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!attr_set[dev][ki]) {
        e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        attr_set[dev][ki] = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>((N + TC_M - 1) / TC_M), static_cast<unsigned>(nparts));
    cfg.blockDim = dim3(TC_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = (flags & MMVQ_PDL) ? 1 : 0;
    e = cudaLaunchKernelEx(&cfg, fn, prm, wmap);
    if (e != cudaSuccess || ks == 1 || single) return e;
    void (*cfn)(const float *, float *, int, int64_t, const TcPush) = nparts == 2 ? mmvq_tc_combine_kernel<2>
                                                                    : nparts == 4 ? mmvq_tc_combine_kernel<4>
                                                                                  : mmvq_tc_combine_kernel<8>;
    cudaLaunchConfig_t c2 = cfg;
    const int64_t total = static_cast<int64_t>(TC_N) * N;
    c2.gridDim = dim3(static_cast<unsigned>(std::min<int64_t>((total + 255) / 256, 148 * 8)));
    c2.blockDim = dim3(256);
    c2.dynamicSmemBytes = 0;
    return cudaLaunchKernelEx(&c2, cfn, static_cast<const float *>(part), y, static_cast<int>(N), ldy, push);
}

}  // namespace abra

ABRA_ERROR_WORD_ACCESSOR(error_word_mmvq_tc)
