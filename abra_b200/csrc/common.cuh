// common.cuh -- formats, PTX helpers and error reporting shared by the
// abra_b200 sm_100a kernels.
//
// Block layouts are the ggml ones the reference fixes
// (kernels/q4k/q4k_q8_mmvq.cuh:42-57): a Q4_K superblock is 256 weights in
// 144 B (fp16 d, fp16 dmin, 12 B of packed 6-bit scales/mins, 128 B of
// nibbles); a Q8_1 block is 32 int8 in 36 B (fp16 d, fp16 s, 32 x int8).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace abra {

constexpr int QK_K = 256;
constexpr int QK8_1 = 32;
constexpr int Q4K_BYTES = 144;
constexpr int Q81_BYTES = 36;

struct block_q4_K {
    __half d;
    __half dmin;
    uint8_t scales[12];
    uint8_t qs[QK_K / 2];
};
struct block_q8_1 {
    __half d;
    __half s;
    int8_t qs[QK8_1];
};
static_assert(sizeof(block_q4_K) == Q4K_BYTES, "block_q4_K must be 144 bytes");
static_assert(sizeof(block_q8_1) == Q81_BYTES, "block_q8_1 must be 36 bytes");

// Error bits written by kernels into the device error word.
enum : unsigned {
    ERR_WAIT_TIMEOUT = 1u << 0,  // a consumer's wait for staged data gave up
    ERR_FLAG_TIMEOUT = 1u << 1,  // a cross-rank flag wait gave up
    ERR_WAIT_EMPTY = 1u << 2,    // a producer's wait for a free stage gave up
    ERR_GRID_TIMEOUT = 1u << 3,  // a grid-wide barrier of the persistent decode gave up
    ERR_BAD_INDEX = 1u << 4,     // a data-dependent index (a token id) was out of range; its access was skipped
};

// Wall-clock bound of every spin-wait in these kernels (nanoseconds).
constexpr uint64_t WAIT_LIMIT_NS = 1000000000ull;

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Each translation unit has its own error word (internal linkage, so no
// relocatable device code is needed); ABRA_ERROR_WORD_ACCESSOR defines the
// host function that reads and optionally clears it.
static __device__ unsigned int g_abra_device_error = 0;

__device__ __forceinline__ void report_error(unsigned bits) {
    atomicOr(&g_abra_device_error, bits);
}

// ---------------------------------------------------------------- PTX ---
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(
                     smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait: returns false (and reports `err`) if the phase did not
// complete within WAIT_LIMIT_NS of wall time.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity,
                                          unsigned err = ERR_WAIT_TIMEOUT) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 63u) == 0 && globaltimer_ns() - t0 > WAIT_LIMIT_NS) break;
    }
    report_error(err);
    return false;
}
// Bulk (non-tensor) async copy global -> this CTA's shared memory.  Both
// addresses 16-byte aligned, size a multiple of 16.  No multicast.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes,
                                         uint64_t *bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
        "[%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}
// Asynchronous prefetch of [src, src + bytes) into L2 (16-byte aligned,
// bytes a multiple of 16); nothing waits for it.
__device__ __forceinline__ void prefetch_l2_bulk(const void *src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t policy_evict_normal() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}
// Programmatic dependent launch: wait for the preceding grid in the stream
// (no-op when launched without the attribute) / let the next one start.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// dp4a with unsigned bytes in a and signed bytes in b.
__device__ __forceinline__ int dp4a_us(uint32_t a, int b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp4a_ss(int a, int b, int c) { return __dp4a(a, b, c); }

__device__ __forceinline__ float half_lo(uint32_t w) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(w & 0xffffu)));
}
__device__ __forceinline__ float half_hi(uint32_t w) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(w >> 16)));
}

// 6-bit scales and mins of sub-blocks 2p and 2p+1 from the 12 scale bytes
// s0 = bytes 0..3, s1 = bytes 4..7, s2 = bytes 8..11 (same unpacking as the
// reference's get_scale_min_k4, tests/q4k_q8_test.cu:44-52).
__device__ __forceinline__ void scale_min_pair(uint32_t s0, uint32_t s1, uint32_t s2, int p,
                                               int &sc0, int &m0, int &sc1, int &m1) {
    const int sh = 16 * (p & 1);
    const uint32_t a = s0 >> sh, b = s1 >> sh;
    if (p < 2) {
        sc0 = a & 63;
        sc1 = (a >> 8) & 63;
        m0 = b & 63;
        m1 = (b >> 8) & 63;
    } else {
        const uint32_t c = s2 >> sh;
        sc0 = (c & 0xF) | (((a & 0xFF) >> 6) << 4);
        sc1 = ((c >> 8) & 0xF) | ((((a >> 8) & 0xFF) >> 6) << 4);
        m0 = ((c & 0xFF) >> 4) | (((b & 0xFF) >> 6) << 4);
        m1 = (((c >> 8) & 0xFF) >> 4) | ((((b >> 8) & 0xFF) >> 6) << 4);
    }
}

// 6-bit scale and min of sub-block j (get_scale_min_k4, tests/q4k_q8_test.cu:44-52).
__host__ __device__ __forceinline__ void scale_min_one(const uint8_t *q, int j, int &sc, int &m) {
    if (j < 4) {
        sc = q[j] & 63;
        m = q[j + 4] & 63;
    } else {
        sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

// Release add / acquire load at system scope (peer GPUs over NVLink).
__device__ __forceinline__ void red_release_sys_add(unsigned long long *p, unsigned long long v) {
    asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long atom_add_acq_rel_gpu(unsigned long long *p,
                                                                   unsigned long long v) {
    unsigned long long old;
    asm volatile("atom.acq_rel.gpu.global.add.u64 %0, [%1], %2;" : "=l"(old) : "l"(p), "l"(v) : "memory");
    return old;
}
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ unsigned long long ld_relaxed_sys(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Order-preserving 64-bit key of (value, row): the float's bits mapped to an
// unsigned order in the high word, ~row in the low word, so the largest key
// is the largest value and, among equal values, the lowest row.
__device__ __forceinline__ unsigned long long argmax_key(float v, int row) {
    unsigned u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return (static_cast<unsigned long long>(u) << 32) | (0xFFFFFFFFu - static_cast<unsigned>(row));
}

// Spins until *cnt >= target or WAIT_LIMIT_NS passes (then flags
// ERR_FLAG_TIMEOUT and returns false); polls with relaxed loads and acquires
// once at the end.  Once a cross-rank wait of this translation unit has
// given up, later ones return at once: a rank that is gone costs one time
// limit, not one per wait.
__device__ __forceinline__ bool wait_count(const unsigned long long *cnt, unsigned long long target) {
    if (ld_acquire_sys(cnt) >= target) return true;
    if (*static_cast<volatile unsigned *>(&g_abra_device_error) & ERR_FLAG_TIMEOUT) return false;
    const unsigned long long t0 = globaltimer_ns();
    for (unsigned i = 1;; ++i) {
        if (ld_relaxed_sys(cnt) >= target) return ld_acquire_sys(cnt) >= target;
        if ((i & 255u) == 0 && globaltimer_ns() - t0 > WAIT_LIMIT_NS) {
            report_error(ERR_FLAG_TIMEOUT);
            return false;
        }
    }
}

// Up to eight fp32 partial deltas summed in a fixed tree before a residual
// add: G = 1: p0; 2: p0+p1; 4: (p0+p1)+(p2+p3); 8: three levels.  G = 0: none.
// With p_g the K-shard partial of rank g (shards on canonical slice
// boundaries), the tree is the top of the unsharded slice tree.  Loads go
// through L2 (.cg): the partials may have been written by peer GPUs.
struct DeltaSet {
    const float *p[8];
    int G;
};

__device__ __forceinline__ float delta_tree(const DeltaSet &ds, int64_t i) {
    const float *const *p = ds.p;
    switch (ds.G) {
        case 1: return __ldcg(p[0] + i);
        case 2: return __fadd_rn(__ldcg(p[0] + i), __ldcg(p[1] + i));
        case 4:
            return __fadd_rn(__fadd_rn(__ldcg(p[0] + i), __ldcg(p[1] + i)),
                             __fadd_rn(__ldcg(p[2] + i), __ldcg(p[3] + i)));
        default:
            return __fadd_rn(__fadd_rn(__fadd_rn(__ldcg(p[0] + i), __ldcg(p[1] + i)),
                                       __fadd_rn(__ldcg(p[2] + i), __ldcg(p[3] + i))),
                             __fadd_rn(__fadd_rn(__ldcg(p[4] + i), __ldcg(p[5] + i)),
                                       __fadd_rn(__ldcg(p[6] + i), __ldcg(p[7] + i))));
    }
}

// Canonical K-slices: eight contiguous superblock ranges, the first nsb % 8
// one superblock longer.  Slice i starts at slice_start(nsb, i).
__host__ __device__ __forceinline__ int slice_start(int nsb, int i) {
    const int q = nsb / 8, r = nsb % 8;
    return i * q + (i < r ? i : r);
}

// ---------------------------------------------------------------- exp ---
// Cody & Waite range reduction x = k ln2 + r (ln2 split into a 16-bit head
// and a tail), e^r by the degree-7 Taylor polynomial in Horner form, then
// scaling by 2^k.  Every step is one IEEE fp32 operation, mirrored operation
// for operation by the CPU oracle (orc_expf), so both return the same bits.
__device__ __forceinline__ float pow2i(int k) { return __int_as_float((k + 127) << 23); }

__device__ __forceinline__ float abra_expf(float x) {
    if (x != x) return x;
    if (x > 88.75f) return __int_as_float(0x7f800000);
    if (x < -104.0f) return 0.0f;
    const float kf = rintf(__fmul_rn(x, 0x1.715476p+0f));
    float r = __fmaf_rn(kf, -0x1.62e400p-1f, x);
    r = __fmaf_rn(kf, -0x1.7f7d1cp-20f, r);
    float p = 0x1.a01a02p-13f;
    p = __fmaf_rn(p, r, 0x1.6c16c2p-10f);
    p = __fmaf_rn(p, r, 0x1.111112p-7f);
    p = __fmaf_rn(p, r, 0x1.555556p-5f);
    p = __fmaf_rn(p, r, 0x1.555556p-3f);
    p = __fmaf_rn(p, r, 0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    const int k = static_cast<int>(kf);
    if (k > 127) return __fmul_rn(__fmul_rn(p, pow2i(127)), pow2i(k - 127));
    if (k < -126) return __fmul_rn(__fmul_rn(p, pow2i(k + 64)), pow2i(-64));
    return __fmul_rn(p, pow2i(k));
}

// silu(g) = g / (1 + exp(-g)), the formula of ggml's silu.
__device__ __forceinline__ float abra_silu(float g) {
    return __fdiv_rn(g, __fadd_rn(1.0f, abra_expf(-g)));
}

// ---------------------------------------------------------- generator ---
__host__ __device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
__host__ __device__ __forceinline__ uint64_t stream_key(uint64_t seed, uint64_t tensor_id) {
    return mix64(seed + 0x9E3779B97F4A7C15ull) ^ mix64(tensor_id * 0xD1B54A32D192ED03ull + 1ull);
}
__host__ __device__ __forceinline__ uint64_t stream_word(uint64_t key, uint64_t i) {
    return mix64(key + (i + 1ull) * 0x9E3779B97F4A7C15ull);
}
__device__ __forceinline__ float unit24(uint64_t bits24) {
    return __fmul_rn(static_cast<float>(static_cast<uint32_t>(bits24)), 5.9604644775390625e-08f);
}

}  // namespace abra

namespace abra {
using ErrorWordFn = cudaError_t (*)(unsigned *value, bool clear);
// Host-side registry of the per-translation-unit error words (api.cu).
int register_error_word(ErrorWordFn fn);
}  // namespace abra

#define ABRA_ERROR_WORD_ACCESSOR(fname)                                              \
    namespace abra {                                                                 \
    cudaError_t fname(unsigned *value, bool clear) {                                 \
        unsigned v = 0;                                                              \
        cudaError_t e = cudaMemcpyFromSymbol(&v, g_abra_device_error, sizeof v);     \
        if (e != cudaSuccess) return e;                                              \
        if (clear && v) {                                                            \
            const unsigned z = 0;                                                    \
            e = cudaMemcpyToSymbol(g_abra_device_error, &z, sizeof z);               \
            if (e != cudaSuccess) return e;                                          \
        }                                                                            \
        *value |= v;                                                                 \
        return cudaSuccess;                                                          \
    }                                                                                \
    static const int fname##_registered = register_error_word(fname);               \
    }
