// tc_common.cuh -- 5th-generation tensor core (tcgen05) helpers for sm_100a:
// tensor-memory allocation, the kind::i8 MMA with shared-memory operand
// descriptors, commit to an mbarrier, tensor-memory loads and the fences
// between them.  Formats follow the PTX ISA's tcgen05 descriptors:
//
// Shared-memory matrix descriptor (64 bit), no swizzle, K-major:
//   [0,14)  start address >> 4     [16,30) leading-dimension byte offset >> 4
//   [32,46) stride-dimension byte offset >> 4   [46,48) version = 1
//   [49,52) base offset = 0        [52]    LBO mode = 0   [61,64) layout = 0
// The canonical K-major no-swizzle operand is built of 8-row x 16-byte
// "core matrices" (128 contiguous bytes, row r at +16 r): the two 16-byte
// halves of a K = 32-byte slab sit LBO apart, consecutive 8-row groups SBO
// apart.
//
// Instruction descriptor (32 bit) of kind::i8: [4,6) D format (2 = s32),
// [7,10) A format (0 = u8, 1 = s8), [10,13) B format, [15] A major, [16] B
// major (0 = K), [17,23) N >> 3, [24,29) M >> 4.
#pragma once
#include <stdint.h>

#include "common.cuh"

namespace abra {

__host__ __device__ constexpr uint32_t tc_idesc_i8(int M, int N, bool a_signed, bool b_signed) {
    return (2u << 4) | ((a_signed ? 1u : 0u) << 7) | ((b_signed ? 1u : 0u) << 10) |
           (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

__device__ __forceinline__ uint64_t tc_smem_desc(const void *smem, uint32_t lbo_bytes,
                                                 uint32_t sbo_bytes) {
    const uint64_t addr = smem_u32(smem);
    return ((addr >> 4) & 0x3FFFull) | (static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFF) << 16) |
           (static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFF) << 32) | (1ull << 46);
}

// Allocation by one whole warp; the TMEM address is written to *holder.
__device__ __forceinline__ void tmem_alloc(uint32_t *holder, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(holder)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// D[tmem] (=|+=) A[smem] x B[smem], one elected thread.
__device__ __forceinline__ void tc_mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                          uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}
// The mbarrier gets one arrival once every prior tcgen05 op of this thread completed.
__device__ __forceinline__ void tc_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Generic-proxy shared-memory writes made visible to the tensor core (async proxy).
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Thread i of the warp reads TMEM lane (taddr.lane + i), 8 consecutive columns.
__device__ __forceinline__ void tmem_ld_x8(uint32_t taddr, int32_t (&v)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
                   "=r"(v[7])
                 : "r"(taddr)
                 : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

}  // namespace abra
