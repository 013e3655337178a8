// lane_gemv.cuh -- the lane-per-superblock Q4_K x Q8_1 arithmetic shared by
// the persistent decode kernel (decode_persistent.cu) and the standalone
// lane-mapped MMVQ (mmvq_lane.cu).
//
// A lane computes whole superblock values (all eight sub-blocks of one
// superblock of one row) against an activation record staged in shared
// memory; the values of a unit of rows meet in a per-warp buffer, and eight
// lanes per row form the eight canonical K-slice sums and their fixed tree.
// The fp32 order is the canonical one of mmvq_q4k_kernel and the CPU oracle
// (oracle/q4k_oracle.c), so results are bit-identical to both.
#pragma once

#include "common.cuh"

namespace abra {

// Activation record of one superblock in shared memory: its 256 int8 quants,
// then d8[8] and A[8] = d8 * sum(q) per 32-block (fp32), padded to 336 bytes
// = 21 16-byte chunks, so eight consecutive superblocks' records start in
// eight distinct bank groups.
constexpr int LG_AREC = 336;

// Value of one superblock of NMAT weight rows against the staged activation
// record: the arithmetic of vec_dot_q4_K_q8_1 in the canonical order of
// mmvq_q4k_kernel (exact int32 sub-block dots by dp4a, t_s = d8_s *
// float(P_s * sc_s), u_s = A_s * float(m_s), S = ((0+1)+(2+3))+((4+5)+(6+7)),
// fmaf(d, S_t, -(dmin * S_u))), all eight sub-blocks in one lane.
template <int NMAT>
__device__ __forceinline__ void pk_sb_value(const uint8_t *const (&wsb)[NMAT], const uint8_t *arec,
                                            float (&v)[NMAT]) {
    uint4 hdr[NMAT];
#pragma unroll
    for (int m = 0; m < NMAT; ++m) hdr[m] = *reinterpret_cast<const uint4 *>(wsb[m]);
    float t[NMAT][8], u[NMAT][8];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const float2 d8 = *reinterpret_cast<const float2 *>(arec + 256 + 8 * q);
        const float2 A = *reinterpret_cast<const float2 *>(arec + 288 + 8 * q);
        const uint4 a0 = *reinterpret_cast<const uint4 *>(arec + 64 * q);
        const uint4 a1 = *reinterpret_cast<const uint4 *>(arec + 64 * q + 16);
        const uint4 a2 = *reinterpret_cast<const uint4 *>(arec + 64 * q + 32);
        const uint4 a3 = *reinterpret_cast<const uint4 *>(arec + 64 * q + 48);
#pragma unroll
        for (int m = 0; m < NMAT; ++m) {
            int sc0, m0, sc1, m1;
            scale_min_pair(hdr[m].y, hdr[m].z, hdr[m].w, q, sc0, m0, sc1, m1);
            const uint4 qa = *reinterpret_cast<const uint4 *>(wsb[m] + 16 + 32 * q);
            const uint4 qb = *reinterpret_cast<const uint4 *>(wsb[m] + 32 + 32 * q);
            int s0 = 0, s1 = 0;
            s0 = dp4a_ss(static_cast<int>(qa.x & 0x0F0F0F0Fu), static_cast<int>(a0.x), s0);
            s1 = dp4a_us(qa.x & 0xF0F0F0F0u, static_cast<int>(a2.x), s1);
            s0 = dp4a_ss(static_cast<int>(qa.y & 0x0F0F0F0Fu), static_cast<int>(a0.y), s0);
            s1 = dp4a_us(qa.y & 0xF0F0F0F0u, static_cast<int>(a2.y), s1);
            s0 = dp4a_ss(static_cast<int>(qa.z & 0x0F0F0F0Fu), static_cast<int>(a0.z), s0);
            s1 = dp4a_us(qa.z & 0xF0F0F0F0u, static_cast<int>(a2.z), s1);
            s0 = dp4a_ss(static_cast<int>(qa.w & 0x0F0F0F0Fu), static_cast<int>(a0.w), s0);
            s1 = dp4a_us(qa.w & 0xF0F0F0F0u, static_cast<int>(a2.w), s1);
            s0 = dp4a_ss(static_cast<int>(qb.x & 0x0F0F0F0Fu), static_cast<int>(a1.x), s0);
            s1 = dp4a_us(qb.x & 0xF0F0F0F0u, static_cast<int>(a3.x), s1);
            s0 = dp4a_ss(static_cast<int>(qb.y & 0x0F0F0F0Fu), static_cast<int>(a1.y), s0);
            s1 = dp4a_us(qb.y & 0xF0F0F0F0u, static_cast<int>(a3.y), s1);
            s0 = dp4a_ss(static_cast<int>(qb.z & 0x0F0F0F0Fu), static_cast<int>(a1.z), s0);
            s1 = dp4a_us(qb.z & 0xF0F0F0F0u, static_cast<int>(a3.z), s1);
            s0 = dp4a_ss(static_cast<int>(qb.w & 0x0F0F0F0Fu), static_cast<int>(a1.w), s0);
            s1 = dp4a_us(qb.w & 0xF0F0F0F0u, static_cast<int>(a3.w), s1);
            s1 >>= 4;  // exact: the masked high nibbles carry a factor of 16
            t[m][2 * q] = __fmul_rn(d8.x, __int2float_rn(s0 * sc0));
            t[m][2 * q + 1] = __fmul_rn(d8.y, __int2float_rn(s1 * sc1));
            u[m][2 * q] = __fmul_rn(A.x, static_cast<float>(m0));
            u[m][2 * q + 1] = __fmul_rn(A.y, static_cast<float>(m1));
        }
    }
#pragma unroll
    for (int m = 0; m < NMAT; ++m) {
        const float St = __fadd_rn(__fadd_rn(__fadd_rn(t[m][0], t[m][1]), __fadd_rn(t[m][2], t[m][3])),
                                   __fadd_rn(__fadd_rn(t[m][4], t[m][5]), __fadd_rn(t[m][6], t[m][7])));
        const float Su = __fadd_rn(__fadd_rn(__fadd_rn(u[m][0], u[m][1]), __fadd_rn(u[m][2], u[m][3])),
                                   __fadd_rn(__fadd_rn(u[m][4], u[m][5]), __fadd_rn(u[m][6], u[m][7])));
        const float d = half_lo(hdr[m].x), dmin = half_hi(hdr[m].x);
        v[m] = __fmaf_rn(d, St, -__fmul_rn(dmin, Su));
    }
}

// The reference's 148-byte packed superblock (kernels/q4k/abra-packed-q4.cuh:
// 3-8): fp16 d and dmin, then for each pair j of sub-blocks one 32-bit word of
// bytes [sc_2j, sc_2j+1, m_2j, m_2j+1] (the 6-bit scales and mins unpacked),
// then the 128 bytes of nibbles.  Rows of packed superblocks are only 4-byte
// aligned, so everything is read as 32-bit words.
constexpr int LG_PACKED_BYTES = 148;

// pk_sb_value on packed superblocks: the same integers (the unpacked bytes
// equal scale_min_pair's), the same fp32 operations in the same order.
template <int NMAT>
__device__ __forceinline__ void pk_sb_value_packed(const uint8_t *const (&wsb)[NMAT], const uint8_t *arec,
                                                   float (&v)[NMAT]) {
    uint32_t dm[NMAT];
#pragma unroll
    for (int m = 0; m < NMAT; ++m) dm[m] = *reinterpret_cast<const uint32_t *>(wsb[m]);
    float t[NMAT][8], u[NMAT][8];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const float2 d8 = *reinterpret_cast<const float2 *>(arec + 256 + 8 * q);
        const float2 A = *reinterpret_cast<const float2 *>(arec + 288 + 8 * q);
        const uint4 a0 = *reinterpret_cast<const uint4 *>(arec + 64 * q);
        const uint4 a1 = *reinterpret_cast<const uint4 *>(arec + 64 * q + 16);
        const uint4 a2 = *reinterpret_cast<const uint4 *>(arec + 64 * q + 32);
        const uint4 a3 = *reinterpret_cast<const uint4 *>(arec + 64 * q + 48);
#pragma unroll
        for (int m = 0; m < NMAT; ++m) {
            const uint32_t *w32 = reinterpret_cast<const uint32_t *>(wsb[m]);
            const uint32_t smp = w32[1 + q];
            const int sc0 = smp & 0xff, sc1 = (smp >> 8) & 0xff, m0 = (smp >> 16) & 0xff, m1 = smp >> 24;
            uint32_t qw[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) qw[k] = w32[5 + 8 * q + k];
            const int lo[8] = {static_cast<int>(a0.x), static_cast<int>(a0.y), static_cast<int>(a0.z),
                               static_cast<int>(a0.w), static_cast<int>(a1.x), static_cast<int>(a1.y),
                               static_cast<int>(a1.z), static_cast<int>(a1.w)};
            const int hi[8] = {static_cast<int>(a2.x), static_cast<int>(a2.y), static_cast<int>(a2.z),
                               static_cast<int>(a2.w), static_cast<int>(a3.x), static_cast<int>(a3.y),
                               static_cast<int>(a3.z), static_cast<int>(a3.w)};
            int s0 = 0, s1 = 0;
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                s0 = dp4a_ss(static_cast<int>(qw[k] & 0x0F0F0F0Fu), lo[k], s0);
                s1 = dp4a_us(qw[k] & 0xF0F0F0F0u, hi[k], s1);
            }
            s1 >>= 4;  // exact: the masked high nibbles carry a factor of 16
            t[m][2 * q] = __fmul_rn(d8.x, __int2float_rn(s0 * sc0));
            t[m][2 * q + 1] = __fmul_rn(d8.y, __int2float_rn(s1 * sc1));
            u[m][2 * q] = __fmul_rn(A.x, static_cast<float>(m0));
            u[m][2 * q + 1] = __fmul_rn(A.y, static_cast<float>(m1));
        }
    }
#pragma unroll
    for (int m = 0; m < NMAT; ++m) {
        const float St = __fadd_rn(__fadd_rn(__fadd_rn(t[m][0], t[m][1]), __fadd_rn(t[m][2], t[m][3])),
                                   __fadd_rn(__fadd_rn(t[m][4], t[m][5]), __fadd_rn(t[m][6], t[m][7])));
        const float Su = __fadd_rn(__fadd_rn(__fadd_rn(u[m][0], u[m][1]), __fadd_rn(u[m][2], u[m][3])),
                                   __fadd_rn(__fadd_rn(u[m][4], u[m][5]), __fadd_rn(u[m][6], u[m][7])));
        const float d = half_lo(dm[m]), dmin = half_hi(dm[m]);
        v[m] = __fmaf_rn(d, St, -__fmul_rn(dmin, Su));
    }
}

// Sum of canonical K-slice i of a row from its staged superblock values
// (sequential within the slice).
__device__ __forceinline__ float pk_slice_sum(const float *vrow, int nsb, int i) {
    const int b0 = slice_start(nsb, i), b1 = slice_start(nsb, i + 1);
    float acc = 0.0f;
    for (int b = b0; b < b1; ++b) acc = b == b0 ? vrow[b] : __fadd_rn(acc, vrow[b]);
    return acc;
}

// The fixed tree over eight slice sums held by lanes 8g .. 8g+7 (slice i in
// lane 8g + i): xor 1, 2, 4 give ((s0+s1)+(s2+s3))+((s4+s5)+(s6+s7)) in every
// lane of the group (IEEE addition commutes, so both partners form the same
// bits).
__device__ __forceinline__ float pk_slice_tree(float v) {
    v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 1));
    v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 2));
    return __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 4));
}

}  // namespace abra
