// gdn_umma.cuh -- tcgen05 (5th-generation tensor core) helpers for sm_100a:
// shared-memory matrix descriptors for K-major bf16 tiles, the instruction
// descriptor of kind::f16 (bf16 x bf16 -> f32), TMEM allocation, MMA issue,
// commit to an mbarrier, and TMEM <-> register moves.
//
// Tile layout used by every operand (no swizzle, "interleaved" core matrices):
// an R x COLS bf16 tile is stored as core matrices of 8 rows x 8 elements
// (8 x 16 B, rows contiguous), ordered [row/8][col/8]:
//     byte offset(r, c) = (r/8)*(COLS/8)*128 + (c/8)*128 + (r%8)*16 + (c%8)*2
// The same tile serves an MMA either K-major (K along the columns: LBO 128 B
// between the two 16-byte K chunks of a k-step, SBO COLS*16 B between 8-row
// groups, next k-step +256 B) or MN-major (K along the rows: SBO 128 B between
// 8-column groups, LBO COLS*16 B between 8-row groups, next k-step +2*LBO).
//
// Accumulator layout in TMEM (cta_group::1): for M = 128, row m is TMEM lane m;
// for M = 64, row m is lane 32*(m/16) + m%16 (the first 16 lanes of each warp's
// quarter).  Column n of the result is TMEM column base + n (32-bit).
#pragma once

#include <stdint.h>

#include "gdn_ptx.cuh"

namespace gdn {

__device__ __forceinline__ uint32_t umma_tile_off(int r, int k, int KT) {
    return (uint32_t)((r >> 3) * (KT >> 3) * 128 + (k >> 3) * 128 + (r & 7) * 16 + (k & 7) * 2);
}

__device__ __forceinline__ uint64_t umma_desc_raw(uint32_t start, uint32_t lbo, uint32_t sbo) {
    uint64_t d = (uint64_t)((start >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;  // descriptor version of sm_100; base offset 0, layout SWIZZLE_NONE
    return d;
}

// Descriptor of a 128-byte-swizzled K-major tile (the layout a SWIZZLE_128B tensor load writes): rows of 64 bf16
// (128 B) whose 16-byte chunks are permuted by row % 8, 8-row atoms of 1024 B (SBO), atom-aligned base.  A k-step
// of 16 elements within the 64-element row advances the start address by 32 B.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
    uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)1 << 16;          // LBO: not used by swizzled K-major layouts
    d |= (uint64_t)(1024 >> 4) << 32;
    d |= (uint64_t)1 << 46;          // descriptor version of sm_100
    d |= (uint64_t)2 << 61;          // SWIZZLE_128B
    return d;
}

// Descriptor of a tile [R][KT] read K-major (the MMA's K runs along the tile's columns),
// advanced by `kstep` k-steps of 16 elements: LBO 128 B, SBO KT*16 B, step 256 B.
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, int KT, int kstep) {
    return umma_desc_raw(saddr + (uint32_t)kstep * 256u, 128u, (uint32_t)KT * 16u);
}

// Descriptor of a tile [K rows][COLS] read MN-major (the MMA's K runs along the tile's rows,
// M or N along its columns): SBO 128 B between 8-element column groups, LBO COLS*16 B between
// 8-row groups, so one k-step of 16 rows advances 2 * LBO.
__device__ __forceinline__ uint64_t umma_desc_mn(uint32_t saddr, int COLS, int kstep) {
    const uint32_t lbo = (uint32_t)COLS * 16u;
    return umma_desc_raw(saddr + (uint32_t)kstep * 2u * lbo, lbo, 128u);
}

// One k-step of the descriptors above, in units of their 16-byte start-address field: adding
// kstep * KSTEP_K (K-major) or kstep * umma_kstep_mn(COLS) (MN-major) to a kstep-0 descriptor gives
// the kstep descriptor (shared-memory addresses stay below 2^18, so the field cannot carry over).
constexpr uint64_t KSTEP_K = 256u >> 4;
__host__ __device__ constexpr uint64_t umma_kstep_mn(int COLS) { return (uint64_t)(2 * COLS * 16) >> 4; }

// kind::f16 instruction descriptor: A = B = bf16, D = f32, M x N; a_mn / b_mn select an
// MN-major operand (bits 15 / 16), K-major otherwise.
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int M, int N, bool a_mn = false, bool b_mn = false) {
    return (1u << 4) | (1u << 7) | (1u << 10) | (a_mn ? (1u << 15) : 0u) | (b_mn ? (1u << 16) : 0u) |
           ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// D (TMEM) (+)= A (smem) * B (smem)^T for one k-step; issued by a single thread.
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n"
        " .reg .pred p;\n"
        " setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n"
        "}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// D (TMEM) (+)= A (TMEM) * B (smem)^T for one k-step: A is M x 16 bf16 with row m in TMEM lane m and two
// consecutive k values per 32-bit column (8 columns per k-step); issued by a single thread.
__device__ __forceinline__ void umma_bf16_ta(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
    asm volatile(
        "{\n"
        " .reg .pred p;\n"
        " setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n"
        "}\n" ::"r"(d_tmem),
        "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// All MMAs issued so far by this thread arrive on `bar` when complete.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(slot)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }

// 16 consecutive 32-bit TMEM columns of this thread's lane (warp-collective).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r[j]);
}

// tmem_ld16 without the completion wait: several loads can be in flight; call tmem_ld_wait() before the
// registers are used (the values are undefined until then).
__device__ __forceinline__ void tmem_ld16_async(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory"); }

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n" ::"r"(
            taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
        "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
        "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
        "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
        "r"(__float_as_uint(v[15]))
        : "memory");
}

// 8 consecutive 32-bit TMEM columns of this thread's lane from two 16-byte vectors (warp-collective).
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint4& a, const uint4& b) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};\n" ::"r"(taddr), "r"(a.x),
                 "r"(a.y), "r"(a.z), "r"(a.w), "r"(b.x), "r"(b.y), "r"(b.z), "r"(b.w)
                 : "memory");
}

__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory"); }

}  // namespace gdn
