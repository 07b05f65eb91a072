// umma.cuh - thin wrappers over the sm_100a tensor-core (tcgen05) instructions
// used by the block-scaled GEMM: TMEM allocation, shared-memory matrix
// descriptors, the kind::mxf8f6f4 block-scaled MMA, the scale-factor copy
// into TMEM, commit-to-mbarrier and the TMEM -> register load.
//
// Layout facts this file relies on (PTX ISA, tcgen05 chapter):
//  - shared-memory matrix descriptor (64 bit): start address >> 4 in [0,14),
//    leading byte offset >> 4 in [16,30), stride byte offset >> 4 in [32,46),
//    descriptor version 1 in [46,48), base offset in [49,52), swizzle mode in
//    [61,64) (0 none, 2 = 128-byte swizzle);
//  - K-major operand with 128-byte swizzle: rows of 128 bytes, 8-row groups
//    1024 bytes apart (stride byte offset 1024); the K = 32 sub-tile k of a
//    128-byte row starts 32 * k bytes further;
//  - block-scaled instruction descriptor (32 bit): B scale id [4,6), A format
//    [7,10), B format [10,13), A/B major bits 15/16 (0 = K-major), N >> 3 in
//    [17,23), scale type bit 23 (1 = UE8M0), M >> 4 in [24,29), A scale id
//    [29,31); formats: E4M3 = 0, E2M1 = 5;
//  - scale factors in TMEM: for an M = 128 (or N <= 128) operand, row m uses
//    lane (m mod 32) of every lane quarter, column (m / 32) of the scale block,
//    and byte k (the scale id) selects the K = 32 block inside a 128-wide K
//    chunk. tcgen05.cp .32x128b.warpx4 fills exactly that from a 512-byte
//    shared-memory block laid out as byte (m mod 32) * 16 + (m / 32) * 4 + k;
//  - FP4 operands of kind::mxf8f6f4 occupy one byte slot per element in shared
//    memory (16 values in the low 8 bytes of every 16 bytes), which the TMA
//    data type 16U4_ALIGN16B produces from the packed global layout.
#pragma once

#include <stdint.h>

#include "common.cuh"

namespace dsv4cu {
namespace umma {

DSV4CU_DEV uint32_t saddr(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

// Whole warp; writes the TMEM base address into *holder (shared memory).
DSV4CU_DEV void tmem_alloc(uint32_t *holder, uint32_t ncols)
{
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(saddr(holder)),
                 "r"(ncols)
                 : "memory");
}
DSV4CU_DEV void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory"); }
DSV4CU_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols)
{
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

DSV4CU_DEV void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
DSV4CU_DEV void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Arrive once on `bar` when every tcgen05 operation this thread issued so far
// has completed.
DSV4CU_DEV void commit(uint64_t *bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(saddr(bar))
                 : "memory");
}

// 32 rows x 16 bytes of scale factors, replicated into all four lane quarters.
DSV4CU_DEV void cp_sf(uint32_t taddr, uint64_t sdesc)
{
    asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

// D[tmem] (+)= (A * SFA) x (B * SFB)^T for one M x N x 32 step.
DSV4CU_DEV void mma_mx(uint32_t d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate, uint32_t sfa,
                       uint32_t sfb)
{
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}"
                 ::"r"(d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa), "r"(sfb)
                 : "memory");
}

// 32 lanes x 8 consecutive fp32 columns (this warp's lane quarter).
DSV4CU_DEV void ld_x8(uint32_t taddr, float (&v)[8])
{
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr)
                 : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 8; i++) v[i] = __uint_as_float(r[i]);
}

// K-major operand tile, 128-byte rows, 128-byte swizzle, 1024-byte aligned
// tile base; `p` may point k * 32 bytes into the first row.
DSV4CU_DEV uint64_t desc_sw128(const void *p)
{
    const uint64_t a = saddr(p);
    return ((a >> 4) & 0x3FFFull) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
}

// 32 rows x 16 bytes, rows contiguous (no swizzle): 8-row core matrices are
// 128 bytes apart.
DSV4CU_DEV uint64_t desc_sf(const void *p)
{
    const uint64_t a = saddr(p);
    return ((a >> 4) & 0x3FFFull) | (1ull << 16) | ((uint64_t)(128 >> 4) << 32) | (1ull << 46);
}

constexpr uint32_t FMT_E4M3 = 0, FMT_E2M1 = 5;

// Block-scaled instruction descriptor, scale ids 0 (OR in (k << 4) | (k << 29)).
__host__ __device__ constexpr uint32_t idesc_mx(uint32_t afmt, uint32_t bfmt, int M, int N)
{
    return (afmt << 7) | (bfmt << 10) | ((uint32_t)(N >> 3) << 17) | (1u << 23) | ((uint32_t)(M >> 4) << 24);
}

}  // namespace umma
}  // namespace dsv4cu
