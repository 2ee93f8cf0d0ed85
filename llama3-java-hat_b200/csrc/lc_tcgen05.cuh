// lc_tcgen05.cuh -- PTX wrappers for the 5th-generation tensor cores of
// sm_100a: tensor-memory (TMEM) allocation, tcgen05.mma with shared-memory
// operand descriptors, completion through mbarriers, TMEM loads, and the
// fences that order tcgen05 work against thread synchronisation.
//
// Operand layout used throughout: K-major, no swizzle.  A "core matrix" is 8
// rows x 16 bytes (8 halves) stored as 128 contiguous bytes; the core
// matrices of one operand tile sit 128 B apart along K (leading byte offset)
// and 1024 B apart along M / N (stride byte offset), i.e. a tile of R rows x
// 64 columns is [R/8 row groups][8 column octets][8 rows][8 halves].  This is
// the order of the tiled weight layout (lc_internal.h) and of the pre-split
// activations, so a TMA box of either lands in shared memory ready for the
// MMA, without a swizzle.
#pragma once

#include "lc_common.cuh"

namespace lc {

// Shared-memory matrix descriptor (tcgen05 "matrix descriptor"): start
// address >> 4 in bits 0-13, leading byte offset >> 4 in 16-29, stride byte
// offset >> 4 in 32-45, descriptor version 1 in bits 46-47, base offset 0,
// absolute leading-offset mode 0, layout type 0 (no swizzle) in bits 61-63.
LC_DEV uint64_t tc_desc_kmajor(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
    return (uint64_t)((smem_addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

// Instruction descriptor of kind::f16 with f16 A and B (formats 0), fp32
// accumulation (D format 1, bits 4-5), both operands K-major (bits 15, 16 =
// 0), N >> 3 in bits 17-22 and M >> 4 in bits 24-28.
__host__ __device__ constexpr uint32_t tc_idesc_f16_f32(int M, int N) {
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// Tiled TMA loads (cp.async.bulk.tensor, no multicast) of one box into this
// CTA's shared memory, completion as transaction bytes on `bar`.  `tmap` is
// the generic address of a __grid_constant__ CUtensorMap; the innermost
// coordinate c0 is 0 at every call site (the box spans the whole 128-byte
// inner dimension), so it is always 16-byte aligned.
LC_DEV void tma_load_4d(void* dst, const void* tmap, int c0, int c1, int c2, int c3, uint64_t* bar,
                        uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(smem_u32(dst)),
        "l"(tmap), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

LC_DEV void tma_load_3d(void* dst, const void* tmap, int c0, int c1, int c2, uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_u32(dst)),
        "l"(tmap), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// TMEM allocation by one full warp: the base address is written to *slot.
// ncols is a power of two >= 32.
LC_DEV void tmem_alloc(uint32_t* slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
                 "r"(ncols)
                 : "memory");
}

LC_DEV void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory"); }

LC_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

LC_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
LC_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Generic-proxy shared-memory writes become visible to the tensor cores
// (async proxy) after this fence and a synchronisation.
LC_DEV void fence_async_shared() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// D[tmem] (+)= A[adesc] * B[bdesc]^T, one thread issues; accumulate != 0
// adds to D, 0 overwrites it.
LC_DEV void tc_mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// 128 TMEM lanes x 256 bits (8 columns from taddr) from the shared-memory
// matrix of descriptor `desc` (row r -> lane r); asynchronous, ordered with
// the thread's other tcgen05 operations, tracked by tc_commit.
LC_DEV void tc_cp_128x256b(uint32_t taddr, uint64_t desc) {
    asm volatile("tcgen05.cp.cta_group::1.128x256b [%0], %1;" ::"r"(taddr), "l"(desc) : "memory");
}

// The mbarrier receives one arrival when every tcgen05 operation this thread
// issued before has completed.
LC_DEV void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// 16 consecutive 32-bit columns of the warp's 32 TMEM lanes (thread i: lane
// base + i).  The values are valid after tmem_wait_ld, which takes them as
// operands so no use can be scheduled before it.
LC_DEV void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
}

LC_DEV void tmem_wait_ld(uint32_t (&v)[16]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]), "+r"(v[6]), "+r"(v[7]),
                   "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]), "+r"(v[12]), "+r"(v[13]), "+r"(v[14]),
                   "+r"(v[15])
                 :
                 : "memory");
}

// ---------------------------------------------- hi / lo split of operand A --
//
// An fp32 activation row becomes two f16 rows under a power-of-two row scale
// 2^e chosen so that max |a| * 2^e lies in [2^14, 2^15): hi = f16(a * 2^e),
// lo = f16(a * 2^e - hi).  The subtraction is exact (hi is a * 2^e rounded to
// 11 bits), hi + lo = a * 2^e to 2^-22 relative, and both stay in f16 range.
LC_DEV int split_row_exp(float m) {
    if (!(m > 0.0f)) return 0;
    int e = 14 - (((__float_as_int(m) >> 23) & 0xff) - 127);
    return e < -126 ? -126 : (e > 126 ? 126 : e);
}

LC_DEV float pow2f(int e) { return __int_as_float((127 + e) << 23); }

// Eight scaled values -> the hi and lo 16-byte rows of one core matrix.
LC_DEV void split_octet(const float (&f)[8], uint4& hi, uint4& lo) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const __half2 hh = __floats2half2_rn(f[2 * k], f[2 * k + 1]);
        const float2 hf = __half22float2(hh);
        const __half2 ll = __floats2half2_rn(f[2 * k] - hf.x, f[2 * k + 1] - hf.y);
        h[k] = *reinterpret_cast<const uint32_t*>(&hh);
        l[k] = *reinterpret_cast<const uint32_t*>(&ll);
    }
    hi = make_uint4(h[0], h[1], h[2], h[3]);
    lo = make_uint4(l[0], l[1], l[2], l[3]);
}

// Byte offset of octet o of activation row s in the pre-split layout with K
// columns: row group s / 4, MMA row 2 (s % 4) (hi; +16 bytes: lo).
__host__ __device__ inline size_t split_offset(int s, int o, int K) {
    return ((size_t)(s >> 2) * (size_t)(K >> 3) + (size_t)o) * 128 + (size_t)(2 * (s & 3)) * 16;
}

}  // namespace lc
