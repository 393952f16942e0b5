// tc_common.cuh -- 5th-generation tensor core (tcgen05) helpers for sm_100a:
// tensor-memory (TMEM) allocation, register <-> TMEM moves, the shared-memory
// matrix descriptor, the instruction descriptor of the integer MMA, MMA issue
// and completion tracking.  Inline PTX, written from the PTX ISA's
// description of these instructions.
//
// TMEM addresses: bits 31..16 lane, 15..0 column (32-bit columns).  A warp
// reaches the 32 lanes 32 * (warp % 4) .. + 31 with the .32x32b shapes.
#pragma once
#include "device_common.cuh"

namespace chpe {
namespace tc {

// Allocate ncols TMEM columns (a power of two >= 32) for this CTA; one warp
// executes it, and the base address lands in *dst (shared memory).
CHPE_DEV void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)),
               "r"(ncols)
               : "memory");
}
CHPE_DEV void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
CHPE_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// Ordering of tcgen05 operations around thread synchronisation.
CHPE_DEV void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
CHPE_DEV void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 16 consecutive 32-bit columns of this thread's lane <- v.
CHPE_DEV void st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
      "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}
CHPE_DEV void st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// v <- 16 consecutive 32-bit columns of this thread's lane.
CHPE_DEV void ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr)
      : "memory");
}
CHPE_DEV void ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Instruction descriptor of tcgen05.mma .kind::i8: D s32, A u8, B s8, both
// K-major, dense, M x N (M 64 or 128; N 8, or 16..256 in steps of 16).
__host__ __device__ constexpr uint32_t idesc_i8_u8s8(uint32_t M, uint32_t N) {
  return (2u << 4)            // D format: s32
         | (0u << 7)          // A: unsigned 8-bit
         | (1u << 10)         // B: signed 8-bit
         | ((N >> 3) << 17)   // N / 8
         | ((M >> 4) << 24);  // M / 16
}

// Shared-memory matrix descriptor, K-major, no swizzle: 8-row x 16-byte core
// matrices (128 contiguous bytes each); lbo = byte distance between the two
// core matrices along K, sbo = between core matrices 8 rows apart.
CHPE_DEV uint64_t smem_desc_kmajor(const void* base, uint32_t lbo, uint32_t sbo) {
  const uint64_t a = (uint64_t)((smem_u32(base) >> 4) & 0x3FFFu);
  return a | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) | ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) |
         (1ull << 46);  // descriptor version of sm_100; base offset 0, no swizzle
}

// D (TMEM) [+]= A (TMEM) x B (shared memory), one elected thread.
CHPE_DEV void mma_i8_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on `bar` when every MMA this thread issued so far has completed.
CHPE_DEV void commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// Arrive (count 1) on an mbarrier from a thread.
CHPE_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

}  // namespace tc
}  // namespace chpe
