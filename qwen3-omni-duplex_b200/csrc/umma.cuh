// Fifth-generation tensor core (tcgen05) helpers: tensor-memory allocation, register
// <-> tensor-memory copies, the MMA with A in tensor memory and B in shared memory, its
// completion through an mbarrier, and the two descriptors it takes.  Hand-written
// inline PTX of documented instructions (PTX ISA 8.6+, sm_100a).
//
// Layouts used here (cta_group::1, M = 128):
//   A [128 x K] 16-bit, tensor memory: lane m = row m, 32-bit column c = the pair
//     (k = 2c low half, k = 2c + 1 high half); one MMA (K = 16) reads 8 columns.
//   B [N x K] 16-bit, shared memory, K-major without swizzle: core matrices of 8 rows
//     x 16 bytes (8 values), rows 16 bytes apart; element (n, k) of a tile laid out as
//     [k / 8][n][k % 8] sits at ((k / 8) * N + n) * 16 + (k % 8) * 2, so the two K
//     halves of one MMA are N * 16 bytes apart (leading byte offset) and consecutive
//     8-row groups 128 bytes apart (stride byte offset).
//   D [128 x N] fp32, tensor memory: lane m = row m, column n.
#pragma once

#include "common.cuh"

namespace duplex {

// tensor-memory address of (lane, column)
DEVI uint32_t tmem_addr(uint32_t base, uint32_t lane, uint32_t col) { return base + (lane << 16) + col; }

// One warp: allocate `ncols` (power of two >= 32) columns; the address lands in *dst.
template <int NCOLS>
DEVI void tmem_alloc(uint32_t* dst) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)),
               "n"(NCOLS)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

template <int NCOLS>
DEVI void tmem_dealloc(uint32_t base) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(base), "n"(NCOLS) : "memory");
}

DEVI void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
DEVI void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
DEVI void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
DEVI void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Warp store: thread i writes 8 consecutive 32-bit columns of lane (lane base + i).
DEVI void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
               "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}

// Warp load: thread i reads 16 consecutive 32-bit columns of lane (lane base + i).
DEVI void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

// Warp load: thread i reads 8 consecutive 32-bit columns of lane (lane base + i).
DEVI void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr)
               : "memory");
}

// Shared-memory matrix descriptor: K-major, no swizzle (layout type 0), version 1.
DEVI uint64_t smem_desc_kmajor(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

// Instruction descriptor of kind::f16: fp32 accumulate, A and B both fp16 (bf = 0) or
// both bf16 (bf = 1), both K-major, M x N.
__host__ __device__ constexpr uint32_t idesc_f16(int bf, int M, int N) {
  return (1u << 4) | ((uint32_t)bf << 7) | ((uint32_t)bf << 10) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}

// D (+)= A B^T, A in tensor memory, B in shared memory; issued by one thread.
DEVI void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// One arrival on `bar` once every tcgen05 operation this thread issued so far is done.
DEVI void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

}  // namespace duplex
