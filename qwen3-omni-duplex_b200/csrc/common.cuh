// Shared device helpers for the sm_100a int4 dequant-GEMV / MoE kernels.
//
// Everything here is hand-written inline PTX around documented instructions:
// mbarrier (arrive / expect_tx / try_wait.parity), the non-tensor bulk copy
// cp.async.bulk (global -> shared, completion by mbarrier transaction bytes, no
// multicast), ldmatrix, the warp-level mma.sync m16n8k16 used as a register dot
// product, and griddepcontrol for programmatic dependent launch.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "duplex_b200.h"

#define DEVI __device__ __forceinline__

namespace duplex {

// ----------------------------------------------------------------- smem / barriers
DEVI uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

DEVI void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

DEVI void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

DEVI void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

DEVI void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

DEVI bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(20000u)
      : "memory");
  return ok != 0;
}

// Bounded wait on an mbarrier phase.  Returns false (and never blocks again) once
// `abort` is set or the wait has spun for ~kWaitLimitCycles; the caller records
// the error.  No wait in these kernels is unbounded.
constexpr long long kWaitLimitCycles = 4000000000LL;  // ~2 s at 2 GHz

DEVI bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, volatile int* abort) {
  if (*abort) return false;
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort) return false;
    if (clock64() - t0 > kWaitLimitCycles) {
      *abort = 1;
      return false;
    }
  }
}

// 1-D bulk copy global -> this CTA's shared memory; completion is signalled as
// transaction bytes on `bar`.  Both addresses 16-byte aligned, bytes % 16 == 0.
DEVI void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Same, with an L2 eviction-priority hint for data that is streamed exactly once.
DEVI void bulk_g2s_stream(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar,
                          uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

DEVI uint64_t policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// order this thread's view of generic-proxy global writes (made visible to it by an
// acquire) before its subsequent async-proxy (bulk copy) reads of global memory
DEVI void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

DEVI void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ----------------------------------------------------------------- PDL
DEVI void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
DEVI void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ----------------------------------------------------------------- fragments
DEVI void ldsm_x2(uint32_t& r0, uint32_t& r1, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];"
               : "=r"(r0), "=r"(r1)
               : "r"(addr));
}

DEVI void ldsm_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

DEVI uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c) {  // (a & b) | c
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

template <typename T> struct MmaOp;

template <> struct MmaOp<__half> {
  static DEVI void run(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                       uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
};

template <> struct MmaOp<__nv_bfloat16> {
  static DEVI void run(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                       uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
};

// ----------------------------------------------------------------- int4 -> 16-bit
// The nibbles of one packed word (reference order: nibble i = column 8m+i) are
// turned into exact 16-bit integers (n - z) by OR-ing them into the mantissa of
// a power-of-two constant and subtracting (power + z): for fp16 1024 + n is exact
// (10-bit mantissa), and a nibble left at bit 4 gives 1024 + 16 n, which a
// fused multiply by 1/16 brings back to 64 + n; for bf16 (7-bit mantissa) every
// nibble is shifted to bits 0..3 and 128 + n is used.  The products are exact, so
// (n - z) is exact in the 16-bit type for every nibble and zero point in 0..15.
//
// Pair order produced per word w: k-step A = {(n0,n4) , (n1,n5)}, k-step B =
// {(n2,n6) , (n3,n7)}; the activation fragments use the same column permutation.
template <typename T> struct Dq;

template <> struct Dq<__half> {
  // per-row constants for one group: lo = (1024+z) x2, hi = -(64+z) x2
  static DEVI void consts(uint32_t z, uint32_t& lo, uint32_t& hi) {
    const uint32_t l = 0x6400u | z;
    const uint32_t h = 0xD400u | (z << 4);
    lo = l | (l << 16);
    hi = h | (h << 16);
  }
  // word of row g (wa) and row g+8 (wb) -> A fragments of two k16 steps
  static DEVI void expand(uint32_t wa, uint32_t wb, uint32_t loa, uint32_t hia, uint32_t lob,
                          uint32_t hib, uint32_t (&A)[4], uint32_t (&B)[4]) {
    const uint32_t MAG = 0x64006400u;
    const uint32_t M_LO = 0x000F000Fu, M_HI = 0x00F000F0u;
    const __half2 sixteenth = __halves2half2(__float2half_rn(0.0625f), __float2half_rn(0.0625f));
    uint32_t v;
    __half2 t;
    // k-step A
    v = lop3_and_or(wa, M_LO, MAG);
    t = __hsub2(*reinterpret_cast<__half2*>(&v), *reinterpret_cast<const __half2*>(&loa));
    A[0] = *reinterpret_cast<uint32_t*>(&t);
    v = lop3_and_or(wb, M_LO, MAG);
    t = __hsub2(*reinterpret_cast<__half2*>(&v), *reinterpret_cast<const __half2*>(&lob));
    A[1] = *reinterpret_cast<uint32_t*>(&t);
    v = lop3_and_or(wa, M_HI, MAG);
    t = __hfma2(*reinterpret_cast<__half2*>(&v), sixteenth, *reinterpret_cast<const __half2*>(&hia));
    A[2] = *reinterpret_cast<uint32_t*>(&t);
    v = lop3_and_or(wb, M_HI, MAG);
    t = __hfma2(*reinterpret_cast<__half2*>(&v), sixteenth, *reinterpret_cast<const __half2*>(&hib));
    A[3] = *reinterpret_cast<uint32_t*>(&t);
    // k-step B
    const uint32_t wa8 = wa >> 8, wb8 = wb >> 8;
    v = lop3_and_or(wa8, M_LO, MAG);
    t = __hsub2(*reinterpret_cast<__half2*>(&v), *reinterpret_cast<const __half2*>(&loa));
    B[0] = *reinterpret_cast<uint32_t*>(&t);
    v = lop3_and_or(wb8, M_LO, MAG);
    t = __hsub2(*reinterpret_cast<__half2*>(&v), *reinterpret_cast<const __half2*>(&lob));
    B[1] = *reinterpret_cast<uint32_t*>(&t);
    v = lop3_and_or(wa8, M_HI, MAG);
    t = __hfma2(*reinterpret_cast<__half2*>(&v), sixteenth, *reinterpret_cast<const __half2*>(&hia));
    B[2] = *reinterpret_cast<uint32_t*>(&t);
    v = lop3_and_or(wb8, M_HI, MAG);
    t = __hfma2(*reinterpret_cast<__half2*>(&v), sixteenth, *reinterpret_cast<const __half2*>(&hib));
    B[3] = *reinterpret_cast<uint32_t*>(&t);
  }
};

template <> struct Dq<__nv_bfloat16> {
  // lo = (128+z) x2 ; hi unused
  static DEVI void consts(uint32_t z, uint32_t& lo, uint32_t& hi) {
    const uint32_t l = 0x4300u | z;
    lo = l | (l << 16);
    hi = 0u;
  }
  static DEVI void expand(uint32_t wa, uint32_t wb, uint32_t loa, uint32_t, uint32_t lob,
                          uint32_t, uint32_t (&A)[4], uint32_t (&B)[4]) {
    const uint32_t MAG = 0x43004300u;
    const uint32_t M_LO = 0x000F000Fu;
    const __nv_bfloat162 ca = *reinterpret_cast<const __nv_bfloat162*>(&loa);
    const __nv_bfloat162 cb = *reinterpret_cast<const __nv_bfloat162*>(&lob);
    uint32_t v;
    __nv_bfloat162 t;
#define DQ_BF16(dst, word, cst)                              \
  v = lop3_and_or((word), M_LO, MAG);                        \
  t = __hsub2(*reinterpret_cast<__nv_bfloat162*>(&v), cst); \
  dst = *reinterpret_cast<uint32_t*>(&t);
    DQ_BF16(A[0], wa, ca)
    DQ_BF16(A[1], wb, cb)
    DQ_BF16(A[2], wa >> 4, ca)
    DQ_BF16(A[3], wb >> 4, cb)
    DQ_BF16(B[0], wa >> 8, ca)
    DQ_BF16(B[1], wb >> 8, cb)
    DQ_BF16(B[2], wa >> 12, ca)
    DQ_BF16(B[3], wb >> 12, cb)
#undef DQ_BF16
  }
};

// Offset dequant (no subtraction in the inner loop): the A operands hold M + n,
// exact in the 16-bit type.  fp16: M = 1024 for the low nibble of each byte and
// 1024 + 16n for the high nibble, whose activations are stored pre-divided by 16,
// so sum_k A.x = 1024 X_even + 64 X_odd + sum n.x over a group (X_even / X_odd: the
// group's activation sums over even / odd columns).  bf16 (7-bit mantissa):
// every nibble is shifted down first and M = 128, giving 128 X + sum n.x.  One
// extra MMA per column pair with `corr_a` coefficients and exact multi-part sums
// as B subtracts (M + z) X, which also applies the zero point.  The column sums
// are kept per 64-column pair, so the correction is exact however a group's pairs
// are split between warps.
template <typename T> struct DqOff;

template <> struct DqOff<__half> {
  static constexpr bool kOddDiv16 = true;
  static DEVI void expand(uint32_t wa, uint32_t wb, uint32_t (&A)[4], uint32_t (&B)[4]) {
    const uint32_t MAG = 0x64006400u, M_LO = 0x000F000Fu, M_HI = 0x00F000F0u;
    A[0] = lop3_and_or(wa, M_LO, MAG);
    A[1] = lop3_and_or(wb, M_LO, MAG);
    A[2] = lop3_and_or(wa, M_HI, MAG);
    A[3] = lop3_and_or(wb, M_HI, MAG);
    const uint32_t sa = wa >> 8, sb = wb >> 8;
    B[0] = lop3_and_or(sa, M_LO, MAG);
    B[1] = lop3_and_or(sb, M_LO, MAG);
    B[2] = lop3_and_or(sa, M_HI, MAG);
    B[3] = lop3_and_or(sb, M_HI, MAG);
  }
  // correction coefficients of one column pair, lane (g, t): k = 2t, 2t+1 carry
  // window t/2; even t -> -(1024 + z), odd t -> -(64 + z), rows g (a0) and g+8 (a1).
  // `wmask` bit h keeps window h (both set unless each window is its own group).
  static DEVI void corr_a(uint32_t za, uint32_t zb, int t, uint32_t wmask, uint32_t& a0,
                          uint32_t& a1) {
    uint32_t ca = 0, cb = 0;
    if ((wmask >> (t >> 1)) & 1u) {
      if ((t & 1) == 0) {
        ca = 0xE400u | za;
        cb = 0xE400u | zb;
      } else {
        ca = 0xD400u | (za << 4);
        cb = 0xD400u | (zb << 4);
      }
    }
    a0 = ca | (ca << 16);
    a1 = cb | (cb << 16);
  }
};

template <> struct DqOff<__nv_bfloat16> {
  static constexpr bool kOddDiv16 = false;
  static DEVI void expand(uint32_t wa, uint32_t wb, uint32_t (&A)[4], uint32_t (&B)[4]) {
    const uint32_t MAG = 0x43004300u, M_LO = 0x000F000Fu;
    A[0] = lop3_and_or(wa, M_LO, MAG);
    A[1] = lop3_and_or(wb, M_LO, MAG);
    A[2] = lop3_and_or(wa >> 4, M_LO, MAG);
    A[3] = lop3_and_or(wb >> 4, M_LO, MAG);
    B[0] = lop3_and_or(wa >> 8, M_LO, MAG);
    B[1] = lop3_and_or(wb >> 8, M_LO, MAG);
    B[2] = lop3_and_or(wa >> 12, M_LO, MAG);
    B[3] = lop3_and_or(wb >> 12, M_LO, MAG);
  }
  // -(128 + z) on every lane of a kept window (three-part column sum per window:
  // k = 4h .. 4h+2 for window h)
  static DEVI void corr_a(uint32_t za, uint32_t zb, int t, uint32_t wmask, uint32_t& a0,
                          uint32_t& a1) {
    uint32_t ca = 0, cb = 0;
    if ((wmask >> (t >> 1)) & 1u) {
      ca = 0xC300u | za;
      cb = 0xC300u | zb;
    }
    a0 = ca | (ca << 16);
    a1 = cb | (cb << 16);
  }
};

// Activation fragments for one 32-column window: 8 consecutive 16-bit values
// x[c0 .. c0+8) (c0 = window*32 + 8*t) -> B registers of k-step A and B.
DEVI void x_frags(uint4 v, uint32_t& a0, uint32_t& a1, uint32_t& b0, uint32_t& b1) {
  a0 = __byte_perm(v.x, v.z, 0x5410);  // (x0, x4)
  a1 = __byte_perm(v.x, v.z, 0x7632);  // (x1, x5)
  b0 = __byte_perm(v.y, v.w, 0x5410);  // (x2, x6)
  b1 = __byte_perm(v.y, v.w, 0x7632);  // (x3, x7)
}

// ----------------------------------------------------------------- conversions
template <typename T> DEVI float to_f32(T v);
template <> DEVI float to_f32<__half>(__half v) { return __half2float(v); }
template <> DEVI float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <> DEVI float to_f32<float>(float v) { return v; }

template <typename T> DEVI T from_f32(float v);
template <> DEVI __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <> DEVI __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <> DEVI float from_f32<float>(float v) { return v; }

DEVI float silu_f32(float g) { return g / (1.0f + expf(-g)); }

DEVI void set_error(int* err, int bit) {
  if (err) atomicOr(err, bit);
}

}  // namespace duplex
