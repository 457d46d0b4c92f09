// kvcu_tcgen05.cuh — PTX helpers for the sm_100a kernels that drive the
// tcgen05 tensor cores (the decode kernel and the MLA-step GEMM): mbarriers,
// proxy and tcgen05 fences, UMMA shared-memory descriptors, commits, TMEM
// loads and stores, and the 128B / 64B swizzled shared-memory layouts.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace kvtc {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_tx(uint32_t bar, uint32_t tx) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(tx)
               : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// One lane of a converged warp (the lane that issues tcgen05 work).
__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n .reg .b32 r;\n .reg .pred p;\n elect.sync r|p, 0xffffffff;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(pred));
  return pred != 0;
}
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// UMMA shared-memory descriptor (sm_100): start>>4 @0, LBO>>4 @16, SBO>>4 @32,
// version 1 @46, layout type @61 (0 = none, 2 = 128B swizzle, 4 = 64B swizzle).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo,
                                              uint32_t layout) {
  return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | ((uint64_t)layout << 61);
}
constexpr uint32_t LAYOUT_NONE = 0, LAYOUT_SW128 = 2, LAYOUT_SW64 = 4;

__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

// TMEM loads / stores of N consecutive 32-bit columns of the warp's 32 lanes.
__device__ __forceinline__ void tld1(uint32_t ta, uint32_t* r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r[0]) : "r"(ta));
}
__device__ __forceinline__ void tld2(uint32_t ta, uint32_t* r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x2.b32 {%0,%1}, [%2];" : "=r"(r[0]), "=r"(r[1]) : "r"(ta));
}
__device__ __forceinline__ void tld4(uint32_t ta, uint32_t* r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(ta));
}
__device__ __forceinline__ void tld8(uint32_t ta, uint32_t* r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
                 "=r"(r[7])
               : "r"(ta));
}
template <int N>
__device__ __forceinline__ void tmem_ld(uint32_t ta, uint32_t* r) {
  if constexpr (N >= 8) {
    tld8(ta, r);
    tmem_ld<N - 8>(ta + 8, r + 8);
  } else if constexpr (N >= 4) {
    tld4(ta, r);
    tmem_ld<N - 4>(ta + 4, r + 4);
  } else if constexpr (N >= 2) {
    tld2(ta, r);
    tmem_ld<N - 2>(ta + 2, r + 2);
  } else if constexpr (N == 1) {
    tld1(ta, r);
  }
}
__device__ __forceinline__ void tst1(uint32_t ta, const uint32_t* r) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x1.b32 [%0], {%1};" ::"r"(ta), "r"(r[0]) : "memory");
}
__device__ __forceinline__ void tst2(uint32_t ta, const uint32_t* r) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x2.b32 [%0], {%1,%2};" ::"r"(ta), "r"(r[0]), "r"(r[1])
               : "memory");
}
__device__ __forceinline__ void tst4(uint32_t ta, const uint32_t* r) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1,%2,%3,%4};" ::"r"(ta), "r"(r[0]),
               "r"(r[1]), "r"(r[2]), "r"(r[3])
               : "memory");
}
__device__ __forceinline__ void tst8(uint32_t ta, const uint32_t* r) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(ta),
               "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}
template <int N>
__device__ __forceinline__ void tmem_st(uint32_t ta, const uint32_t* r) {
  if constexpr (N >= 8) {
    tst8(ta, r);
    tmem_st<N - 8>(ta + 8, r + 8);
  } else if constexpr (N >= 4) {
    tst4(ta, r);
    tmem_st<N - 4>(ta + 4, r + 4);
  } else if constexpr (N >= 2) {
    tst2(ta, r);
    tmem_st<N - 2>(ta + 2, r + 2);
  } else if constexpr (N == 1) {
    tst1(ta, r);
  }
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// Ties registers written by an earlier tcgen05.ld to a point after
// tcgen05.wait::ld, so no use of them is scheduled before the wait.
template <int N>
__device__ __forceinline__ void reg_fence(uint32_t (&r)[N]) {
#pragma unroll
  for (int i = 0; i < N; ++i) asm volatile("" : "+r"(r[i]));
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Byte offset of (row, byte) inside a K-major 128B-swizzled region whose rows
// are 128 B and whose 8-row atoms are 1024 B apart (region base 1024-aligned).
__device__ __forceinline__ uint32_t sw128_off(uint32_t row, uint32_t byte) {
  return (row >> 3) * 1024u + (row & 7u) * 128u + ((((byte >> 4) ^ row) & 7u) << 4) + (byte & 15u);
}
// Same for 64-byte rows with the 64B swizzle (8-row atoms of 512 B).
__device__ __forceinline__ uint32_t sw64_off(uint32_t row, uint32_t byte) {
  return (row >> 3) * 512u + (row & 7u) * 64u + ((((byte >> 4) ^ ((row & 7u) >> 1)) & 3u) << 4) +
         (byte & 15u);
}


}  // namespace kvtc
