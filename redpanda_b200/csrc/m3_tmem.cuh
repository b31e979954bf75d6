// Tensor Memory (TMEM) as per-thread scratch for the backward scan.
//
// The backward needs the forward state P[t-1] of every cell of a kCK-step chunk
// in reverse order.  Each warp of the 128-thread CTA owns one 32-lane TMEM
// sub-partition (lanes 32*warp .. 32*warp+31); each thread keeps its cells of a
// timestep in consecutive columns of its own lane, written with tcgen05.st and
// read back with tcgen05.ld (32x32b shape: one lane per thread, one 32-bit
// column per register).  No MMA is involved; TMEM is used as 256 KB/SM of
// addressable storage next to the register file.
#pragma once

#include <stdint.h>

namespace m3 {

__device__ __forceinline__ void tmem_alloc(uint32_t* smem_slot, uint32_t ncols) {
  const uint32_t dst = static_cast<uint32_t>(__cvta_generic_to_shared(smem_slot));
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tmem_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_st8(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
      "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7])
      : "memory");
}

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float* v) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
      : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3]), "=f"(v[4]), "=f"(v[5]), "=f"(v[6]),
        "=f"(v[7])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_st4(uint32_t taddr, const float* v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};" ::"r"(taddr),
               "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3])
               : "memory");
}

__device__ __forceinline__ void tmem_ld4(uint32_t taddr, float* v) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3])
               : "r"(taddr)
               : "memory");
}

// Store / load C consecutive 32-bit values (C a multiple of 4): 8-column
// pieces, then one 4-column piece.
template <int C>
__device__ __forceinline__ void tmem_store(uint32_t taddr, const float (&v)[C]) {
  static_assert(C % 4 == 0, "TMEM rows are written 4 columns at a time");
#pragma unroll
  for (int i = 0; i < C / 8; ++i) tmem_st8(taddr + 8 * i, &v[8 * i]);
  if constexpr (C % 8 != 0) tmem_st4(taddr + 8 * (C / 8), &v[8 * (C / 8)]);
}

template <int C>
__device__ __forceinline__ void tmem_load(uint32_t taddr, float (&v)[C]) {
  static_assert(C % 4 == 0, "TMEM rows are read 4 columns at a time");
#pragma unroll
  for (int i = 0; i < C / 8; ++i) tmem_ld8(taddr + 8 * i, &v[8 * i]);
  if constexpr (C % 8 != 0) tmem_ld4(taddr + 8 * (C / 8), &v[8 * (C / 8)]);
}

}  // namespace m3
