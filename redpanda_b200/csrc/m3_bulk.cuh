// Bulk asynchronous copies (global -> shared, completion on an mbarrier) with
// bounded waits.  Used by the pipelined step kernel to stream whole state rows
// into shared memory several rows ahead of the compute, by the forward scan for
// its input rows and by the backward for its checkpoint tiles.
//
// Every copy is the plain single-destination form: it reads this GPU's own
// memory into the issuing CTA's own shared memory (a CTA-local shared address
// is a valid shared::cluster address of the issuing CTA).
#pragma once

#include <stdint.h>

namespace m3 {

// Upper bound on mbarrier polls before a wait gives up and reports an error
// (each try_wait may itself suspend for a short, hardware-defined time).
constexpr int kMbarMaxPolls = 1 << 22;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

// Makes mbarrier initialisation visible to the async (bulk copy) proxy.
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

// Arrives without expecting bytes (completes a phase that has no copy).
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// Waits for phase `parity` of the barrier to complete; false after
// kMbarMaxPolls unsuccessful polls.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t a = smem_addr(bar);
  for (int i = 0; i < kMbarMaxPolls; ++i) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}

// Orders this thread's earlier generic-proxy view of global memory (including
// writes by other threads made visible to it by a barrier) before its later
// bulk copies, which read through the async proxy.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// bytes (a multiple of 16) from global src (16-byte aligned) to shared dst
// (16-byte aligned); completion is counted on bar's transaction count.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// A 2D tile of a tensor map (TMA) into shared memory, completion counted on
// bar's transaction count; c0 is the inner coordinate (elements), c1 the outer.
// The map must be a __grid_constant__ kernel parameter (its address is a
// parameter-space address, valid as the tensor-map operand).
__device__ __forceinline__ void tma_load_2d(void* dst, const void* tmap, int c0, int c1,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3}], [%4];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(c0), "r"(c1), "r"(smem_addr(bar))
      : "memory");
}

}  // namespace m3
