// Shared-memory staging helpers (cp.async) and staged-row readers.
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

namespace m3 {

__device__ __forceinline__ void cp_async4(void* smem, const void* gmem, bool valid) {
  uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  int sz = valid ? 4 : 0;  // src-size 0 => zero fill
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(s), "l"(gmem), "r"(sz)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;\n" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait1() {
  asm volatile("cp.async.wait_group 1;\n" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait_n() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}
__device__ __forceinline__ void cp_async_wait0() {
  asm volatile("cp.async.wait_group 0;\n" ::: "memory");
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
  uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  int sz = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(sz)
               : "memory");
}

// Lane-wise maximum of two pairs of unsigned 16-bit integers.
__device__ __forceinline__ uint32_t max_u16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("max.u16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// ND channel values of one staged row, converted to fp32.
template <int ND>
__device__ __forceinline__ void read_chan(const unsigned char* base, bool bf16, float (&v)[ND]) {
  if (bf16) {
    if constexpr (ND % 2 == 0) {
      const __nv_bfloat162* p2 = reinterpret_cast<const __nv_bfloat162*>(base);
#pragma unroll
      for (int i = 0; i < ND / 2; ++i) {
        float2 f = __bfloat1622float2(p2[i]);
        v[2 * i] = f.x;
        v[2 * i + 1] = f.y;
      }
    } else {
      const __nv_bfloat16* p1 = reinterpret_cast<const __nv_bfloat16*>(base);
#pragma unroll
      for (int i = 0; i < ND; ++i) v[i] = __bfloat162float(p1[i]);
    }
  } else {
    const float* pf = reinterpret_cast<const float*>(base);
    if constexpr (ND % 4 == 0) {
#pragma unroll
      for (int i = 0; i < ND / 4; ++i) {
        float4 f = reinterpret_cast<const float4*>(pf)[i];
        v[4 * i] = f.x; v[4 * i + 1] = f.y; v[4 * i + 2] = f.z; v[4 * i + 3] = f.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < ND; ++i) v[i] = pf[i];
    }
  }
}

}  // namespace m3
