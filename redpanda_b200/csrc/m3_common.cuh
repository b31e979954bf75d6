// Shared device code of the Mamba-3 trapezoidal scan, backward and step kernels.
//
// Recurrence (reference: redpanda/engine/mamba.py:382-423 and 466-493,
// redpanda/engine/triton_scan.py:7-12), per (row b, channel d, state lane n):
//
//   gate[t] = exp(delta*A_real) * cos(delta*A_imag)   rotational lanes n <  n_rot
//           = tanh(theta)                             tracking lanes   n >= n_rot
//   dBu[t]  = delta[t] * u[t] * B[t]
//   h[t]    = gate[t]*h[t-1] + 0.5*dBu[t] + 0.5*gate[t]*dBu[t-1]
//   y[t]    = sum_n h[t] * C[t]
//
// The kernels carry one register per cell, P = 2*h + dBu, so that the update is
//   H = fma(gate, P_prev, dBu)      (H = 2*h[t], exact power-of-two scaling)
//   P = H + dBu
//   y = 0.5 * sum_n H * C
// which is the same mathematics with one register per cell instead of two.
// The cached state handed to the O(1) step is the reference's (h, dBu) pair:
// h = 0.5*H, so the step rebuilds H = 2*h exactly and P = H + dBu with the same
// rounded add the scan performs.  Every multiply/add below is an explicitly
// rounded intrinsic (no compiler contraction), and the scan and the step call
// the same functions, so the step is bit-identical to the scan.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "m3_math.cuh"
#include "m3scan.h"

namespace m3 {

constexpr int kThreads = 128;   // threads per CTA for every scan/step kernel
constexpr int kQ = 4;           // threads that share one channel d (state-lane quarters)
constexpr int kCK = 16;         // checkpoint / recompute chunk length (timesteps)

// ---------------------------------------------------------------- dtype io
__device__ __forceinline__ float ld_f(const void* p, size_t i, int dt) {
  if (dt == M3_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  return reinterpret_cast<const float*>(p)[i];
}

__device__ __forceinline__ void st_f(void* p, size_t i, int dt, float v) {
  if (dt == M3_BF16) reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else reinterpret_cast<float*>(p)[i] = v;
}

// ---------------------------------------------------------------- lane map
// A thread with quarter index q (0..3) owns R rotational lanes
//   n = q*R + j            (j < R, real when n < NR)
// and T tracking lanes
//   n = NR + q*T + j       (j < T, real when q*T + j < NT).
// Lanes past the real counts are virtual: their B/C/params read as zero, so
// their state stays exactly zero and they are never stored.
template <int R, int T>
struct LaneMap {
  static constexpr int NL = R + T;        // lanes per thread per channel
  static constexpr int NP = kQ * NL;      // padded lanes per channel
  // memory state index of local lane j for quarter q, or -1 when virtual
  __device__ __forceinline__ static int mem_lane(int q, int j, int NR, int NT) {
    if (j < R) {
      int n = q * R + j;
      return n < NR ? n : -1;
    }
    int k = q * T + (j - R);
    return k < NT ? NR + k : -1;
  }
};

// ---------------------------------------------------------------- cell math
// Rotational gate exp(dl*A_real) * cos(dl*A_imag) from a2 = A_real*log2(e)
// (m3_math.cuh: ~1e-7 absolute error, no MUFU cosine).
__device__ __forceinline__ float rot_gate(float dl, float a2, float ai) {
  return __fmul_rn(gate_exp(dl, a2), gate_cos(dl, ai));
}

// Per-cell constant of the exponential, computed identically by every kernel.
__device__ __forceinline__ float exp_const(float ar) { return __fmul_rn(ar, kLog2e); }

// One cell update: returns H = 2*h[t]; P becomes 2*h[t] + dBu[t].
__device__ __forceinline__ float cell_update(float g, float& P, float du, float b) {
  float dbu = __fmul_rn(du, b);
  float H = __fmaf_rn(g, P, dbu);
  P = __fadd_rn(H, dbu);
  return H;
}

// Two cells (channels k, k+1 of one state lane) in one packed update: the
// lane-wise twin of cell_update().
__device__ __forceinline__ float2 cell_update2(float2 g, float2& P, float2 du, float b) {
  const float2 dbu = __fmul2_rn(du, f2(b));
  const float2 H = __ffma2_rn(g, P, dbu);
  P = __fadd2_rn(H, dbu);
  return H;
}

// The same packed update with B already held as a (b, b) pair.
__device__ __forceinline__ float2 cell_update2p(float2 g, float2& P, float2 du, float2 b) {
  const float2 dbu = __fmul2_rn(du, b);
  const float2 H = __ffma2_rn(g, P, dbu);
  P = __fadd2_rn(H, dbu);
  return H;
}

// Sum of a per-thread partial over the kQ threads of a channel group
// (fixed pairing: (s0+s1)+(s2+s3) on every lane).
__device__ __forceinline__ float quad_sum(float s) {
  s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, 1));
  s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, 2));
  return s;
}

// quad_sum() of ND channel partials at once, transposed: each round keeps
// the channels of its own lane bit and adds the partner's copy of them, so
// quarter q ends with the totals of its channels k = 4i + q in v[i] (ND >= 4;
// ND = 2: quarters 0/2 hold channel 0 and 1/3 channel 1 in v[0]).  Every total
// is summed in quad_sum()'s order (s0+s1)+(s2+s3), so the bits are the same.
template <int ND>
__device__ __forceinline__ void quad_sum_t(float (&v)[ND], int q) {
  static_assert(ND % 2 == 0, "channel pairs");
  const int b0 = q & 1, b1 = (q >> 1) & 1;
#pragma unroll
  for (int i = 0; i < ND / 2; ++i) {
    const float keep = b0 ? v[2 * i + 1] : v[2 * i];
    const float send = b0 ? v[2 * i] : v[2 * i + 1];
    v[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, 1));
  }
  if constexpr (ND >= 4) {
#pragma unroll
    for (int i = 0; i < ND / 4; ++i) {
      const float keep = b1 ? v[2 * i + 1] : v[2 * i];
      const float send = b1 ? v[2 * i] : v[2 * i + 1];
      v[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, 2));
    }
  } else {
    v[0] = __fadd_rn(v[0], __shfl_xor_sync(0xffffffffu, v[0], 2));
  }
}

// Per-thread channel partial of y: sum_j H_j * C_j over the thread's lanes in
// the fixed order rotational lanes first, then tracking lanes.
template <int NL>
__device__ __forceinline__ float y_partial(const float (&H)[NL], const float* C) {
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < NL; ++j) s = __fmaf_rn(H[j], C[j], s);
  return s;
}

// Device-side error word: first error wins.
__device__ __forceinline__ void set_err(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

}  // namespace m3
