// The scan's per-token prologue (redpanda/engine/mamba.py:284-301, 336-337),
// shared by the standalone prologue kernel (m3_layer.cu) and the scan kernels
// that fuse it into their staging, so that both produce the same bits:
//   delta  = softplus(dt)                 torch's threshold 20: x > 20 ? x : log1p(exp(x))
//   rs     = rsqrt(mean(x^2) + eps)       over the N*p vector of B_raw (or C_raw)
//   Bc[n]  = sum_k (x[n*p + k] * rs) * w[n*p + k]     k = 0..p-1 in order
// (RMSNorm, mamba.py:82-89, then the MIMO fold).  The sum of squares is one
// warp's: lane l accumulates x[l], x[l+32], ... by FMA, then an xor butterfly
// over 16, 8, 4, 2, 1 lanes.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace m3 {

__device__ __forceinline__ float softplus20(float x) { return x > 20.f ? x : log1pf(expf(x)); }

// d softplus(x) / dx applied to g, as torch's softplus backward (threshold 20)
__device__ __forceinline__ float softplus20_grad(float g, float x) {
  if (x > 20.f) return g;
  const float e = expf(x);
  return __fdiv_rn(__fmul_rn(g, e), __fadd_rn(e, 1.f));
}

// rs of one row, computed by a full warp; ld(k) returns element k as fp32.
// Without weights (use_bcnorm=False) the fold is a plain sum: rs = 1.
template <class Ld>
__device__ __forceinline__ float bcnorm_scale(Ld ld, int np, float eps, bool has_w, int lane) {
  if (!has_w) return 1.f;
  float ss = 0.f;
  for (int k = lane; k < np; k += 32) {
    const float v = ld(k);
    ss = __fmaf_rn(v, v, ss);
  }
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, m));
  return rsqrtf(__fadd_rn(__fdiv_rn(ss, (float)np), eps));
}

// Bc[n] of one row from its scale rs (w == nullptr: plain sum over p)
template <class Ld>
__device__ __forceinline__ float bcnorm_fold(Ld ld, int n, int p, float rs, const float* w) {
  float a = 0.f;
  for (int k = 0; k < p; ++k) {
    const int i = n * p + k;
    float v = ld(i);
    if (w != nullptr) v = __fmul_rn(__fmul_rn(v, rs), w[i]);
    a = k == 0 ? v : __fadd_rn(a, v);
  }
  return a;
}

}  // namespace m3
