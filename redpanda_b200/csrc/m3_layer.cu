// Per-token inputs of the recurrent step, computed from the layer's projection
// outputs in one launch (the elementwise part of Mamba3Block.step,
// redpanda/engine/mamba.py:455-469, that the reference runs as a dozen torch
// ops per layer):
//   delta  = softplus(dt)                       dt = dt_proj(dt_raw), bias included
//   Bc[n]  = sum_k RMSNorm_wb(B_raw)[n*p + k]   BCNorm over the N*p vector, MIMO fold
//   Cc[n]  = sum_k RMSNorm_wc(C_raw)[n*p + k]
// RMSNorm(x) = x * rsqrt(mean(x^2) + eps) * w (mamba.py:82-89), applied per
// element in that rounding order; softplus(x) = x for x > 20, else
// log1p(exp(x)) (torch's threshold).  One warp normalises one row.
//
// Also the gated activation after a scan (mamba.py:262-265):
//   out = (y + coef * u*D) * silu(z),  coef 1 (one direction) or 2 (the
//   bidirectional pair adds u*D once per direction).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "m3_internal.h"

namespace m3 {
namespace {

constexpr int kRowsPerCta = 8;   // one warp per row

__global__ void __launch_bounds__(32 * kRowsPerCta) step_inputs_kernel(const InputsParams p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r0 = blockIdx.x * kRowsPerCta;
  const int rows = min(kRowsPerCta, p.B - r0);
  for (int i = threadIdx.x; i < rows * p.D; i += blockDim.x) {
    const int r = i / p.D, d = i - r * p.D;
    const size_t b = (size_t)(r0 + r);
    const float x = p.dt[b * p.ld_dt + d];
    p.delta[b * p.D + d] = x > 20.f ? x : log1pf(expf(x));
  }
  if (warp >= rows) return;
  const size_t b = (size_t)(r0 + warp);
  const int np = p.N * p.P;
  const float* xb = p.xbc + b * p.ld_x + p.off_b;
  const float* xc = p.xbc + b * p.ld_x + p.off_c;
  float rb = 1.f, rc = 1.f;
  if (p.wb != nullptr) {
    float sb = 0.f, sc = 0.f;
    for (int k = lane; k < np; k += 32) {
      sb = __fmaf_rn(xb[k], xb[k], sb);
      sc = __fmaf_rn(xc[k], xc[k], sc);
    }
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) {
      sb = __fadd_rn(sb, __shfl_xor_sync(0xffffffffu, sb, m));
      sc = __fadd_rn(sc, __shfl_xor_sync(0xffffffffu, sc, m));
    }
    rb = rsqrtf(__fadd_rn(__fdiv_rn(sb, (float)np), p.eps));
    rc = rsqrtf(__fadd_rn(__fdiv_rn(sc, (float)np), p.eps));
  }
  for (int n = lane; n < p.N; n += 32) {
    float ab = 0.f, ac = 0.f;
    for (int k = 0; k < p.P; ++k) {
      const int i = n * p.P + k;
      float vb = xb[i], vc = xc[i];
      if (p.wb != nullptr) {
        vb = __fmul_rn(__fmul_rn(vb, rb), p.wb[i]);
        vc = __fmul_rn(__fmul_rn(vc, rc), p.wc[i]);
      }
      ab = k == 0 ? vb : __fadd_rn(ab, vb);
      ac = k == 0 ? vc : __fadd_rn(ac, vc);
    }
    p.Bc[b * p.N + n] = ab;
    p.Cc[b * p.N + n] = ac;
  }
}

// out = (y + coef*(u*d_skip)) * silu(z) over (rows, D), grid-stride over the
// elements (consecutive threads take consecutive channels: coalesced rows).
__global__ void gate_kernel(const GateParams p) {
  const size_t D = (size_t)p.D;
  const size_t total = (size_t)p.rows * D;
  auto one = [&](size_t i) {
    const size_t r = i / D, d = i - r * D;
    const float u = p.u_bf16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(p.u)[i])
                             : static_cast<const float*>(p.u)[i];
    const float z = p.z[r * p.ld_z + d];
    const float sz = __fdiv_rn(z, __fadd_rn(1.0f, expf(-z)));
    const float ud = __fmul_rn(p.coef, __fmul_rn(u, p.d_skip[d]));
    p.out[i] = __fmul_rn(__fadd_rn(p.y[i], ud), sz);
  };
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += stride) one(i);
}

}  // namespace

cudaError_t launch_gate(const GateParams& p, cudaStream_t s) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const size_t total = (size_t)p.rows * p.D;
  size_t grid = (total + 255) / 256;
  if (grid > (size_t)sms * 16) grid = (size_t)sms * 16;
  gate_kernel<<<(unsigned)grid, 256, 0, s>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_step_inputs(const InputsParams& p, cudaStream_t s) {
  const int grid = (p.B + kRowsPerCta - 1) / kRowsPerCta;
  step_inputs_kernel<<<grid, 32 * kRowsPerCta, 0, s>>>(p);
  return cudaGetLastError();
}

}  // namespace m3
