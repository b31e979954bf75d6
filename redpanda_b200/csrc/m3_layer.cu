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
#include <stdint.h>

#include "m3_internal.h"
#include "m3_prologue.cuh"

namespace m3 {
namespace {

constexpr int kRowsPerCta = 8;   // one warp per row

__global__ void __launch_bounds__(32 * kRowsPerCta) step_inputs_kernel(const InputsParams p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r0 = blockIdx.x * kRowsPerCta;
  const int rows = min(kRowsPerCta, p.B - r0);
  if (warp >= rows) return;
  const size_t b = (size_t)(r0 + warp);
  auto ldv = [](const void* base, size_t i, int bf) {
    return bf ? __bfloat162float(static_cast<const __nv_bfloat16*>(base)[i])
              : static_cast<const float*>(base)[i];
  };
  auto stv = [](void* base, size_t i, float v, int bf) {
    if (bf) static_cast<__nv_bfloat16*>(base)[i] = __float2bfloat16_rn(v);
    else static_cast<float*>(base)[i] = v;
  };
  if (p.du_bf16) {   // bf16 dt and delta: fp32 arithmetic, delta rounded once
    const size_t i0 = b * p.ld_dt, o0 = b * p.D;
    const float* bias = p.dt_bias;
    for (int d = lane; d < p.D; d += 32) {
      const float x = ldv(p.dt, i0 + d, 1);
      stv(p.delta, o0 + d, softplus20(bias != nullptr ? __fadd_rn(x, bias[d]) : x), 1);
    }
  } else {   // softplus of this warp's row (after the dt_proj bias, when given)
    const float* dt = static_cast<const float*>(p.dt) + b * p.ld_dt;
    float* delta = static_cast<float*>(p.delta) + b * p.D;
    const float* bias = p.dt_bias;
    if (p.vec4) {
      const float4* dt4 = reinterpret_cast<const float4*>(dt);
      const float4* b4 = reinterpret_cast<const float4*>(bias);
      float4* de4 = reinterpret_cast<float4*>(delta);
      for (int c = lane; c < p.D / 4; c += 32) {
        float4 x = dt4[c];
        if (b4 != nullptr) {
          const float4 bb = b4[c];
          x = make_float4(__fadd_rn(x.x, bb.x), __fadd_rn(x.y, bb.y), __fadd_rn(x.z, bb.z),
                          __fadd_rn(x.w, bb.w));
        }
        de4[c] = make_float4(softplus20(x.x), softplus20(x.y), softplus20(x.z), softplus20(x.w));
      }
    } else {
      for (int d = lane; d < p.D; d += 32)
        delta[d] = softplus20(bias != nullptr ? __fadd_rn(dt[d], bias[d]) : dt[d]);
    }
  }
  const int np = p.N * p.P;
  const size_t xb = b * p.ld_x + p.off_b, xc = b * p.ld_x + p.off_c;
  const bool has_w = p.wb != nullptr;
  const int xbf = p.bc_bf16;
  auto ldb = [&](int k) { return ldv(p.xbc, xb + k, xbf); };
  auto ldc = [&](int k) { return ldv(p.xbc, xc + k, xbf); };
  const float rb = bcnorm_scale(ldb, np, p.eps, has_w, lane);
  const float rc = bcnorm_scale(ldc, np, p.eps, has_w, lane);
  for (int n = lane; n < p.N; n += 32) {
    stv(p.Bc, b * p.N + n, bcnorm_fold(ldb, n, p.P, rb, p.wb), xbf);
    stv(p.Cc, b * p.N + n, bcnorm_fold(ldc, n, p.P, rc, p.wc), xbf);
  }
}

// out = (y + coef*(u*d_skip)) * silu(z) over (rows, D): each warp walks rows
// (grid-stride), its lanes the channels, four at a time when VEC (D % 4 == 0,
// 16-byte aligned rows of fp32 y, u, z and out).
__device__ __forceinline__ float gate_one(float y, float u, float z, float ds, float coef,
                                         bool round_silu = false) {
  float sz = __fdiv_rn(z, __fadd_rn(1.0f, expf(-z)));
  if (round_silu) sz = __bfloat162float(__float2bfloat16_rn(sz));
  return __fmul_rn(__fadd_rn(y, __fmul_rn(coef, __fmul_rn(u, ds))), sz);
}

template <bool VEC>
__global__ void gate_kernel(const GateParams p) {
  const int lane = threadIdx.x & 31;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long r = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < p.rows;
       r += warps) {
    const size_t row = (size_t)r * p.D;
    if constexpr (VEC) {
      const float* z = static_cast<const float*>(p.z) + (size_t)r * p.ld_z;
      const float4* y4 = reinterpret_cast<const float4*>(static_cast<const float*>(p.y) + row);
      const float4* u4 = reinterpret_cast<const float4*>(static_cast<const float*>(p.u) + row);
      const float4* z4 = reinterpret_cast<const float4*>(z);
      const float4* d4 = reinterpret_cast<const float4*>(p.d_skip);
      float4* o4 = reinterpret_cast<float4*>(static_cast<float*>(p.out) + row);
      for (int c = lane; c < p.D / 4; c += 32) {
        const float4 y = y4[c], u = u4[c], zz = z4[c], ds = d4[c];
        o4[c] = make_float4(gate_one(y.x, u.x, zz.x, ds.x, p.coef),
                            gate_one(y.y, u.y, zz.y, ds.y, p.coef),
                            gate_one(y.z, u.z, zz.z, ds.z, p.coef),
                            gate_one(y.w, u.w, zz.w, ds.w, p.coef));
      }
    } else {
      // element types per operand: fp32 or bf16 (a bf16 layer's y, z and out)
      auto ld = [](const void* base, size_t i, int bf) {
        return bf ? __bfloat162float(static_cast<const __nv_bfloat16*>(base)[i])
                  : static_cast<const float*>(base)[i];
      };
      const size_t zrow = (size_t)r * p.ld_z;
      for (int d = lane; d < p.D; d += 32) {
        const float v = gate_one(ld(p.y, row + d, p.y_bf16), ld(p.u, row + d, p.u_bf16),
                                 ld(p.z, zrow + d, p.z_bf16), p.d_skip[d], p.coef,
                                 p.round_silu && p.z_bf16);
        if (p.out_bf16) static_cast<__nv_bfloat16*>(p.out)[row + d] = __float2bfloat16_rn(v);
        else static_cast<float*>(p.out)[row + d] = v;
      }
    }
  }
}

// Backward of step_inputs_kernel over `rows` rows:
//   d_dt   = g_delta * softplus'(dt)  (1 above torch's threshold 20, else
//            e/(e+1) with e = exp(dt), as torch's softplus backward)
//   BCNorm with the MIMO fold, per row: y_i = (x_i*rs)*w_i, Bc[n] = sum_k y_{n*p+k},
//   rs = (mean(x^2) + eps)^-1/2, so with gy_i = gBc[i/p], gx_i = gy_i*w_i:
//     d_x_i = rs*gx_i - (rs^3/np) * x_i * sum_j gx_j*x_j
//     d_w_i = sum over rows of gy_i * (x_i*rs)
// One warp per row (grid-stride); the weight gradients accumulate per warp in
// shared memory, are summed over the CTA's warps in warp order into one partial
// per CTA, and reduce_w_kernel sums the partials in CTA order: deterministic.
// XT: element type of the x_proj rows xbc and their gradient d_xbc (float, or
// __nv_bfloat16 for the fused bf16 scan, whose rows are bf16); every
// computation is fp32 and d_xbc is rounded once.  p.dt == nullptr skips the
// softplus part (the fused scan backward applies it in its own flush).
template <class XT>
__device__ __forceinline__ float ldx(const XT* x, size_t i) {
  if constexpr (sizeof(XT) == 2) return __bfloat162float(x[i]);
  else return x[i];
}
template <class XT>
__device__ __forceinline__ void stx(XT* x, size_t i, float v) {
  if constexpr (sizeof(XT) == 2) x[i] = __float2bfloat16_rn(v);
  else x[i] = v;
}

template <class XT>
__global__ void __launch_bounds__(256) step_inputs_bwd_kernel(const InputsBwdParams p) {
  extern __shared__ float s_w[];             // [8 warps][2][np]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int np = p.N * p.P;
  const XT* xbc = static_cast<const XT*>(p.xbc);
  XT* d_xbc = static_cast<XT*>(p.d_xbc);
  auto ldv = [](const void* base, size_t i, int bf) {
    return bf ? __bfloat162float(static_cast<const __nv_bfloat16*>(base)[i])
              : static_cast<const float*>(base)[i];
  };
  float* wacc = s_w + (size_t)warp * 2 * np;
  for (int i = lane; i < 2 * np; i += 32) wacc[i] = 0.f;
  const long long nwarps = (long long)gridDim.x * 8;
  for (long long r = (long long)blockIdx.x * 8 + warp; r < p.rows; r += nwarps) {
    const size_t b = (size_t)r;
    if (p.dt != nullptr) {
      const int bf = p.du_bf16;
      for (int d = lane; d < p.D; d += 32) {
        const float v = softplus20_grad(ldv(p.g_delta, b * p.D + d, bf),
                                        ldv(p.dt, b * p.ld_dt + d, bf));
        if (bf) static_cast<__nv_bfloat16*>(p.d_dt)[b * p.D + d] = __float2bfloat16_rn(v);
        else static_cast<float*>(p.d_dt)[b * p.D + d] = v;
      }
    }
#pragma unroll
    for (int which = 0; which < 2; ++which) {
      const size_t x0 = b * p.ld_x + (which ? p.off_c : p.off_b);
      const void* gsrc = which ? p.g_Cc : p.g_Bc;
      const size_t g0 = b * p.N;
      const int gbf = p.gbc_bf16;
      auto gbc_at = [&](int n) { return ldv(gsrc, g0 + n, gbf); };
      const float* w = which ? p.wc : p.wb;
      if (w == nullptr) {   // no BCNorm: the fold is a plain sum
        for (int i = lane; i < np; i += 32) stx(d_xbc, x0 + i, gbc_at(i / p.P));
        continue;
      }
      float ss = 0.f, sg = 0.f;
      for (int i = lane; i < np; i += 32) {
        const float xi = ldx(xbc, x0 + i);
        ss = __fmaf_rn(xi, xi, ss);
        sg = __fmaf_rn(__fmul_rn(gbc_at(i / p.P), w[i]), xi, sg);
      }
#pragma unroll
      for (int m = 16; m > 0; m >>= 1) {
        ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, m));
        sg = __fadd_rn(sg, __shfl_xor_sync(0xffffffffu, sg, m));
      }
      const float rs = rsqrtf(__fadd_rn(__fdiv_rn(ss, (float)np), p.eps));
      const float coef = __fdiv_rn(__fmul_rn(__fmul_rn(rs, rs), rs), (float)np);
      const float cs = __fmul_rn(coef, sg);
      float* wa = wacc + which * np;
      for (int i = lane; i < np; i += 32) {
        const float xi = ldx(xbc, x0 + i), gy = gbc_at(i / p.P);
        stx(d_xbc, x0 + i, __fsub_rn(__fmul_rn(rs, __fmul_rn(gy, w[i])), __fmul_rn(cs, xi)));
        wa[i] = __fmaf_rn(gy, __fmul_rn(xi, rs), wa[i]);
      }
    }
  }
  __syncthreads();
  if (p.wb != nullptr) {
    for (int i = threadIdx.x; i < 2 * np; i += blockDim.x) {
      float v = s_w[i];
      for (int w = 1; w < 8; ++w) v = __fadd_rn(v, s_w[(size_t)w * 2 * np + i]);
      p.part_w[(size_t)blockIdx.x * 2 * np + i] = v;
    }
  }
}

__global__ void reduce_w_kernel(const float* part, int nparts, int np, float* d_wb, float* d_wc) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < 2 * np; i += gridDim.x * blockDim.x) {
    float v = 0.f;
    for (int g = 0; g < nparts; ++g) v = __fadd_rn(v, part[(size_t)g * 2 * np + i]);
    if (i < np) d_wb[i] = v;
    else d_wc[i - np] = v;
  }
}

}  // namespace

int step_inputs_bwd_ctas(long long rows) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  long long g = (rows + 7) / 8;
  if (g > (long long)sms * 4) g = (long long)sms * 4;
  return (int)(g < 1 ? 1 : g);
}

cudaError_t launch_step_inputs_bwd(const InputsBwdParams& p, cudaStream_t s) {
  const int grid = step_inputs_bwd_ctas(p.rows);
  const int np = p.N * p.P;
  const size_t smem = (size_t)8 * 2 * np * sizeof(float);
  auto kern = p.x_bf16 ? step_inputs_bwd_kernel<__nv_bfloat16> : step_inputs_bwd_kernel<float>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
  }
  kern<<<grid, 256, smem, s>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || p.wb == nullptr) return e;
  reduce_w_kernel<<<(2 * np + 255) / 256, 256, 0, s>>>(p.part_w, grid, np, p.d_wb, p.d_wc);
  return cudaGetLastError();
}

cudaError_t launch_gate(const GateParams& p, cudaStream_t s) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  long long grid = (p.rows + 7) / 8;   // 8 warps (rows) per CTA
  if (grid > (long long)sms * 16) grid = (long long)sms * 16;
  auto a16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  const bool vec = !p.u_bf16 && !p.y_bf16 && !p.z_bf16 && !p.out_bf16 && (p.D % 4) == 0 &&
                   !p.round_silu &&
                   (p.ld_z % 4) == 0 && a16(p.y) && a16(p.u) &&
                   a16(p.z) && a16(p.d_skip) && a16(p.out);
  if (vec) gate_kernel<true><<<(unsigned)grid, 256, 0, s>>>(p);
  else gate_kernel<false><<<(unsigned)grid, 256, 0, s>>>(p);
  return cudaGetLastError();
}

// Backward of the gated output out = (y + coef*u*ds) * s, s = silu(z)
// (mamba.py:262-265, 496-497), everything in fp32 and each gradient rounded once
// to its input's element type:
//   ga = g * s                     d y  = ga
//   d u = (ga * ds) * coef         d ds = sum over rows of ga * (coef * u)
//   d z = (g * a) * sig * (1 + z * (1 - sig)),  a = y + coef*u*ds, sig = 1/(1+exp(-z))
// A thread owns kGateVec consecutive channels (one 8- or 16-byte access per
// operand and row), CTA (x, y) = rows chunk x of channel block y, so the d ds
// partial of each (chunk, channel) is one sequential sum over the chunk's rows;
// gate_bwd_reduce adds the chunks in order: deterministic.
constexpr int kGateVec = 4;
constexpr int kGateThreads = 128;

template <int V>
__device__ __forceinline__ void gate_ld(const void* base, size_t i, int bf, float (&v)[V]) {
  if constexpr (V == 4) {   // one 8- or 16-byte access (the caller checked the alignment)
    if (bf) {
      const uint2 w = *reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(base) + i);
      const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w.x));
      const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w.y));
      v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
    } else {
      const float4 f = *reinterpret_cast<const float4*>(static_cast<const float*>(base) + i);
      v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
    }
    return;
  }
  if (bf) {
    const __nv_bfloat16* b = static_cast<const __nv_bfloat16*>(base) + i;
#pragma unroll
    for (int k = 0; k < V; ++k) v[k] = __bfloat162float(b[k]);
  } else {
    const float* f = static_cast<const float*>(base) + i;
#pragma unroll
    for (int k = 0; k < V; ++k) v[k] = f[k];
  }
}
template <int V>
__device__ __forceinline__ void gate_st(void* base, size_t i, int bf, const float (&v)[V]) {
  if constexpr (V == 4) {
    if (bf) {
      const __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]);
      const __nv_bfloat162 b = __floats2bfloat162_rn(v[2], v[3]);
      uint2 w;
      w.x = *reinterpret_cast<const uint32_t*>(&a);
      w.y = *reinterpret_cast<const uint32_t*>(&b);
      *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(base) + i) = w;
    } else {
      *reinterpret_cast<float4*>(static_cast<float*>(base) + i) = make_float4(v[0], v[1], v[2], v[3]);
    }
    return;
  }
  if (bf) {
    __nv_bfloat16* b = static_cast<__nv_bfloat16*>(base) + i;
#pragma unroll
    for (int k = 0; k < V; ++k) b[k] = __float2bfloat16_rn(v[k]);
  } else {
    float* f = static_cast<float*>(base) + i;
#pragma unroll
    for (int k = 0; k < V; ++k) f[k] = v[k];
  }
}

// VEC: kGateVec channels per thread (D % kGateVec == 0 and every row of every
// operand aligned to kGateVec elements); otherwise one channel per thread.
template <bool VEC>
__global__ void __launch_bounds__(kGateThreads) gate_bwd_kernel(const GateBwdParams p) {
  constexpr int V = VEC ? kGateVec : 1;
  const int d0 = (blockIdx.y * kGateThreads + threadIdx.x) * V;
  if (d0 >= p.D) return;   // no barrier in this kernel
  const long long per = (p.rows + p.gx - 1) / p.gx;
  const long long r0 = (long long)blockIdx.x * per;
  const long long r1 = r0 + per < p.rows ? r0 + per : p.rows;
  const bool rs = p.round_silu && p.z_bf16;
  float ds[V], acc[V];
#pragma unroll
  for (int k = 0; k < V; ++k) {
    ds[k] = p.d_skip[d0 + k];
    acc[k] = 0.f;
  }
#pragma unroll 2
  for (long long r = r0; r < r1; ++r) {
    const size_t i = (size_t)r * p.D + d0;
    float y[V], u[V], z[V], g[V], oy[V], ou[V], oz[V];
    gate_ld<V>(p.y, i, p.y_bf16, y);
    gate_ld<V>(p.u, i, p.u_bf16, u);
    gate_ld<V>(p.z, (size_t)r * p.ld_z + d0, p.z_bf16, z);
    gate_ld<V>(p.g, i, p.g_bf16, g);
#pragma unroll
    for (int k = 0; k < V; ++k) {
      const float e1 = __fadd_rn(1.0f, expf(-z[k]));
      float s = __fdiv_rn(z[k], e1);
      if (rs) s = __bfloat162float(__float2bfloat16_rn(s));
      const float sig = __fdiv_rn(1.0f, e1);
      const float a = __fadd_rn(y[k], __fmul_rn(p.coef, __fmul_rn(u[k], ds[k])));
      const float ga = __fmul_rn(g[k], s);
      oy[k] = ga;
      ou[k] = __fmul_rn(__fmul_rn(ga, ds[k]), p.coef);
      acc[k] = __fmaf_rn(ga, __fmul_rn(p.coef, u[k]), acc[k]);
      const float dsz =
          __fmul_rn(sig, __fadd_rn(1.0f, __fmul_rn(z[k], __fsub_rn(1.0f, sig))));
      oz[k] = __fmul_rn(__fmul_rn(g[k], a), dsz);
    }
    gate_st<V>(p.dy, i, p.y_bf16, oy);
    gate_st<V>(p.du, i, p.u_bf16, ou);
    gate_st<V>(p.dz, i, p.z_bf16, oz);
  }
#pragma unroll
  for (int k = 0; k < V; ++k) p.part[(size_t)blockIdx.x * p.D + d0 + k] = acc[k];
}

__global__ void gate_bwd_reduce(const float* part, int gx, int D, float* out) {
  const int d = blockIdx.x * blockDim.x + threadIdx.x;
  if (d >= D) return;
  float s = part[d];
  for (int x = 1; x < gx; ++x) s = __fadd_rn(s, part[(size_t)x * D + d]);
  out[d] = s;
}

int gate_bwd_row_ctas(long long rows, int d) {
  const int cb = (d + kGateThreads * kGateVec - 1) / (kGateThreads * kGateVec);
  long long gx = (148LL * 4 + cb - 1) / cb;   // about four CTAs per SM of a 148-SM B200
  if (gx > rows) gx = rows;
  return gx < 1 ? 1 : (int)gx;
}

cudaError_t launch_gate_bwd(const GateBwdParams& p, cudaStream_t s) {
  auto al = [](const void* q, int bf) {
    return (reinterpret_cast<uintptr_t>(q) & (bf ? 2 * kGateVec - 1 : 4 * kGateVec - 1)) == 0;
  };
  const bool vec = p.D % kGateVec == 0 && p.ld_z % kGateVec == 0 && al(p.y, p.y_bf16) &&
                   al(p.u, p.u_bf16) && al(p.z, p.z_bf16) && al(p.g, p.g_bf16) &&
                   al(p.dy, p.y_bf16) && al(p.du, p.u_bf16) && al(p.dz, p.z_bf16);
  const int per_block = kGateThreads * (vec ? kGateVec : 1);
  dim3 grid(p.gx, (p.D + per_block - 1) / per_block);
  if (vec) gate_bwd_kernel<true><<<grid, kGateThreads, 0, s>>>(p);
  else gate_bwd_kernel<false><<<grid, kGateThreads, 0, s>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  gate_bwd_reduce<<<(p.D + 255) / 256, 256, 0, s>>>(p.part, p.gx, p.D, p.d_dskip);
  return cudaGetLastError();
}

// u = silu(x) over (rows, D) of a row-strided x (the x half of in_proj's
// output, mamba.py:243/452): z / (1 + exp(-z)) in that rounding order; each
// warp walks rows (grid-stride), its lanes the channels, four at a time when
// vec4.
__global__ void silu_kernel(const SiluParams p) {
  const int lane = threadIdx.x & 31;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  auto silu = [](float z) { return __fdiv_rn(z, __fadd_rn(1.0f, expf(-z))); };
  for (long long r = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < p.rows;
       r += warps) {
    const float* x = p.x + (size_t)r * p.ld_x;
    float* o = p.out + (size_t)r * p.D;
    if (p.vec4) {
      const float4* x4 = reinterpret_cast<const float4*>(x);
      float4* o4 = reinterpret_cast<float4*>(o);
      for (int c = lane; c < p.D / 4; c += 32) {
        const float4 v = x4[c];
        o4[c] = make_float4(silu(v.x), silu(v.y), silu(v.z), silu(v.w));
      }
    } else {
      for (int d = lane; d < p.D; d += 32) o[d] = silu(x[d]);
    }
  }
}

cudaError_t launch_silu(const SiluParams& p, cudaStream_t s) {
  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
    return e;
  const long long want = (p.rows + 7) / 8;
  const int grid = (int)(want < (long long)sms * 8 ? (want > 0 ? want : 1) : (long long)sms * 8);
  silu_kernel<<<grid, 256, 0, s>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_step_inputs(const InputsParams& p, cudaStream_t s) {
  const int grid = (p.B + kRowsPerCta - 1) / kRowsPerCta;
  step_inputs_kernel<<<grid, 32 * kRowsPerCta, 0, s>>>(p);
  return cudaGetLastError();
}

}  // namespace m3
