// Small-batch projections of the recurrent step layer, for lockstep batches of
// at most kSmallRows rows (a search evaluating one node, or a few lines).
//
// At these sizes each projection of Mamba3Block.step is a matrix-vector
// product whose time is launch and memory latency rather than arithmetic, so
// the element-wise work around each product is folded into it and one step
// layer runs as four launches:
//
//   rows_linear: RMSNorm + in_proj + silu of the x half  (mamba.py:82-89, 450-452)
//   rows_linear: x_proj (+ bias)                          (mamba.py:454)
//   m3_step_gated_fused_proj: dt_proj's product, softplus, BCNorm, MIMO fold,
//                recurrence, gated output                 (mamba.py:455-497)
//   rows_linear: out_proj + the residual add              (mamba.py:497, 591-595)
//
// xdt_proj (x_proj and dt_proj's product in one launch) serves the lane
// splits the fused step kernel does not, whose step takes dt as an input.
//
// One warp computes one output column for every row: its lanes stride the
// weight row in 16-byte chunks (512-byte coalesced loads), each lane sums its
// products in input order, then the warp adds the lanes by a fixed butterfly,
// so results are deterministic run to run.  The input rows (at most
// kSmallStage floats) are staged once per CTA in shared memory, where the
// RMSNorm is applied.  The weights are read through the read-only path; across
// the layers of a replayed step they stay resident in L2.
#include <cuda_runtime.h>
#include <stdint.h>

#include "m3_internal.h"
#include "m3_pdl.cuh"

namespace m3 {
namespace {

constexpr int kLinThreads = 256;
constexpr int kLinWarps = kLinThreads / 32;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, m));
  return v;
}

// torch's silu in fp32: z / (1 + exp(-z))
__device__ __forceinline__ float silu_f(float z) {
  return __fdiv_rn(z, __fadd_rn(1.0f, expf(-z)));
}

// Dot products of one weight row w (K floats, 16-byte aligned, K % 4 == 0)
// with the RW staged rows of s; every lane returns the warp totals.  Each
// lane loads the row in batches of kBatch 16-byte loads issued before they are
// used, so a row of up to kBatch * 512 bytes costs one memory latency; `a`
// holds the first batch on entry (load_batch), which lets a kernel issue it
// before it waits for its inputs.
constexpr int kBatch = 8;

__device__ __forceinline__ void load_batch(const float* __restrict__ w, int K4, int k0,
                                           float4 (&a)[kBatch]) {
  const float4* w4 = reinterpret_cast<const float4*>(w);
#pragma unroll
  for (int j = 0; j < kBatch; ++j)
    if (k0 + 32 * j < K4) a[j] = __ldg(w4 + k0 + 32 * j);
}

template <int RW>
__device__ __forceinline__ void row_dots(const float* __restrict__ w, const float* s, int K,
                                         int lane, float4 (&a)[kBatch], float (&acc)[RW]) {
  const float4* s4 = reinterpret_cast<const float4*>(s);
  const int K4 = K >> 2;
#pragma unroll
  for (int r = 0; r < RW; ++r) acc[r] = 0.f;
  for (int k0 = lane; k0 < K4; k0 += 32 * kBatch) {
    if (k0 != lane) load_batch(w, K4, k0, a);
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      if (k0 + 32 * j < K4) {
#pragma unroll
        for (int r = 0; r < RW; ++r) {
          const float4 x = s4[r * K4 + k0 + 32 * j];
          acc[r] = __fmaf_rn(a[j].x, x.x, acc[r]);
          acc[r] = __fmaf_rn(a[j].y, x.y, acc[r]);
          acc[r] = __fmaf_rn(a[j].z, x.z, acc[r]);
          acc[r] = __fmaf_rn(a[j].w, x.w, acc[r]);
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < RW; ++r) acc[r] = warp_sum(acc[r]);
}

// The total of row `lane` (lanes >= RW get row 0's; callers mask them).
template <int RW>
__device__ __forceinline__ float lane_row(const float (&acc)[RW], int lane) {
  float v = acc[0];
#pragma unroll
  for (int r = 1; r < RW; ++r)
    if (lane == r) v = acc[r];
  return v;
}

// Stage RW rows of x into s (rows past `rows` read zero), RMS-normalised when
// norm_w is given: x * rsqrt(mean(x^2) + eps) * w  (mamba.py:88-89).  NT: the
// CTA's threads.  vec (x rows and norm_w 16-byte aligned): one 16-byte load
// per thread and row, every row's load issued before any is used.
template <int RW, int NT>
__device__ void stage_rows(float* s, const float* x, long long ld_x, int rows, int K,
                           const float* norm_w, float eps, bool vec) {
  __shared__ float s_rstd[RW];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int K4 = K >> 2;
  float4* s4 = reinterpret_cast<float4*>(s);
  if (vec) {
    for (int k = tid; k < K4; k += NT) {
      float4 v[RW];
#pragma unroll
      for (int r = 0; r < RW; ++r)
        v[r] = r < rows ? reinterpret_cast<const float4*>(x + (size_t)r * ld_x)[k]
                        : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int r = 0; r < RW; ++r) s4[r * K4 + k] = v[r];
    }
  } else {
    for (int i = tid; i < RW * K; i += NT) {
      const int r = i / K, k = i - r * K;
      s[i] = r < rows ? x[(size_t)r * ld_x + k] : 0.f;
    }
  }
  __syncthreads();
  if (norm_w == nullptr) return;
  for (int r = warp; r < RW; r += NT / 32) {
    float ss = 0.f;
    for (int k = lane; k < K; k += 32) ss = __fmaf_rn(s[r * K + k], s[r * K + k], ss);
    ss = warp_sum(ss);
    if (lane == 0) s_rstd[r] = rsqrtf(__fadd_rn(__fdiv_rn(ss, (float)K), eps));
  }
  __syncthreads();
  if (vec) {
    for (int k = tid; k < K4; k += NT) {
      const float4 w = reinterpret_cast<const float4*>(norm_w)[k];
#pragma unroll
      for (int r = 0; r < RW; ++r) {
        float4 v = s4[r * K4 + k];
        const float rs = s_rstd[r];
        v.x = __fmul_rn(__fmul_rn(v.x, rs), w.x);
        v.y = __fmul_rn(__fmul_rn(v.y, rs), w.y);
        v.z = __fmul_rn(__fmul_rn(v.z, rs), w.z);
        v.w = __fmul_rn(__fmul_rn(v.w, rs), w.w);
        s4[r * K4 + k] = v;
      }
    }
  } else {
    for (int i = tid; i < RW * K; i += NT) {
      const int r = i / K, k = i - r * K;
      s[i] = __fmul_rn(__fmul_rn(s[i], s_rstd[r]), norm_w[k]);
    }
  }
  __syncthreads();
}

// out = act(residual + (bias + norm(x) W^T)); the residual is added last, as
// the reference adds the layer's output to its input (mamba.py:595).
// Launched as a programmatic dependent launch (p.pdl), the first batch of
// each warp's weight row is loaded before the kernel waits for the kernel
// ahead of it, so that load overlaps the previous layer's tail.
template <int RW>
__global__ void __launch_bounds__(kLinThreads) rows_linear_kernel(const RowsLinearParams p) {
  extern __shared__ __align__(16) float s_x[];   // [RW][d_in]
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int o0 = blockIdx.x * kLinWarps + warp;
  float4 a[kBatch];
  if (o0 < p.d_out) load_batch(p.W + (size_t)o0 * p.d_in, p.d_in >> 2, lane, a);
  pdl_wait();
  stage_rows<RW, kLinThreads>(s_x, p.x, p.ld_x, p.rows, p.d_in, p.norm_w, p.eps, p.vec != 0);
  for (int o = o0; o < p.d_out; o += gridDim.x * kLinWarps) {
    if (o != o0) load_batch(p.W + (size_t)o * p.d_in, p.d_in >> 2, lane, a);
    float acc[RW];
    row_dots<RW>(p.W + (size_t)o * p.d_in, s_x, p.d_in, lane, a, acc);
    float v = lane_row<RW>(acc, lane);
    if (lane < p.rows) {
      if (p.bias) v = __fadd_rn(v, p.bias[o]);
      if (p.residual) v = __fadd_rn(p.residual[(size_t)lane * p.ld_r + o], v);
      if (o < p.split) {
        if (p.silu) v = silu_f(v);
        p.out0[(size_t)lane * p.ld0 + o] = v;
      } else {
        p.out1[(size_t)lane * p.ld1 + (o - p.split)] = v;
      }
    }
  }
}

// x_dbl = u W_x^T + b_x, dt = x_dbl[:, :r] W_dt^T (r <= kMaxDtRank).  Every
// CTA computes the r dt_raw columns itself (each dt needs all of them; CTA 0
// stores them) and the other x_proj columns are spread over the grid's warps;
// then each warp computes dt for groups of kDtGroup channels, its lanes
// striding each W_dt row (coalesced), all of a group's loads issued first.
constexpr int kXdtThreads = 512;
constexpr int kXdtWarps = kXdtThreads / 32;
constexpr int kDtGroup = 8;

template <int RW>
__global__ void __launch_bounds__(kXdtThreads) xdt_proj_kernel(const XdtParams p) {
  extern __shared__ __align__(16) float s_u[];   // [RW][D], then [RW][r] dt_raw
  float* s_raw = s_u + RW * p.D;
  pdl_launch_dependents();
  pdl_wait();
  stage_rows<RW, kXdtThreads>(s_u, p.u, p.D, p.rows, p.D, nullptr, 0.f, p.vec != 0);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float4 a[kBatch];
  for (int j = warp; j < p.r; j += kXdtWarps) {
    float acc[RW];
    load_batch(p.Wx + (size_t)j * p.D, p.D >> 2, lane, a);
    row_dots<RW>(p.Wx + (size_t)j * p.D, s_u, p.D, lane, a, acc);
    float v = lane_row<RW>(acc, lane);
    if (p.bx) v = __fadd_rn(v, p.bx[j]);
    if (lane < RW) s_raw[lane * p.r + j] = v;
    if (blockIdx.x == 0 && lane < p.rows) p.x_dbl[(size_t)lane * p.n_x + j] = v;
  }
  for (int j = p.r + blockIdx.x * kXdtWarps + warp; j < p.n_x; j += gridDim.x * kXdtWarps) {
    float acc[RW];
    load_batch(p.Wx + (size_t)j * p.D, p.D >> 2, lane, a);
    row_dots<RW>(p.Wx + (size_t)j * p.D, s_u, p.D, lane, a, acc);
    float v = lane_row<RW>(acc, lane);
    if (p.bx) v = __fadd_rn(v, p.bx[j]);
    if (lane < p.rows) p.x_dbl[(size_t)lane * p.n_x + j] = v;
  }
  __syncthreads();
  const int r = p.r;
  for (int d0 = (blockIdx.x * kXdtWarps + warp) * kDtGroup; d0 < p.D;
       d0 += gridDim.x * kXdtWarps * kDtGroup) {
    float wv[kDtGroup][2];
#pragma unroll
    for (int c = 0; c < kDtGroup; ++c)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int i = lane + 32 * h;
        wv[c][h] = (d0 + c < p.D && i < r) ? __ldg(p.Wdt + (size_t)(d0 + c) * r + i) : 0.f;
      }
#pragma unroll
    for (int c = 0; c < kDtGroup; ++c) {
      float acc[RW];
#pragma unroll
      for (int q = 0; q < RW; ++q) {
        float a = lane < r ? __fmul_rn(wv[c][0], s_raw[q * r + lane]) : 0.f;
        if (lane + 32 < r) a = __fmaf_rn(wv[c][1], s_raw[q * r + lane + 32], a);
        acc[q] = warp_sum(a);
      }
      const float v = lane_row<RW>(acc, lane);
      if (d0 + c < p.D && lane < p.rows) p.dt[(size_t)lane * p.D + d0 + c] = v;
    }
  }
}

template <int RW>
cudaError_t rows_linear_impl(const RowsLinearParams& p, cudaStream_t s) {
  const int grid = (p.d_out + kLinWarps - 1) / kLinWarps;
  const size_t smem = (size_t)RW * p.d_in * sizeof(float);
  return launch_maybe_pdl(p.pdl != 0, rows_linear_kernel<RW>, dim3(grid), dim3(kLinThreads), smem,
                          s, p);
}

template <int RW>
cudaError_t xdt_proj_impl(const XdtParams& p, cudaStream_t s) {
  const int g1 = (p.n_x - p.r + kXdtWarps - 1) / kXdtWarps;
  const int g2 = (p.D + kXdtWarps * kDtGroup - 1) / (kXdtWarps * kDtGroup);
  int grid = g1 > g2 ? g1 : g2;
  grid = grid < 1 ? 1 : (grid > 64 ? 64 : grid);
  const size_t smem = (size_t)RW * (p.D + p.r) * sizeof(float);
  return launch_maybe_pdl(p.pdl != 0, xdt_proj_kernel<RW>, dim3(grid), dim3(kXdtThreads), smem,
                          s, p);
}

}  // namespace

int small_rows_pad(int rows) { return rows <= 1 ? 1 : rows <= 2 ? 2 : rows <= 4 ? 4 : 8; }

cudaError_t launch_rows_linear(const RowsLinearParams& p, cudaStream_t s) {
  switch (small_rows_pad(p.rows)) {
    case 1: return rows_linear_impl<1>(p, s);
    case 2: return rows_linear_impl<2>(p, s);
    case 4: return rows_linear_impl<4>(p, s);
    default: return rows_linear_impl<8>(p, s);
  }
}

cudaError_t launch_xdt_proj(const XdtParams& p, cudaStream_t s) {
  switch (small_rows_pad(p.rows)) {
    case 1: return xdt_proj_impl<1>(p, s);
    case 2: return xdt_proj_impl<2>(p, s);
    case 4: return xdt_proj_impl<4>(p, s);
    default: return xdt_proj_impl<8>(p, s);
  }
}

}  // namespace m3
