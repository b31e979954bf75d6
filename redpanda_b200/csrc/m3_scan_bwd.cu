// K2 dispatch: tile and element-type selection for the analytic backward, the
// element-wise-staging variants (run-time element types) and the fixed-order
// reductions of the partials.  The bulk-staged variants, one per combination
// of delta/u and dy element types, are compiled in m3_scan_bwd_bulk_*.cu (in
// parallel) from the kernel template in m3_scan_bwd.cuh.
#include "m3_scan_bwd.cuh"

namespace m3 {

// defined in m3_scan_bwd_bulk_<du><dy>.cu: launch the bulk-staged kernel of
// tile t; *handled is false when the tile's bulk layout does not fit
cudaError_t launch_bwd_bulk_bf16_bf16(const Tile& t, const BwdParams& p, cudaStream_t s,
                                      bool* handled);
cudaError_t launch_bwd_bulk_bf16_f32(const Tile& t, const BwdParams& p, cudaStream_t s,
                                     bool* handled);
cudaError_t launch_bwd_bulk_f32_bf16(const Tile& t, const BwdParams& p, cudaStream_t s,
                                     bool* handled);
cudaError_t launch_bwd_bulk_f32_f32(const Tile& t, const BwdParams& p, cudaStream_t s,
                                    bool* handled);

namespace {

// ---------------------------------------------------------------- reductions
// Lane index (q*NL + j) of memory state lane n.
__device__ __forceinline__ int pad_lane(int n, int NR, int R, int T) {
  if (n < NR) return (n / R) * (R + T) + (n % R);
  const int k = n - NR;
  return (k / T) * (R + T) + R + (k % T);
}

// Position (j*4 + q) of memory state lane n in the dB/dC partial rows.
__device__ __forceinline__ int part_lane(int n, int NR, int R, int T) {
  if (n < NR) return (n % R) * 4 + n / R;
  const int k = n - NR;
  return (R + k % T) * 4 + k / T;
}

__global__ void reduce_bc_kernel(const ReduceParams p, int R, int T) {
  const size_t total = (size_t)p.B * p.L * p.N;
  const int NP = 4 * (R + T);
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const int n = (int)(i % p.N);
    const size_t bt = i / p.N;
    const int ln = part_lane(n, p.NR, R, T);
    float vb = 0.f, vc = 0.f;
    for (int g = 0; g < p.G * p.ndirs; ++g) {   // channel tiles x directions, fixed order
      const float* src = p.part_bc + (((size_t)g * p.B * p.L + bt) * 2) * NP + ln;
      vb = __fadd_rn(vb, src[0]);
      vc = __fadd_rn(vc, src[NP]);
    }
    if (p.bc_f32_of_bf16) {   // the fused prologue's backward reads them (fp32 of the bf16 grads)
      static_cast<float*>(p.d_Bc)[i] = __bfloat162float(__float2bfloat16_rn(vb));
      static_cast<float*>(p.d_Cc)[i] = __bfloat162float(__float2bfloat16_rn(__fmul_rn(0.5f, vc)));
    } else {
      st_f(p.d_Bc, i, p.dt_bc, vb);
      st_f(p.d_Cc, i, p.dt_bc, __fmul_rn(0.5f, vc));
    }
  }
}

__global__ void reduce_a_kernel(const ReduceParams p, int R, int T) {
  const size_t total = (size_t)p.D * p.N;
  const int NP = 4 * (R + T);
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const int n = (int)(i % p.N);
    const size_t d = i / p.N;
    const int ln = pad_lane(n, p.NR, R, T);
    float v0 = 0.f, v1 = 0.f, v2 = 0.f;
    for (int g = 0; g < p.Bg; ++g) {
      const float* src = p.part_a + ((size_t)g * 3 * p.D + d) * NP + ln;
      v0 = __fadd_rn(v0, src[0]);
      v1 = __fadd_rn(v1, src[(size_t)p.D * NP]);
      v2 = __fadd_rn(v2, src[2 * (size_t)p.D * NP]);
    }
    const bool rot = n < p.NR;
    p.dAr[i] = rot ? __fmul_rn(0.5f, v0) : 0.f;
    p.dAi[i] = rot ? __fmul_rn(0.5f, v1) : 0.f;
    p.dTk[i] = rot ? 0.f : __fmul_rn(0.5f, v2);
  }
}

}  // namespace

cudaError_t launch_bwd_bulk_pro(const Tile& t, const BwdParams& p, cudaStream_t s,
                                bool* handled);

cudaError_t launch_scan_bwd(const Tile& t, const BwdParams& p, cudaStream_t s) {
  if (p.pro) {   // bf16 bulk-staged kernels only (the C ABI checks eligibility first)
    bool handled = false;
    const cudaError_t e = launch_bwd_bulk_pro(t, p, s, &handled);
    return handled ? e : cudaErrorNotSupported;
  }
  if (p.bulk) {
    bool handled = false;
    const bool du = p.dt_du == M3_BF16, dy = p.dt_dy == M3_BF16;
    const cudaError_t e = du ? (dy ? launch_bwd_bulk_bf16_bf16(t, p, s, &handled)
                                   : launch_bwd_bulk_bf16_f32(t, p, s, &handled))
                             : (dy ? launch_bwd_bulk_f32_bf16(t, p, s, &handled)
                                   : launch_bwd_bulk_f32_f32(t, p, s, &handled));
    if (handled) return e;
  }
#define M3_X(r, tt, nd, ndb, nthb, gs)                                              \
  if constexpr (ndb > 0)                                                            \
    if (t.R == r && t.T == tt && t.ND == nd)                                        \
      return bwd::launch_bwd_impl<r, tt, ndb, nthb, (gs != 0), false, -1, -1>(p, s);
  M3_TILE_LIST(M3_X)
  M3_SMALL_TILE_LIST(M3_X)
#undef M3_X
  return cudaErrorInvalidValue;
}
cudaError_t launch_bwd_reduce(const Tile& t, const ReduceParams& p, cudaStream_t s) {
  const int threads = 256;
  const size_t nbc = (size_t)p.B * p.L * p.N;
  const size_t na = (size_t)p.D * p.N;
  const int gbc = (int)((nbc + threads - 1) / threads < 148 * 16 ? (nbc + threads - 1) / threads
                                                                  : 148 * 16);
  const int ga = (int)((na + threads - 1) / threads < 148 * 16 ? (na + threads - 1) / threads
                                                                : 148 * 16);
  reduce_bc_kernel<<<gbc, threads, 0, s>>>(p, t.R, t.T);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  reduce_a_kernel<<<ga, threads, 0, s>>>(p, t.R, t.T);
  return cudaGetLastError();
}

}  // namespace m3
