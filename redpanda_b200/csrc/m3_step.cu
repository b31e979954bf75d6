// K4: batched lockstep O(1) recurrent step, in place on the caller's (h, dBu).
//
// Replaces the recurrence part of Mamba3Block.step (redpanda/engine/mamba.py:466-493):
// gate, dBu_t, trapezoidal token, state update and y = sum_n h*C, for B rows at
// once (the MARS batched rollout, redpanda/engine/mars_search.py:440-446).
//
// The thread -> (channel, state lane) map and every rounded operation are the
// ones of the forward scan (m3_common.cuh), so a step from the scan's state
// reproduces the scan's next output bit for bit.  The kernel is HBM-bound:
// per cell it reads h and dBu (8 B) and writes them back (8 B).
#include "m3_common.cuh"
#include "m3_internal.h"
#include "m3_tiles.h"

namespace m3 {
namespace {

template <int R, int T>
__global__ void __launch_bounds__(kThreads) step_kernel(const StepParams p) {
  using LM = LaneMap<R, T>;
  constexpr int NL = R + T;
  const int tid = threadIdx.x, q = tid & 3, grp = tid >> 2;
  const int b = blockIdx.x;
  const int d = blockIdx.y * 32 + grp;
  const int D = p.D, N = p.N;
  const bool dok = d < D;

  const size_t rd = (size_t)b * D + (dok ? d : 0);
  const float dl = dok ? ld_f(p.delta, rd, p.dt_du) : 0.f;
  const float uu = dok ? ld_f(p.u, rd, p.dt_du) : 0.f;
  const float du = __fmul_rn(dl, uu);

  int lane[NL];
  float Bv[NL], Cv[NL], h[NL], dbp[NL];
#pragma unroll
  for (int j = 0; j < NL; ++j) {
    const int n = LM::mem_lane(q, j, p.NR, p.NT);
    lane[j] = (dok && n >= 0) ? n : -1;
    const size_t gb = (size_t)b * N + (n >= 0 ? n : 0);
    Bv[j] = n >= 0 ? ld_f(p.Bc, gb, p.dt_bc) : 0.f;
    Cv[j] = n >= 0 ? ld_f(p.Cc, gb, p.dt_bc) : 0.f;
    const size_t gs = (rd * N) + (lane[j] >= 0 ? lane[j] : 0);
    h[j] = lane[j] >= 0 ? p.h[gs] : 0.f;
    dbp[j] = lane[j] >= 0 ? p.dbu[gs] : 0.f;
  }

  float H[NL];
#pragma unroll
  for (int j = 0; j < NL; ++j) {
    // P = 2h + dBu_prev, the scan's carried register (2h is exact)
    float P = __fadd_rn(__fmul_rn(2.f, h[j]), dbp[j]);
    const size_t gp = (size_t)(dok ? d : 0) * N + (lane[j] >= 0 ? lane[j] : 0);
    float g;
    if (j < R) {
      const float ar = lane[j] >= 0 ? exp_const(p.Ar[gp]) : 0.f;
      const float ai = lane[j] >= 0 ? p.Ai[gp] : 0.f;
      g = rot_gate(dl, ar, ai);
    } else {
      g = lane[j] >= 0 ? p.Tk[gp] : 0.f;
    }
    H[j] = cell_update(g, P, du, Bv[j]);
  }
  const float tot = __fmul_rn(0.5f, quad_sum(y_partial<NL>(H, Cv)));
  if (q == 0 && dok) p.y[rd] = tot;
#pragma unroll
  for (int j = 0; j < NL; ++j) {
    if (lane[j] >= 0) {
      const size_t gs = rd * N + lane[j];
      p.h[gs] = __fmul_rn(0.5f, H[j]);
      p.dbu[gs] = __fmul_rn(du, Bv[j]);
    }
  }
}

template <int R, int T>
cudaError_t launch_step_impl(const StepParams& p, cudaStream_t stream) {
  dim3 grid(p.B, (p.D + 31) / 32);
  step_kernel<R, T><<<grid, kThreads, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_step(const Tile& t, const StepParams& p, cudaStream_t s) {
#define M3_X(r, tt, nd, ndb, nthb) \
  if (t.R == r && t.T == tt) return launch_step_impl<r, tt>(p, s);
  M3_TILE_LIST(M3_X)
#undef M3_X
  return cudaErrorInvalidValue;
}

}  // namespace m3
