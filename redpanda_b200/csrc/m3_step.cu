// K4: batched lockstep O(1) recurrent step, in place on the caller's state.
//
// Replaces the recurrence part of Mamba3Block.step (redpanda/engine/mamba.py:466-493):
// gate, dBu_t, trapezoidal token, state update and y = sum_n h*C, for B rows at
// once (the MARS batched rollout, redpanda/engine/mars_search.py:440-446).
//
// The thread -> (channel, state lane) map and every rounded operation are the
// ones of the forward scan (m3_common.cuh), so a step from the scan's state
// reproduces the scan's next output bit for bit.  The kernel is HBM-bound.
// A CTA owns 32 channels of kRowsPerCta consecutive rows: eigenvalues are
// loaded once per CTA, the next row's state and inputs are prefetched into
// registers while the current row computes, and state rows move as
// float2/float4 where the lane layout allows.
//
// Two state formats:
//  * full (the reference's cache contract): h and dBu, both (B, D, N) fp32;
//    16 bytes of HBM traffic per cell.
//  * factored: h (B, D, N) and fac (B, D + N) = [delta*u (D) | B (N)] of the
//    last token.  dBu = (delta*u)*B is recomputed with the same rounded
//    multiply the scan uses, so results are identical; 8 bytes per cell.
//    h is updated in place; the factors go from fac_in to a separate fac_out
//    (every channel tile of a row reads the row's B factors, so they cannot be
//    overwritten while the step runs).
#include "m3_common.cuh"
#include "m3_internal.h"
#include "m3_stage.cuh"
#include "m3_tiles.h"

namespace m3 {
namespace {

#ifndef M3_STEP_ROWS
#define M3_STEP_ROWS 4
#endif
constexpr int kRowsPerCta = M3_STEP_ROWS;

// Resident CTAs per SM asked of the register allocator: the step is bound by
// the bytes in flight, so small lane tiles trade registers for more warps
// (at 8 lanes per thread, 4 CTAs of 128 threads beat 3 by 4 %); larger tiles
// keep enough registers to hold two rows without spilling.
constexpr int step_min_blocks(int lanes) { return lanes <= 8 ? 4 : (lanes <= 16 ? 2 : 1); }

// Load / store n consecutive floats with the widest access the compile-time
// layout allows (VW = 4, 2 or 1 floats; the caller guarantees alignment).
template <int n, int VW>
__device__ __forceinline__ void ld_vec(const float* src, float* v) {
  if constexpr (VW == 4) {
#pragma unroll
    for (int i = 0; i < n / 4; ++i) {
      const float4 x = reinterpret_cast<const float4*>(src)[i];
      v[4 * i] = x.x; v[4 * i + 1] = x.y; v[4 * i + 2] = x.z; v[4 * i + 3] = x.w;
    }
  } else if constexpr (VW == 2) {
#pragma unroll
    for (int i = 0; i < n / 2; ++i) {
      const float2 x = reinterpret_cast<const float2*>(src)[i];
      v[2 * i] = x.x; v[2 * i + 1] = x.y;
    }
  } else {
#pragma unroll
    for (int i = 0; i < n; ++i) v[i] = src[i];
  }
}

template <int n, int VW>
__device__ __forceinline__ void st_vec(float* dst, const float* v) {
  if constexpr (VW == 4) {
#pragma unroll
    for (int i = 0; i < n / 4; ++i)
      reinterpret_cast<float4*>(dst)[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
  } else if constexpr (VW == 2) {
#pragma unroll
    for (int i = 0; i < n / 2; ++i)
      reinterpret_cast<float2*>(dst)[i] = make_float2(v[2 * i], v[2 * i + 1]);
  } else {
#pragma unroll
    for (int i = 0; i < n; ++i) dst[i] = v[i];
  }
}

// n consecutive bf16 widened to fp32: pairs when n is even (the caller
// guarantees 4-byte alignment of src then), single elements otherwise.
template <int n>
__device__ __forceinline__ void ld_vec_bf16(const __nv_bfloat16* src, float* v) {
  if constexpr (n % 2 == 0) {
#pragma unroll
    for (int i = 0; i < n / 2; ++i) {
      const float2 x = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(src)[i]);
      v[2 * i] = x.x; v[2 * i + 1] = x.y;
    }
  } else {
#pragma unroll
    for (int i = 0; i < n; ++i) v[i] = __bfloat162float(src[i]);
  }
}

constexpr int vec_width(int n) { return n % 4 == 0 ? 4 : (n % 2 == 0 ? 2 : 1); }

template <int R, int T, bool FACT>
__global__ void __launch_bounds__(kThreads, step_min_blocks(R + T)) step_kernel(const StepParams p) {
  using LM = LaneMap<R, T>;
  constexpr int NL = R + T;
  constexpr int RR = R > 0 ? R : 1;
  constexpr int TT = T > 0 ? T : 1;
  constexpr int VR = vec_width(RR), VT = vec_width(TT);
  const int tid = threadIdx.x, q = tid & 3, grp = tid >> 2;
  const int row0 = blockIdx.x * kRowsPerCta;
  const int d = blockIdx.y * 32 + grp;
  const int D = p.D, N = p.N;
  const bool dok = d < D;
  const bool vec = p.NR == 4 * R && p.NT == 4 * T && (N % 4) == 0;

  int lane[NL];
  float a2[RR], ai[RR], tk[TT];
  float maxai = 0.f;
#pragma unroll
  for (int j = 0; j < NL; ++j) {
    const int n = LM::mem_lane(q, j, p.NR, p.NT);
    lane[j] = (dok && n >= 0) ? n : -1;
    const size_t gp = (size_t)(dok ? d : 0) * N + (n >= 0 ? n : 0);
    if (j < R) {
      a2[j] = lane[j] >= 0 ? exp_const(p.Ar[gp]) : 0.f;
      ai[j] = lane[j] >= 0 ? p.Ai[gp] : 0.f;
      maxai = fmaxf(maxai, fabsf(ai[j]));
    } else {
      tk[j - R] = lane[j] >= 0 ? p.Tk[gp] : 0.f;
    }
  }

  auto load_state = [&](int b, float (&h)[NL], float (&dbp)[NL]) {
    const size_t rd = (size_t)b * D + (dok ? d : 0);
    if (vec && dok) {
      const float* hs = p.h + rd * N;
      if constexpr (R > 0) ld_vec<R, VR>(hs + q * R, h);
      if constexpr (T > 0) ld_vec<T, VT>(hs + 4 * R + q * T, h + R);
      if constexpr (!FACT) {
        const float* ds = p.dbu + rd * N;
        if constexpr (R > 0) ld_vec<R, VR>(ds + q * R, dbp);
        if constexpr (T > 0) ld_vec<T, VT>(ds + 4 * R + q * T, dbp + R);
      }
    } else {
#pragma unroll
      for (int j = 0; j < NL; ++j) {
        const size_t gs = rd * N + (lane[j] >= 0 ? lane[j] : 0);
        h[j] = lane[j] >= 0 ? p.h[gs] : 0.f;
        if constexpr (!FACT) dbp[j] = lane[j] >= 0 ? p.dbu[gs] : 0.f;
      }
    }
    if constexpr (FACT) {
      const float* fac = p.fac_in + (size_t)b * (D + N);
      const float dup = dok ? fac[d] : 0.f;
      float bf[NL];
      if (vec && p.vec_fac) {
        if constexpr (R > 0) ld_vec<R, VR>(fac + D + q * R, bf);
        if constexpr (T > 0) ld_vec<T, VT>(fac + D + 4 * R + q * T, bf + R);
      } else {
#pragma unroll
        for (int j = 0; j < NL; ++j) {
          const int n = LM::mem_lane(q, j, p.NR, p.NT);
          bf[j] = n >= 0 ? fac[D + n] : 0.f;
        }
      }
#pragma unroll
      for (int j = 0; j < NL; ++j) dbp[j] = (lane[j] >= 0) ? __fmul_rn(dup, bf[j]) : 0.f;
    }
  };

  // per-row inputs (delta, u, B, C) of one row; B and C rows move as vectors
  // when the lane layout and the pointers allow
  auto load_inputs = [&](int b, float& dl, float& uu, float (&Bv)[NL], float (&Cv)[NL]) {
    const size_t rd = (size_t)b * D + (dok ? d : 0);
    dl = dok ? ld_f(p.delta, rd, p.dt_du) : 0.f;
    uu = dok ? ld_f(p.u, rd, p.dt_du) : 0.f;
    const size_t rb = (size_t)b * N;
    if (vec && p.vec_bc && p.dt_bc == M3_F32) {
      const float* bs = static_cast<const float*>(p.Bc) + rb;
      const float* cs = static_cast<const float*>(p.Cc) + rb;
      if constexpr (R > 0) { ld_vec<R, VR>(bs + q * R, Bv); ld_vec<R, VR>(cs + q * R, Cv); }
      if constexpr (T > 0) {
        ld_vec<T, VT>(bs + 4 * R + q * T, Bv + R);
        ld_vec<T, VT>(cs + 4 * R + q * T, Cv + R);
      }
    } else if (vec && p.vec_bc) {
      const __nv_bfloat16* bs = static_cast<const __nv_bfloat16*>(p.Bc) + rb;
      const __nv_bfloat16* cs = static_cast<const __nv_bfloat16*>(p.Cc) + rb;
      if constexpr (R > 0) { ld_vec_bf16<R>(bs + q * R, Bv); ld_vec_bf16<R>(cs + q * R, Cv); }
      if constexpr (T > 0) {
        ld_vec_bf16<T>(bs + 4 * R + q * T, Bv + R);
        ld_vec_bf16<T>(cs + 4 * R + q * T, Cv + R);
      }
    } else {
#pragma unroll
      for (int j = 0; j < NL; ++j) {
        const int n = LM::mem_lane(q, j, p.NR, p.NT);
        const size_t gb = rb + (n >= 0 ? n : 0);
        Bv[j] = n >= 0 ? ld_f(p.Bc, gb, p.dt_bc) : 0.f;
        Cv[j] = n >= 0 ? ld_f(p.Cc, gb, p.dt_bc) : 0.f;
      }
    }
  };

  float h[NL], dbp[NL], dl = 0.f, uu = 0.f, Bv[NL], Cv[NL];
  const int nrows = min(kRowsPerCta, p.B - row0);
  if (nrows > 0) {
    load_state(row0, h, dbp);
    load_inputs(row0, dl, uu, Bv, Cv);
  }
  for (int r = 0; r < nrows; ++r) {
    const int b = row0 + r;
    const size_t rd = (size_t)b * D + (dok ? d : 0);
    // prefetch the next row's state and inputs while this row computes
    float hn[NL], dbn[NL], dln = 0.f, uun = 0.f, Bn[NL], Cn[NL];
    if (r + 1 < nrows) {
      load_state(b + 1, hn, dbn);
      load_inputs(b + 1, dln, uun, Bn, Cn);
    }

    const float du = __fmul_rn(dl, uu);
    float H[NL];
    if (__fmul_rn(fabsf(dl), maxai) <= kFastArgBound) {
#pragma unroll
      for (int j = 0; j < R; ++j) {
        float P = __fadd_rn(__fmul_rn(2.f, h[j]), dbp[j]);
        const float g = __fmul_rn(gate_exp(dl, a2[j]),
                                  gate_cos2_nocheck(f2(dl), f2(ai[j])).x);
        H[j] = cell_update(g, P, du, Bv[j]);
      }
    } else {
#pragma unroll
      for (int j = 0; j < R; ++j) {
        float P = __fadd_rn(__fmul_rn(2.f, h[j]), dbp[j]);
        H[j] = cell_update(rot_gate(dl, a2[j], ai[j]), P, du, Bv[j]);
      }
    }
#pragma unroll
    for (int j = R; j < NL; ++j) {
      float P = __fadd_rn(__fmul_rn(2.f, h[j]), dbp[j]);
      H[j] = cell_update(tk[j - R], P, du, Bv[j]);
    }
    const float tot = __fmul_rn(0.5f, quad_sum(y_partial<NL>(H, Cv)));
    if (q == 0 && dok) p.y[rd] = tot;

    float hs[NL], ds[NL];
#pragma unroll
    for (int j = 0; j < NL; ++j) {
      hs[j] = __fmul_rn(0.5f, H[j]);
      ds[j] = __fmul_rn(du, Bv[j]);
    }
    if (vec && dok) {
      float* ho = p.h + rd * N;
      if constexpr (R > 0) st_vec<R, VR>(ho + q * R, hs);
      if constexpr (T > 0) st_vec<T, VT>(ho + 4 * R + q * T, hs + R);
      if constexpr (!FACT) {
        float* dout = p.dbu + rd * N;
        if constexpr (R > 0) st_vec<R, VR>(dout + q * R, ds);
        if constexpr (T > 0) st_vec<T, VT>(dout + 4 * R + q * T, ds + R);
      }
    } else {
#pragma unroll
      for (int j = 0; j < NL; ++j) {
        if (lane[j] >= 0) {
          const size_t gs = rd * N + lane[j];
          p.h[gs] = hs[j];
          if constexpr (!FACT) p.dbu[gs] = ds[j];
        }
      }
    }
    if constexpr (FACT) {
      float* fac = p.fac_out + (size_t)b * (D + N);
      if (q == 0 && dok) fac[d] = du;
      if (blockIdx.y == 0 && grp == 0) {
#pragma unroll
        for (int j = 0; j < NL; ++j) {
          const int n = LM::mem_lane(q, j, p.NR, p.NT);
          if (n >= 0) fac[D + n] = Bv[j];
        }
      }
    }
#pragma unroll
    for (int j = 0; j < NL; ++j) {
      h[j] = hn[j]; dbp[j] = dbn[j]; Bv[j] = Bn[j]; Cv[j] = Cn[j];
    }
    dl = dln;
    uu = uun;
  }
}

template <int R, int T, bool FACT>
cudaError_t launch_step_impl(const StepParams& p, cudaStream_t stream) {
  dim3 grid((p.B + kRowsPerCta - 1) / kRowsPerCta, (p.D + 31) / 32);
  step_kernel<R, T, FACT><<<grid, kThreads, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_step(const Tile& t, const StepParams& p, cudaStream_t s) {
#define M3_X(r, tt, nd, ndb, nthb)                                                 \
  if (t.R == r && t.T == tt)                                                       \
    return p.factored ? launch_step_impl<r, tt, true>(p, s)                        \
                      : launch_step_impl<r, tt, false>(p, s);
  M3_TILE_LIST(M3_X)
#undef M3_X
  return cudaErrorInvalidValue;
}

}  // namespace m3
