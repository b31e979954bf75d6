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
#include <cuda.h>
#include <cudaTypedefs.h>
#include <stdlib.h>
#include <string.h>

#include "m3_common.cuh"
#include "m3_pdl.cuh"
#include "m3_internal.h"
#include "m3_bulk.cuh"
#include "m3_prologue.cuh"
#include "m3_tma.h"
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

// Output of one (row, channel): y, or with the gated epilogue of
// Mamba3Block.step (mamba.py:493-497) (y + u*D) * silu(z), in that rounding order;
// silu(z) = z / (1 + exp(-z)).
__device__ __forceinline__ float step_out(const StepParams& p, float y, float u, float ds,
                                          float z) {
  if (!p.gated) return y;
  const float sz = __fdiv_rn(z, __fadd_rn(1.0f, expf(-z)));
  return __fmul_rn(__fadd_rn(y, __fmul_rn(u, ds)), sz);
}

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
    if (q == 0 && dok)
      p.y[rd] = step_out(p, tot, uu, p.gated ? p.d_skip[d] : 0.f,
                         p.gated ? p.z[(size_t)b * p.ld_z + d] : 0.f);

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

// ---------------------------------------------------------------------------
// Pipelined fast path for dense lane tiles (N == 4*(R+T), no virtual lanes),
// D % 32 == 0 and 16-byte aligned rows.  A CTA owns one 32-channel tile for
// the whole launch (eigenvalues loaded once) and a contiguous range of row
// pairs.  Thread 0 streams each row pair's state tile (32 x N fp32 of h and of
// dBu, or of h plus the [delta*u | B] factors) and its inputs into shared
// memory with bulk asynchronous copies, kBulkStages pairs ahead of the
// compute; completion is tracked per stage on an mbarrier.  For 32-lane tiles
// the state tiles move as 2D TMA tiles with the 128-byte swizzle, so that the
// warp's 8 channel rows (128 bytes apart) do not read the same shared-memory
// banks; other tiles use 1D bulk copies of the contiguous 32 x N block.  The two rows of a
// pair are computed as the two lanes of packed FP32 instructions, with the
// rounding of the scalar cell functions, so outputs equal step_kernel's bit
// for bit.  New state goes straight from registers to global memory.
constexpr int kBulkRows = 2;   // rows per stage, one per packed lane
// Stages in flight: the factored state moves half the bytes per row, so it
// keeps more rows in flight to cover the same memory latency.
constexpr int bulk_stages(bool fact) { return fact ? 5 : 3; }

// Stage layout of a row pair.  Unswizzled: row after row, [h | S2 | delta | u |
// Bc | Cc].  Swizzled (SWZ, 32 lanes = 128-byte tile rows): the two h tiles,
// then the two S2 parts, then the small rows, padded to 1 KB, so that every
// state tile starts on the 1024-byte boundary the 128-byte swizzle needs.
// PRO (prologue fused): the delta slot holds dt, and each row also stages its
// raw B and C rows of x_proj (N*p fp32 each, p <= 2) after Cc; Bc and Cc are
// then written by the CTA from the raw rows.  Sized so that the 32-lane tile
// keeps 4 CTAs per SM (3 stages of 18 KB): a larger stage costs a resident CTA
// and with it a quarter of the bytes in flight.
template <int NP, bool FACT, bool SWZ, bool PRO = false>
struct BulkStage {
  static constexpr int kH = 32 * NP * 4;                        // h tile of one row
  static constexpr int kS2 = FACT ? 32 * 4 + NP * 4 : kH;       // dBu tile, or [du | B]
  static constexpr int kDL = 32 * 4;                            // delta or u (<= fp32)
  static constexpr int kBC = NP * 4;                            // Bc or Cc (<= fp32)
  static constexpr int kRaw = PRO ? 2 * NP * 4 : 0;             // raw B or C row (fp32)
  static constexpr int kSmall = 2 * kDL + 2 * kBC + 2 * kRaw;
  static constexpr int kRow = kH + kS2 + kSmall;
  static constexpr int kBytes = SWZ ? (kBulkRows * kRow + 1023) / 1024 * 1024 : kBulkRows * kRow;
  __device__ static constexpr int oH(int r) { return SWZ ? r * kH : r * kRow; }
  __device__ static constexpr int oS2(int r) { return SWZ ? 2 * kH + r * kS2 : r * kRow + kH; }
  __device__ static constexpr int oDL(int r) {
    return SWZ ? 2 * (kH + kS2) + r * kSmall : r * kRow + kH + kS2;
  }
  __device__ static constexpr int oU(int r) { return oDL(r) + kDL; }
  __device__ static constexpr int oB(int r) { return oDL(r) + 2 * kDL; }
  __device__ static constexpr int oC(int r) { return oB(r) + kBC; }
  __device__ static constexpr int oRB(int r) { return oC(r) + kBC; }
  __device__ static constexpr int oRC(int r) { return oRB(r) + kRaw; }
  static_assert(kS2 % 16 == 0 && kBC % 16 == 0, "bulk copy destinations are 16-byte aligned");
  static_assert(!SWZ || NP * 4 == 128, "the swizzled layout has 128-byte tile rows");
};

// n consecutive floats from float f0 of row `row` of a staged 32 x 32 fp32
// tile written by a TMA copy with the 128-byte swizzle: the 16-byte chunk c of
// tile row r lies at chunk c ^ (r & 7) (the tile starts on a 1 KB boundary).
// Each VW-float piece is VW*4-byte aligned, so it stays inside one chunk.
template <int n, int VW>
__device__ __forceinline__ void ld_vec_swz(const unsigned char* tile, int row, int f0, float* v) {
#pragma unroll
  for (int i = 0; i < n / VW; ++i) {
    const int byte = (f0 + i * VW) * 4;
    const int phys = row * 128 + ((((byte >> 4) ^ (row & 7)) << 4) | (byte & 15));
    if constexpr (VW == 4) {
      const float4 x = *reinterpret_cast<const float4*>(tile + phys);
      v[4 * i] = x.x; v[4 * i + 1] = x.y; v[4 * i + 2] = x.z; v[4 * i + 3] = x.w;
    } else if constexpr (VW == 2) {
      const float2 x = *reinterpret_cast<const float2*>(tile + phys);
      v[2 * i] = x.x; v[2 * i + 1] = x.y;
    } else {
      v[i] = *reinterpret_cast<const float*>(tile + phys);
    }
  }
}

// n fp32 (dt == M3_F32) or bf16 values of a staged row, widened to fp32.
template <int n>
__device__ __forceinline__ void ld_staged(const unsigned char* base, int off, bool bf16, float* v) {
  if (bf16) ld_vec_bf16<n>(reinterpret_cast<const __nv_bfloat16*>(base) + off, v);
  else ld_vec<n, vec_width(n)>(reinterpret_cast<const float*>(base) + off, v);
}

template <int R, int T, bool FACT, bool SWZ, bool PRO>
__global__ void __launch_bounds__(kThreads, step_min_blocks(R + T))
    step_bulk_kernel(const StepParams p, int pairs_per_cta,
                     const __grid_constant__ CUtensorMap tmap_h,
                     const __grid_constant__ CUtensorMap tmap_d) {
  using LM = LaneMap<R, T>;
  constexpr int NL = R + T;
  constexpr int NP = LM::NP;
  constexpr int RR = R > 0 ? R : 1;
  constexpr int TT = T > 0 ? T : 1;
  constexpr int VR = vec_width(RR), VT = vec_width(TT);
  using SL = BulkStage<NP, FACT, SWZ, PRO>;
  static_assert(!PRO || kThreads == 128, "the fused prologue uses one warp per (row, B|C)");
  constexpr int kBulkStages = bulk_stages(FACT);
  extern __shared__ __align__(128) unsigned char smem_raw[];
  // launched as a programmatic dependent launch (p.pdl), the kernel starts
  // while the one ahead of it finishes and waits here before reading anything
  pdl_launch_dependents();
  pdl_wait();
  // stage buffers (from the first 1 KB boundary when swizzled), then one
  // mbarrier per stage
  unsigned char* smem =
      SWZ ? smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u) : smem_raw;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kBulkStages * SL::kBytes);

  const int tid = threadIdx.x, q = tid & 3, grp = tid >> 2;
  const int D = p.D;
  const int d0 = blockIdx.y * 32, d = d0 + grp;
  const int npairs = (p.B + 1) / 2;
  const int pair0 = blockIdx.x * pairs_per_cta;
  const int n = min(pairs_per_cta, npairs - pair0);
  const bool bf_du = p.dt_du == M3_BF16, bf_bc = !PRO && p.dt_bc == M3_BF16;
  const int esd = bf_du ? 2 : 4, esb = bf_bc ? 2 : 4;
  const int np_raw = PRO ? p.N * p.P : 0;   // raw B/C row length (PRO)

  float a2[RR], ai[RR], tk[TT];
  float maxai = 0.f;
  const float dskip = p.gated ? p.d_skip[d] : 0.f;
#pragma unroll
  for (int j = 0; j < NL; ++j) {
    const int m = LM::mem_lane(q, j, p.NR, p.NT);   // dense tile: never virtual
    const size_t gp = (size_t)d * NP + m;
    if (j < R) {
      a2[j] = exp_const(p.Ar[gp]);
      ai[j] = p.Ai[gp];
      maxai = fmaxf(maxai, fabsf(ai[j]));
    } else {
      tk[j - R] = p.Tk[gp];
    }
  }

  if (tid == 0) {
#pragma unroll
    for (int s = 0; s < kBulkStages; ++s) mbar_init(&full[s], 1);
    mbar_fence_init();
  }
  __syncthreads();

  // PRO: dt (fp32; none when the kernel forms dt itself) and u, then the raw
  // B and C rows instead of Bc and Cc
  const bool dtproj = PRO && p.wdt != nullptr;
  const uint32_t row_tx = SL::kH + (FACT ? 32 * 4 + NP * 4 : SL::kH) +
                          (PRO ? (dtproj ? 0 : 32 * 4) + 32 * esd + 2 * np_raw * 4
                               : 2 * 32 * esd + 2 * NP * esb);
  auto issue = [&](int i) {   // thread 0: stage the row pair pair0 + i
    const int s = i % kBulkStages;
    unsigned char* st = smem + s * SL::kBytes;
    const int b0 = 2 * (pair0 + i);
    const int nr = min(2, p.B - b0);
    mbar_arrive_expect_tx(&full[s], nr * row_tx);
    for (int r = 0; r < nr; ++r) {
      const size_t b = (size_t)(b0 + r);
      if constexpr (SWZ) {
        tma_load_2d(st + SL::oH(r), &tmap_h, 0, (int)(b * D + d0), &full[s]);
      } else {
        bulk_g2s(st + SL::oH(r), p.h + (b * D + d0) * NP, SL::kH, &full[s]);
      }
      if constexpr (FACT) {
        const float* fac = p.fac_in + b * (D + NP);
        bulk_g2s(st + SL::oS2(r), fac + d0, 32 * 4, &full[s]);
        bulk_g2s(st + SL::oS2(r) + 32 * 4, fac + D, NP * 4, &full[s]);
      } else if constexpr (SWZ) {
        tma_load_2d(st + SL::oS2(r), &tmap_d, 0, (int)(b * D + d0), &full[s]);
      } else {
        bulk_g2s(st + SL::oS2(r), p.dbu + (b * D + d0) * NP, SL::kH, &full[s]);
      }
      if constexpr (PRO) {
        if (!dtproj) bulk_g2s(st + SL::oDL(r), p.dt + b * p.ld_dt + d0, 32 * 4, &full[s]);
        bulk_g2s(st + SL::oU(r), (const char*)p.u + (b * D + d0) * esd, 32 * esd, &full[s]);
        bulk_g2s(st + SL::oRB(r), p.xbc + b * p.ld_x + p.off_b, np_raw * 4, &full[s]);
        bulk_g2s(st + SL::oRC(r), p.xbc + b * p.ld_x + p.off_c, np_raw * 4, &full[s]);
      } else {
        bulk_g2s(st + SL::oDL(r), (const char*)p.delta + (b * D + d0) * esd, 32 * esd,
                 &full[s]);
        bulk_g2s(st + SL::oU(r), (const char*)p.u + (b * D + d0) * esd, 32 * esd, &full[s]);
        bulk_g2s(st + SL::oB(r), (const char*)p.Bc + b * NP * esb, NP * esb, &full[s]);
        bulk_g2s(st + SL::oC(r), (const char*)p.Cc + b * NP * esb, NP * esb, &full[s]);
      }
    }
  };

  if (tid == 0) {
    for (int i = 0; i < min(kBulkStages, n); ++i) issue(i);
  }

  int fail_at = -1;
  for (int i = 0; i < n; ++i) {
    const int s = i % kBulkStages;
    const int b0 = 2 * (pair0 + i);
    const bool two = b0 + 1 < p.B;
    // dtproj: dt of channel d for the pair's rows, x_proj's dt_raw columns
    // times the channel's dt_proj row, the 4 quarters striding the dt_rank
    // terms and summed in quad_sum's order; loaded and formed before the wait
    // so their latency overlaps the stage's copies
    float dtw[2] = {0.f, 0.f};
    if (dtproj) {
      const float* wr = p.wdt + (size_t)d * p.dt_rank;
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const float* xr = p.xbc + (size_t)(r == 1 && !two ? b0 : b0 + r) * p.ld_x;
        float acc = 0.f;
#pragma unroll
        for (int k = 0; k < kMaxDtRank / 4; ++k) {
          const int j = q + 4 * k;
          if (j < p.dt_rank) acc = __fmaf_rn(__ldg(wr + j), xr[j], acc);
        }
        dtw[r] = quad_sum(acc);
      }
    }
    const bool ok = mbar_wait(&full[s], (uint32_t)((i / kBulkStages) & 1));
    if constexpr (PRO) {
      // Bc / Cc of the pair from the staged raw rows: warp w normalises and
      // folds (row w/2, B or C) exactly as step_inputs_kernel does (one warp
      // per row, the same lane order), so the values equal the unfused
      // chain's; the whole warp takes part (warp-uniform condition)
      const int w = tid >> 5, lane = tid & 31, r = w >> 1;
      if (r == 0 || two) {
        unsigned char* st = smem + s * SL::kBytes;
        const float* x = reinterpret_cast<const float*>(st + ((w & 1) ? SL::oRC(r) : SL::oRB(r)));
        const float* wv = (w & 1) ? p.wc : p.wb;
        auto ld = [&](int k) { return x[k]; };
        const float rs = bcnorm_scale(ld, np_raw, p.eps, wv != nullptr, lane);
        float* dst = reinterpret_cast<float*>(st + ((w & 1) ? SL::oC(r) : SL::oB(r)));
        for (int nn = lane; nn < NP; nn += 32) dst[nn] = bcnorm_fold(ld, nn, p.P, rs, wv);
      }
      __syncthreads();
    }

    // ---- staged row pair -> registers (row 0 in .x, row 1 in .y)
    float2 h2[NL], db2[NL], B2[NL], C2[NL], dl2, uu2;
    {
      float hv[2][NL], dv[2][NL], bv[2][NL], cv[2][NL], dlv[2], uv[2];
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const unsigned char* st = smem + s * SL::kBytes;
        if (r == 1 && !two) {
#pragma unroll
          for (int j = 0; j < NL; ++j) { hv[r][j] = 0.f; dv[r][j] = 0.f; bv[r][j] = 0.f; cv[r][j] = 0.f; }
          dlv[r] = 0.f; uv[r] = 0.f;
          continue;
        }
        if constexpr (SWZ) {
          if constexpr (R > 0) ld_vec_swz<R, VR>(st + SL::oH(r), grp, q * R, hv[r]);
          if constexpr (T > 0) ld_vec_swz<T, VT>(st + SL::oH(r), grp, 4 * R + q * T, hv[r] + R);
        } else {
          const float* hs = reinterpret_cast<const float*>(st + SL::oH(r)) + grp * NP;
          if constexpr (R > 0) ld_vec<R, VR>(hs + q * R, hv[r]);
          if constexpr (T > 0) ld_vec<T, VT>(hs + 4 * R + q * T, hv[r] + R);
        }
        if constexpr (FACT) {
          const float dup = reinterpret_cast<const float*>(st + SL::oS2(r))[grp];
          const float* bp = reinterpret_cast<const float*>(st + SL::oS2(r) + 32 * 4);
          float bf[NL];
          if constexpr (R > 0) ld_vec<R, VR>(bp + q * R, bf);
          if constexpr (T > 0) ld_vec<T, VT>(bp + 4 * R + q * T, bf + R);
#pragma unroll
          for (int j = 0; j < NL; ++j) dv[r][j] = __fmul_rn(dup, bf[j]);
        } else if constexpr (SWZ) {
          if constexpr (R > 0) ld_vec_swz<R, VR>(st + SL::oS2(r), grp, q * R, dv[r]);
          if constexpr (T > 0) ld_vec_swz<T, VT>(st + SL::oS2(r), grp, 4 * R + q * T, dv[r] + R);
        } else {
          const float* ds = reinterpret_cast<const float*>(st + SL::oS2(r)) + grp * NP;
          if constexpr (R > 0) ld_vec<R, VR>(ds + q * R, dv[r]);
          if constexpr (T > 0) ld_vec<T, VT>(ds + 4 * R + q * T, dv[r] + R);
        }
        if constexpr (PRO) {   // delta = softplus(dt + bias), as step_inputs_kernel
          const float dtv = dtproj ? dtw[r] : reinterpret_cast<const float*>(st + SL::oDL(r))[grp];
          dlv[r] = softplus20(p.dt_bias != nullptr ? __fadd_rn(dtv, p.dt_bias[d]) : dtv);
        } else {
          dlv[r] = bf_du ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(st + SL::oDL(r))[grp])
                         : reinterpret_cast<const float*>(st + SL::oDL(r))[grp];
        }
        uv[r] = bf_du ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(st + SL::oU(r))[grp])
                      : reinterpret_cast<const float*>(st + SL::oU(r))[grp];
        if constexpr (R > 0) {
          ld_staged<R>(st + SL::oB(r), q * R, bf_bc, bv[r]);
          ld_staged<R>(st + SL::oC(r), q * R, bf_bc, cv[r]);
        }
        if constexpr (T > 0) {
          ld_staged<T>(st + SL::oB(r), 4 * R + q * T, bf_bc, bv[r] + R);
          ld_staged<T>(st + SL::oC(r), 4 * R + q * T, bf_bc, cv[r] + R);
        }
      }
#pragma unroll
      for (int j = 0; j < NL; ++j) {
        h2[j] = make_float2(hv[0][j], hv[1][j]);
        db2[j] = make_float2(dv[0][j], dv[1][j]);
        B2[j] = make_float2(bv[0][j], bv[1][j]);
        C2[j] = make_float2(cv[0][j], cv[1][j]);
      }
      dl2 = make_float2(dlv[0], dlv[1]);
      uu2 = make_float2(uv[0], uv[1]);
    }
    // gated epilogue: z of the pair, loaded now, used after the recurrence
    float zz[2] = {0.f, 0.f};
    if (p.gated && q == 0) {
      zz[0] = p.z[(size_t)b0 * p.ld_z + d];
      if (two) zz[1] = p.z[(size_t)(b0 + 1) * p.ld_z + d];
    }
    // every thread has read stage s: it may be refilled (or the launch gives up)
    if (__syncthreads_or(!ok)) { fail_at = i; break; }
    if (tid == 0 && i + kBulkStages < n) issue(i + kBulkStages);

    // ---- recurrence (the cell arithmetic of m3_common.cuh, two rows per instruction)
    const float2 du2 = __fmul2_rn(dl2, uu2);
    float2 H2[NL], ds2[NL];
    const bool fast = __fmul_rn(fmaxf(fabsf(dl2.x), fabsf(dl2.y)), maxai) <= kFastArgBound;
#pragma unroll
    for (int j = 0; j < NL; ++j) {
      const float2 P = __fadd2_rn(__fmul2_rn(f2(2.f), h2[j]), db2[j]);
      float2 g;
      if (j < R) {
        if (fast) {
          g = __fmul2_rn(gate_exp2(dl2, f2(a2[j % RR])), gate_cos2_nocheck(dl2, f2(ai[j % RR])));
        } else {
          g = make_float2(rot_gate(dl2.x, a2[j % RR], ai[j % RR]),
                          rot_gate(dl2.y, a2[j % RR], ai[j % RR]));
        }
      } else {
        g = f2(tk[(j - R) % TT]);
      }
      ds2[j] = __fmul2_rn(du2, B2[j]);
      H2[j] = __ffma2_rn(g, P, ds2[j]);
    }
    float2 acc = f2(0.f);
#pragma unroll
    for (int j = 0; j < NL; ++j) acc = __ffma2_rn(H2[j], C2[j], acc);
    const float y0 = __fmul_rn(0.5f, quad_sum(acc.x));
    const float y1 = __fmul_rn(0.5f, quad_sum(acc.y));

    // ---- new state, factors and y
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      if (r == 1 && !two) break;
      const size_t b = (size_t)(b0 + r);
      float hs[NL], dsv[NL];
#pragma unroll
      for (int j = 0; j < NL; ++j) {
        const float2 hh = __fmul2_rn(f2(0.5f), H2[j]);
        hs[j] = r ? hh.y : hh.x;
        dsv[j] = r ? ds2[j].y : ds2[j].x;
      }
      float* ho = p.h + (b * D + d) * NP;
      if constexpr (R > 0) st_vec<R, VR>(ho + q * R, hs);
      if constexpr (T > 0) st_vec<T, VT>(ho + 4 * R + q * T, hs + R);
      if constexpr (FACT) {
        float* fac = p.fac_out + b * (D + NP);
        if (q == 0) fac[d] = r ? du2.y : du2.x;
        if (blockIdx.y == 0 && grp == 0) {
          float bvv[NL];
#pragma unroll
          for (int j = 0; j < NL; ++j) bvv[j] = r ? B2[j].y : B2[j].x;
          if constexpr (R > 0) st_vec<R, VR>(fac + D + q * R, bvv);
          if constexpr (T > 0) st_vec<T, VT>(fac + D + 4 * R + q * T, bvv + R);
        }
      } else {
        float* dout = p.dbu + (b * D + d) * NP;
        if constexpr (R > 0) st_vec<R, VR>(dout + q * R, dsv);
        if constexpr (T > 0) st_vec<T, VT>(dout + 4 * R + q * T, dsv + R);
      }
      if (q == 0) p.y[b * D + d] = step_out(p, r ? y1 : y0, r ? uu2.y : uu2.x, dskip, zz[r]);
    }
  }

  if (fail_at >= 0 && tid == 0) {
    set_err(p.err, M3_ERR_DEVICE);
    // let the copies still in flight land before the CTA's shared memory goes away
    for (int i = fail_at; i < min(fail_at + kBulkStages, n); ++i)
      mbar_wait(&full[i % kBulkStages], (uint32_t)((i / kBulkStages) & 1));
  }
}

// A (rows, 32) fp32 state tensor as a 2D tensor map whose box is one 32-channel
// tile (32 rows of 128 bytes) with the 128-byte swizzle.
bool encode_state_map(CUtensorMap* map, const float* base, size_t rows) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  if (enc == nullptr) return false;
  const cuuint64_t dims[2] = {32, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {32 * sizeof(float)};
  const cuuint32_t box[2] = {32, 32};
  const cuuint32_t elem[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides,
             box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

template <int R, int T, bool FACT, bool SWZ, bool PRO>
cudaError_t launch_step_bulk_kernel(const StepParams& p, cudaStream_t stream,
                                    const CUtensorMap& mh, const CUtensorMap& md) {
  using SL = BulkStage<4 * (R + T), FACT, SWZ, PRO>;
  constexpr int kBulkStages = bulk_stages(FACT);
  auto kern = step_bulk_kernel<R, T, FACT, SWZ, PRO>;
  const int smem = kBulkStages * SL::kBytes + kBulkStages * (int)sizeof(uint64_t) +
                   (SWZ ? 1024 : 0);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 0, occ = 0;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
  if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
    return e;
  if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kThreads, smem)) !=
      cudaSuccess)
    return e;
  if (occ < 1) occ = 1;
  const int tiles = p.D / 32;
  const int npairs = (p.B + 1) / 2;
  int g = (sms * occ) / tiles;          // one resident wave when the tiles allow it
  if (g < 1) g = 1;
  if (g > npairs) g = npairs;
  const int per = (npairs + g - 1) / g;
  g = (npairs + per - 1) / per;
  dim3 grid(g, tiles);
  return launch_maybe_pdl(p.pdl != 0, kern, grid, dim3(kThreads), (size_t)smem, stream, p, per,
                          mh, md);
}


template <int R, int T, bool FACT, bool PRO>
cudaError_t launch_step_bulk_pro(const StepParams& p, cudaStream_t stream) {
  CUtensorMap mh, md;
  memset(&mh, 0, sizeof(mh));
  memset(&md, 0, sizeof(md));
  if constexpr (4 * (R + T) == 32) {
    const size_t rows = (size_t)p.B * p.D;
    if (getenv("M3_NO_SWIZZLE") == nullptr && encode_state_map(&mh, p.h, rows) &&
        (FACT || encode_state_map(&md, p.dbu, rows)))
      return launch_step_bulk_kernel<R, T, FACT, true, PRO>(p, stream, mh, md);
  }
  return launch_step_bulk_kernel<R, T, FACT, false, PRO>(p, stream, mh, md);
}

// The fused prologue is compiled for the 32-lane tiles (the Search-Mamba and
// Eval-Mamba shapes); other tiles report cudaErrorNotSupported (nothing is
// launched) and the caller runs the prologue kernel and the step separately.
template <int R, int T, bool FACT>
cudaError_t launch_step_bulk_impl(const StepParams& p, cudaStream_t stream) {
  if (p.pro) {
    if constexpr (4 * (R + T) == 32) return launch_step_bulk_pro<R, T, FACT, true>(p, stream);
    return cudaErrorNotSupported;
  }
  return launch_step_bulk_pro<R, T, FACT, false>(p, stream);
}

template <int R, int T, bool FACT>
cudaError_t launch_step_impl(const StepParams& p, cudaStream_t stream) {
  dim3 grid((p.B + kRowsPerCta - 1) / kRowsPerCta, (p.D + 31) / 32);
  step_kernel<R, T, FACT><<<grid, kThreads, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_step(const Tile& t, const StepParams& p, cudaStream_t s) {
#define M3_X(r, tt, nd, ndb, nthb, gs)                                             \
  if (t.R == r && t.T == tt) {                                                     \
    if (p.pro && !p.bulk) return cudaErrorNotSupported;                            \
    if (p.bulk)                                                                    \
      return p.factored ? launch_step_bulk_impl<r, tt, true>(p, s)                 \
                        : launch_step_bulk_impl<r, tt, false>(p, s);               \
    return p.factored ? launch_step_impl<r, tt, true>(p, s)                        \
                      : launch_step_impl<r, tt, false>(p, s);                      \
  }
  M3_TILE_LIST(M3_X)
#undef M3_X
  return cudaErrorInvalidValue;
}

}  // namespace m3
