// K2: analytic backward of the trapezoidal scan, causal / reverse / both
// directions, with deterministic reductions.
//
// Replaces _bwd_kernel (redpanda/engine/triton_scan.py:100-241) and the
// backward half of _TrapezoidalScanFn (triton_scan.py:283-315).  Gradients, per
// cell, with q[t] = dL/dh[t] and P[t] = 2h[t] + dBu[t]:
//   q[t]     = dy[t]*C[t] + gate[t+1]*q[t+1]
//   dgate[t] = 0.5*q[t]*P[t-1]                  (= q*h[t-1] + 0.5*q*dBu[t-1])
//   ddBu[t]  = 0.5*q[t] + 0.5*gate[t+1]*q[t+1]  (= q[t] - 0.5*dy[t]*C[t])
//   dA_real += dgate*delta*gate,  dA_imag -= dgate*delta*exp*sin,  dtrack += dgate
//   ddelta   = sum_n dgate*(A_real*gate - A_imag*exp*sin) + u*sum_n ddBu*B
//   du       = delta*sum_n ddBu*B
//   dB[t,n]  = sum_d ddBu*delta*u,   dC[t,n] = sum_d dy*h[t]
//
// Work split: CTA (batch group bg, channel tile g) walks its rows b = bg,
// bg + Bg, ... and, per row and direction, the kCK-step chunks from last to
// first.  Each chunk restarts from the forward's checkpoint of P, recomputes
// the chunk forward storing P[t-1] of every cell in Tensor Memory, then runs
// the reverse recurrence reading P back.  dA_real/dA_imag/dtrack accumulate in
// registers over the CTA's rows and land in one partial per batch group;
// dB/dC are reduced over the CTA's channels (warp shuffles + shared memory)
// into one partial per channel tile.  A second kernel sums both partial sets in
// a fixed order, so results are bitwise reproducible run to run.
#include "m3_common.cuh"
#include "m3_internal.h"
#include "m3_tiles.h"
#include "m3_tmem.cuh"

namespace m3 {
namespace {

constexpr int pow2ceil(int x) {
  int p = 1;
  while (p < x) p <<= 1;
  return p;
}

template <int R, int T, int ND>
struct BwdCfg {
  static constexpr int NL = R + T;
  static constexpr int NP = 4 * NL;
  static constexpr int DT = 32 * ND;
  static constexpr int C = ND * NL;                 // cells per thread
  static constexpr int CS = pow2ceil(C);            // TMEM columns per timestep
  static constexpr int NCOLS = (kCK * CS < 32) ? 32 : kCK * CS;
  static constexpr size_t smem_floats =
      3 * (size_t)kCK * DT + 2 * (size_t)kCK * NP + (size_t)kCK * 4 * 2 * NP;
  static constexpr size_t smem_bytes = smem_floats * 4 + 16;
};

template <int R, int T, int ND>
__global__ void __launch_bounds__(kThreads, 1) scan_bwd_kernel(const BwdParams p) {
  using LM = LaneMap<R, T>;
  using CF = BwdCfg<R, T, ND>;
  constexpr int NL = CF::NL, NP = CF::NP, DT = CF::DT, C = CF::C, CS = CF::CS;
  constexpr int RR = R > 0 ? R : 1;
  constexpr int TT = T > 0 ? T : 1;
  static_assert(CF::NCOLS <= 512, "TMEM holds at most 512 columns");

  extern __shared__ __align__(16) float sm[];
  float* s_dl = sm;                          // [kCK][DT]
  float* s_u = s_dl + kCK * DT;              // [kCK][DT]
  float* s_dy = s_u + kCK * DT;              // [kCK][DT]
  float* s_b = s_dy + kCK * DT;              // [kCK][NP]
  float* s_c = s_b + kCK * NP;               // [kCK][NP]
  float* s_red = s_c + kCK * NP;             // [kCK][4 warps][2][NP]
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(s_red + kCK * 4 * 2 * NP);

  const int tid = threadIdx.x, q = tid & 3, grp = tid >> 2;
  const int warp = tid >> 5, lane = tid & 31;
  const int bg = blockIdx.x, gt = blockIdx.y;
  const int d0 = gt * DT, dbase = d0 + grp * ND;
  const int B = p.B, L = p.L, D = p.D, N = p.N;
  const bool bidir = p.direction == M3_DIR_BIDIR;
  const int ndirs = bidir ? 2 : 1;

  if (warp == 0) tmem_alloc(s_tmem, CF::NCOLS);
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  const uint32_t tbase = *s_tmem + ((uint32_t)(warp * 32) << 16);

  float ar[ND][RR], ai[ND][RR], tk[ND][TT];
#pragma unroll
  for (int k = 0; k < ND; ++k) {
    const int d = dbase + k;
#pragma unroll
    for (int j = 0; j < NL; ++j) {
      const int n = LM::mem_lane(q, j, p.NR, p.NT);
      const bool ok = (d < D) && (n >= 0);
      const size_t gi = ok ? (size_t)d * N + n : 0;
      if (j < R) {
        ar[k][j] = ok ? p.Ar[gi] : 0.f;
        ai[k][j] = ok ? p.Ai[gi] : 0.f;
      } else {
        tk[k][j - R] = ok ? p.Tk[gi] : 0.f;
      }
    }
  }

  float gAr[ND][RR], gAi[ND][RR], gTk[ND][TT];
#pragma unroll
  for (int k = 0; k < ND; ++k) {
#pragma unroll
    for (int j = 0; j < RR; ++j) { gAr[k][j] = 0.f; gAi[k][j] = 0.f; }
#pragma unroll
    for (int j = 0; j < TT; ++j) gTk[k][j] = 0.f;
  }

  const int cta = gt * p.Bg + bg;
  float* scratch = p.scratch_du ? p.scratch_du + (size_t)cta * L * DT * 2 : nullptr;

  for (int b = bg; b < B; b += p.Bg) {
    for (int pass = 0; pass < ndirs; ++pass) {
      const int dir = bidir ? pass : p.direction;
      const int dslot = bidir ? dir : 0;
      const bool first_of_two = bidir && pass == 0;
      const bool second_of_two = bidir && pass == 1;

      float qv[ND][NL], gn[ND][RR];
#pragma unroll
      for (int k = 0; k < ND; ++k) {
#pragma unroll
        for (int j = 0; j < NL; ++j) qv[k][j] = 0.f;
#pragma unroll
        for (int j = 0; j < RR; ++j) gn[k][j] = 0.f;
      }

      for (int c = p.nch - 1; c >= 0; --c) {
        const int s0 = c * kCK;
        const int ns = min(kCK, L - s0);
        __syncthreads();  // previous chunk's shared-memory readers are done
        for (int i = tid; i < kCK * DT; i += kThreads) {
          const int tt = i / DT, dd = i - tt * DT;
          const int s = s0 + tt, d = d0 + dd;
          const bool ok = (s < L) && (d < D);
          const int t = dir ? L - 1 - s : s;
          const size_t gi = ok ? ((size_t)b * L + t) * D + d : 0;
          s_dl[i] = ok ? ld_f(p.delta, gi, p.dt_du) : 0.f;
          s_u[i] = ok ? ld_f(p.u, gi, p.dt_du) : 0.f;
          s_dy[i] = ok ? ld_f(p.dy, gi, p.dt_dy) : 0.f;
        }
        for (int i = tid; i < kCK * NP; i += kThreads) {
          const int tt = i / NP, ln = i - tt * NP;
          const int s = s0 + tt;
          const int n = LM::mem_lane(ln / NL, ln % NL, p.NR, p.NT);
          const bool ok = (s < L) && (n >= 0);
          const int t = dir ? L - 1 - s : s;
          const size_t gi = ok ? ((size_t)b * L + t) * N + n : 0;
          s_b[i] = ok ? ld_f(p.Bc, gi, p.dt_bc) : 0.f;
          s_c[i] = ok ? ld_f(p.Cc, gi, p.dt_bc) : 0.f;
        }
        float P[C];
#pragma unroll
        for (int k = 0; k < ND; ++k) {
          const int d = dbase + k;
          const float* src =
              (c > 0 && d < D)
                  ? p.ckpt + ((((size_t)b * ndirs + dslot) * (p.nch - 1) + (c - 1)) * D + d) * NP +
                        q * NL
                  : nullptr;
#pragma unroll
          for (int j = 0; j < NL; ++j) P[k * NL + j] = src ? src[j] : 0.f;
        }
        __syncthreads();

        // ---- forward recompute of the chunk; P[t-1] of every cell -> TMEM
        for (int tt = 0; tt < ns; ++tt) {
          tmem_store<C>(tbase + (uint32_t)(tt * CS), P);
          const float* rdl = s_dl + tt * DT + grp * ND;
          const float* ru = s_u + tt * DT + grp * ND;
          const float* rb = s_b + tt * NP + q * NL;
#pragma unroll
          for (int k = 0; k < ND; ++k) {
            const float dl = rdl[k];
            const float du = __fmul_rn(dl, ru[k]);
#pragma unroll
            for (int j = 0; j < R; ++j)
              cell_update(rot_gate(dl, ar[k][j], ai[k][j]), P[k * NL + j], du, rb[j]);
#pragma unroll
            for (int j = R; j < NL; ++j) cell_update(tk[k][j - R], P[k * NL + j], du, rb[j]);
          }
        }
        tmem_wait_st();

        // ---- reverse recurrence
        for (int tt = ns - 1; tt >= 0; --tt) {
          float Pp[C];
          tmem_load<C>(tbase + (uint32_t)(tt * CS), Pp);
          tmem_wait_ld();
          const int s = s0 + tt;
          const int t = dir ? L - 1 - s : s;
          const float* rdl = s_dl + tt * DT + grp * ND;
          const float* ru = s_u + tt * DT + grp * ND;
          const float* rdy = s_dy + tt * DT + grp * ND;
          const float* rb = s_b + tt * NP + q * NL;
          const float* rc = s_c + tt * NP + q * NL;
          float Bv[NL], Cv[NL], pB[NL], pC[NL];
#pragma unroll
          for (int j = 0; j < NL; ++j) {
            Bv[j] = rb[j];
            Cv[j] = rc[j];
            pB[j] = 0.f;
            pC[j] = 0.f;
          }
          float gsum[ND], sbs[ND];
#pragma unroll
          for (int k = 0; k < ND; ++k) {
            const float dl = rdl[k], uu = ru[k], dyv = rdy[k];
            const float du = __fmul_rn(dl, uu);
            float gs = 0.f, sB = 0.f;
#pragma unroll
            for (int j = 0; j < R; ++j) {
              const float pp = Pp[k * NL + j];
              const float e = expf(__fmul_rn(dl, ar[k][j]));
              float sn, cs;
              sincosf(__fmul_rn(dl, ai[k][j]), &sn, &cs);
              const float g = __fmul_rn(e, cs);
              const float es = __fmul_rn(e, sn);
              const float dbu = __fmul_rn(du, Bv[j]);
              const float H = __fmaf_rn(g, pp, dbu);
              const float dyC = __fmul_rn(dyv, Cv[j]);
              const float qn = __fmaf_rn(gn[k][j], qv[k][j], dyC);
              const float ddbu = __fmaf_rn(-0.5f, dyC, qn);
              const float wp = __fmul_rn(qn, pp);
              const float wg = __fmul_rn(wp, g);
              const float ws = __fmul_rn(wp, es);
              gAr[k][j] = __fmaf_rn(dl, wg, gAr[k][j]);
              gAi[k][j] = __fmaf_rn(-dl, ws, gAi[k][j]);
              gs = __fmaf_rn(ar[k][j], wg, gs);
              gs = __fmaf_rn(-ai[k][j], ws, gs);
              sB = __fmaf_rn(ddbu, Bv[j], sB);
              pB[j] = __fmaf_rn(ddbu, du, pB[j]);
              pC[j] = __fmaf_rn(dyv, H, pC[j]);
              qv[k][j] = qn;
              gn[k][j] = g;
            }
#pragma unroll
            for (int j = R; j < NL; ++j) {
              const float pp = Pp[k * NL + j];
              const float g = tk[k][j - R];
              const float dbu = __fmul_rn(du, Bv[j]);
              const float H = __fmaf_rn(g, pp, dbu);
              const float dyC = __fmul_rn(dyv, Cv[j]);
              const float qn = __fmaf_rn(g, qv[k][j], dyC);
              const float ddbu = __fmaf_rn(-0.5f, dyC, qn);
              const float wp = __fmul_rn(qn, pp);
              gTk[k][j - R] = __fadd_rn(gTk[k][j - R], wp);
              sB = __fmaf_rn(ddbu, Bv[j], sB);
              pB[j] = __fmaf_rn(ddbu, du, pB[j]);
              pC[j] = __fmaf_rn(dyv, H, pC[j]);
              qv[k][j] = qn;
            }
            gsum[k] = gs;
            sbs[k] = sB;
          }
          // per-channel outputs: reduce over the 4 lane quarters
#pragma unroll
          for (int k = 0; k < ND; ++k) {
            const float gsv = quad_sum(gsum[k]);
            const float sBv = quad_sum(sbs[k]);
            const int d = dbase + k;
            if ((k & 3) == q && d < D) {
              float ddl = __fmaf_rn(0.5f, gsv, __fmul_rn(sBv, ru[k]));
              float ddu = __fmul_rn(sBv, rdl[k]);
              const size_t oi = ((size_t)b * L + t) * D + d;
              float* sc = scratch ? scratch + ((size_t)t * DT + (d - d0)) * 2 : nullptr;
              if (first_of_two) {
                sc[0] = ddl;
                sc[1] = ddu;
              } else {
                if (second_of_two) {
                  ddl = __fadd_rn(sc[0], ddl);
                  ddu = __fadd_rn(sc[1], ddu);
                }
                st_f(p.d_delta, oi, p.dt_du, ddl);
                st_f(p.d_u, oi, p.dt_du, ddu);
              }
            }
          }
          // dB/dC partial over this warp's 8 channel groups
#pragma unroll
          for (int j = 0; j < NL; ++j) {
#pragma unroll
            for (int m = 4; m < 32; m <<= 1) {
              pB[j] = __fadd_rn(pB[j], __shfl_xor_sync(0xffffffffu, pB[j], m));
              pC[j] = __fadd_rn(pC[j], __shfl_xor_sync(0xffffffffu, pC[j], m));
            }
          }
          if (lane < 4) {
            float* r0 = s_red + ((size_t)(tt * 4 + warp) * 2) * NP + q * NL;
#pragma unroll
            for (int j = 0; j < NL; ++j) {
              r0[j] = pB[j];
              r0[NP + j] = pC[j];
            }
          }
        }
        __syncthreads();
        // flush this chunk's dB/dC partials: fixed order over the 4 warps
        for (int i = tid; i < ns * 2 * NP; i += kThreads) {
          const int tt = i / (2 * NP), rem = i - tt * 2 * NP;
          const int which = rem / NP, ln = rem - which * NP;
          const float* r = s_red + ((size_t)tt * 4 * 2 + which) * NP + ln;
          const float v = __fadd_rn(__fadd_rn(__fadd_rn(r[0], r[2 * NP]), r[4 * NP]), r[6 * NP]);
          const int s = s0 + tt;
          const int t = dir ? L - 1 - s : s;
          float* dst = p.part_bc + ((((size_t)gt * B + b) * L + t) * 2 + which) * NP + ln;
          *dst = second_of_two ? __fadd_rn(*dst, v) : v;
        }
      }
    }
  }

  // dA partial of this batch group
#pragma unroll
  for (int k = 0; k < ND; ++k) {
    const int d = dbase + k;
    if (d < D) {
      float* a0 = p.part_a + (((size_t)bg * 3 + 0) * D + d) * NP + q * NL;
      float* a1 = p.part_a + (((size_t)bg * 3 + 1) * D + d) * NP + q * NL;
      float* a2 = p.part_a + (((size_t)bg * 3 + 2) * D + d) * NP + q * NL;
#pragma unroll
      for (int j = 0; j < R; ++j) { a0[j] = gAr[k][j]; a1[j] = gAi[k][j]; a2[j] = 0.f; }
#pragma unroll
      for (int j = R; j < NL; ++j) { a0[j] = 0.f; a1[j] = 0.f; a2[j] = gTk[k][j - R]; }
    }
  }

  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  if (warp == 0) tmem_dealloc(*s_tmem, CF::NCOLS);
}

// ---------------------------------------------------------------- reductions
// Lane index (q*NL + j) of memory state lane n.
__device__ __forceinline__ int pad_lane(int n, int NR, int R, int T) {
  if (n < NR) return (n / R) * (R + T) + (n % R);
  const int k = n - NR;
  return (k / T) * (R + T) + R + (k % T);
}

__global__ void reduce_bc_kernel(const ReduceParams p, int R, int T) {
  const size_t total = (size_t)p.B * p.L * p.N;
  const int NP = 4 * (R + T);
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
       i += (size_t)gridDim.x * blockDim.x) {
    const int n = (int)(i % p.N);
    const size_t bt = i / p.N;
    const int ln = pad_lane(n, p.NR, R, T);
    float vb = 0.f, vc = 0.f;
    for (int g = 0; g < p.G; ++g) {
      const float* src = p.part_bc + (((size_t)g * p.B * p.L + bt) * 2) * NP + ln;
      vb = __fadd_rn(vb, src[0]);
      vc = __fadd_rn(vc, src[NP]);
    }
    st_f(p.d_Bc, i, p.dt_bc, vb);
    st_f(p.d_Cc, i, p.dt_bc, __fmul_rn(0.5f, vc));
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

template <int R, int T, int ND>
cudaError_t launch_bwd_impl(const BwdParams& p, cudaStream_t stream) {
  using CF = BwdCfg<R, T, ND>;
  auto kern = scan_bwd_kernel<R, T, ND>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)CF::smem_bytes);
  if (e != cudaSuccess) return e;
  dim3 grid(p.Bg, p.G);
  kern<<<grid, kThreads, CF::smem_bytes, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_scan_bwd(const Tile& t, const BwdParams& p, cudaStream_t s) {
#define M3_X(r, tt, nd) \
  if (t.R == r && t.T == tt && t.ND == nd) return launch_bwd_impl<r, tt, nd>(p, s);
  M3_TILE_LIST(M3_X)
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
