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
#include "m3_stage.cuh"
#include "m3_tiles.h"
#include "m3_tmem.cuh"

namespace m3 {
namespace {

constexpr int pow2ceil(int x) {
  int p = 1;
  while (p < x) p <<= 1;
  return p;
}

template <int R, int T, int ND, int NTH>
struct BwdCfg {
  static constexpr int NL = R + T;
  static constexpr int NP = 4 * NL;
  static constexpr int NW = NTH / 32;               // warps
  static constexpr int DT = NTH / 4 * ND;           // channels per CTA
  static constexpr int C = ND * NL;                 // cells per thread
  static constexpr int CS = pow2ceil(C);            // TMEM columns per timestep
  static constexpr int WG_COLS = kCK * CS;          // TMEM columns per warpgroup
  static constexpr int NCOLS = (NTH / 128) * WG_COLS < 32 ? 32 : (NTH / 128) * WG_COLS;
  static constexpr size_t raw_bytes = (size_t)kCK * DT * 4;   // one staged (kCK x DT) tile
  static constexpr size_t smem_bytes =
      3 * 2 * raw_bytes                       // delta, u, dy (HBM dtype), double-buffered
      + 2 * (size_t)DT * NP * 4               // checkpoint tile, double-buffered
      + 2 * 2 * (size_t)kCK * NP * 4          // B, C (fp32), double-buffered
      + (size_t)kCK * NW * 2 * NP * 4         // dB/dC warp partials
      + 16;                                   // TMEM address slot
};

// Stage a (kCK x DT) tile of a (B, L, D) tensor for processing steps
// [s0, s0 + kCK) in its HBM dtype; rows past L and channels past D read zero.
template <int DT, int NTH>
__device__ __forceinline__ void stage_tile(unsigned char* dst, const void* src, int esz,
                                           bool async_ok, int b, int d0, int s0, int dir,
                                           int L, int D) {
  if (async_ok) {
    const int epw = 4 / esz, wpr = DT / epw;
    for (int i = threadIdx.x; i < kCK * wpr; i += NTH) {
      const int tt = i / wpr, w = i - tt * wpr;
      const int s = s0 + tt, d = d0 + w * epw;
      const bool ok = (s < L) && (d < D);
      const int t = dir ? L - 1 - s : s;
      const size_t gi = ok ? ((size_t)b * L + t) * D + d : 0;
      cp_async4(dst + (size_t)i * 4, (const char*)src + gi * esz, ok);
    }
  } else {
    for (int i = threadIdx.x; i < kCK * DT; i += NTH) {
      const int tt = i / DT, dd = i - tt * DT;
      const int s = s0 + tt, d = d0 + dd;
      const bool ok = (s < L) && (d < D);
      const int t = dir ? L - 1 - s : s;
      const size_t gi = ok ? ((size_t)b * L + t) * D + d : 0;
      if (esz == 2) ((uint16_t*)dst)[i] = ok ? ((const uint16_t*)src)[gi] : (uint16_t)0;
      else ((float*)dst)[i] = ok ? ((const float*)src)[gi] : 0.f;
    }
  }
}

template <int R, int T, int ND, int NTH>
__global__ void __launch_bounds__(NTH, 1) scan_bwd_kernel(const BwdParams p) {
  using LM = LaneMap<R, T>;
  using CF = BwdCfg<R, T, ND, NTH>;
  constexpr int NL = CF::NL, NP = CF::NP, DT = CF::DT, C = CF::C, CS = CF::CS, NW = CF::NW;
  constexpr int RR = R > 0 ? R : 1;
  constexpr int TT = T > 0 ? T : 1;
  constexpr int BCE = (kCK * NP + NTH - 1) / NTH;
  constexpr int V = 2 * NL;                  // dB + dC partials per thread per step
  constexpr int V8 = (V + 7) / 8 * 8;        // padded to the 8-group butterfly
  static_assert(CF::NCOLS <= 512, "TMEM holds at most 512 columns");

  extern __shared__ __align__(16) unsigned char smem[];
  unsigned char* s_dl = smem;                                   // [2][raw]
  unsigned char* s_u = s_dl + 2 * CF::raw_bytes;                // [2][raw]
  unsigned char* s_dy = s_u + 2 * CF::raw_bytes;                // [2][raw]
  float* s_ck = reinterpret_cast<float*>(s_dy + 2 * CF::raw_bytes);  // [2][DT][NP]
  float* s_b = s_ck + 2 * DT * NP;                              // [2][kCK][NP]
  float* s_c = s_b + 2 * kCK * NP;                              // [2][kCK][NP]
  float* s_red = s_c + 2 * kCK * NP;                            // [kCK][NW][2][NP]
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(s_red + kCK * NW * 2 * NP);

  const int tid = threadIdx.x, q = tid & 3, grp = tid >> 2;
  const int warp = tid >> 5, lane = tid & 31;
  const int bg = blockIdx.x, gt = blockIdx.y;
  const int d0 = gt * DT, dbase = d0 + grp * ND;
  const int B = p.B, L = p.L, D = p.D, N = p.N;
  const bool bidir = p.direction == M3_DIR_BIDIR;
  const int ndirs = bidir ? 2 : 1;
  const int nch = p.nch;
  const bool bf_du = p.dt_du == M3_BF16, bf_dy = p.dt_dy == M3_BF16;
  const int es_du = bf_du ? 2 : 4, es_dy = bf_dy ? 2 : 4;
  const bool async_du = p.async_du, async_dy = p.async_dy;

  if (warp == 0) tmem_alloc(s_tmem, CF::NCOLS);
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  // warp w reads/writes TMEM lanes 32*(w%4).. of column block w/4
  const uint32_t tbase =
      *s_tmem + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)((warp >> 2) * CF::WG_COLS);

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

  // work items in processing order: rows b = bg, bg+Bg, ...; per row the
  // directions; per direction the chunks from last to first
  const int rows = bg < B ? (B - bg + p.Bg - 1) / p.Bg : 0;
  const int per_row = ndirs * nch;
  const int nitems = rows * per_row;
  auto item = [&](int i, int& b, int& pass, int& c) {
    const int r = i / per_row, rem = i - r * per_row;
    b = bg + r * p.Bg;
    pass = rem / nch;
    c = nch - 1 - (rem - pass * nch);
  };
  auto dir_of = [&](int pass) { return bidir ? pass : p.direction; };

  float rb[BCE], rc[BCE];
  auto load_bc = [&](int b, int dir, int s0) {
#pragma unroll
    for (int e = 0; e < BCE; ++e) {
      const int i = tid + e * NTH;
      const int tt = i / NP, ln = i - tt * NP;
      const int s = s0 + tt;
      const int n = LM::mem_lane(ln / NL, ln % NL, p.NR, p.NT);
      const bool ok = (i < kCK * NP) && (s < L) && (n >= 0);
      const int t = dir ? L - 1 - s : s;
      const size_t gi = ok ? ((size_t)b * L + t) * N + n : 0;
      rb[e] = ok ? ld_f(p.Bc, gi, p.dt_bc) : 0.f;
      rc[e] = ok ? ld_f(p.Cc, gi, p.dt_bc) : 0.f;
    }
  };
  auto store_bc = [&](int buf) {
#pragma unroll
    for (int e = 0; e < BCE; ++e) {
      const int i = tid + e * NTH;
      if (i < kCK * NP) {
        s_b[buf * kCK * NP + i] = rb[e];
        s_c[buf * kCK * NP + i] = rc[e];
      }
    }
  };
  auto stage = [&](int i, int buf) {
    int b, pass, c;
    item(i, b, pass, c);
    const int dir = dir_of(pass), s0 = c * kCK;
    stage_tile<DT, NTH>(s_dl + buf * CF::raw_bytes, p.delta, es_du, async_du, b, d0, s0, dir, L, D);
    stage_tile<DT, NTH>(s_u + buf * CF::raw_bytes, p.u, es_du, async_du, b, d0, s0, dir, L, D);
    stage_tile<DT, NTH>(s_dy + buf * CF::raw_bytes, p.dy, es_dy, async_dy, b, d0, s0, dir, L, D);
    if (c > 0) {
      const int dslot = bidir ? dir : 0;
      const float* src = p.ckpt + ((((size_t)b * ndirs + dslot) * (nch - 1) + (c - 1)) * D + d0) * NP;
      float* dst = s_ck + buf * DT * NP;
      for (int v = tid; v < DT * NP / 4; v += NTH) {
        const bool ok = d0 + (v * 4) / NP < D;
        cp_async16(dst + v * 4, ok ? src + v * 4 : p.ckpt, ok);
      }
    }
  };

  float qv[C], gn[ND * RR];
  if (nitems > 0) {
    stage(0, 0);
    cp_async_commit();
    {
      int b, pass, c;
      item(0, b, pass, c);
      load_bc(b, dir_of(pass), c * kCK);
      store_bc(0);
    }
  }
  for (int it = 0; it < nitems; ++it) {
    const int buf = it & 1;
    int b, pass, c;
    item(it, b, pass, c);
    const int dir = dir_of(pass);
    const bool first_of_two = bidir && pass == 0;
    const bool second_of_two = bidir && pass == 1;
    const int s0 = c * kCK;
    const int ns = min(kCK, L - s0);
    const bool more = it + 1 < nitems;
    if (more) stage(it + 1, buf ^ 1);
    cp_async_commit();
    if (more) {
      int b2, pass2, c2;
      item(it + 1, b2, pass2, c2);
      load_bc(b2, dir_of(pass2), c2 * kCK);
    }
    cp_async_wait1();
    __syncthreads();

    if (c == nch - 1) {   // first chunk of a direction pass: adjoint state starts at zero
#pragma unroll
      for (int i = 0; i < C; ++i) qv[i] = 0.f;
#pragma unroll
      for (int i = 0; i < ND * RR; ++i) gn[i] = 0.f;
    }

    const unsigned char* bdl = s_dl + buf * CF::raw_bytes;
    const unsigned char* bu = s_u + buf * CF::raw_bytes;
    const unsigned char* bdy = s_dy + buf * CF::raw_bytes;
    const float* bb = s_b + buf * kCK * NP;
    const float* bc = s_c + buf * kCK * NP;

    // ---- forward recompute of the chunk; P[t-1] of every cell -> TMEM
    float P[C];
    {
      const float* ck = s_ck + buf * DT * NP + grp * ND * NP + q * NL;
#pragma unroll
      for (int k = 0; k < ND; ++k)
#pragma unroll
        for (int j = 0; j < NL; ++j) P[k * NL + j] = c > 0 ? ck[k * NP + j] : 0.f;
    }
    for (int tt = 0; tt < ns; ++tt) {
      tmem_store<C>(tbase + (uint32_t)(tt * CS), P);
      float dl[ND], uu[ND];
      read_chan<ND>(bdl + (size_t)(tt * DT + grp * ND) * es_du, bf_du, dl);
      read_chan<ND>(bu + (size_t)(tt * DT + grp * ND) * es_du, bf_du, uu);
      const float* rbv = bb + tt * NP + q * NL;
#pragma unroll
      for (int k = 0; k < ND; ++k) {
        const float du = __fmul_rn(dl[k], uu[k]);
#pragma unroll
        for (int j = 0; j < R; ++j)
          cell_update(rot_gate(dl[k], exp_const(ar[k][j]), ai[k][j]), P[k * NL + j], du, rbv[j]);
#pragma unroll
        for (int j = R; j < NL; ++j) cell_update(tk[k][j - R], P[k * NL + j], du, rbv[j]);
      }
    }
    tmem_wait_st();

    // ---- reverse recurrence
    for (int tt = ns - 1; tt >= 0; --tt) {
      float Pp[C];
      tmem_load<C>(tbase + (uint32_t)(tt * CS), Pp);
      const int s = s0 + tt;
      const int t = dir ? L - 1 - s : s;
      float dl[ND], uu[ND], dyv[ND];
      read_chan<ND>(bdl + (size_t)(tt * DT + grp * ND) * es_du, bf_du, dl);
      read_chan<ND>(bu + (size_t)(tt * DT + grp * ND) * es_du, bf_du, uu);
      read_chan<ND>(bdy + (size_t)(tt * DT + grp * ND) * es_dy, bf_dy, dyv);
      const float* rbv = bb + tt * NP + q * NL;
      const float* rcv = bc + tt * NP + q * NL;
      float Bv[NL], Cv[NL], pB[NL], pC[NL];
#pragma unroll
      for (int j = 0; j < NL; ++j) {
        Bv[j] = rbv[j];
        Cv[j] = rcv[j];
        pB[j] = 0.f;
        pC[j] = 0.f;
      }
      tmem_wait_ld();
      float gsum[ND], sbs[ND];
#pragma unroll
      for (int k = 0; k < ND; ++k) {
        const float dlk = dl[k], dyk = dyv[k];
        const float du = __fmul_rn(dlk, uu[k]);
        float gs = 0.f, sB = 0.f;
#pragma unroll
        for (int j = 0; j < R; ++j) {
          const float pp = Pp[k * NL + j];
          const float e = gate_exp(dlk, exp_const(ar[k][j]));
          float sn, cs;
          gate_sincos(dlk, ai[k][j], sn, cs);
          const float g = __fmul_rn(e, cs);
          const float es = __fmul_rn(e, sn);
          const float dbu = __fmul_rn(du, Bv[j]);
          const float H = __fmaf_rn(g, pp, dbu);
          const float dyC = __fmul_rn(dyk, Cv[j]);
          const float qn = __fmaf_rn(gn[k * RR + j], qv[k * NL + j], dyC);
          const float ddbu = __fmaf_rn(-0.5f, dyC, qn);
          const float wp = __fmul_rn(qn, pp);
          const float wg = __fmul_rn(wp, g);
          const float ws = __fmul_rn(wp, es);
          gAr[k][j] = __fmaf_rn(dlk, wg, gAr[k][j]);
          gAi[k][j] = __fmaf_rn(-dlk, ws, gAi[k][j]);
          gs = __fmaf_rn(ar[k][j], wg, gs);
          gs = __fmaf_rn(-ai[k][j], ws, gs);
          sB = __fmaf_rn(ddbu, Bv[j], sB);
          pB[j] = __fmaf_rn(ddbu, du, pB[j]);
          pC[j] = __fmaf_rn(dyk, H, pC[j]);
          qv[k * NL + j] = qn;
          gn[k * RR + j] = g;
        }
#pragma unroll
        for (int j = R; j < NL; ++j) {
          const float pp = Pp[k * NL + j];
          const float g = tk[k][j - R];
          const float dbu = __fmul_rn(du, Bv[j]);
          const float H = __fmaf_rn(g, pp, dbu);
          const float dyC = __fmul_rn(dyk, Cv[j]);
          const float qn = __fmaf_rn(g, qv[k * NL + j], dyC);
          const float ddbu = __fmaf_rn(-0.5f, dyC, qn);
          const float wp = __fmul_rn(qn, pp);
          gTk[k][j - R] = __fadd_rn(gTk[k][j - R], wp);
          sB = __fmaf_rn(ddbu, Bv[j], sB);
          pB[j] = __fmaf_rn(ddbu, du, pB[j]);
          pC[j] = __fmaf_rn(dyk, H, pC[j]);
          qv[k * NL + j] = qn;
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
          float ddl = __fmaf_rn(0.5f, gsv, __fmul_rn(sBv, uu[k]));
          float ddu = __fmul_rn(sBv, dl[k]);
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
      // dB/dC over this warp's 8 channel groups (lanes q, q+4, ..., q+28):
      // transposed butterfly, after which each lane holds V8/8 fully reduced
      // values; value i of lane l is original index
      // ((l>>2)&1)*V8/2 + ((l>>3)&1)*V8/4 + ((l>>4)&1)*V8/8 + i.
      {
        float v[V8];
#pragma unroll
        for (int j = 0; j < NL; ++j) { v[j] = pB[j]; v[NL + j] = pC[j]; }
#pragma unroll
        for (int j = V; j < V8; ++j) v[j] = 0.f;
#pragma unroll
        for (int lvl = 0; lvl < 3; ++lvl) {
          const int m = 4 << lvl;
          const int half = V8 >> (lvl + 1);
          const bool hi = (lane & m) != 0;
#pragma unroll
          for (int i = 0; i < half; ++i) {
            const float send = hi ? v[i] : v[i + half];
            const float keep = hi ? v[i + half] : v[i];
            v[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, m));
          }
        }
        const int obase = ((lane >> 2) & 1) * (V8 / 2) + ((lane >> 3) & 1) * (V8 / 4) +
                          ((lane >> 4) & 1) * (V8 / 8);
        float* r0 = s_red + (size_t)(tt * NW + warp) * 2 * NP + q * NL;
#pragma unroll
        for (int i = 0; i < V8 / 8; ++i) {
          const int o = obase + i;
          if (o < NL) r0[o] = v[i];
          else if (o < V) r0[NP + (o - NL)] = v[i];
        }
      }
    }
    __syncthreads();
    // flush this chunk's dB/dC partials: fixed order over the 4 warps
    for (int i = tid; i < ns * 2 * NP; i += NTH) {
      const int tt = i / (2 * NP), rem = i - tt * 2 * NP;
      const int which = rem / NP, ln = rem - which * NP;
      const float* r = s_red + ((size_t)tt * NW * 2 + which) * NP + ln;
      float v = r[0];
#pragma unroll
      for (int w = 1; w < NW; ++w) v = __fadd_rn(v, r[(size_t)w * 2 * NP]);
      const int s = s0 + tt;
      const int t = dir ? L - 1 - s : s;
      float* dst = p.part_bc + ((((size_t)gt * B + b) * L + t) * 2 + which) * NP + ln;
      *dst = second_of_two ? __fadd_rn(*dst, v) : v;
    }
    if (more) store_bc(buf ^ 1);
  }
  cp_async_wait0();

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

template <int R, int T, int ND, int NTH>
cudaError_t launch_bwd_impl(const BwdParams& p, cudaStream_t stream) {
  using CF = BwdCfg<R, T, ND, NTH>;
  auto kern = scan_bwd_kernel<R, T, ND, NTH>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)CF::smem_bytes);
  if (e != cudaSuccess) return e;
  dim3 grid(p.Bg, p.G);
  kern<<<grid, NTH, CF::smem_bytes, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_scan_bwd(const Tile& t, const BwdParams& p, cudaStream_t s) {
#define M3_X(r, tt, nd, ndb, nthb) \
  if (t.R == r && t.T == tt && t.ND == nd) return launch_bwd_impl<r, tt, ndb, nthb>(p, s);
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
