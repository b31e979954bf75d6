#pragma once
// K2 (kernel template): analytic backward of the trapezoidal scan, causal / reverse / both
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
// bg + Bg, ... and, per row and direction, the KC-step chunks from last to
// first.  Each chunk restarts from the forward's checkpoint of P, recomputes
// the chunk forward storing P[t-1] of every cell in Tensor Memory, then runs
// the reverse recurrence reading P back.  dA_real/dA_imag/dtrack accumulate in
// registers over the CTA's rows and land in one partial per batch group;
// dB/dC are reduced over the CTA's channels (warp shuffles + shared memory)
// into one partial per channel tile.  A second kernel sums both partial sets in
// a fixed order, so results are bitwise reproducible run to run.
#include <string.h>

#include <type_traits>

#include "m3_bulk.cuh"
#include "m3_common.cuh"
#include "m3_internal.h"
#include "m3_prologue.cuh"
#include "m3_stage.cuh"
#include "m3_tiles.h"
#include "m3_tma.h"
#include "m3_tmem.cuh"

#ifndef M3_BWD_UNROLL_RECOMPUTE
#define M3_BWD_UNROLL_RECOMPUTE 2
#endif
#ifndef M3_BWD_UNROLL_REVERSE
#define M3_BWD_UNROLL_REVERSE 1
#endif


namespace m3 {
namespace bwd {

constexpr int kUnrollRecompute = M3_BWD_UNROLL_RECOMPUTE;
constexpr int kUnrollReverse = M3_BWD_UNROLL_REVERSE;
// BULK: warps whose lane 0 issues a share of each work item's copies
constexpr int kStageWarps = 4;

constexpr int pow2ceil(int x) {
  int p = 1;
  while (p < x) p <<= 1;
  return p;
}

// Backward tiling: NDP channel pairs per thread (packed FP32), NTH threads.
// GS: the recompute pass also keeps each step's rotational gates (exp*cos and
// exp*sin) in Tensor Memory, so the reverse pass evaluates no transcendental;
// the chunk is then KC = 8 steps so that state and gates fit.
// PRO: the layer's prologue fused into the staging (bf16 bulk variant): raw dt
// tiles and raw B/C rows are staged besides the delta and B/C tiles the math
// reads (m3_prologue.cuh).
template <int R, int T, int ND, int NTH, bool GS, bool BULK, bool PRO = false>
struct BwdCfg {
  static_assert(ND % 2 == 0, "the backward processes channel pairs");
  static constexpr int KC = GS ? M3_GS_CHUNK : kCK; // chunk length (= checkpoint interval)
  static constexpr int NL = R + T;
  static constexpr int NP = 4 * NL;
  static constexpr int NG = NTH / 4;                // channel groups
  static constexpr int DT = NG * ND;                // channels per CTA
  static constexpr int NDP = ND / 2;                // channel pairs per thread
  static constexpr int C = ND * NL;                 // cells per thread
  static constexpr int CG = GS ? ND * R * 2 : 0;    // gate values per thread and step
  static constexpr int CS = pow2ceil(C + CG);       // TMEM columns per timestep
  static constexpr int WG_COLS = KC * CS;           // TMEM columns per warpgroup
  static constexpr int NCOLS = (NTH / 128) * WG_COLS < 32 ? 32 : (NTH / 128) * WG_COLS;
  static constexpr int CPS = 512 / NCOLS < 1 ? 1 : 512 / NCOLS;   // CTAs per SM by TMEM
  // WR: dB/dC partials are first reduced over the 8 channel groups of a warp
  // with a transposed shuffle butterfly (2*NL values halved over lane bits
  // 4, 3, 2), leaving one value per (step, B|C, lane, warp, quarter) in shared
  // memory; the flush then sums the warps once per chunk.  Otherwise every
  // thread stores its partials and the flush sums all groups every 4 steps.
  static constexpr bool WR = (2 * (R + T)) % 8 == 0;
  static constexpr int NW = NTH / 32;               // warps
  static constexpr int FL = WR ? (KC < 8 ? KC : 8) : 4;   // steps per dB/dC/ddelta flush
  static constexpr size_t raw_bytes = (size_t)KC * DT * 4;    // one staged (KC x DT) tile
  // Reduction staging rows hold one value per thread (group-major, quarter-minor),
  // so per-step stores are bank-conflict free; the row pitches are padded so
  // the float4 reads of the flush hit distinct banks.
  static constexpr int SR = NG * 4 + 16;                       // dB/dC row pitch
  static constexpr int SG = NG * 4 + (16 / ND < 4 ? 4 : 16 / ND);  // ddelta row pitch
  static constexpr size_t red_floats =
      WR ? (size_t)FL * 2 * NL * NW * 4                           // [FL][2*NL][NW][4]
         : (size_t)FL * 2 * NL * SR;                              // [FL][2][NL][SR]
  static constexpr size_t gs_floats = (size_t)FL * ND * 2 * SG;    // [FL][ND][2][SG]
  // BULK (copy-engine staging): the delta/u/dy tiles land in memory row order
  // (TMA boxes of KC rows), B/C rows land raw (HBM dtype, memory order) and are
  // widened into the padded fp32 tiles after the copy; the bidirectional second
  // pass stages the first pass's ddelta/du rows of the chunk.
  static constexpr size_t braw_floats = BULK ? 2 * 2 * (size_t)KC * NP : 0;  // [2][B|C][KC][NP]
  static constexpr size_t scr_floats = BULK ? (size_t)KC * DT * 2 : 0;       // [KC][DT][2]
  // PRO: [2][KC][DT] bf16 raw dt, [2][B|C][KC][4*NP] bf16 raw x_proj rows
  // (the host admits N*p <= 4*NP)
  static constexpr size_t dtr_bytes = PRO ? 2 * (size_t)KC * DT * 2 : 0;
  static constexpr size_t xraw_bytes = PRO ? 2 * 2 * (size_t)KC * 4 * NP * 2 : 0;
  static constexpr size_t base_bytes =
      dtr_bytes + xraw_bytes +
      3 * 2 * raw_bytes                       // delta, u, dy (HBM dtype), double-buffered
      + 2 * (size_t)DT * NP * 4               // checkpoint tile, double-buffered
      + 2 * 2 * (size_t)KC * NP * 4           // B, C (fp32), double-buffered
      + red_floats * 4 + gs_floats * 4
      + braw_floats * 4 + scr_floats * 4;
  // dA/dtrack totals: each thread's fp32 register sums of one row (both
  // directions, every step) are folded into its own float64 totals here when
  // the CTA moves to its next row, so the parameter gradients carry the
  // rounding of one row's fp32 sum instead of one sequential fp32 sum over
  // every (row, step) of the CTA (tens of thousands of terms at large batch;
  // measured at B=2048: 1.2-1.4e-6 of float64 without it).  Once per row
  // costs ~0.2 % of the kernel; once per chunk measured 7 %.  [pair][thread]
  // double2 layout (conflict-free 16-byte accesses).  Tilings whose shared
  // memory cannot hold it keep the fp32 register sums.
  static constexpr int NPAIR = NDP * (2 * (R > 0 ? R : 1) + (T > 0 ? T : 1));
  static constexpr size_t acc_bytes = (size_t)NPAIR * NTH * 16;
  static constexpr bool F64ACC = base_bytes + acc_bytes + 32 <= 227 * 1024;
  static constexpr size_t smem_bytes =
      base_bytes + (F64ACC ? acc_bytes : 0)
      + 32;                                   // TMEM address slot, 3 mbarriers (BULK)
};

// Stage a (KC x DT) tile of a (B, L, D) tensor for processing steps
// [s0, s0 + KC) in its HBM dtype; rows past L and channels past D read zero.
template <int DT, int NTH, int KC>
__device__ __forceinline__ void stage_tile(unsigned char* dst, const void* src, int esz,
                                           bool async_ok, int b, int d0, int s0, int dir,
                                           int L, int D) {
  if (async_ok) {
    const int epw = 4 / esz, wpr = DT / epw;
    for (int i = threadIdx.x; i < KC * wpr; i += NTH) {
      const int tt = i / wpr, w = i - tt * wpr;
      const int s = s0 + tt, d = d0 + w * epw;
      const bool ok = (s < L) && (d < D);
      const int t = dir ? L - 1 - s : s;
      const size_t gi = ok ? ((size_t)b * L + t) * D + d : 0;
      cp_async4(dst + (size_t)i * 4, (const char*)src + gi * esz, ok);
    }
  } else {
    for (int i = threadIdx.x; i < KC * DT; i += NTH) {
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

// One element of a staged (KC x DT) tile, converted to fp32.
__device__ __forceinline__ float tile_at(const unsigned char* base, bool bf16, int idx) {
  if (bf16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(base)[idx]);
  return reinterpret_cast<const float*>(base)[idx];
}

// DU, DY: element types of delta/u and of dy fixed at compile time (0 fp32,
// 1 bf16), or -1 to read them from the parameters (element-wise staging path).
template <int R, int T, int ND, int NTH, bool GS, bool BULK, int DU, int DY, bool PRO = false>
__global__ void __launch_bounds__(
    NTH, (M3_BWD_MIN_BLOCKS > 0 && M3_BWD_MIN_BLOCKS < BwdCfg<R, T, ND, NTH, GS, BULK, PRO>::CPS)
             ? M3_BWD_MIN_BLOCKS
             : BwdCfg<R, T, ND, NTH, GS, BULK, PRO>::CPS)
    scan_bwd_kernel(const BwdParams p, const __grid_constant__ CUtensorMap tm_dl,
                    const __grid_constant__ CUtensorMap tm_u,
                    const __grid_constant__ CUtensorMap tm_dy,
                    const __grid_constant__ CUtensorMap tm_x) {
  using LM = LaneMap<R, T>;
  using CF = BwdCfg<R, T, ND, NTH, GS, BULK, PRO>;
  static_assert(!PRO || (BULK && DU == 1), "the fused prologue is a bf16 bulk-staging variant");
  constexpr int KC = CF::KC;
  constexpr int NL = CF::NL, NP = CF::NP, DT = CF::DT, C = CF::C, CS = CF::CS, CG = CF::CG;
  constexpr int NG = CF::NG, NDP = CF::NDP, FL = CF::FL, SR = CF::SR, SG = CF::SG;
  constexpr int RR = R > 0 ? R : 1;
  constexpr int TT = T > 0 ? T : 1;
  constexpr int BCE = (KC * NP + NTH - 1) / NTH;
  static_assert(CF::NCOLS <= 512, "TMEM holds at most 512 columns");
  static_assert(!BULK || NTH / 32 >= kStageWarps, "bulk staging issues from 4 warps");

  extern __shared__ __align__(128) unsigned char smem[];
  // PRO staging first: raw dt [2][KC][DT] bf16, raw x_proj rows [2][B|C][KC][4*NP] bf16
  __nv_bfloat16* s_dtr = reinterpret_cast<__nv_bfloat16*>(smem);
  __nv_bfloat16* s_xraw = reinterpret_cast<__nv_bfloat16*>(smem + CF::dtr_bytes);
  unsigned char* s_dl = smem + CF::dtr_bytes + CF::xraw_bytes;       // [2][raw]
  unsigned char* s_u = s_dl + 2 * CF::raw_bytes;                     // [2][raw]
  unsigned char* s_dy = s_u + 2 * CF::raw_bytes;                     // [2][raw]
  float* s_ck = reinterpret_cast<float*>(s_dy + 2 * CF::raw_bytes);  // [2][DT][NP]
  float* s_b = s_ck + 2 * DT * NP;                                   // [2][KC][NP]
  float* s_c = s_b + 2 * KC * NP;                                    // [2][KC][NP]
  float* s_red = s_c + 2 * KC * NP;                                  // dB/dC staging (CF::WR)
  float* s_gs = s_red + CF::red_floats;                              // [FL][ND][2][SG]
  float* s_braw = s_gs + CF::gs_floats;                              // [2][B|C][KC][NP] (BULK)
  float* s_scr = s_braw + CF::braw_floats;                           // [KC][DT][2] (BULK)
  double2* s_acc = reinterpret_cast<double2*>(s_scr + CF::scr_floats);   // [NPAIR][NTH] (F64ACC)
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(
      reinterpret_cast<unsigned char*>(s_acc) + (CF::F64ACC ? CF::acc_bytes : 0));
  uint64_t* s_bar = reinterpret_cast<uint64_t*>(s_tmem) + 1;          // [3] (BULK)

  const int tid = threadIdx.x, q = tid & 3, grp = tid >> 2;
  const int warp = tid >> 5;
  const int bg = blockIdx.x, gt = blockIdx.y;
  const int d0 = gt * DT, dbase = d0 + grp * ND;
  const int B = p.B, L = p.L, D = p.D, N = p.N;
  const bool bidir = p.direction == M3_DIR_BIDIR;
  const int ndirs = bidir ? 2 : 1;
  const int nch = p.nch;
  const bool bf_du = DU < 0 ? p.dt_du == M3_BF16 : DU == 1;
  const bool bf_dy = DY < 0 ? p.dt_dy == M3_BF16 : DY == 1;
  const int es_du = bf_du ? 2 : 4, es_dy = bf_dy ? 2 : 4;
  const bool async_du = p.async_du, async_dy = p.async_dy;

  if constexpr (BULK) {
    // TMA boxes land at 128-byte aligned shared addresses (the raw tiles are
    // multiples of 128 bytes, so the base decides); uniform over the CTA
    if (smem_addr(smem) & 127u) {
      if (tid == 0) set_err(p.err, M3_ERR_DEVICE);
      return;
    }
    if (tid == 0) {   // one barrier per staging buffer, one for the scratch rows
      mbar_init(&s_bar[0], kStageWarps);
      mbar_init(&s_bar[1], kStageWarps);
      mbar_init(&s_bar[2], 1);
      mbar_fence_init();
    }
  }
  if (warp == 0) tmem_alloc(s_tmem, CF::NCOLS);
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  // warp w reads/writes TMEM lanes 32*(w%4).. of column block w/4
  const uint32_t tbase =
      *s_tmem + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)((warp >> 2) * CF::WG_COLS);

  // parameters of the thread's cells, as channel pairs (k, k+1)
  float2 AR[NDP][RR], A2[NDP][RR], AI[NDP][RR], TK[NDP][TT];
  float maxai = 0.f;
#pragma unroll
  for (int k = 0; k < ND; ++k) {
    const int d = dbase + k;
#pragma unroll
    for (int j = 0; j < NL; ++j) {
      const int n = LM::mem_lane(q, j, p.NR, p.NT);
      const bool ok = (d < D) && (n >= 0);
      const size_t gi = ok ? (size_t)d * N + n : 0;
      if (j < R) {
        const float ar = ok ? p.Ar[gi] : 0.f, ai = ok ? p.Ai[gi] : 0.f;
        maxai = fmaxf(maxai, fabsf(ai));
        float2& r_ = AR[k >> 1][j]; float2& e_ = A2[k >> 1][j]; float2& i_ = AI[k >> 1][j];
        if (k & 1) { r_.y = ar; e_.y = exp_const(ar); i_.y = ai; }
        else       { r_.x = ar; e_.x = exp_const(ar); i_.x = ai; }
      } else {
        const float tv = ok ? p.Tk[gi] : 0.f;
        if (k & 1) TK[k >> 1][j - R].y = tv; else TK[k >> 1][j - R].x = tv;
      }
    }
  }

  // dA accumulators: sum_t dl*wp*gate, sum_t dl*wp*exp*sin, sum_t wp (x 0.5 at the end;
  // the second carries the sign of dA_imag)
  float2 gAr[NDP][RR], gAi[NDP][RR], gTk[NDP][TT];
#pragma unroll
  for (int k = 0; k < NDP; ++k) {
#pragma unroll
    for (int j = 0; j < RR; ++j) { gAr[k][j] = f2(0.f); gAi[k][j] = f2(0.f); }
#pragma unroll
    for (int j = 0; j < TT; ++j) gTk[k][j] = f2(0.f);
  }

  // the thread's accumulator pairs in a fixed order: gAr, gAi, gTk
  auto acc_pair = [&](int i) -> float2& {
    constexpr int NR2 = NDP * RR;
    if (i < NR2) return gAr[i / RR][i % RR];
    if (i < 2 * NR2) return gAi[(i - NR2) / RR][(i - NR2) % RR];
    return gTk[(i - 2 * NR2) / TT][(i - 2 * NR2) % TT];
  };
  // add the fp32 chunk sums to the float64 totals and restart them from zero
  auto fold_acc = [&]() {
    if constexpr (CF::F64ACC) {
#pragma unroll
      for (int i = 0; i < CF::NPAIR; ++i) {
        float2& a = acc_pair(i);
        double2 t = s_acc[i * NTH + tid];
        t.x += (double)a.x;
        t.y += (double)a.y;
        s_acc[i * NTH + tid] = t;
        a = f2(0.f);
      }
    }
  };
  if constexpr (CF::F64ACC) {
#pragma unroll
    for (int i = 0; i < CF::NPAIR; ++i) s_acc[i * NTH + tid] = make_double2(0.0, 0.0);
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
      const bool ok = (i < KC * NP) && (s < L) && (n >= 0);
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
      if (i < KC * NP) {
        s_b[buf * KC * NP + i] = rb[e];
        s_c[buf * KC * NP + i] = rc[e];
      }
    }
  };
  auto stage = [&](int i, int buf) {
    int b, pass, c;
    item(i, b, pass, c);
    const int dir = dir_of(pass), s0 = c * KC;
    stage_tile<DT, NTH, KC>(s_dl + buf * CF::raw_bytes, p.delta, es_du, async_du, b, d0, s0, dir, L, D);
    stage_tile<DT, NTH, KC>(s_u + buf * CF::raw_bytes, p.u, es_du, async_du, b, d0, s0, dir, L, D);
    stage_tile<DT, NTH, KC>(s_dy + buf * CF::raw_bytes, p.dy, es_dy, async_dy, b, d0, s0, dir, L, D);
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

  // BULK staging of work item (b, pass, c) into buffer buf, all by thread 0
  // on the copy engine, completing on the buffer's mbarrier: the delta/u/dy
  // tiles as TMA boxes of KC memory rows x DT channels starting at the chunk's
  // first memory row (rows past the chunk are never read; rows past the tensor
  // are zero-filled), the checkpoint tile and the chunk's B and C rows as one
  // contiguous block each (memory order).
  const int es_bc = p.dt_bc == M3_BF16 ? 2 : 4;
  auto stage_vec = [&](int b, int pass, int c, int buf) {
    // lane 0 of warps 0..3 each registers its own bytes and issues its copies
    // (an issuing thread waits on every copy instruction, so four issue in
    // parallel); the buffer's barrier expects kStageWarps arrivals per item
    const int w = tid >> 5;
    if ((tid & 31) != 0 || w >= kStageWarps) return;
    const int dir = dir_of(pass), s0 = c * KC;
    const int ns = min(KC, L - s0);
    const int t_lo = dir ? L - s0 - ns : s0;             // first memory row of the chunk
    const int y0 = b * L + t_lo;
    if (w == 0) {
      mbar_arrive_expect_tx(&s_bar[buf], (uint32_t)(KC * DT * es_du));
      // PRO: the raw dt tile; the widen step writes delta into s_dl
      tma_load_2d(PRO ? static_cast<void*>(s_dtr + (size_t)buf * KC * DT)
                      : static_cast<void*>(s_dl + buf * CF::raw_bytes),
                  &tm_dl, d0, y0, &s_bar[buf]);
    } else if (w == 1) {
      mbar_arrive_expect_tx(&s_bar[buf], (uint32_t)(KC * DT * es_du));
      tma_load_2d(s_u + buf * CF::raw_bytes, &tm_u, d0, y0, &s_bar[buf]);
    } else if (w == 2) {
      mbar_arrive_expect_tx(&s_bar[buf], (uint32_t)(KC * DT * es_dy) +
                                             (c > 0 ? (uint32_t)(DT * NP * 4) : 0u));
      tma_load_2d(s_dy + buf * CF::raw_bytes, &tm_dy, d0, y0, &s_bar[buf]);
      if (c > 0) {
        const int dslot = bidir ? dir : 0;
        const float* src =
            p.ckpt + ((((size_t)b * ndirs + dslot) * (nch - 1) + (c - 1)) * D + d0) * NP;
        bulk_g2s(s_ck + buf * DT * NP, src, DT * NP * 4, &s_bar[buf]);
      }
    } else if (PRO) {
      // raw B_raw / C_raw boxes (KC rows x N*p bf16) of the x_proj rows
      const int npr = N * p.P;
      mbar_arrive_expect_tx(&s_bar[buf], (uint32_t)(2 * KC * npr * 2));
      __nv_bfloat16* raw = s_xraw + (size_t)buf * 2 * KC * 4 * NP;
      tma_load_2d(raw, &tm_x, p.off_b, y0, &s_bar[buf]);
      tma_load_2d(raw + (size_t)KC * 4 * NP, &tm_x, p.off_c, y0, &s_bar[buf]);
    } else {
      const uint32_t bc_bytes = (uint32_t)(ns * N * es_bc);
      mbar_arrive_expect_tx(&s_bar[buf], 2 * bc_bytes);
      const size_t bc_off = ((size_t)b * L + t_lo) * N * es_bc;
      bulk_g2s(s_braw + ((size_t)(buf * 2 + 0) * KC) * NP, (const char*)p.Bc + bc_off, bc_bytes,
               &s_bar[buf]);
      bulk_g2s(s_braw + ((size_t)(buf * 2 + 1) * KC) * NP, (const char*)p.Cc + bc_off, bc_bytes,
               &s_bar[buf]);
    }
  };
  // widen the raw B/C rows of buffer buf into the padded fp32 lane layout
  // (processing step tt is memory row tt, or ns-1-tt for the reversed scan).
  // When NP divides the block, a thread always fills the same padded lane.
  constexpr bool kFixedLane = NTH % NP == 0;
  const int wl = tid % NP;
  const int wn = LM::mem_lane(wl / NL, wl % NL, p.NR, p.NT);
  const bool bc16 = p.dt_bc == M3_BF16;
  auto widen_bc = [&](int buf, int ns, int dir) {
    if constexpr (PRO) {
      // delta = bf16(softplus(dt)) over the tile (memory order, as TMA left it)
      __nv_bfloat16* dlt = reinterpret_cast<__nv_bfloat16*>(s_dl + buf * CF::raw_bytes);
      const __nv_bfloat16* dtr = s_dtr + (size_t)buf * KC * DT;
      for (int i = tid; i < KC * DT; i += NTH)
        dlt[i] = __float2bfloat16_rn(softplus20(__bfloat162float(dtr[i])));
      // BCNorm + MIMO fold of each staged row, one warp per (step, B|C); the
      // fold is rounded to bf16 as the unfused bf16 layer's cast does
      const int np = N * p.P, lane = tid & 31;
      const __nv_bfloat16* raw = s_xraw + (size_t)buf * 2 * KC * 4 * NP;
      for (int r = tid >> 5; r < 2 * ns; r += NTH / 32) {
        const int which = r & 1, tt = r >> 1;
        const int mr = dir ? ns - 1 - tt : tt;
        // box rows are packed at a pitch of np elements
        const __nv_bfloat16* x = raw + (size_t)which * KC * 4 * NP + (size_t)mr * np;
        auto ld = [&](int k) { return __bfloat162float(x[k]); };
        const float* w = which ? p.wc : p.wb;
        const float rs = bcnorm_scale(ld, np, p.eps, w != nullptr, lane);
        float* dst = (which ? s_c : s_b) + buf * KC * NP + tt * NP;
        for (int ln = lane; ln < NP; ln += 32) {
          const int n = LM::mem_lane(ln / NL, ln % NL, p.NR, p.NT);
          dst[ln] = n >= 0 ? __bfloat162float(__float2bfloat16_rn(
                                 bcnorm_fold(ld, n, p.P, rs, w)))
                           : 0.f;
        }
      }
      return;
    }
    const float* rb0 = s_braw + ((size_t)(buf * 2 + 0) * KC) * NP;
    const float* rc0 = s_braw + ((size_t)(buf * 2 + 1) * KC) * NP;
    if constexpr (kFixedLane) {
      for (int tt = tid / NP; tt < ns; tt += NTH / NP) {
        const int r = (dir ? ns - 1 - tt : tt) * N + (wn >= 0 ? wn : 0);
        float bv = 0.f, cv = 0.f;
        if (wn >= 0) {
          if (bc16) {
            bv = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(rb0)[r]);
            cv = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(rc0)[r]);
          } else {
            bv = rb0[r];
            cv = rc0[r];
          }
        }
        s_b[buf * KC * NP + tt * NP + wl] = bv;
        s_c[buf * KC * NP + tt * NP + wl] = cv;
      }
    } else {
      for (int i = tid; i < ns * NP; i += NTH) {
        const int tt = i / NP, ln = i - tt * NP;
        const int n = LM::mem_lane(ln / NL, ln % NL, p.NR, p.NT);
        const size_t r = (size_t)(dir ? ns - 1 - tt : tt) * N + (n >= 0 ? n : 0);
        s_b[buf * KC * NP + i] = n >= 0 ? ld_f(rb0, r, p.dt_bc) : 0.f;
        s_c[buf * KC * NP + i] = n >= 0 ? ld_f(rc0, r, p.dt_bc) : 0.f;
      }
    }
  };

  float2 qv[NDP][NL], gn[NDP][RR];
  // the current work item, advanced without divisions: chunks from last to
  // first, then the next direction, then the next row
  int b = bg, pass = 0, c = nch - 1;
  auto advance = [&](int& ib, int& ipass, int& ic) {
    if (ic > 0) { --ic; return; }
    ic = nch - 1;
    if (++ipass < ndirs) return;
    ipass = 0;
    ib += p.Bg;
  };
  if (nitems > 0) {
    if constexpr (BULK) {
      stage_vec(b, pass, c, 0);
    } else {
      stage(0, 0);
      cp_async_commit();
      int b, pass, c;
      item(0, b, pass, c);
      load_bc(b, dir_of(pass), c * KC);
      store_bc(0);
    }
  }
  bool fail = false;   // a staging copy did not complete (BULK)
  int nscr = 0;        // scratch-row copies issued (BULK barrier 2 phases)
  for (int it = 0; it < nitems; ++it, advance(b, pass, c)) {
    const int buf = it & 1;
    const int dir = dir_of(pass);
    const bool first_of_two = bidir && pass == 0;
    const bool second_of_two = bidir && pass == 1;
    const int s0 = c * KC;
    const int ns = min(KC, L - s0);
    const bool more = it + 1 < nitems;
    // staged rows are in processing order (cp.async staging) or in memory
    // order (BULK: processing step tt is memory row ns-1-tt when reversed)
    const int mrow0 = (BULK && dir) ? ns - 1 : 0, mstep = (BULK && dir) ? -1 : 1;
    [[maybe_unused]] const uint32_t scr_par = (uint32_t)(nscr & 1);
    if constexpr (BULK) {
      // the first pass's ddelta/du rows of this chunk, written by this CTA
      // before the previous barrier (generic stores, hence the proxy fence),
      // needed from the first flush on
      if (second_of_two) {
        if (tid == 32) {   // lane 0 of warp 1, which issues one TMA box per item
          const int t_lo = dir ? L - s0 - ns : s0;
          fence_proxy_async_global();
          mbar_arrive_expect_tx(&s_bar[2], (uint32_t)(ns * DT * 8));
          bulk_g2s(s_scr, scratch + (size_t)t_lo * DT * 2, (uint32_t)(ns * DT * 8), &s_bar[2]);
        }
        ++nscr;
      }
      if (more) {   // the next work item
        int b2 = b, pass2 = pass, c2 = c;
        advance(b2, pass2, c2);
        stage_vec(b2, pass2, c2, buf ^ 1);
      }
      // item it is use it/2 of its buffer's barrier
      const bool ok = mbar_wait(&s_bar[buf], (uint32_t)((it >> 1) & 1));
      if (__syncthreads_or(!ok)) {
        // give up: let the copies still in flight land before the CTA exits
        if (tid == 0) {
          mbar_wait(&s_bar[buf], (uint32_t)((it >> 1) & 1));
          if (more) mbar_wait(&s_bar[buf ^ 1], (uint32_t)(((it + 1) >> 1) & 1));
          if (second_of_two) mbar_wait(&s_bar[2], scr_par);
        }
        fail = true;
        break;
      }
      widen_bc(buf, ns, dir);
      __syncthreads();
    } else {
      if (more) stage(it + 1, buf ^ 1);
      cp_async_commit();
      if (more) {
        int b2, pass2, c2;
        item(it + 1, b2, pass2, c2);
        load_bc(b2, dir_of(pass2), c2 * KC);
      }
      cp_async_wait1();
      __syncthreads();
    }

    if (c == nch - 1) {   // first chunk of a direction pass: adjoint state starts at zero
#pragma unroll
      for (int k = 0; k < NDP; ++k) {
#pragma unroll
        for (int j = 0; j < NL; ++j) qv[k][j] = f2(0.f);
#pragma unroll
        for (int j = 0; j < RR; ++j) gn[k][j] = f2(0.f);
      }
    }

    const unsigned char* bdl = s_dl + buf * CF::raw_bytes;
    const unsigned char* bu = s_u + buf * CF::raw_bytes;
    const unsigned char* bdy = s_dy + buf * CF::raw_bytes;
    const float* bb = s_b + buf * KC * NP;
    const float* bc = s_c + buf * KC * NP;

    // ---- forward recompute of the chunk; P[t-1] of every cell -> TMEM
    float2 P[NDP][NL];
    {
      const float* ck = s_ck + buf * DT * NP + grp * ND * NP + q * NL;
#pragma unroll
      for (int k = 0; k < ND; ++k)
#pragma unroll
        for (int j = 0; j < NL; ++j) {
          const float v = c > 0 ? ck[k * NP + j] : 0.f;
          if (k & 1) P[k >> 1][j].y = v; else P[k >> 1][j].x = v;
        }
    }
#pragma unroll kUnrollRecompute
    for (int tt = 0; tt < ns; ++tt) {
      tmem_store<C>(tbase + (uint32_t)(tt * CS), reinterpret_cast<const float(&)[C]>(P));
      float dl[ND], uu[ND];
      const int mr = mrow0 + mstep * tt;
      read_chan<ND>(bdl + (size_t)(mr * DT + grp * ND) * es_du, bf_du, dl);
      read_chan<ND>(bu + (size_t)(mr * DT + grp * ND) * es_du, bf_du, uu);
      const float* rbv = bb + tt * NP + q * NL;
      float mdl = 0.f;
#pragma unroll
      for (int k = 0; k < ND; ++k) mdl = fmaxf(mdl, fabsf(dl[k]));
      // The fast/exact choice is made once per step (not per cell) so that the
      // compiler emits two branch-free bodies instead of predicating both.
      // GS: gates of this step, [channel pair][lane][exp*cos, exp*sin]
      float2 GG[NDP][RR][2];
      auto recompute = [&](auto fast_tag) {
        [[maybe_unused]] constexpr bool FAST = decltype(fast_tag)::value;
#pragma unroll
        for (int kp = 0; kp < NDP; ++kp) {
          const float2 dl2 = make_float2(dl[2 * kp], dl[2 * kp + 1]);
          const float2 du2 = __fmul2_rn(dl2, make_float2(uu[2 * kp], uu[2 * kp + 1]));
#pragma unroll
          for (int j = 0; j < R; ++j) {
            float2 g;
            if constexpr (GS) {
              if constexpr (FAST) {
                gate_es2_nocheck(dl2, A2[kp][j], AI[kp][j], g, GG[kp][j][1]);
              } else {
                const float2 e = gate_exp2(dl2, A2[kp][j]);
                float2 sn, cs;
                gate_sincos_pi(dl2.x, AI[kp][j].x, sn.x, cs.x);
                gate_sincos_pi(dl2.y, AI[kp][j].y, sn.y, cs.y);
                g = __fmul2_rn(e, cs);
                GG[kp][j][1] = __fmul2_rn(e, sn);
              }
              GG[kp][j][0] = g;
            } else if constexpr (FAST) {
              g = __fmul2_rn(gate_exp2(dl2, A2[kp][j]), gate_cos2_nocheck(dl2, AI[kp][j]));
            } else {
              g = make_float2(rot_gate(dl2.x, A2[kp][j].x, AI[kp][j].x),
                              rot_gate(dl2.y, A2[kp][j].y, AI[kp][j].y));
            }
            cell_update2(g, P[kp][j], du2, rbv[j]);
          }
#pragma unroll
          for (int j = R; j < NL; ++j) cell_update2(TK[kp][j - R], P[kp][j], du2, rbv[j]);
        }
      };
      if (__fmul_rn(mdl, maxai) <= kFastArgBound) recompute(std::true_type{});
      else recompute(std::false_type{});
      if constexpr (GS)
        tmem_store<CG>(tbase + (uint32_t)(tt * CS + C), reinterpret_cast<const float(&)[CG]>(GG));
    }
    tmem_wait_st();

    // ---- reverse recurrence, flushing dB/dC and ddelta/du every FL steps
#pragma unroll kUnrollReverse
    for (int tt = ns - 1; tt >= 0; --tt) {
      const int slot = (ns - 1 - tt) % FL;
      float2 Pp[NDP][NL];
      float2 GG[NDP][RR][2];
      tmem_load<C>(tbase + (uint32_t)(tt * CS), reinterpret_cast<float(&)[C]>(Pp));
      if constexpr (GS)
        tmem_load<CG>(tbase + (uint32_t)(tt * CS + C), reinterpret_cast<float(&)[CG]>(GG));
      float dl[ND], uu[ND], dyv[ND];
      const int mr = mrow0 + mstep * tt;
      read_chan<ND>(bdl + (size_t)(mr * DT + grp * ND) * es_du, bf_du, dl);
      read_chan<ND>(bu + (size_t)(mr * DT + grp * ND) * es_du, bf_du, uu);
      read_chan<ND>(bdy + (size_t)(mr * DT + grp * ND) * es_dy, bf_dy, dyv);
      const float* rbv = bb + tt * NP + q * NL;
      const float* rcv = bc + tt * NP + q * NL;
      float Bv[NL], Cv[NL];
#pragma unroll
      for (int j = 0; j < NL; ++j) { Bv[j] = rbv[j]; Cv[j] = rcv[j]; }
      float mdl = 0.f;
#pragma unroll
      for (int k = 0; k < ND; ++k) mdl = fmaxf(mdl, fabsf(dl[k]));
      tmem_wait_ld();
      float2 pB[NL], pC[NL];
      float* gsrow = s_gs + (size_t)slot * ND * 2 * SG + grp * 4 + q;
      auto reverse_cells = [&](auto fast_tag) {
      [[maybe_unused]] constexpr bool FAST = decltype(fast_tag)::value;
#pragma unroll
      for (int kp = 0; kp < NDP; ++kp) {
        const float2 dl2 = make_float2(dl[2 * kp], dl[2 * kp + 1]);
        const float2 du2 = __fmul2_rn(dl2, make_float2(uu[2 * kp], uu[2 * kp + 1]));
        const float2 dy2 = make_float2(dyv[2 * kp], dyv[2 * kp + 1]);
        float2 gs = f2(0.f), gsi = f2(0.f), sB = f2(0.f);
#pragma unroll
        for (int j = 0; j < R; ++j) {
          const float2 pp = Pp[kp][j];
          float2 g, es;
          if constexpr (GS) {
            g = GG[kp][j][0];
            es = GG[kp][j][1];
          } else if constexpr (FAST) {
            gate_es2_nocheck(dl2, A2[kp][j], AI[kp][j], g, es);
          } else {
            const float2 e = gate_exp2(dl2, A2[kp][j]);
            float2 sn, cs;
            gate_sincos_pi(dl2.x, AI[kp][j].x, sn.x, cs.x);
            gate_sincos_pi(dl2.y, AI[kp][j].y, sn.y, cs.y);
            g = __fmul2_rn(e, cs);
            es = __fmul2_rn(e, sn);
          }
          const float2 dbu = __fmul2_rn(du2, f2(Bv[j]));
          const float2 H = __ffma2_rn(g, pp, dbu);
          const float2 dyC = __fmul2_rn(dy2, f2(Cv[j]));
          const float2 qn = __ffma2_rn(gn[kp][j], qv[kp][j], dyC);
          const float2 ddbu = __ffma2_rn(f2(-0.5f), dyC, qn);
          const float2 wp = __fmul2_rn(qn, pp);
          const float2 wg = __fmul2_rn(wp, g);
          const float2 ws = __fmul2_rn(wp, es);
          gAr[kp][j] = __ffma2_rn(dl2, wg, gAr[kp][j]);
          gAi[kp][j] = __ffma2_rn(dl2, ws, gAi[kp][j]);
          gs = __ffma2_rn(AR[kp][j], wg, gs);
          gsi = __ffma2_rn(AI[kp][j], ws, gsi);
          sB = __ffma2_rn(ddbu, f2(Bv[j]), sB);
          pB[j] = kp == 0 ? __fmul2_rn(ddbu, du2) : __ffma2_rn(ddbu, du2, pB[j]);
          pC[j] = kp == 0 ? __fmul2_rn(dy2, H) : __ffma2_rn(dy2, H, pC[j]);
          qv[kp][j] = qn;
          gn[kp][j] = g;
        }
#pragma unroll
        for (int j = R; j < NL; ++j) {
          const float2 pp = Pp[kp][j];
          const float2 g = TK[kp][j - R];
          const float2 dbu = __fmul2_rn(du2, f2(Bv[j]));
          const float2 H = __ffma2_rn(g, pp, dbu);
          const float2 dyC = __fmul2_rn(dy2, f2(Cv[j]));
          const float2 qn = __ffma2_rn(g, qv[kp][j], dyC);
          const float2 ddbu = __ffma2_rn(f2(-0.5f), dyC, qn);
          const float2 wp = __fmul2_rn(qn, pp);
          gTk[kp][j - R] = __fadd2_rn(gTk[kp][j - R], wp);
          sB = __ffma2_rn(ddbu, f2(Bv[j]), sB);
          pB[j] = kp == 0 ? __fmul2_rn(ddbu, du2) : __ffma2_rn(ddbu, du2, pB[j]);
          pC[j] = kp == 0 ? __fmul2_rn(dy2, H) : __ffma2_rn(dy2, H, pC[j]);
          qv[kp][j] = qn;
        }
        // channel partials over this thread's lanes: gsum = sum(ar*wg) - sum(ai*ws), sB
        const float2 gsum = __fadd2_rn(gs, __fmul2_rn(gsi, f2(-1.f)));
        gsrow[(2 * (2 * kp) + 0) * SG] = gsum.x;
        gsrow[(2 * (2 * kp) + 1) * SG] = sB.x;
        gsrow[(2 * (2 * kp + 1) + 0) * SG] = gsum.y;
        gsrow[(2 * (2 * kp + 1) + 1) * SG] = sB.y;
      }
      };
      if (GS || __fmul_rn(mdl, maxai) <= kFastArgBound) reverse_cells(std::true_type{});
      else reverse_cells(std::false_type{});
      // dB/dC partial of this thread's channels
      if constexpr (CF::WR) {
        // transposed butterfly over the warp's 8 channel groups (lane bits 4..2):
        // each round keeps half of the values and adds the partner's copy of it
        constexpr int V = 2 * NL;
        float v[V];
#pragma unroll
        for (int j = 0; j < NL; ++j) {
          v[j] = __fadd_rn(pB[j].x, pB[j].y);
          v[NL + j] = __fadd_rn(pC[j].x, pC[j].y);
        }
        const int lane = tid & 31;
#pragma unroll
        for (int r = 0; r < 3; ++r) {
          const int m = 16 >> r, h = V >> (r + 1);
          const bool up = (lane & m) != 0;
#pragma unroll
          for (int i = 0; i < h; ++i) {
            const float keep = up ? v[h + i] : v[i];
            const float send = up ? v[i] : v[h + i];
            v[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, m));
          }
        }
        // lane (g, q) now holds values base .. base + V/8 - 1 of its quarter q
        const int g = lane >> 2;
        const int base = ((g >> 2) & 1) * (V / 2) + ((g >> 1) & 1) * (V / 4) + (g & 1) * (V / 8);
#pragma unroll
        for (int i = 0; i < V / 8; ++i)
          s_red[(((size_t)slot * V + base + i) * CF::NW + warp) * 4 + q] = v[i];
      } else {
        float* r0 = s_red + (size_t)slot * 2 * NL * SR + grp * 4 + q;
#pragma unroll
        for (int j = 0; j < NL; ++j) {
          r0[j * SR] = __fadd_rn(pB[j].x, pB[j].y);
          r0[(NL + j) * SR] = __fadd_rn(pC[j].x, pC[j].y);
        }
      }
      if (slot == FL - 1 || tt == 0) {
        bool okf = true;
        if constexpr (BULK) {
          if (second_of_two) okf = mbar_wait(&s_bar[2], scr_par);
        }
        if (__syncthreads_or(!okf)) {
          // give up (leaves the step loop, then the item loop): let the copies
          // still in flight land before the CTA exits
          if (tid == 0) {
            mbar_wait(&s_bar[2], scr_par);
            if (more) mbar_wait(&s_bar[buf ^ 1], (uint32_t)(((it + 1) >> 1) & 1));
          }
          fail = true;
          break;
        }
        const int nsl = slot + 1;                 // slots in this flush
        const int tt_hi = tt + slot;              // step of slot 0
        if constexpr (CF::WR) {
          // dB/dC: sum the warps' float4 (4 quarters) of each (slot, which, j)
          // in warp order, write lanes j*4 + q of the partial
          for (int row = tid; row < nsl * 2 * NL; row += NTH) {
            const float4* src = reinterpret_cast<const float4*>(s_red) + (size_t)row * CF::NW;
            float4 acc = src[0];
#pragma unroll
            for (int w = 1; w < CF::NW; ++w) {
              const float4 v = src[w];
              acc.x = __fadd_rn(acc.x, v.x); acc.y = __fadd_rn(acc.y, v.y);
              acc.z = __fadd_rn(acc.z, v.z); acc.w = __fadd_rn(acc.w, v.w);
            }
            const int sl = row / (2 * NL), rem = row - sl * 2 * NL;
            const int which = rem / NL, j = rem - which * NL;
            const int s = s0 + tt_hi - sl;
            const int t = dir ? L - 1 - s : s;
            const int dslot = bidir ? dir : 0;
            float4* dst = reinterpret_cast<float4*>(
                p.part_bc + (((((size_t)gt * ndirs + dslot) * B + b) * L + t) * 2 + which) * NP +
                j * 4);
            *dst = acc;
          }
        }
        // dB/dC: each (slot, which, j) row holds one value per (group, quarter);
        // 4 threads sum it over the groups as float4s of the 4 quarters, in a
        // fixed order, and write lanes j*4 + q of the partial.
        for (int base = 0; !CF::WR && base < nsl * 2 * NL; base += NTH / 4) {
          const int row = base + (tid >> 2), part = tid & 3;
          const bool rok = row < nsl * 2 * NL;
          float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
          if (rok) {
            const float* src = s_red + (size_t)row * SR;
#pragma unroll 4
            for (int g = part; g < NG; g += 4) {
              const float4 v = *reinterpret_cast<const float4*>(src + g * 4);
              acc.x = __fadd_rn(acc.x, v.x); acc.y = __fadd_rn(acc.y, v.y);
              acc.z = __fadd_rn(acc.z, v.z); acc.w = __fadd_rn(acc.w, v.w);
            }
          }
#pragma unroll
          for (int m = 1; m < 4; m <<= 1) {
            acc.x = __fadd_rn(acc.x, __shfl_xor_sync(0xffffffffu, acc.x, m));
            acc.y = __fadd_rn(acc.y, __shfl_xor_sync(0xffffffffu, acc.y, m));
            acc.z = __fadd_rn(acc.z, __shfl_xor_sync(0xffffffffu, acc.z, m));
            acc.w = __fadd_rn(acc.w, __shfl_xor_sync(0xffffffffu, acc.w, m));
          }
          if (rok && part == 0) {
            const int sl = row / (2 * NL), rem = row - sl * 2 * NL;
            const int which = rem / NL, j = rem - which * NL;
            const int s = s0 + tt_hi - sl;
            const int t = dir ? L - 1 - s : s;
            // one partial per (channel tile, direction): no read-modify-write
            const int dslot = bidir ? dir : 0;
            float4* dst = reinterpret_cast<float4*>(
                p.part_bc + (((((size_t)gt * ndirs + dslot) * B + b) * L + t) * 2 + which) * NP +
                j * 4);
            *dst = acc;
          }
        }
        // ddelta / du per channel: sum the 4 lane-quarter partials
        auto flush_du = [&](int sl, int dd) {
          const int d = d0 + dd;
          if (d >= D) return;
          const int tts = tt_hi - sl;
          const float* g4p = s_gs + ((size_t)(sl * ND + dd % ND) * 2) * SG + (dd / ND) * 4;
          const float4 g4 = *reinterpret_cast<const float4*>(g4p);
          const float4 b4 = *reinterpret_cast<const float4*>(g4p + SG);
          const float gsv = __fadd_rn(__fadd_rn(g4.x, g4.y), __fadd_rn(g4.z, g4.w));
          const float sBv = __fadd_rn(__fadd_rn(b4.x, b4.y), __fadd_rn(b4.z, b4.w));
          const int mr = mrow0 + mstep * tts;
          const float dlv = tile_at(bdl, bf_du, mr * DT + dd);
          const float uv = tile_at(bu, bf_du, mr * DT + dd);
          float ddl = __fmaf_rn(0.5f, gsv, __fmul_rn(sBv, uv));
          float ddu = __fmul_rn(sBv, dlv);
          const int s = s0 + tts;
          const int t = dir ? L - 1 - s : s;
          float* sc = scratch ? scratch + ((size_t)t * DT + dd) * 2 : nullptr;
          if (first_of_two) {
            *reinterpret_cast<float2*>(sc) = make_float2(ddl, ddu);
          } else {
            if (second_of_two) {
              const float2 sv = *reinterpret_cast<const float2*>(
                  BULK ? s_scr + ((size_t)mr * DT + dd) * 2 : sc);
              ddl = __fadd_rn(sv.x, ddl);
              ddu = __fadd_rn(sv.y, ddu);
            }
            if constexpr (PRO) {   // d dt = softplus'(dt) * (d delta rounded as the bf16 grad)
              ddl = softplus20_grad(__bfloat162float(__float2bfloat16_rn(ddl)),
                                    __bfloat162float(s_dtr[(size_t)buf * KC * DT + mr * DT + dd]));
            }
            const size_t oi = ((size_t)b * L + t) * D + d;
            if (bf_du) {
              reinterpret_cast<__nv_bfloat16*>(p.d_delta)[oi] = __float2bfloat16_rn(ddl);
              reinterpret_cast<__nv_bfloat16*>(p.d_u)[oi] = __float2bfloat16_rn(ddu);
            } else {
              reinterpret_cast<float*>(p.d_delta)[oi] = ddl;
              reinterpret_cast<float*>(p.d_u)[oi] = ddu;
            }
          }
        };
        if constexpr (BULK && DT % 4 == 0) {
          // 4 consecutive channels of one step per thread (whole channel
          // tiles and 16-byte aligned rows: vector loads and stores)
          for (int i = tid; i < nsl * (DT / 4); i += NTH) {
            const int sl = i / (DT / 4), dd0 = (i - sl * (DT / 4)) * 4;
            const int tts = tt_hi - sl;
            float dlv[4], uv[4], ddl[4], ddu[4];
            const int mr = mrow0 + mstep * tts;
            read_chan<4>(bdl + (size_t)(mr * DT + dd0) * es_du, bf_du, dlv);
            read_chan<4>(bu + (size_t)(mr * DT + dd0) * es_du, bf_du, uv);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const int dd = dd0 + k;
              const float* g4p = s_gs + ((size_t)(sl * ND + dd % ND) * 2) * SG + (dd / ND) * 4;
              const float4 g4 = *reinterpret_cast<const float4*>(g4p);
              const float4 b4 = *reinterpret_cast<const float4*>(g4p + SG);
              const float gsv = __fadd_rn(__fadd_rn(g4.x, g4.y), __fadd_rn(g4.z, g4.w));
              const float sBv = __fadd_rn(__fadd_rn(b4.x, b4.y), __fadd_rn(b4.z, b4.w));
              ddl[k] = __fmaf_rn(0.5f, gsv, __fmul_rn(sBv, uv[k]));
              ddu[k] = __fmul_rn(sBv, dlv[k]);
            }
            const int s = s0 + tts;
            const int t = dir ? L - 1 - s : s;
            if (first_of_two) {
              float4* sc = reinterpret_cast<float4*>(scratch + ((size_t)t * DT + dd0) * 2);
              sc[0] = make_float4(ddl[0], ddu[0], ddl[1], ddu[1]);
              sc[1] = make_float4(ddl[2], ddu[2], ddl[3], ddu[3]);
            } else {
              if (second_of_two) {
                const float4* sv = reinterpret_cast<const float4*>(s_scr + ((size_t)mr * DT + dd0) * 2);
                const float4 v0 = sv[0], v1 = sv[1];
                ddl[0] = __fadd_rn(v0.x, ddl[0]); ddu[0] = __fadd_rn(v0.y, ddu[0]);
                ddl[1] = __fadd_rn(v0.z, ddl[1]); ddu[1] = __fadd_rn(v0.w, ddu[1]);
                ddl[2] = __fadd_rn(v1.x, ddl[2]); ddu[2] = __fadd_rn(v1.y, ddu[2]);
                ddl[3] = __fadd_rn(v1.z, ddl[3]); ddu[3] = __fadd_rn(v1.w, ddu[3]);
              }
              if constexpr (PRO) {   // d dt = softplus'(dt) * (d delta rounded as the bf16 grad)
                const __nv_bfloat16* dtr = s_dtr + (size_t)buf * KC * DT + (size_t)mr * DT + dd0;
#pragma unroll
                for (int k = 0; k < 4; ++k)
                  ddl[k] = softplus20_grad(__bfloat162float(__float2bfloat16_rn(ddl[k])),
                                           __bfloat162float(dtr[k]));
              }
              const size_t oi = ((size_t)b * L + t) * D + d0 + dd0;
              if (bf_du) {
                auto pack = [](float x, float y) {
                  const __nv_bfloat162 h = __floats2bfloat162_rn(x, y);
                  return *reinterpret_cast<const uint32_t*>(&h);
                };
                *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(p.d_delta) + oi) =
                    make_uint2(pack(ddl[0], ddl[1]), pack(ddl[2], ddl[3]));
                *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(p.d_u) + oi) =
                    make_uint2(pack(ddu[0], ddu[1]), pack(ddu[2], ddu[3]));
              } else {
                *reinterpret_cast<float4*>(reinterpret_cast<float*>(p.d_delta) + oi) =
                    make_float4(ddl[0], ddl[1], ddl[2], ddl[3]);
                *reinterpret_cast<float4*>(reinterpret_cast<float*>(p.d_u) + oi) =
                    make_float4(ddu[0], ddu[1], ddu[2], ddu[3]);
              }
            }
          }
        } else if constexpr (NTH % DT == 0) {
          // a thread keeps one channel; its steps are independent, so unroll
          const int dd = tid % DT;
#pragma unroll 4
          for (int sl = tid / DT; sl < nsl; sl += NTH / DT) flush_du(sl, dd);
        } else {
          for (int i = tid; i < nsl * DT; i += NTH) {
            const int sl = i / DT;
            flush_du(sl, i - sl * DT);
          }
        }
        __syncthreads();
      }
    }
    if (fail) break;
    if (c == 0 && pass == ndirs - 1) fold_acc();   // the row's last work item
    if constexpr (!BULK) {
      if (more) store_bc(buf ^ 1);
    }
  }
  cp_async_wait0();
  if (fail && tid == 0) set_err(p.err, M3_ERR_DEVICE);

  // dA partial of this batch group (F64ACC: the float64 totals, rounded once)
  if constexpr (CF::F64ACC) {
#pragma unroll
    for (int i = 0; i < CF::NPAIR; ++i) {
      const double2 t = s_acc[i * NTH + tid];
      acc_pair(i) = make_float2((float)t.x, (float)t.y);
    }
  }
#pragma unroll
  for (int k = 0; k < ND; ++k) {
    const int d = dbase + k;
    if (d < D) {
      float* a0 = p.part_a + (((size_t)bg * 3 + 0) * D + d) * NP + q * NL;
      float* a1 = p.part_a + (((size_t)bg * 3 + 1) * D + d) * NP + q * NL;
      float* a2 = p.part_a + (((size_t)bg * 3 + 2) * D + d) * NP + q * NL;
#pragma unroll
      for (int j = 0; j < R; ++j) {
        a0[j] = (k & 1) ? gAr[k >> 1][j].y : gAr[k >> 1][j].x;
        a1[j] = -((k & 1) ? gAi[k >> 1][j].y : gAi[k >> 1][j].x);
        a2[j] = 0.f;
      }
#pragma unroll
      for (int j = R; j < NL; ++j) {
        a0[j] = 0.f;
        a1[j] = 0.f;
        a2[j] = (k & 1) ? gTk[k >> 1][j - R].y : gTk[k >> 1][j - R].x;
      }
    }
  }

  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  if (warp == 0) tmem_dealloc(*s_tmem, CF::NCOLS);
}

// Largest dynamic shared memory of one CTA on sm_100 (227 KB); tiles whose
// bulk-staging layout does not fit use the cp.async staging.
constexpr size_t kMaxSmemPerCta = 227 * 1024;

template <int R, int T, int ND, int NTH, bool GS, bool BULK, int DU, int DY, bool PRO = false>
cudaError_t launch_bwd_impl(const BwdParams& p, cudaStream_t stream) {
  using CF = BwdCfg<R, T, ND, NTH, GS, BULK, PRO>;
  static_assert(CF::smem_bytes <= kMaxSmemPerCta, "backward tile exceeds shared memory");
  // BULK: delta, u, dy as (B*L, D) row-major matrices with a (DT x KC) box;
  // cudaErrorNotSupported (nothing launched) when the maps cannot be built
  CUtensorMap maps[4];
  memset(maps, 0, sizeof(maps));
  if constexpr (BULK) {
    static_assert(DU >= 0 && DY >= 0, "bulk staging needs compile-time element types");
    if constexpr (PRO) {   // the bf16 x_proj rows, a (KC x N*P) box per B/C load
      if (!encode_rows_map(&maps[3], p.xbc, 2, (size_t)p.B * p.L, (size_t)p.ld_x, p.N * p.P,
                           CF::KC))
        return cudaErrorNotSupported;
    }
    // TMA staging only for tiles of at most 128 channels (the configurations
    // validated on the GPU); wider tiles take the element-wise staging
    if constexpr (CF::DT > 128) return cudaErrorNotSupported;
    const size_t rows = (size_t)p.B * p.L;
    const int edu = DU == 1 ? 2 : 4, edy = DY == 1 ? 2 : 4;
    if (!encode_rows_map(&maps[0], p.delta, edu, rows, p.D, CF::DT, CF::KC) ||
        !encode_rows_map(&maps[1], p.u, edu, rows, p.D, CF::DT, CF::KC) ||
        !encode_rows_map(&maps[2], p.dy, edy, rows, p.D, CF::DT, CF::KC))
      return cudaErrorNotSupported;
  }
  auto kern = scan_bwd_kernel<R, T, ND, NTH, GS, BULK, DU, DY, PRO>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)CF::smem_bytes);
  if (e != cudaSuccess) return e;
  dim3 grid(p.Bg, p.G);
  kern<<<grid, NTH, CF::smem_bytes, stream>>>(p, maps[0], maps[1], maps[2], maps[3]);
  return cudaGetLastError();
}

}  // namespace bwd
}  // namespace m3
