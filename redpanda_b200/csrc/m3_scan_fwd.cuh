#pragma once
// K1/K3 (kernel template): forward trapezoidal scan (causal, reverse, or both directions fused
// into one launch) with optional chunk checkpoints for the backward and the
// final (h, dBu) state for the O(1) step.
//
// Replaces _fwd_kernel (redpanda/engine/triton_scan.py:44-98) and the two
// flipped launches of the bidirectional Eval Mamba (redpanda/engine/mamba.py:254-260).
//
// CTA = 128 threads = 32 channel groups x 4 state-lane quarters.  A thread owns
// ND consecutive channels x (R rotational + T tracking) state lanes and walks
// the sequence in registers.  delta/u tiles of kCK timesteps are staged into
// shared memory with cp.async (double-buffered, in their HBM dtype); B/C are
// register-prefetched one chunk ahead, converted to fp32 and padded to the
// thread lane layout.  y is reduced over the 4 lane quarters with shuffles.
#include "m3_bulk.cuh"
#include "m3_common.cuh"
#include "m3_internal.h"
#include "m3_prologue.cuh"
#include "m3_stage.cuh"
#include "m3_tiles.h"
#include "m3_tma.h"

#include <string.h>

#include <type_traits>

namespace m3 {
namespace fwd {

// Stage delta and u for processing steps [s0, s0 + kCK) of row b, channels
// [d0, d0 + DT), in their HBM dtype, into one shared buffer pair.  Rows past the
// sequence end and channels past D are zero-filled.
template <int DT>
__device__ __forceinline__ void stage_du(unsigned char* s_dl, unsigned char* s_u,
                                         const FwdParams& p, int b, int d0, int s0,
                                         int dir, int esz) {
  if (p.async_ok) {
    const int epw = 4 / esz;        // elements per 4-byte word
    const int wpr = DT / epw;       // words per staged row
    for (int i = threadIdx.x; i < kCK * wpr; i += kThreads) {
      const int tt = i / wpr, w = i - tt * wpr;
      const int s = s0 + tt, d = d0 + w * epw;
      const bool ok = (s < p.L) && (d < p.D);
      const int t = dir ? p.L - 1 - s : s;
      const size_t gi = ok ? ((size_t)b * p.L + t) * p.D + d : 0;
      cp_async4(s_dl + (size_t)i * 4, (const char*)p.delta + gi * esz, ok);
      cp_async4(s_u + (size_t)i * 4, (const char*)p.u + gi * esz, ok);
    }
  } else {
    for (int i = threadIdx.x; i < kCK * DT; i += kThreads) {
      const int tt = i / DT, dd = i - tt * DT;
      const int s = s0 + tt, d = d0 + dd;
      const bool ok = (s < p.L) && (d < p.D);
      const int t = dir ? p.L - 1 - s : s;
      const size_t gi = ok ? ((size_t)b * p.L + t) * p.D + d : 0;
      if (esz == 2) {
        const uint16_t* a = (const uint16_t*)p.delta;
        const uint16_t* c = (const uint16_t*)p.u;
        ((uint16_t*)s_dl)[i] = ok ? a[gi] : 0;
        ((uint16_t*)s_u)[i] = ok ? c[gi] : 0;
      } else {
        ((float*)s_dl)[i] = ok ? ((const float*)p.delta)[gi] : 0.f;
        ((float*)s_u)[i] = ok ? ((const float*)p.u)[gi] : 0.f;
      }
    }
  }
}

// Stage y of processing steps [s0, s0 + kCK) for the second pass of the
// bidirectional scan, which adds the first pass's output; the tile is fp32
// in processing order (a bf16 y is widened by plain loads).
template <int DT>
__device__ __forceinline__ void stage_y(float* s_y, const FwdParams& p, int b, int d0, int s0,
                                        int dir) {
  for (int i = threadIdx.x; i < kCK * DT; i += kThreads) {
    const int tt = i / DT, dd = i - tt * DT;
    const int s = s0 + tt, d = d0 + dd;
    const bool ok = (s < p.L) && (d < p.D);
    const int t = dir ? p.L - 1 - s : s;
    const size_t gi = ok ? ((size_t)b * p.L + t) * p.D + d : 0;
    if (p.y_bf16)
      s_y[i] = ok ? __bfloat162float(static_cast<const __nv_bfloat16*>(p.y)[gi]) : 0.f;
    else
      cp_async4(s_y + i, static_cast<const float*>(p.y) + gi, ok);
  }
}

#ifndef M3_FWD_UNROLL
#define M3_FWD_UNROLL 2
#endif
constexpr int kFwdUnroll = M3_FWD_UNROLL;

#ifndef M3_FWD_MIN_BLOCKS
#define M3_FWD_MIN_BLOCKS 3
#endif

// Shared memory of the forward kernel (bytes): delta, u (HBM dtype, 4 bytes
// reserved per element), B, C (padded fp32), raw B/C rows and two mbarriers
// (BULK staging), y of the first pass (bidirectional second pass only).  The
// tiles that TMA boxes land in (delta, u, y) start on 128-byte boundaries.
template <int NP, int DT, bool BULK>
struct FwdSmem {
  static constexpr size_t du = (size_t)kCK * DT * 4;             // one buffer of delta or u
  static constexpr size_t bc = (size_t)kCK * NP * 8;             // one buffer of B or C pairs
  static constexpr size_t braw = BULK ? 2 * 2 * (size_t)kCK * NP * 4 : 0;   // [2][B|C][kCK][NP]
  static constexpr size_t off_bar = 2 * 2 * du + 2 * 2 * bc + braw;
  static constexpr size_t off_y = off_bar + 128;
  static size_t bytes(bool bidir) { return off_y + (bidir ? 2 * (size_t)kCK * DT * 4 : 0); }
};

// STATE: the launch writes the final (h, dBu) (return_state); compiled apart so
// that launches without it carry no code for the state-writing last step.
// DU: element type of delta and u fixed at compile time (0 fp32, 1 bf16), or
// -1 to read it from the parameters (the element-wise staging path).
// BULK: delta, u and the first pass's y arrive as TMA boxes (tm_dl, tm_u, tm_y:
// (B*L, D) row-major maps with a DT x kCK box), in memory row order.
// YB: y stored as bf16 (1) or fp32 (0) fixed at compile time, or -1 to read it
// from the parameters (the element-wise staging path).
// PRO: the layer's prologue is fused into the staging (BULK, bf16 only): tm_dl
// maps dt, the dt_proj output before softplus, and tm_x the bf16 x_proj rows;
// each landed chunk is turned into delta = bf16(softplus(dt)) in place and
// into the padded B/C pairs by BCNorm + MIMO fold (m3_prologue.cuh), the same
// values the standalone prologue followed by a cast to bf16 gives.
template <int R, int T, int ND, bool BULK, bool STATE, int DU, int YB, bool PRO = false>
__global__ void __launch_bounds__(kThreads, M3_FWD_MIN_BLOCKS)
    scan_fwd_kernel(const FwdParams p, const __grid_constant__ CUtensorMap tm_dl,
                    const __grid_constant__ CUtensorMap tm_u,
                    const __grid_constant__ CUtensorMap tm_y,
                    const __grid_constant__ CUtensorMap tm_x) {
  static_assert(!PRO || (BULK && DU == 1), "the fused prologue is a bf16 bulk-staging variant");
  using LM = LaneMap<R, T>;
  constexpr int NL = R + T;
  constexpr int NP = LM::NP;
  constexpr int DT = 32 * ND;
  constexpr int RR = R > 0 ? R : 1;
  constexpr int TT = T > 0 ? T : 1;
  constexpr int BCE = (kCK * NP + kThreads - 1) / kThreads;   // B/C prefetch per thread

  using SM = FwdSmem<NP, DT, BULK>;
  extern __shared__ __align__(128) unsigned char smem[];
  unsigned char* s_dl = smem;                                 // [2][kCK*DT*4]
  unsigned char* s_u = s_dl + 2 * kCK * DT * 4;               // [2][kCK*DT*4]
  // B and C of each staged step in the padded lane layout, as (b, b) pairs so
  // that packed instructions take them without a broadcast
  float2* s_b = reinterpret_cast<float2*>(s_u + 2 * kCK * DT * 4);  // [2][kCK][NP]
  float2* s_c = s_b + 2 * kCK * NP;
  float* s_braw = reinterpret_cast<float*>(s_c + 2 * kCK * NP);     // [2][B|C][kCK][NP] (BULK)
  uint64_t* s_bar = reinterpret_cast<uint64_t*>(smem + SM::off_bar);   // [2] (BULK)
  float* s_y = reinterpret_cast<float*>(smem + SM::off_y);    // [2][kCK][DT] (bidir pass 2)

  const int tid = threadIdx.x, q = tid & 3, grp = tid >> 2;
  const int b = blockIdx.x;
  const int d0 = blockIdx.y * DT;
  const int dbase = d0 + grp * ND;
  const bool bf16 = DU < 0 ? p.dt_du == M3_BF16 : DU == 1;
  const bool ybf = YB < 0 ? p.y_bf16 != 0 : YB == 1;
  const int esz = bf16 ? 2 : 4;
  const int L = p.L, D = p.D, N = p.N;

  // Eigenvalues of this thread's cells (zero for virtual lanes / channels),
  // held as channel pairs (k, k+1) so the packed FP32 path can use them.
  constexpr int NDP = (ND + 1) / 2;
  float2 A2[NDP][RR], AI[NDP][RR], TK[NDP][TT];
  float maxai = 0.f;   // max |A_imag| over the thread's cells (fast-path bound)
#pragma unroll
  for (int k = 0; k < 2 * NDP; ++k) {
    const int d = dbase + k;
#pragma unroll
    for (int j = 0; j < NL; ++j) {
      const int n = LM::mem_lane(q, j, p.NR, p.NT);
      const bool ok = (k < ND) && (d < D) && (n >= 0);
      const size_t gi = ok ? (size_t)d * N + n : 0;
      if (j < R) {
        const float a2 = ok ? exp_const(p.Ar[gi]) : 0.f;   // A_real * log2(e)
        const float ai = ok ? p.Ai[gi] : 0.f;
        maxai = fmaxf(maxai, fabsf(ai));
        if (k & 1) { A2[k >> 1][j].y = a2; AI[k >> 1][j].y = ai; }
        else       { A2[k >> 1][j].x = a2; AI[k >> 1][j].x = ai; }
      } else {
        const float tv = ok ? p.Tk[gi] : 0.f;
        if (k & 1) TK[k >> 1][j - R].y = tv;
        else       TK[k >> 1][j - R].x = tv;
      }
    }
  }

  const int es_bc = p.dt_bc == M3_BF16 ? 2 : 4;
  if constexpr (BULK) {
    // TMA boxes land at 128-byte aligned shared addresses; uniform over the CTA
    if (smem_addr(smem) & 127u) {
      if (tid == 0) set_err(p.err, M3_ERR_DEVICE);
      return;
    }
    if (tid == 0) {
      mbar_init(&s_bar[0], 1);
      mbar_init(&s_bar[1], 1);
      mbar_fence_init();
    }
    __syncthreads();
  }
  int phase[2] = {0, 0};   // completed uses of each staging buffer (BULK)
  int fail = 0;

  const int npass = p.direction == M3_DIR_BIDIR ? 2 : 1;
  for (int pass = 0; pass < npass && !fail; ++pass) {
    const int dir = p.direction == M3_DIR_BIDIR ? (pass == 0 ? 1 : 0) : p.direction;
    const bool accumulate = p.direction == M3_DIR_BIDIR && pass == 1;
    const int dslot = p.direction == M3_DIR_BIDIR ? dir : 0;
    const int ndirs = p.direction == M3_DIR_BIDIR ? 2 : 1;

    float2 P[NDP][NL];   // P = 2h + dBu of cells (k, j): component k&1 of P[k/2][j]
#pragma unroll
    for (int k = 0; k < NDP; ++k)
#pragma unroll
      for (int j = 0; j < NL; ++j) P[k][j] = make_float2(0.f, 0.f);

    float rb[BCE], rc[BCE];
    auto load_bc = [&](int s0) {
#pragma unroll
      for (int e = 0; e < BCE; ++e) {
        const int i = tid + e * kThreads;
        const int tt = i / NP, lane = i - tt * NP;
        const int s = s0 + tt;
        const int n = LM::mem_lane(lane / NL, lane % NL, p.NR, p.NT);
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
        const int i = tid + e * kThreads;
        if (i < kCK * NP) {
          s_b[buf * kCK * NP + i] = f2(rb[e]);
          s_c[buf * kCK * NP + i] = f2(rc[e]);
        }
      }
    };

    // BULK: thread 0 stages chunk c on the copy engine, completing on the
    // buffer's mbarrier: delta, u (and, in the second pass, the first pass's
    // y) as TMA boxes of kCK memory rows from the chunk's first memory row
    // (rows past the chunk are never read; rows past the tensor read zero),
    // the chunk's B and C rows as one contiguous block each.  y was written by
    // this CTA's first pass with generic stores before an earlier barrier,
    // hence the proxy fence.
    auto stage_bulk = [&](int c, int buf) {
      const int s0 = c * kCK, ns = min(kCK, L - s0);
      const int t_lo = dir ? L - s0 - ns : s0;
      const uint32_t bcb = PRO ? (uint32_t)(kCK * N * p.P * 2) : (uint32_t)(ns * N * es_bc);
      const uint32_t bytes = (uint32_t)(2 * kCK * DT * esz) + 2 * bcb +
                             (accumulate ? (uint32_t)(kCK * DT * (ybf ? 2 : 4)) : 0u);
      if (accumulate) fence_proxy_async_global();
      mbar_arrive_expect_tx(&s_bar[buf], bytes);
      const int y0 = b * L + t_lo;
      tma_load_2d(s_dl + buf * kCK * DT * 4, &tm_dl, d0, y0, &s_bar[buf]);
      tma_load_2d(s_u + buf * kCK * DT * 4, &tm_u, d0, y0, &s_bar[buf]);
      if constexpr (PRO) {
        // B_raw and C_raw boxes (kCK rows x N*P bf16) into the single raw
        // buffer: the previous chunk's raw rows were widened before the
        // barrier that precedes this issue
        __nv_bfloat16* raw = reinterpret_cast<__nv_bfloat16*>(s_braw);
        tma_load_2d(raw, &tm_x, p.off_b, y0, &s_bar[buf]);
        tma_load_2d(raw + (size_t)kCK * N * p.P, &tm_x, p.off_c, y0, &s_bar[buf]);
      } else {
        const size_t bc_off = ((size_t)b * L + t_lo) * N * es_bc;
        bulk_g2s(s_braw + (size_t)(buf * 2 + 0) * kCK * NP, (const char*)p.Bc + bc_off, bcb,
                 &s_bar[buf]);
        bulk_g2s(s_braw + (size_t)(buf * 2 + 1) * kCK * NP, (const char*)p.Cc + bc_off, bcb,
                 &s_bar[buf]);
      }
      if (accumulate) tma_load_2d(s_y + (size_t)buf * kCK * DT, &tm_y, d0, y0, &s_bar[buf]);
    };
    // raw B/C rows (memory order, N elements each) -> (b, b) pairs of the
    // padded lane layout in processing order
    auto widen_bc = [&](int buf, int ns) {
      if constexpr (PRO) {
        // delta = bf16(softplus(dt)) in place over the landed dt tile
        __nv_bfloat16* dlt = reinterpret_cast<__nv_bfloat16*>(s_dl + buf * kCK * DT * 4);
        for (int i = tid; i < kCK * DT; i += kThreads)
          dlt[i] = __float2bfloat16_rn(softplus20(__bfloat162float(dlt[i])));
        // BCNorm + MIMO fold of each staged row, one warp per (step, B|C)
        const int np = N * p.P, lane = tid & 31;
        const __nv_bfloat16* raw = reinterpret_cast<const __nv_bfloat16*>(s_braw);
        for (int r = tid >> 5; r < 2 * ns; r += kThreads / 32) {
          const int which = r & 1, tt = r >> 1;
          const int mr = dir ? ns - 1 - tt : tt;   // raw rows are in memory order
          const __nv_bfloat16* x = raw + ((size_t)which * kCK + mr) * np;
          auto ld = [&](int k) { return __bfloat162float(x[k]); };
          const float* w = which ? p.wc : p.wb;
          const float rs = bcnorm_scale(ld, np, p.eps, w != nullptr, lane);
          float2* dst = (which ? s_c : s_b) + buf * kCK * NP + tt * NP;
          for (int ln = lane; ln < NP; ln += 32) {
            const int n = LM::mem_lane(ln / NL, ln % NL, p.NR, p.NT);
            const float v = n >= 0 ? __bfloat162float(__float2bfloat16_rn(
                                         bcnorm_fold(ld, n, p.P, rs, w)))
                                   : 0.f;
            dst[ln] = f2(v);
          }
        }
        return;
      }
      const float* rb0 = s_braw + (size_t)(buf * 2 + 0) * kCK * NP;
      const float* rc0 = s_braw + (size_t)(buf * 2 + 1) * kCK * NP;
      for (int i = tid; i < ns * NP; i += kThreads) {
        const int tt = i / NP, ln = i - tt * NP;
        const int n = LM::mem_lane(ln / NL, ln % NL, p.NR, p.NT);
        const size_t r = (size_t)(dir ? ns - 1 - tt : tt) * N + (n >= 0 ? n : 0);
        s_b[buf * kCK * NP + i] = f2(n >= 0 ? ld_f(rb0, r, p.dt_bc) : 0.f);
        s_c[buf * kCK * NP + i] = f2(n >= 0 ? ld_f(rc0, r, p.dt_bc) : 0.f);
      }
    };

    // prologue: chunk 0 into buffer 0 (BULK: landed and widened before the
    // loop; each chunk then waits for and widens its successor at its end,
    // under the barrier that closes it)
    if constexpr (BULK) {
      if (tid == 0) stage_bulk(0, 0);
      const bool ok = mbar_wait(&s_bar[0], (uint32_t)(phase[0] & 1));
      ++phase[0];
      // (the fused widen uses warp shuffles: enter it warp-uniformly)
      if (PRO ? __all_sync(0xffffffffu, ok) : ok) widen_bc(0, min(kCK, L));
      if (__syncthreads_or(!ok)) {
        if (tid == 0) mbar_wait(&s_bar[0], (uint32_t)((phase[0] - 1) & 1));
        fail = 1;
        break;
      }
    } else {
      stage_du<DT>(s_dl, s_u, p, b, d0, 0, dir, esz);
      if (accumulate) stage_y<DT>(s_y, p, b, d0, 0, dir);
      cp_async_commit();
      load_bc(0);
      store_bc(0);
    }

    for (int c = 0; c < p.nch; ++c) {
      const int buf = c & 1;
      const bool more = c + 1 < p.nch;
      if constexpr (BULK) {
        if (more && tid == 0) stage_bulk(c + 1, buf ^ 1);
      } else {
        if (more) {
          stage_du<DT>(s_dl + (buf ^ 1) * kCK * DT * 4, s_u + (buf ^ 1) * kCK * DT * 4, p, b, d0,
                       (c + 1) * kCK, dir, esz);
          if (accumulate) stage_y<DT>(s_y + (buf ^ 1) * kCK * DT, p, b, d0, (c + 1) * kCK, dir);
        }
        cp_async_commit();
        if (more) load_bc((c + 1) * kCK);
        cp_async_wait1();
        __syncthreads();
      }

      const unsigned char* bdl = s_dl + buf * kCK * DT * 4;
      const unsigned char* bu = s_u + buf * kCK * DT * 4;
      const float2* bb = s_b + buf * kCK * NP;
      const float2* bc = s_c + buf * kCK * NP;
      const float* by = s_y + buf * kCK * DT;
      const int ns = min(kCK, L - c * kCK);
      // staged delta/u/y rows: processing order (cp.async staging) or memory
      // order (BULK: processing step tt is memory row ns-1-tt when reversed)
      const int mrow0 = (BULK && dir) ? ns - 1 : 0, mstep = (BULK && dir) ? -1 : 1;
      // checkpoint of P = 2h + dBu before processing step s (the start of a
      // backward chunk: every p.cki steps)
      auto write_ckpt = [&](int s) {
#pragma unroll
        for (int k = 0; k < ND; ++k) {
          const int d = dbase + k;
          if (d < D) {
            float* dst = p.ckpt +
                ((((size_t)b * ndirs + dslot) * p.nck + (s / p.cki - 1)) * D + d) * NP + q * NL;
            if constexpr (NL % 4 == 0) {   // 16-byte aligned: NP*4 and NL*4 are multiples of 16
#pragma unroll
              for (int j = 0; j < NL; j += 4)
                *reinterpret_cast<float4*>(dst + j) =
                    (k & 1) ? make_float4(P[k >> 1][j].y, P[k >> 1][j + 1].y,
                                          P[k >> 1][j + 2].y, P[k >> 1][j + 3].y)
                            : make_float4(P[k >> 1][j].x, P[k >> 1][j + 1].x,
                                          P[k >> 1][j + 2].x, P[k >> 1][j + 3].x);
            } else {
#pragma unroll
              for (int j = 0; j < NL; ++j) dst[j] = (k & 1) ? P[k >> 1][j].y : P[k >> 1][j].x;
            }
          }
        }
      };
      // One processing step.  FASTC: the caller proved |delta*A_imag| <=
      // kFastArgBound for the whole chunk and that it holds no state output,
      // so the packed path runs without a per-step check.
      auto step = [&](int tt, auto fast_tag) {
        constexpr bool FASTC = decltype(fast_tag)::value;
        const int s = c * kCK + tt;
        const int t = dir ? L - 1 - s : s;
        const int mr = mrow0 + mstep * tt;
        float dl[ND], uu[ND];
        read_chan<ND>(bdl + (size_t)(mr * DT + grp * ND) * esz, bf16, dl);
        read_chan<ND>(bu + (size_t)(mr * DT + grp * ND) * esz, bf16, uu);
        float2 Bv[NL], Cv[NL];   // B, C of the thread's lanes as (b, b) pairs
#pragma unroll
        for (int j = 0; j < NL; ++j) {
          Bv[j] = bb[tt * NP + q * NL + j];
          Cv[j] = bc[tt * NP + q * NL + j];
        }
        const bool last = STATE && !FASTC && (s == L - 1) && (p.h_last != nullptr);
        float mdl = 0.f;
        if constexpr (!FASTC) {
#pragma unroll
          for (int k = 0; k < ND; ++k) mdl = fmaxf(mdl, fabsf(dl[k]));
        }
        float part[2 * NDP];
        if (FASTC || ((ND % 2 == 0) && !last && __fmul_rn(mdl, maxai) <= kFastArgBound)) {
          // packed path: channel pairs, no per-cell range checks
#pragma unroll
          for (int kp = 0; kp < NDP; ++kp) {
            const float2 dl2 = make_float2(dl[2 * kp], dl[(2 * kp + 1) % ND]);
            const float2 du2 = __fmul2_rn(dl2, make_float2(uu[2 * kp], uu[(2 * kp + 1) % ND]));
            float2 acc = make_float2(0.f, 0.f);
#pragma unroll
            for (int j = 0; j < R; ++j) {
              const float2 g = __fmul2_rn(gate_exp2(dl2, A2[kp][j]), gate_cos2_nocheck(dl2, AI[kp][j]));
              const float2 H = cell_update2p(g, P[kp][j], du2, Bv[j]);
              acc = __ffma2_rn(H, Cv[j], acc);
            }
#pragma unroll
            for (int j = R; j < NL; ++j) {
              const float2 H = cell_update2p(TK[kp][j - R], P[kp][j], du2, Bv[j]);
              acc = __ffma2_rn(H, Cv[j], acc);
            }
            part[2 * kp] = acc.x;
            part[2 * kp + 1] = acc.y;
          }
        } else {
          // scalar path: per-cell range checks (large arguments, the last step)
          float du[ND];
#pragma unroll
          for (int k = 0; k < ND; ++k) du[k] = __fmul_rn(dl[k], uu[k]);
          float Cs[NL];
#pragma unroll
          for (int j = 0; j < NL; ++j) Cs[j] = Cv[j].x;
#pragma unroll
          for (int k = 0; k < ND; ++k) {
            float H[NL];
#pragma unroll
            for (int j = 0; j < NL; ++j) {
              float& Pk = (k & 1) ? P[k >> 1][j].y : P[k >> 1][j].x;
              float g;
              if (j < R) {
                g = rot_gate(dl[k], (k & 1) ? A2[k >> 1][j].y : A2[k >> 1][j].x,
                             (k & 1) ? AI[k >> 1][j].y : AI[k >> 1][j].x);
              } else {
                g = (k & 1) ? TK[k >> 1][j - R].y : TK[k >> 1][j - R].x;
              }
              H[j] = cell_update(g, Pk, du[k], Bv[j].x);
            }
            part[k] = y_partial<NL>(H, Cs);
            if (last) {
              const int d = dbase + k;
              if (d < D) {
#pragma unroll
                for (int j = 0; j < NL; ++j) {
                  const int n = LM::mem_lane(q, j, p.NR, p.NT);
                  if (n >= 0) {
                    const size_t gi = ((size_t)b * D + d) * N + n;
                    p.h_last[gi] = __fmul_rn(0.5f, H[j]);
                    p.dbu_last[gi] = __fmul_rn(du[k], Bv[j].x);
                  }
                }
              }
            }
          }
        }
        const size_t yrow = ((size_t)b * L + t) * D;
        // channel totals over the 4 quarters; quarter q writes channels k = 4i + q
        constexpr int NY = ND >= 4 ? ND / 4 : 1;   // channels written per thread
        if constexpr (ND % 2 == 0) quad_sum_t<ND>(reinterpret_cast<float(&)[ND]>(part), q);
        else part[0] = quad_sum(part[0]);
#pragma unroll
        for (int i = 0; i < NY; ++i) {
          const int k = ND >= 4 ? 4 * i + q : q;
          const float tot = __fmul_rn(0.5f, part[i]);
          const int d = dbase + k;
          if (k < ND && d < D) {
            float v = tot;
            if (accumulate) {
              // BULK with a bf16 y: the staged first-pass rows are bf16
              const int si = mr * DT + grp * ND + k;
              v = __fadd_rn(tot, (BULK && ybf)
                                     ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(by)[si])
                                     : by[si]);
            }
            if (ybf) static_cast<__nv_bfloat16*>(p.y)[yrow + d] = __float2bfloat16_rn(v);
            else static_cast<float*>(p.y)[yrow + d] = v;
          }
        }
      };
      // the range decision once per chunk: max |delta| of the thread's channels
      bool chunk_fast = false;
      if constexpr (ND % 2 == 0) {
        float mdl = 0.f;
        if (bf16) {
          // bf16 rows: |x| orders like the unsigned bits x & 0x7fff, so the
          // maximum is taken on packed 16-bit halves of the raw words (a NaN
          // sorts above every number and selects the checked path)
          uint32_t m = 0;
          for (int tt = 0; tt < ns; ++tt) {
            const uint32_t* w =
                reinterpret_cast<const uint32_t*>(bdl + (size_t)(tt * DT + grp * ND) * 2);
#pragma unroll
            for (int i = 0; i < ND / 2; ++i) m = max_u16x2(m, w[i] & 0x7fff7fffu);
          }
          mdl = __uint_as_float(max(m & 0xffffu, m >> 16) << 16);
        } else {
          for (int tt = 0; tt < ns; ++tt) {
            float dl[ND];
            read_chan<ND>(bdl + (size_t)(tt * DT + grp * ND) * 4, false, dl);
#pragma unroll
            for (int k = 0; k < ND; ++k) mdl = fmaxf(mdl, fabsf(dl[k]));
          }
        }
        chunk_fast = __fmul_rn(mdl, maxai) <= kFastArgBound;
      }
      // the step that writes the final state (return_state) takes the checked path
      const bool has_last = STATE && p.h_last != nullptr && c * kCK + ns == L;
      const int nfast = has_last ? ns - 1 : ns;
      // segments between checkpoint positions (p.cki divides kCK)
      const int seg_len = p.cki < kCK ? p.cki : kCK;
      for (int seg = 0; seg < ns; seg += seg_len) {
        const int send = min(ns, seg + seg_len);
        const int s = c * kCK + seg;
        if (p.ckpt != nullptr && s > 0 && (s & (p.cki - 1)) == 0) write_ckpt(s);
        if (chunk_fast) {
          const int fend = min(send, nfast);
#pragma unroll kFwdUnroll
          for (int tt = seg; tt < fend; ++tt) step(tt, std::true_type{});
          for (int tt = fend; tt < send; ++tt) step(tt, std::false_type{});
        } else {
          for (int tt = seg; tt < send; ++tt) step(tt, std::false_type{});
        }
      }
      if constexpr (BULK) {
        bool ok = true;
        if (more) {
          ok = mbar_wait(&s_bar[buf ^ 1], (uint32_t)(phase[buf ^ 1] & 1));
          ++phase[buf ^ 1];
          if (PRO ? __all_sync(0xffffffffu, ok) : ok) widen_bc(buf ^ 1, min(kCK, L - (c + 1) * kCK));
        }
        if (__syncthreads_or(!ok)) {
          // give up: let the copy still in flight land before the CTA exits
          if (tid == 0) mbar_wait(&s_bar[buf ^ 1], (uint32_t)((phase[buf ^ 1] - 1) & 1));
          fail = 1;
          break;
        }
      } else {
        if (more) store_bc(buf ^ 1);
        __syncthreads();
      }
    }
  }
  cp_async_wait0();
  if (fail) set_err(p.err, M3_ERR_DEVICE);
}

template <int R, int T, int ND, bool BULK, bool STATE, int DU, int YB, bool PRO = false>
cudaError_t launch_fwd_impl(const FwdParams& p, cudaStream_t stream) {
  constexpr int NP = 4 * (R + T);
  constexpr int DT = 32 * ND;
  const size_t smem = FwdSmem<NP, DT, BULK>::bytes(p.direction == M3_DIR_BIDIR);
  // BULK: delta, u, y as (B*L, D) row-major maps with a (DT x kCK) box;
  // cudaErrorNotSupported (nothing launched) when the maps cannot be built
  CUtensorMap maps[4];
  memset(maps, 0, sizeof(maps));
  if constexpr (BULK) {
    static_assert(DU >= 0, "bulk staging needs a compile-time element type");
    if constexpr (PRO) {   // the bf16 x_proj rows, a (kCK x N*P) box per B/C load
      if (!encode_rows_map(&maps[3], p.xbc, 2, (size_t)p.B * p.L, (size_t)p.ld_x,
                           p.N * p.P, kCK))
        return cudaErrorNotSupported;
    }
    // TMA staging only for tiles of at most 128 channels (the configurations
    // validated on the GPU); wider tiles take the element-wise staging
    if constexpr (DT > 128) return cudaErrorNotSupported;
    const size_t rows = (size_t)p.B * p.L;
    const int edu = DU == 1 ? 2 : 4;
    if (!encode_rows_map(&maps[0], p.delta, edu, rows, p.D, DT, kCK) ||
        !encode_rows_map(&maps[1], p.u, edu, rows, p.D, DT, kCK) ||
        !encode_rows_map(&maps[2], p.y, p.y_bf16 ? 2 : 4, rows, p.D, DT, kCK))
      return cudaErrorNotSupported;
  }
  auto kern = scan_fwd_kernel<R, T, ND, BULK, STATE, DU, YB, PRO>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid(p.B, (p.D + DT - 1) / DT);
  kern<<<grid, kThreads, smem, stream>>>(p, maps[0], maps[1], maps[2], maps[3]);
  return cudaGetLastError();
}

}  // namespace fwd
}  // namespace m3
