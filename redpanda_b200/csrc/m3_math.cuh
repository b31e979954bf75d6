// Transcendentals of the gate exp(delta*A_real) * cos(delta*A_imag) and of its
// derivative (which also needs sin), written for the scan's accuracy budget.
//
// exp: 2^(delta * A_real*log2(e)) on the MUFU ex2 unit.  The log2(e) factor is
//   folded into the per-cell constant once; the relative error is a few ulp
//   and the absolute error of the gate stays below ~1e-7 because |x| e^x <= 1/e.
//
// cos / sin: Cody-Waite argument reduction (W. J. Cody and W. Waite, "Software
//   Manual for the Elementary Functions", 1980) followed by short polynomials.
//   The multiple of pi (or pi/2) is subtracted from the EXACT product
//   delta*A_imag inside an FMA, using a three-part split of pi whose leading
//   part has 12 significant bits (so k*PI_A is exact for |k| < 2^12).
//   Polynomial coefficients are this project's own least-squares fits on
//   Chebyshev nodes of the reduced interval (fp32 Horner evaluation included):
//     cos on [-pi/2, pi/2], 6 terms in r^2:          max abs error  9.0e-8
//     cos on [-pi/4, pi/4], 5 terms in r^2:          max abs error  5.2e-8
//     sin on [-pi/4, pi/4], r * (5 terms in r^2):    max rel error  9.0e-8
//   Arguments beyond the reduction's exact range (|k| > 2048, i.e.
//   |delta*A_imag| > ~6400) take the accurate libm path instead.
#pragma once

#include <cuda_runtime.h>

namespace m3 {

constexpr float kLog2e = 0x1.715476p+0f;        // log2(e) rounded to fp32
constexpr float kInvPi = 0x1.45f306p-2f;        // 1/pi
constexpr float kTwoOverPi = 0x1.45f306p-1f;    // 2/pi
constexpr float kPiA = 0x1.922p+1f;             // 3217/1024: pi to 12 significant bits
constexpr float kPiB = -0x1.2aeef4p-17f;        // pi - kPiA, rounded
constexpr float kPiC = -0x1.73dcb4p-42f;        // pi - kPiA - kPiB, rounded
constexpr float kMagic = 12582912.0f;           // 1.5 * 2^23: round-to-integer shifter
constexpr float kMaxK = 2048.0f;

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// exp(dl * ar) given a2 = ar * log2(e)
__device__ __forceinline__ float gate_exp(float dl, float a2) {
  return ex2_approx(__fmul_rn(dl, a2));
}

static __device__ __noinline__ float cos_slow(float dl, float ai) { return cosf(__fmul_rn(dl, ai)); }
static __device__ __noinline__ void sincos_slow(float dl, float ai, float* s, float* c) {
  sincosf(__fmul_rn(dl, ai), s, c);
}

// cos(dl * ai): reduction by pi, |r| <= pi/2, sign from the parity of k.
__device__ __forceinline__ float gate_cos(float dl, float ai) {
  const float x = __fmul_rn(dl, ai);
  const float j = __fmaf_rn(x, kInvPi, kMagic);
  const float k = __fsub_rn(j, kMagic);
  if (fabsf(k) > kMaxK) return cos_slow(dl, ai);
  float r = __fmaf_rn(dl, ai, -__fmul_rn(k, kPiA));
  r = __fmaf_rn(-k, kPiB, r);
  r = __fmaf_rn(-k, kPiC, r);
  const float s = __fmul_rn(r, r);
  float p = -0x1.181966p-22f;
  p = __fmaf_rn(p, s, 0x1.9f720cp-16f);
  p = __fmaf_rn(p, s, -0x1.6c1396p-10f);
  p = __fmaf_rn(p, s, 0x1.555548p-5f);
  p = __fmaf_rn(p, s, -0.5f);
  p = __fmaf_rn(p, s, 1.0f);
  const unsigned odd = __float_as_uint(j) << 31;   // k odd -> negate
  return __uint_as_float(__float_as_uint(p) ^ odd);
}

// sin and cos of dl * ai: reduction by pi/2, |r| <= pi/4, quadrant rotation.
__device__ __forceinline__ void gate_sincos(float dl, float ai, float& sn, float& cs) {
  const float x = __fmul_rn(dl, ai);
  const float j = __fmaf_rn(x, kTwoOverPi, kMagic);
  const float k = __fsub_rn(j, kMagic);
  if (fabsf(k) > 2.0f * kMaxK) {
    sincos_slow(dl, ai, &sn, &cs);
    return;
  }
  // pi/2 split = half of the pi split (exact halving)
  float r = __fmaf_rn(dl, ai, -__fmul_rn(k, 0.5f * kPiA));
  r = __fmaf_rn(-k, 0.5f * kPiB, r);
  r = __fmaf_rn(-k, 0.5f * kPiC, r);
  const float s = __fmul_rn(r, r);
  float pc = 0x1.994066p-16f;
  pc = __fmaf_rn(pc, s, -0x1.6c08bep-10f);
  pc = __fmaf_rn(pc, s, 0x1.55553ep-5f);
  pc = __fmaf_rn(pc, s, -0.5f);
  pc = __fmaf_rn(pc, s, 1.0f);
  float ps = 0x1.6ce166p-19f;
  ps = __fmaf_rn(ps, s, -0x1.a00fccp-13f);
  ps = __fmaf_rn(ps, s, 0x1.111108p-7f);
  ps = __fmaf_rn(ps, s, -0x1.555556p-3f);
  ps = __fmaf_rn(__fmul_rn(r, s), ps, r);
  const unsigned q = __float_as_uint(j);
  // quadrant q: (sin, cos) = (s, c), (c, -s), (-s, -c), (-c, s)
  const bool swap = q & 1u;
  const float a = swap ? pc : ps;
  const float b = swap ? ps : pc;
  const unsigned sgn_s = (q & 2u) << 30;            // q = 2, 3 -> negative sin
  const unsigned sgn_c = ((q + 1u) & 2u) << 30;     // q = 1, 2 -> negative cos
  sn = __uint_as_float(__float_as_uint(a) ^ sgn_s);
  cs = __uint_as_float(__float_as_uint(b) ^ sgn_c);
}

}  // namespace m3
