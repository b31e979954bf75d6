// Transcendentals of the gate exp(delta*A_real) * cos(delta*A_imag) and of its
// derivative (which also needs sin), written for the scan's accuracy budget.
//
// exp: 2^(delta * A_real*log2(e)) on the MUFU ex2 unit.  The log2(e) factor is
//   folded into the per-cell constant once; the relative error is a few ulp
//   and the absolute error of the gate stays below ~1e-7 because |x| e^x <= 1/e.
//
// cos / sin: Cody-Waite argument reduction (W. J. Cody and W. Waite, "Software
//   Manual for the Elementary Functions", 1980) followed by short polynomials.
//   The multiple of pi is subtracted from the EXACT product delta*A_imag
//   inside an FMA, using a two-part split of pi whose leading part has 12
//   significant bits (so k*PI_A is exact for |k| < 2^12); the second part is
//   pi - PI_A rounded to fp32, whose rounding error (3.3e-13) leaves r off by
//   at most 7e-10 for |k| <= 2048, far below the polynomials' errors.
//   The reduction is by pi (|r| <= pi/2); sin and cos share the sign (-1)^k.
//   Polynomial coefficients are this project's own least-squares fits on
//   Chebyshev nodes of [-pi/2, pi/2] (errors include the fp32 Horner evaluation):
//     cos: 6 terms in r^2,          max abs error 9.0e-8
//     sin: r * (6 terms in r^2),    max rel error 1.1e-7
//   Arguments beyond the reduction's exact range (|k| > 2048, i.e.
//   |delta*A_imag| > ~6400) take a slow path in double precision: the product
//   of two fp32 values is exact in fp64 (48 significant bits), and the CUDA
//   double-precision cos/sin of it, rounded once to fp32, are within half an
//   fp32 ulp or so of the true values.  All three paths (packed, scalar and
//   slow) therefore evaluate the gate at the EXACT product delta*A_imag; an
//   fp32 evaluation at the rounded product would be off by up to
//   |x| * 2^-24 (~4e-4 at |x| = 6400) in the argument.
#pragma once

#include <cuda_runtime.h>

namespace m3 {

constexpr float kLog2e = 0x1.715476p+0f;        // log2(e) rounded to fp32
constexpr float kInvPi = 0x1.45f306p-2f;        // 1/pi
constexpr float kPiA = 0x1.922p+1f;             // 3217/1024: pi to 12 significant bits
constexpr float kPiB = -0x1.2aeef4p-17f;        // pi - kPiA, rounded
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

// v with its sign flipped when k = j - kMagic is odd.  The low mantissa bit of
// j is the parity of k, so adding (bits(j) << 31) to the bits of v flips the
// sign bit exactly when k is odd (the carry out of bit 31 is dropped): a
// single shift-add.
__device__ __forceinline__ float flip_odd(float v, float j) {
  return __uint_as_float(__float_as_uint(v) + (__float_as_uint(j) << 31));
}

// |k| > 2048: cos / sin of the exact product in double precision.  cos is
// evaluated by the same call in both helpers, so the forward's and the
// backward's gates agree bit for bit on this path too.
static __device__ __noinline__ float cos_slow(float dl, float ai) {
  return (float)cos((double)dl * (double)ai);
}
static __device__ __noinline__ void sincos_slow(float dl, float ai, float* s, float* c) {
  const double x = (double)dl * (double)ai;
  *c = (float)cos(x);
  *s = (float)sin(x);
}

// cos(dl * ai): reduction by pi, |r| <= pi/2, sign from the parity of k.
__device__ __forceinline__ float gate_cos(float dl, float ai) {
  const float x = __fmul_rn(dl, ai);
  const float j = __fmaf_rn(x, kInvPi, kMagic);
  const float k = __fsub_rn(j, kMagic);
  if (fabsf(k) > kMaxK) return cos_slow(dl, ai);
  float r = __fmaf_rn(dl, ai, -__fmul_rn(k, kPiA));
  r = __fmaf_rn(-k, kPiB, r);
  const float s = __fmul_rn(r, r);
  float p = -0x1.181966p-22f;
  p = __fmaf_rn(p, s, 0x1.9f720cp-16f);
  p = __fmaf_rn(p, s, -0x1.6c1396p-10f);
  p = __fmaf_rn(p, s, 0x1.555548p-5f);
  p = __fmaf_rn(p, s, -0.5f);
  p = __fmaf_rn(p, s, 1.0f);
  return flip_odd(p, j);   // k odd -> negate
}

// ---------------------------------------------------------------------------
// Packed two-lane forms (sm_100 FFMA2/FMUL2/FADD2).  Each lane is rounded
// exactly like the scalar intrinsic above, so packed and scalar code paths give
// bit-identical results; only the instruction count differs.
__device__ __forceinline__ float2 f2(float a) { return make_float2(a, a); }

__device__ __forceinline__ float2 gate_exp2(float2 dl, float2 a2) {
  const float2 x = __fmul2_rn(dl, a2);
  return make_float2(ex2_approx(x.x), ex2_approx(x.y));
}

// cos(dl * ai) for two cells WITHOUT the large-argument check: the caller
// guarantees |dl * ai| <= 6000 (so |k| < kMaxK), where it equals gate_cos().
__device__ __forceinline__ float2 gate_cos2_nocheck(float2 dl, float2 ai) {
  const float2 x = __fmul2_rn(dl, ai);
  const float2 j = __ffma2_rn(x, f2(kInvPi), f2(kMagic));
  const float2 k = __fadd2_rn(j, f2(-kMagic));
  float2 r = __ffma2_rn(dl, ai, __fmul2_rn(k, f2(-kPiA)));
  r = __ffma2_rn(k, f2(-kPiB), r);
  const float2 s = __fmul2_rn(r, r);
  float2 p = f2(-0x1.181966p-22f);
  p = __ffma2_rn(p, s, f2(0x1.9f720cp-16f));
  p = __ffma2_rn(p, s, f2(-0x1.6c1396p-10f));
  p = __ffma2_rn(p, s, f2(0x1.555548p-5f));
  p = __ffma2_rn(p, s, f2(-0.5f));
  p = __ffma2_rn(p, s, f2(1.0f));
  return make_float2(flip_odd(p.x, j.x), flip_odd(p.y, j.y));
}

// sin and cos of dl*ai with the reduction by pi: both share the sign (-1)^k,
// cos is computed exactly as gate_cos() (so the backward's gate equals the
// forward's bit for bit) and sin uses a 6-term odd polynomial on [-pi/2, pi/2]
// (this project's least-squares fit, max relative error 1.1e-7).
__device__ __forceinline__ float sin_poly(float r, float s) {
  float p = -0x1.9a6850p-26f;
  p = __fmaf_rn(p, s, 0x1.71707ep-19f);
  p = __fmaf_rn(p, s, -0x1.a017dap-13f);
  p = __fmaf_rn(p, s, 0x1.11110cp-7f);
  p = __fmaf_rn(p, s, -0x1.555556p-3f);
  return __fmaf_rn(__fmul_rn(r, s), p, r);
}

__device__ __forceinline__ void gate_sincos_pi(float dl, float ai, float& sn, float& cs) {
  const float x = __fmul_rn(dl, ai);
  const float j = __fmaf_rn(x, kInvPi, kMagic);
  const float k = __fsub_rn(j, kMagic);
  if (fabsf(k) > kMaxK) {
    sincos_slow(dl, ai, &sn, &cs);
    return;
  }
  float r = __fmaf_rn(dl, ai, -__fmul_rn(k, kPiA));
  r = __fmaf_rn(-k, kPiB, r);
  const float s = __fmul_rn(r, r);
  float p = -0x1.181966p-22f;
  p = __fmaf_rn(p, s, 0x1.9f720cp-16f);
  p = __fmaf_rn(p, s, -0x1.6c1396p-10f);
  p = __fmaf_rn(p, s, 0x1.555548p-5f);
  p = __fmaf_rn(p, s, -0.5f);
  p = __fmaf_rn(p, s, 1.0f);
  cs = flip_odd(p, j);
  sn = flip_odd(sin_poly(r, s), j);
}

// Reduction by pi and both polynomials for two cells, before the sign:
// cos(dl*ai) = (-1)^k p and sin(dl*ai) = (-1)^k q, k's parity in the low bit of j.
__device__ __forceinline__ void sincos_reduced2(float2 dl, float2 ai, float2& j, float2& p,
                                                float2& q) {
  const float2 x = __fmul2_rn(dl, ai);
  j = __ffma2_rn(x, f2(kInvPi), f2(kMagic));
  const float2 k = __fadd2_rn(j, f2(-kMagic));
  float2 r = __ffma2_rn(dl, ai, __fmul2_rn(k, f2(-kPiA)));
  r = __ffma2_rn(k, f2(-kPiB), r);
  const float2 s = __fmul2_rn(r, r);
  p = f2(-0x1.181966p-22f);
  p = __ffma2_rn(p, s, f2(0x1.9f720cp-16f));
  p = __ffma2_rn(p, s, f2(-0x1.6c1396p-10f));
  p = __ffma2_rn(p, s, f2(0x1.555548p-5f));
  p = __ffma2_rn(p, s, f2(-0.5f));
  p = __ffma2_rn(p, s, f2(1.0f));
  q = f2(-0x1.9a6850p-26f);
  q = __ffma2_rn(q, s, f2(0x1.71707ep-19f));
  q = __ffma2_rn(q, s, f2(-0x1.a017dap-13f));
  q = __ffma2_rn(q, s, f2(0x1.11110cp-7f));
  q = __ffma2_rn(q, s, f2(-0x1.555556p-3f));
  q = __ffma2_rn(__fmul2_rn(r, s), q, r);
}

// The backward's two gate values of two cells, g = exp(dl*ar)*cos(dl*ai) and
// es = exp(dl*ar)*sin(dl*ai), without the large-argument check (|dl*ai| <=
// kFastArgBound).  The sign (-1)^k is put on the exponential once instead of
// on both polynomials; round-to-nearest is symmetric in the sign, so g equals
// gate_exp2(dl, a2) * gate_cos2_nocheck(dl, ai) bit for bit.
__device__ __forceinline__ void gate_es2_nocheck(float2 dl, float2 a2, float2 ai, float2& g,
                                                 float2& es) {
  float2 j, p, q;
  sincos_reduced2(dl, ai, j, p, q);
  const float2 e = gate_exp2(dl, a2);
  const float2 se = make_float2(flip_odd(e.x, j.x), flip_odd(e.y, j.y));
  g = __fmul2_rn(se, p);
  es = __fmul2_rn(se, q);
}

__device__ __forceinline__ void gate_sincos2_nocheck(float2 dl, float2 ai, float2& sn, float2& cs) {
  float2 j, p, q;
  sincos_reduced2(dl, ai, j, p, q);
  cs = make_float2(flip_odd(p.x, j.x), flip_odd(p.y, j.y));
  sn = make_float2(flip_odd(q.x, j.x), flip_odd(q.y, j.y));
}

// Largest |dl * ai| for which the packed no-check path is exact-equivalent.
constexpr float kFastArgBound = 6000.0f;

}  // namespace m3
