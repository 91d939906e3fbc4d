// dc_math.cuh -- double-precision exp for the verified elementwise steps.
//
// The reference computes softmax and SiLU with JavaScript's Math.exp
// (public/infer.js:59, :192), which V8 implements by porting the fdlibm 5.3
// method (Sun Microsystems, 1993).  This is an independent restatement of that
// published method, written with explicitly rounded double operations so no
// multiply-add contraction can change a bit:
//   1. reduce x = k*ln2 + r, |r| <= ln2/2, with r carried as hi - lo;
//   2. approximate R(r^2) = r*(e^r + 1)/(e^r - 1) by a degree-5 Remez
//      polynomial in r^2 and rebuild e^r = 1 - ((lo - r*c/(2 - c)) - hi);
//   3. scale by 2^k through the exponent field.
// The coefficients are fdlibm's published Remez values (given as IEEE bit
// patterns).  Its error is below 1 ulp; it is checked against the CPU
// oracle's separate restatement and against CUDA's exp error bound.
#pragma once
#include <stdint.h>

#include "dc_exp2_table.cuh"

namespace dcm {

__device__ __forceinline__ double b2d(uint64_t u) { return __longlong_as_double((long long)u); }

__device__ inline double fdlibm_exp(double x) {
  const double one = 1.0, huge = 1.0e+300;
  const double twom1000 = b2d(0x0170000000000000ULL);
  const double o_threshold = b2d(0x40862E42FEFA39EFULL);
  const double u_threshold = b2d(0xC0874910D52D3051ULL);
  const double ln2HI0 = b2d(0x3FE62E42FEE00000ULL);
  const double ln2LO0 = b2d(0x3DEA39EF35793C76ULL);
  const double invln2 = b2d(0x3FF71547652B82FEULL);
  const double P1 = b2d(0x3FC555555555553EULL), P2 = b2d(0xBF66C16C16BEBD93ULL),
               P3 = b2d(0x3F11566AAF25DE2CULL), P4 = b2d(0xBEBBBD41C5D26BF1ULL),
               P5 = b2d(0x3E66376972BEA4D0ULL);
  const uint64_t bx = (uint64_t)__double_as_longlong(x);
  uint32_t hx = (uint32_t)(bx >> 32);
  const int xsb = (int)((hx >> 31) & 1u);
  hx &= 0x7fffffffu;
  double hi = 0.0, lo = 0.0;
  int k = 0;
  if (hx >= 0x40862E42u) {
    if (hx >= 0x7ff00000u) {
      if (((hx & 0xfffffu) | (uint32_t)bx) != 0) return __dadd_rn(x, x);
      return xsb == 0 ? x : 0.0;
    }
    if (x > o_threshold) return __dmul_rn(huge, huge);
    if (x < u_threshold) return __dmul_rn(twom1000, twom1000);
  }
  if (hx > 0x3fd62e42u) {
    if (hx < 0x3FF0A2B2u) {
      const double l2h = xsb ? -ln2HI0 : ln2HI0;
      hi = __dsub_rn(x, l2h);
      lo = xsb ? -ln2LO0 : ln2LO0;
      k = 1 - xsb - xsb;
    } else {
      k = (int)__dadd_rn(__dmul_rn(invln2, x), xsb ? -0.5 : 0.5);  // truncation toward zero, as (int) in C
      const double t = (double)k;
      hi = __dsub_rn(x, __dmul_rn(t, ln2HI0));
      lo = __dmul_rn(t, ln2LO0);
    }
    x = __dsub_rn(hi, lo);
  } else if (hx < 0x3e300000u) {
    if (__dadd_rn(huge, x) > one) return __dadd_rn(one, x);
  } else {
    k = 0;
  }
  const double t = __dmul_rn(x, x);
  double p = __dadd_rn(P4, __dmul_rn(t, P5));
  p = __dadd_rn(P3, __dmul_rn(t, p));
  p = __dadd_rn(P2, __dmul_rn(t, p));
  p = __dadd_rn(P1, __dmul_rn(t, p));
  const double c = __dsub_rn(x, __dmul_rn(t, p));
  if (k == 0) return __dsub_rn(one, __dsub_rn(__ddiv_rn(__dmul_rn(x, c), __dsub_rn(c, 2.0)), x));
  const double y = __dsub_rn(one, __dsub_rn(__dsub_rn(lo, __ddiv_rn(__dmul_rn(x, c), __dsub_rn(2.0, c))), hi));
  const long long by = __double_as_longlong(y);
  if (k >= -1021) return __longlong_as_double(by + (long long)k * 4503599627370496LL);
  return __dmul_rn(__longlong_as_double(by + (long long)(k + 1000) * 4503599627370496LL), twom1000);
}

// fdlibm_exp without branches (selects only), for the kernels that evaluate
// it over many arguments side by side.  The reduction k = (int)(x/ln2 +- 1/2),
// hi = x - k ln2hi, lo = k ln2lo is fdlibm's general one; for 0.5 ln2 < |x| <
// 1.5 ln2 it yields exactly the k = +-1, hi = x -+ ln2hi, lo = +-ln2lo of
// fdlibm's special case (k*ln2hi and k*ln2lo are exact); up to fdlibm's k = 0
// bound (high word 0x3fd62e42) k is set to 0, where hi = x, lo = 0 and the
// rebuilt 1 - ((0 - xc/(2-c)) - x) equals fdlibm's 1 - (xc/(c-2) - x) bit for
// bit (negation is exact).  Tiny |x| (1 + x), overflow (+inf), underflow (+0),
// the subnormal scaling and non-finite arguments are selected.  Equal to
// fdlibm_exp for every argument (checked on the device against it).
__device__ __forceinline__ double fdlibm_exp_sel(double x) {
  const double one = 1.0;
  const double twom1000 = b2d(0x0170000000000000ULL);
  const double o_threshold = b2d(0x40862E42FEFA39EFULL);
  const double u_threshold = b2d(0xC0874910D52D3051ULL);
  const double ln2HI0 = b2d(0x3FE62E42FEE00000ULL);
  const double ln2LO0 = b2d(0x3DEA39EF35793C76ULL);
  const double invln2 = b2d(0x3FF71547652B82FEULL);
  const double P1 = b2d(0x3FC555555555553EULL), P2 = b2d(0xBF66C16C16BEBD93ULL),
               P3 = b2d(0x3F11566AAF25DE2CULL), P4 = b2d(0xBEBBBD41C5D26BF1ULL),
               P5 = b2d(0x3E66376972BEA4D0ULL);
  const uint64_t bx = (uint64_t)__double_as_longlong(x);
  const uint32_t hx = (uint32_t)(bx >> 32) & 0x7fffffffu;
  const bool neg = (bx >> 63) != 0;
  // (clamped so that the conversion is defined for every argument)
  const double kd = __dadd_rn(__dmul_rn(invln2, fmin(fmax(x, -800.0), 800.0)), neg ? -0.5 : 0.5);
  const int k = hx > 0x3fd62e42u ? (int)kd : 0;  // truncation toward zero, as (int) in C
  const double t = (double)k;
  const double hi = __dsub_rn(x, __dmul_rn(t, ln2HI0));
  const double lo = __dmul_rn(t, ln2LO0);
  const double r = __dsub_rn(hi, lo);
  const double tt = __dmul_rn(r, r);
  double p = __dadd_rn(P4, __dmul_rn(tt, P5));
  p = __dadd_rn(P3, __dmul_rn(tt, p));
  p = __dadd_rn(P2, __dmul_rn(tt, p));
  p = __dadd_rn(P1, __dmul_rn(tt, p));
  const double c = __dsub_rn(r, __dmul_rn(tt, p));
  const double y = __dsub_rn(one, __dsub_rn(__dsub_rn(lo, __ddiv_rn(__dmul_rn(r, c), __dsub_rn(2.0, c))), hi));
  const long long by = __double_as_longlong(y);
  const double yn = __longlong_as_double(by + (long long)k * 4503599627370496LL);
  const double ys = __dmul_rn(__longlong_as_double(by + (long long)(k + 1000) * 4503599627370496LL), twom1000);
  double res = k >= -1021 ? yn : ys;
  res = hx < 0x3e300000u ? __dadd_rn(one, x) : res;
  res = x < u_threshold ? 0.0 : res;
  res = x > o_threshold ? __longlong_as_double(0x7ff0000000000000LL) : res;
  return hx >= 0x7ff00000u ? (isnan(x) ? __dadd_rn(x, x) : (neg ? 0.0 : x)) : res;
}

// ---- a faster exp whose error bound settles the softmax's f32 values -------
// Tang's table-driven method (P. T. P. Tang, "Table-driven implementation of
// the exponential function in IEEE floating-point arithmetic", ACM TOMS 15(2),
// 1989), written here from the mathematics: x = (64 K + j) ln2/64 + r with
// |r| <= ln2/128 (ln2/64 split hi + lo, k * hi exact), e^r - 1 by its Taylor
// polynomial to degree 5 (truncation below 3.6e-17 relative), and
// exp(x) = 2^K * 2^(j/64) * e^r with 2^(j/64) a double-double from
// dc_exp2_table.cuh.  For -700 <= x <= 0.35 the result is normal and within
// 0.9 ulp of e^x; fdlibm's is within 1 ulp, so the two differ by less than
// 2^-51 relative.  It is not fdlibm's value bit for bit: exp_settle uses it
// only where that bound decides the f32 rounding.
// tab: the 64 pairs in shared memory (exp2_tab_load).
__device__ __forceinline__ void exp2_tab_load(double2* tab) {
  for (int i = threadIdx.x; i < 64; i += blockDim.x) tab[i] = make_double2(b2d(kExp2Tab[i][0]), b2d(kExp2Tab[i][1]));
}
__device__ __forceinline__ double exp_tang(double x, const double2* tab) {
  const int k = __double2int_rn(__dmul_rn(x, b2d(kInvLn2Times64)));
  const double kd = (double)k;
  const double r = __dsub_rn(__dsub_rn(x, __dmul_rn(kd, b2d(kLn2Over64Hi))), __dmul_rn(kd, b2d(kLn2Over64Lo)));
  double p = __dadd_rn(1.0 / 24.0, __dmul_rn(r, 1.0 / 120.0));
  p = __dadd_rn(1.0 / 6.0, __dmul_rn(r, p));
  p = __dadd_rn(0.5, __dmul_rn(r, p));
  p = __dadd_rn(1.0, __dmul_rn(r, p));
  p = __dmul_rn(r, p);  // e^r - 1
  const double2 t = tab[k & 63];
  const double y = __dadd_rn(t.x, __dadd_rn(__dmul_rn(t.x, p), t.y));  // 2^(j/64) e^r, in [0.99, 2.02)
  return __longlong_as_double(__double_as_longlong(y) + ((long long)(k >> 6) << 52));
}

// f32(fdlibm_exp(x)) -- the rounding the softmax keeps -- and in *e a double
// within 2^-49 relative of fdlibm_exp(x) (for the sums that are bracketed):
// from exp_tang when both ends of that interval round to the same float,
// otherwise (rarely, and for x < -700) from fdlibm_exp_sel itself.
__device__ __forceinline__ float exp_settle(double x, const double2* tab, double* e) {
  if (x >= -700.0 && x <= 0.0) {
    const double t = exp_tang(x, tab);
    const float lo = __double2float_rn(__dmul_rn(t, 1.0 - 0x1p-49));
    const float hi = __double2float_rn(__dmul_rn(t, 1.0 + 0x1p-49));
    if (lo == hi) {
      *e = t;
      return lo;
    }
  }
  const double f = fdlibm_exp_sel(x);
  *e = f;
  return __double2float_rn(f);
}

// infer.js:59 + :212: f32(silu(g) * u) with silu(v) = v / (1 + exp(-v)) in
// double and the exp above.
__device__ __forceinline__ float swiglu_f32(float gf, float uf) {
  const double v = gf;
  const double sl = __ddiv_rn(v, __dadd_rn(1.0, fdlibm_exp_sel(-v)));
  return __double2float_rn(__dmul_rn(sl, (double)uf));
}

// swiglu_f32's value, settled from exp_tang: e = exp(-v) within 2^-51 of
// fdlibm's, 1/(1 + e) from an f32 reciprocal refined by two Newton steps
// (within 2^-51), so the double product lies within 2^-49.4 relative of the
// exact chain's; unless both ends of a 2^-46 interval around it round to the
// same float (and for v outside [-80, 700], where f32(1 + e) could overflow),
// the exact chain decides.  tab: exp2_tab_load's table.
// swiglu_fast: the same value with no branch, *ok false where only the exact
// chain may decide (the caller then calls swiglu_f32).
__device__ __forceinline__ float swiglu_fast(float gf, float uf, const double2* tab, bool* ok) {
  const double v = gf;
  const bool inr = v >= -80.0 && v <= 700.0;
  const double d = __dadd_rn(1.0, exp_tang(inr ? -v : 0.0, tab));
  const double r0 = (double)__frcp_rn(__double2float_rn(d));
  double r = __fma_rn(r0, __fma_rn(-d, r0, 1.0), r0);
  r = __fma_rn(r, __fma_rn(-d, r, 1.0), r);
  const double y = __dmul_rn(__dmul_rn(v, r), (double)uf);
  const float lo = __double2float_rn(__dmul_rn(y, 1.0 - 0x1p-46));
  const float hi = __double2float_rn(__dmul_rn(y, 1.0 + 0x1p-46));
  *ok = inr && lo == hi;
  return lo;
}
__device__ __forceinline__ float swiglu_settle(float gf, float uf, const double2* tab) {
  bool ok;
  const float y = swiglu_fast(gf, uf, tab, &ok);
  return ok ? y : swiglu_f32(gf, uf);
}

}  // namespace dcm
