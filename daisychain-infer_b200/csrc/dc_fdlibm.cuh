// dc_fdlibm.cuh -- host-side pow / sin / cos for the RoPE tables.
//
// public/infer.js:71-81 builds its rotary tables with Math.pow, Math.cos and
// Math.sin.  V8 implements those with its fdlibm-derived ieee754 routines, so
// the tables here follow the same published method (Sun Microsystems fdlibm
// 5.3, 1993) rather than the C library's:
//   sin/cos: reduce x = n*pi/2 + (y0 + y1) with pi/2 split into 33-bit pieces
//            (three Cody-Waite stages, used as far as cancellation needs),
//            then a degree-13 odd / degree-14 even minimax polynomial on
//            [-pi/4, pi/4] with the tail y1 folded in;
//   pow:     log2(x) in extra precision (x scaled to [1, 2) and reduced by 1 or
//            1.5, log of (1+s)/(1-s) by a degree-12 polynomial in s^2, the
//            result split into high/low parts), times y split likewise, then
//            2^z by range reduction and the exp polynomial.
// The routines take the arguments the tables need: sin/cos for |x| below
// 2^19 * pi/2 (positions up to ~800000 radians; larger ones are refused by
// the table builder), pow for a finite base > 0 and a finite exponent.  Each
// is within 1 ulp of the correctly rounded value (checked against the C
// library in tests/test_rope_tables.py on the oracle's twin of this code).
#pragma once
#include <math.h>
#include <stdint.h>
#include <string.h>

namespace dcf {

inline double from_bits(uint64_t u) {
  double d;
  memcpy(&d, &u, 8);
  return d;
}
inline uint64_t to_bits(double d) {
  uint64_t u;
  memcpy(&u, &d, 8);
  return u;
}
inline int32_t hi_word(double d) { return (int32_t)(to_bits(d) >> 32); }
inline uint32_t lo_word(double d) { return (uint32_t)to_bits(d); }
inline double set_lo(double d, uint32_t lo) { return from_bits((to_bits(d) & 0xFFFFFFFF00000000ull) | lo); }
inline double set_hi(double d, uint32_t hi) { return from_bits((to_bits(d) & 0xFFFFFFFFull) | ((uint64_t)hi << 32)); }
inline double hi_only(uint32_t hi) { return from_bits((uint64_t)hi << 32); }

// sin on [-pi/4, pi/4] of x + y (y the tail of the reduced argument; tail = 0: y is 0)
inline double poly_sin(double x, double y, int tail) {
  const double s1 = from_bits(0xBFC5555555555549ull), s2 = from_bits(0x3F8111111110F8A6ull),
               s3 = from_bits(0xBF2A01A019C161D5ull), s4 = from_bits(0x3EC71DE357B1FE7Dull),
               s5 = from_bits(0xBE5AE5E68A2B9CEBull), s6 = from_bits(0x3DE5D93A5ACFD57Cull);
  if ((hi_word(x) & 0x7fffffff) < 0x3e400000 && (int)x == 0) return x;  // |x| < 2^-27
  const double z = x * x, v = z * x;
  const double r = s2 + z * (s3 + z * (s4 + z * (s5 + z * s6)));
  if (!tail) return x + v * (s1 + z * r);
  return x - ((z * (0.5 * y - v * r) - y) - v * s1);
}

// cos on [-pi/4, pi/4] of x + y
inline double poly_cos(double x, double y) {
  const double c1 = from_bits(0x3FA555555555554Cull), c2 = from_bits(0xBF56C16C16C15177ull),
               c3 = from_bits(0x3EFA01A019CB1590ull), c4 = from_bits(0xBE927E4F809C52ADull),
               c5 = from_bits(0x3E21EE9EBDB4B1C4ull), c6 = from_bits(0xBDA8FAE9BE8838D4ull);
  const int32_t ax = hi_word(x) & 0x7fffffff;
  if (ax < 0x3e400000 && (int)x == 0) return 1.0;
  const double z = x * x;
  const double r = z * (c1 + z * (c2 + z * (c3 + z * (c4 + z * (c5 + z * c6)))));
  if (ax < 0x3FD33333) return 1.0 - (0.5 * z - (z * r - x * y));  // |x| < 0.3
  // 1 - z/2 loses bits: take qx (x^2/8 rounded to a short number, capped) out first
  const double qx = ax > 0x3fe90000 ? 0.28125 : hi_only((uint32_t)(ax - 0x00200000));
  const double hz = 0.5 * z - qx, a = 1.0 - qx;
  return a - (hz - (z * r - x * y));
}

// High words of n * pi/2, n = 1..32: an argument whose high word differs from
// them is far enough from a multiple of pi/2 that one reduction stage suffices.
inline int32_t npio2_high(int n) {
  static const int32_t t[32] = {
      0x3FF921FB, 0x400921FB, 0x4012D97C, 0x401921FB, 0x401F6A7A, 0x4022D97C, 0x4025FDBB, 0x402921FB,
      0x402C463A, 0x402F6A7A, 0x4031475C, 0x4032D97C, 0x40346B9C, 0x4035FDBB, 0x40378FDB, 0x403921FB,
      0x403AB41B, 0x403C463A, 0x403DD85A, 0x403F6A7A, 0x40407E4C, 0x4041475C, 0x4042106C, 0x4042D97C,
      0x4043A28C, 0x40446B9C, 0x404534AC, 0x4045FDBB, 0x4046C6CB, 0x40478FDB, 0x404858EB, 0x404921FB};
  return t[n - 1];
}

// x = n * pi/2 + (y[0] + y[1]), |y| <= pi/4.  Valid for |x| <= 2^19 * pi/2
// (returns false beyond it).
inline bool reduce_pio2(double x, double y[2], int* n_out) {
  const double invpio2 = from_bits(0x3FE45F306DC9C883ull);
  const double p1 = from_bits(0x3FF921FB54400000ull), p1t = from_bits(0x3DD0B4611A626331ull);
  const double p2 = from_bits(0x3DD0B4611A600000ull), p2t = from_bits(0x3BA3198A2E037073ull);
  const double p3 = from_bits(0x3BA3198A2E000000ull), p3t = from_bits(0x397B839A252049C1ull);
  const int32_t hx = hi_word(x), ax = hx & 0x7fffffff;
  if (ax <= 0x3fe921fb) {
    y[0] = x;
    y[1] = 0.0;
    *n_out = 0;
    return true;
  }
  if (ax < 0x4002d97c) {  // |x| < 3pi/4: n = +-1
    const double sg = hx > 0 ? 1.0 : -1.0;
    double z = x - sg * p1;
    if (ax != 0x3ff921fb) {
      y[0] = z - sg * p1t;
      y[1] = (z - y[0]) - sg * p1t;
    } else {  // next to pi/2: one more piece of pi/2
      z -= sg * p2;
      y[0] = z - sg * p2t;
      y[1] = (z - y[0]) - sg * p2t;
    }
    *n_out = hx > 0 ? 1 : -1;
    return true;
  }
  if (ax > 0x413921fb) return false;
  double t = fabs(x);
  const int n = (int)(t * invpio2 + 0.5);
  const double fn = (double)n;
  double r = t - fn * p1, w = fn * p1t;
  y[0] = r - w;
  if (!(n < 32 && ax != npio2_high(n))) {
    const int32_t ex = ax >> 20;
    if (ex - ((hi_word(y[0]) >> 20) & 0x7ff) > 16) {  // cancellation: second stage (118 bits)
      t = r;
      w = fn * p2;
      r = t - w;
      w = fn * p2t - ((t - r) - w);
      y[0] = r - w;
      if (ex - ((hi_word(y[0]) >> 20) & 0x7ff) > 49) {  // third stage (151 bits)
        t = r;
        w = fn * p3;
        r = t - w;
        w = fn * p3t - ((t - r) - w);
        y[0] = r - w;
      }
    }
  }
  y[1] = (r - y[0]) - w;
  if (hx < 0) {
    y[0] = -y[0];
    y[1] = -y[1];
    *n_out = -n;
  } else {
    *n_out = n;
  }
  return true;
}

// sin / cos; *ok = false when |x| is beyond the reduction's range (or not finite).
inline double sin(double x, bool* ok) {
  double y[2];
  int n = 0;
  *ok = (hi_word(x) & 0x7fffffff) < 0x7ff00000 && reduce_pio2(x, y, &n);
  if (!*ok) return 0.0;
  if (n == 0) return poly_sin(x, 0.0, 0);
  switch (n & 3) {
    case 0: return poly_sin(y[0], y[1], 1);
    case 1: return poly_cos(y[0], y[1]);
    case 2: return -poly_sin(y[0], y[1], 1);
    default: return -poly_cos(y[0], y[1]);
  }
}
inline double cos(double x, bool* ok) {
  double y[2];
  int n = 0;
  *ok = (hi_word(x) & 0x7fffffff) < 0x7ff00000 && reduce_pio2(x, y, &n);
  if (!*ok) return 0.0;
  if (n == 0) return poly_cos(x, 0.0);
  switch (n & 3) {
    case 0: return poly_cos(y[0], y[1]);
    case 1: return -poly_sin(y[0], y[1], 1);
    case 2: return -poly_cos(y[0], y[1]);
    default: return poly_sin(y[0], y[1], 1);
  }
}

// x^y for finite x > 0 and finite y (*ok = false otherwise).
inline double pow(double x, double y, bool* ok) {
  *ok = x > 0.0 && (hi_word(x) & 0x7fffffff) < 0x7ff00000 && (hi_word(y) & 0x7fffffff) < 0x7ff00000;
  if (!*ok) return 0.0;
  const double two53 = from_bits(0x4340000000000000ull), huge = 1.0e300, tiny = 1.0e-300;
  const double bp[2] = {1.0, 1.5};
  const double dp_h[2] = {0.0, from_bits(0x3FE2B80340000000ull)}, dp_l[2] = {0.0, from_bits(0x3E4CFDEB43CFD006ull)};
  const double L1 = from_bits(0x3FE3333333333303ull), L2 = from_bits(0x3FDB6DB6DB6FABFFull),
               L3 = from_bits(0x3FD55555518F264Dull), L4 = from_bits(0x3FD17460A91D4101ull),
               L5 = from_bits(0x3FCD864A93C9DB65ull), L6 = from_bits(0x3FCA7E284A454EEFull);
  const double P1 = from_bits(0x3FC555555555553Eull), P2 = from_bits(0xBF66C16C16BEBD93ull),
               P3 = from_bits(0x3F11566AAF25DE2Cull), P4 = from_bits(0xBEBBBD41C5D26BF1ull),
               P5 = from_bits(0x3E66376972BEA4D0ull);
  const double lg2 = from_bits(0x3FE62E42FEFA39EFull), lg2_h = from_bits(0x3FE62E4300000000ull),
               lg2_l = from_bits(0xBE205C610CA86C39ull), ovt = 8.0085662595372944372e-17;
  const double cp = from_bits(0x3FEEC709DC3A03FDull), cp_h = from_bits(0x3FEEC709E0000000ull),
               cp_l = from_bits(0xBE3E2FE0145B01F5ull);
  const double ivln2 = from_bits(0x3FF71547652B82FEull), ivln2_h = from_bits(0x3FF7154760000000ull),
               ivln2_l = from_bits(0x3E54AE0BF85DDF44ull);
  const int32_t hx = hi_word(x), hy = hi_word(y);
  int32_t ix = hx & 0x7fffffff;
  const int32_t iy = hy & 0x7fffffff;
  if ((iy | (int32_t)lo_word(y)) == 0) return 1.0;
  double ax = x;
  if (lo_word(x) == 0 && ix == 0x3ff00000) return 1.0;
  // log2(x) = t1 + t2, extra precise
  double t1, t2;
  if (iy > 0x41e00000) {  // |y| > 2^31
    if (iy > 0x43f00000) return (ix <= 0x3fefffff) == (hy < 0) ? huge * huge : tiny * tiny;
    if (ix < 0x3fefffff) return hy < 0 ? huge * huge : tiny * tiny;
    if (ix > 0x3ff00000) return hy > 0 ? huge * huge : tiny * tiny;
    const double t = ax - 1.0;  // |1 - x| <= 2^-20: a short series
    const double w = (t * t) * (0.5 - t * (0.3333333333333333333333 - t * 0.25));
    const double u = ivln2_h * t, v = t * ivln2_l - w * ivln2;
    t1 = set_lo(u + v, 0);
    t2 = v - (t1 - u);
  } else {
    int32_t n = 0;
    if (ix < 0x00100000) {  // subnormal x
      ax *= two53;
      n -= 53;
      ix = hi_word(ax);
    }
    n += (ix >> 20) - 0x3ff;
    const int32_t j = ix & 0x000fffff;
    int k;
    ix = j | 0x3ff00000;  // x scaled into [1, 2)
    if (j <= 0x3988E) {   // below sqrt(3/2): reduce by 1
      k = 0;
    } else if (j < 0xBB67A) {  // below sqrt(3): reduce by 1.5
      k = 1;
    } else {  // otherwise halve and reduce by 1
      k = 0;
      n += 1;
      ix -= 0x00100000;
    }
    ax = set_hi(ax, (uint32_t)ix);
    // s = (x - b) / (x + b) as s_h + s_l
    double u = ax - bp[k], v = 1.0 / (ax + bp[k]);
    const double ss = u * v, s_h = set_lo(ss, 0);
    double t_h = hi_only((uint32_t)(((ix >> 1) | 0x20000000) + 0x00080000 + (k << 18)));
    double t_l = ax - (t_h - bp[k]);
    const double s_l = v * ((u - s_h * t_h) - s_h * t_l);
    double s2 = ss * ss;
    double r = s2 * s2 * (L1 + s2 * (L2 + s2 * (L3 + s2 * (L4 + s2 * (L5 + s2 * L6)))));
    r += s_l * (s_h + ss);
    s2 = s_h * s_h;
    t_h = set_lo(3.0 + s2 + r, 0);
    t_l = r - ((t_h - 3.0) - s2);
    u = s_h * t_h;
    v = s_l * t_h + t_l * ss;
    const double p_h = set_lo(u + v, 0), p_l = v - (p_h - u);
    const double z_h = cp_h * p_h, z_l = cp_l * p_h + p_l * cp + dp_l[k];
    const double t = (double)n;
    t1 = set_lo(((z_h + z_l) + dp_h[k]) + t, 0);
    t2 = z_l - (((t1 - t) - dp_h[k]) - z_h);
  }
  // y * log2(x) = p_h + p_l, then 2^(p_h + p_l)
  const double y1 = set_lo(y, 0);
  const double p_l = (y - y1) * t1 + y * t2;
  double p_h = y1 * t1;
  double z = p_l + p_h;
  int32_t j = hi_word(z);
  const int32_t i = (int32_t)lo_word(z);
  if (j >= 0x40900000) {  // z >= 1024
    if (((j - 0x40900000) | i) != 0 || p_l + ovt > z - p_h) return huge * huge;
  } else if ((j & 0x7fffffff) >= 0x4090cc00) {  // z <= -1075
    if (((j - (int32_t)0xc090cc00) | i) != 0 || p_l <= z - p_h) return tiny * tiny;
  }
  const int32_t iz = j & 0x7fffffff;
  int32_t k = (iz >> 20) - 0x3ff, n = 0;
  if (iz > 0x3fe00000) {  // |z| > 0.5: n = round(z), taken out of p_h
    n = j + (0x00100000 >> (k + 1));
    k = ((n & 0x7fffffff) >> 20) - 0x3ff;
    const double t = hi_only((uint32_t)(n & ~(0x000fffff >> k)));
    n = ((n & 0x000fffff) | 0x00100000) >> (20 - k);
    if (j < 0) n = -n;
    p_h -= t;
  }
  double t = set_lo(p_l + p_h, 0);
  const double u = t * lg2_h, v = (p_l - (t - p_h)) * lg2 + t * lg2_l;
  z = u + v;
  const double w = v - (z - u);
  t = z * z;
  const double tt = z - t * (P1 + t * (P2 + t * (P3 + t * (P4 + t * P5))));
  const double r = (z * tt) / (tt - 2.0) - (w + z * w);
  z = 1.0 - (r - z);
  j = hi_word(z) + (n << 20);
  if ((j >> 20) <= 0) return scalbn(z, n);  // subnormal result
  return set_hi(z, (uint32_t)j);
}

}  // namespace dcf
