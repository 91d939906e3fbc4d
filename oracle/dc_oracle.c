/*
 * dc_oracle.c -- CPU oracle for DaisyChain-Infer's verified INT8 W8A8 path.
 *
 * TEST INFRASTRUCTURE, NOT PRODUCT CODE.  This file restates in plain C the
 * arithmetic of the reference's JavaScript CPU path so that the CUDA product
 * can be checked against it bit for bit.  Only tests/, __graft_entry__.smoke()
 * and bench.py's CPU-baseline legs load it; the product library never links,
 * loads or calls it, and it is never a fallback.
 *
 * What it restates (reference paths are relative to the reference project):
 *   public/verified_core.js  assertFinite :16-27, accBound/MAX_INT32_K :41-49,
 *                            quantizeRows :108-121, quantizeCols :122-136,
 *                            epi :227-228, bgemmJS :241-266, vgemmBlock :425-449
 *   public/infer.js          rmsNorm :30-39, silu :59, ropeTables :71-81,
 *                            applyRope :83-97, layerForward :114-221,
 *                            embedRows :298-310, logitsAt :324-334,
 *                            pickToken (greedy) :390-396
 *   public/webgpu.js         probeInputs :998-1009, kernelProbe's FNV :1053-1055
 *   public/shard.js          fnv1a :195-200
 *   test_pipeline.js         mulberry32 :32, rnd :33-37 (weight fixtures)
 *
 * Parity status.  The LUT contents are pinned by the sha256 of the reference's
 * LFS objects.  Integer work (quantisation, int32 accumulation, LUT outputs)
 * and every f32/f64 step built from + - * / sqrt are pinned by IEEE-754
 * (correct rounding) and by the reference's known-answer tests.  Values
 * downstream of a transcendental (softmax exp, SiLU exp, RoPE pow/cos/sin)
 * are PARITY UNPINNED against V8: no JavaScript runtime exists on either
 * machine, and the reference stores no golden vectors.  exp() here follows
 * the fdlibm 5.3 method (Sun Microsystems, 1993), the method V8's Math.exp is
 * ported from, and so do pow/cos/sin for the RoPE tables.
 *
 * The requant-LUT output rule is not defined anywhere in the reference (it
 * belonged to a Python kernel that is not in the repository).  This build
 * declares it: out8 = requant[(uint16)sat16(acc)], then relu[(uint8)out8]
 * when the ReLU flag is set.  That output is bit-exact against this declared
 * rule, not against reference code.
 *
 * Build: oracle/Makefile (gcc -O2 -ffp-contract=off, no -march, so no FMA
 * contraction and every double/float operation rounds exactly once).
 */
#ifdef _OPENMP
#include <omp.h>
#endif
#if defined(__x86_64__) && defined(__GNUC__)
#include <immintrin.h>
#define ORC_X86 1
#endif
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_OK 0
#define ORC_E_ACCBOUND 1
#define ORC_E_NONFINITE 2
#define ORC_E_INVAL 3
#define ORC_E_NOMEM 4

#define ORC_RELU 1u
#define ORC_ACC 2u
#define ORC_REQUANT 4u

/* floor((2^31 - 1) / (128 * 128)) -- verified_core.js:41 */
#define ORC_MAX_INT32_K 131071

/* Parallel loops (OpenMP) only above this much work; smaller calls stay serial. */
#define PAR_MIN (1 << 16)
#define BGEMM_JB 512

static double bits2d(uint64_t u) { double d; memcpy(&d, &u, 8); return d; }
static uint64_t d2bits(double d) { uint64_t u; memcpy(&u, &d, 8); return u; }

int orc_max_int32_k(void) { return (int)floor(2147483647.0 / (128.0 * 128.0)); }

/* verified_core.js:42-49: refuse a contraction that could wrap int32. */
int orc_acc_bound(int64_t k) { return k > ORC_MAX_INT32_K ? ORC_E_ACCBOUND : ORC_OK; }

/* verified_core.js:16-27: index of the first non-finite value, or -1. */
int64_t orc_first_nonfinite(const float* x, int64_t n) {
  for (int64_t i = 0; i < n; i++)
    if (!isfinite(x[i])) return i;
  return -1;
}

/* ECMAScript Math.round: nearest integer, ties toward +infinity.
 * floor(v + 0.5) is wrong at 0.49999999999999994, so compare the remainder. */
static double js_round(double v) {
  double r = floor(v);
  if (v - r >= 0.5) r += 1.0;
  return r;
}
static int8_t clamp8(double v) { return v < -128.0 ? (int8_t)-128 : v > 127.0 ? (int8_t)127 : (int8_t)v; }

double orc_js_round(double v) { return js_round(v); }

/* ---- lookup-table units: public/{mul,requant,relu}_lut.bin, reconstructed */
void orc_make_luts(int16_t* mul, int8_t* requant, int8_t* relu) {
  for (int a = 0; a < 256; a++)
    for (int b = 0; b < 256; b++)
      mul[a * 256 + b] = (int16_t)((a > 127 ? a - 256 : a) * (b > 127 ? b - 256 : b));
  for (int u = 0; u < 65536; u++) {
    int s = u > 32767 ? u - 65536 : u;
    requant[u] = (int8_t)(s >> 8); /* arithmetic shift by luts_meta.json "shift": 8 */
  }
  for (int u = 0; u < 256; u++) {
    int s = u > 127 ? u - 256 : u;
    relu[u] = (int8_t)(s > 0 ? s : 0);
  }
}

/* ---- quantisers ------------------------------------------------------------ */
/* verified_core.js:108-121.  The scale is computed in DOUBLE and the quotient
 * uses that double; only the stored copy s[r] is rounded to f32. */
int orc_quantize_rows(const float* X, int64_t rows, int64_t cols, int8_t* q, float* s) {
  if (orc_first_nonfinite(X, rows * cols) >= 0) return ORC_E_NONFINITE;
#pragma omp parallel for schedule(static) if (rows * cols >= PAR_MIN)
  for (int64_t r = 0; r < rows; r++) {
    const float* x = X + r * cols;
    double mx = 0.0;
    for (int64_t c = 0; c < cols; c++) {
      double a = fabs((double)x[c]);
      if (a > mx) mx = a;
    }
    double sc = mx / 127.0;
    if (!(sc > 1e-8)) sc = 1e-8;
    s[r] = (float)sc;
    for (int64_t c = 0; c < cols; c++) q[r * cols + c] = clamp8(js_round((double)x[c] / sc));
  }
  return ORC_OK;
}

/* verified_core.js:122-136.  The scale is stored as f32 and the quotient uses
 * the f32-ROUNDED scale (the asymmetry with quantizeRows is real). */
int orc_quantize_cols(const float* W, int64_t rows, int64_t cols, int8_t* q, float* s) {
  if (orc_first_nonfinite(W, rows * cols) >= 0) return ORC_E_NONFINITE;
#pragma omp parallel for schedule(static) if (rows * cols >= PAR_MIN)
  for (int64_t c = 0; c < cols; c++) {
    double mx = 0.0;
    for (int64_t r = 0; r < rows; r++) {
      double a = fabs((double)W[r * cols + c]);
      if (a > mx) mx = a;
    }
    double sc = mx / 127.0;
    if (!(sc > 1e-8)) sc = 1e-8;
    s[c] = (float)sc;
  }
#pragma omp parallel for schedule(static) if (rows * cols >= PAR_MIN)
  for (int64_t r = 0; r < rows; r++)
    for (int64_t c = 0; c < cols; c++)
      q[r * cols + c] = clamp8(js_round((double)W[r * cols + c] / (double)s[c]));
  return ORC_OK;
}

/* ---- epilogue and GEMM ---------------------------------------------------- */
/* verified_core.js:227-228: f32(f32(f32(s) * a) * b), no fused multiply-add. */
float orc_epi(int32_t s, float a, float b) {
  volatile float t = (float)s;
  t = t * a;
  t = t * b;
  return t;
}

/* verified_core.js:241-266 (bgemmJS), extended with the declared requant rule.
 * X is (batch*m) x k int8, W is batch x (k x n) int8 row-major, rs[batch*m],
 * cs[batch*n].  out is int32 (ACC), int8 (REQUANT) or f32 (default). */
int orc_bgemm(const int8_t* Xq, const int8_t* Wq, const float* rs, const float* cs, int m, int k, int n,
              int batch, unsigned flags, const int16_t* mul, const int8_t* requant, const int8_t* relu,
              void* out) {
  if (m < 0 || k < 0 || n < 0 || batch < 1) return ORC_E_INVAL;
  if (orc_acc_bound(k)) return ORC_E_ACCBOUND;
  /* Each (row, block of BGEMM_JB columns) is one task: its int32 sums run over
   * p in order (each output element is computed by one thread, so the result
   * does not depend on the thread count). */
  const int nb = (n + BGEMM_JB - 1) / BGEMM_JB;
  const int64_t work = (int64_t)batch * m * k * n;
  for (int bz = 0; bz < batch; bz++) {
    const int8_t* xb = Xq + (int64_t)bz * m * k;
    const int8_t* wb = Wq + (int64_t)bz * k * n;
#pragma omp parallel for collapse(2) schedule(static) if (work >= PAR_MIN)
    for (int i = 0; i < m; i++) {
      for (int jbk = 0; jbk < nb; jbk++) {
        const int j0 = jbk * BGEMM_JB, j1 = j0 + BGEMM_JB < n ? j0 + BGEMM_JB : n;
        int32_t acc[BGEMM_JB];
        memset(acc, 0, sizeof(acc));
        const int8_t* xr = xb + (int64_t)i * k;
        for (int p = 0; p < k; p++) {
          const int16_t* row = mul + ((uint8_t)xr[p]) * 256;
          const int8_t* wr = wb + (int64_t)p * n;
          for (int j = j0; j < j1; j++)
            acc[j - j0] = (int32_t)((uint32_t)acc[j - j0] + (uint32_t)(int32_t)row[(uint8_t)wr[j]]);
        }
        int64_t orow = ((int64_t)bz * m + i) * n;
        if (flags & ORC_ACC) {
          memcpy((int32_t*)out + orow + j0, acc, sizeof(int32_t) * (size_t)(j1 - j0));
        } else if (flags & ORC_REQUANT) {
          int8_t* o = (int8_t*)out + orow;
          for (int j = j0; j < j1; j++) {
            int32_t a = acc[j - j0] < -32768 ? -32768 : acc[j - j0] > 32767 ? 32767 : acc[j - j0];
            int8_t v = requant[(uint16_t)(int16_t)a];
            if (flags & ORC_RELU) v = relu[(uint8_t)v];
            o[j] = v;
          }
        } else {
          float* o = (float*)out + orow;
          float rsc = rs[(int64_t)bz * m + i];
          for (int j = j0; j < j1; j++) {
            float v = orc_epi(acc[j - j0], rsc, cs[(int64_t)bz * n + j]);
            o[j] = ((flags & ORC_RELU) && v < 0.0f) ? 0.0f : v;
          }
        }
      }
    }
  }
  return ORC_OK;
}

/* Threads the parallel loops above may use (1 without OpenMP). */
int orc_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* ---- exp: fdlibm 5.3 method (Sun Microsystems, 1993) ------------------------
 * Reduce x = k*ln2 + r with |r| <= ln2/2 (r kept as hi - lo), approximate
 * R(r^2) = r*(e^r + 1)/(e^r - 1) by a degree-5 Remez polynomial, rebuild
 * e^r = 1 - ((lo - r*c/(2 - c)) - hi) and scale by 2^k. */
double orc_exp(double x) {
  const double one = 1.0, huge = 1.0e+300;
  const double halF[2] = {0.5, -0.5};
  const double twom1000 = bits2d(0x0170000000000000ULL);
  const double o_threshold = bits2d(0x40862E42FEFA39EFULL);
  const double u_threshold = bits2d(0xC0874910D52D3051ULL);
  const double ln2HI[2] = {bits2d(0x3FE62E42FEE00000ULL), bits2d(0xBFE62E42FEE00000ULL)};
  const double ln2LO[2] = {bits2d(0x3DEA39EF35793C76ULL), bits2d(0xBDEA39EF35793C76ULL)};
  const double invln2 = bits2d(0x3FF71547652B82FEULL);
  const double P1 = bits2d(0x3FC555555555553EULL), P2 = bits2d(0xBF66C16C16BEBD93ULL),
               P3 = bits2d(0x3F11566AAF25DE2CULL), P4 = bits2d(0xBEBBBD41C5D26BF1ULL),
               P5 = bits2d(0x3E66376972BEA4D0ULL);
  double y, hi = 0.0, lo = 0.0, c, t;
  int k = 0;
  uint64_t bx = d2bits(x);
  uint32_t hx = (uint32_t)(bx >> 32);
  int xsb = (int)((hx >> 31) & 1);
  hx &= 0x7fffffffu;
  if (hx >= 0x40862E42u) { /* |x| >= 709.78... */
    if (hx >= 0x7ff00000u) {
      if (((hx & 0xfffffu) | (uint32_t)bx) != 0) return x + x; /* NaN */
      return xsb == 0 ? x : 0.0;                               /* exp(+-inf) */
    }
    if (x > o_threshold) return huge * huge;
    if (x < u_threshold) return twom1000 * twom1000;
  }
  if (hx > 0x3fd62e42u) {   /* |x| > 0.5 ln2 */
    if (hx < 0x3FF0A2B2u) { /* and |x| < 1.5 ln2 */
      hi = x - ln2HI[xsb];
      lo = ln2LO[xsb];
      k = 1 - xsb - xsb;
    } else {
      k = (int)(invln2 * x + halF[xsb]);
      t = k;
      hi = x - t * ln2HI[0];
      lo = t * ln2LO[0];
    }
    x = hi - lo;
  } else if (hx < 0x3e300000u) { /* |x| < 2^-28 */
    if (huge + x > one) return one + x;
  } else {
    k = 0;
  }
  t = x * x;
  c = x - t * (P1 + t * (P2 + t * (P3 + t * (P4 + t * P5))));
  if (k == 0) return one - ((x * c) / (c - 2.0) - x);
  y = one - ((lo - (x * c) / (2.0 - c)) - hi);
  uint64_t by = d2bits(y);
  /* add k (or k + 1000) to the exponent field of y */
  if (k >= -1021) return bits2d((uint64_t)((int64_t)by + (int64_t)k * 4503599627370496LL));
  return bits2d((uint64_t)((int64_t)by + (int64_t)(k + 1000) * 4503599627370496LL)) * twom1000;
}

/* ---- pow / sin / cos: the fdlibm 5.3 method (Sun Microsystems, 1993) -------
 * The RoPE tables of infer.js:71-81 come from Math.pow, Math.cos and Math.sin,
 * which V8 implements with its fdlibm-derived ieee754 routines; these are a
 * restatement of the same published method (not the C library's):
 * sin/cos reduce x = n*pi/2 + (y0 + y1) with pi/2 in 33-bit pieces (three
 * Cody-Waite stages as cancellation requires; |x| <= 2^19*pi/2, NaN beyond),
 * then minimax polynomials on [-pi/4, pi/4]; pow (x > 0 finite, y finite)
 * forms log2(x) in extra precision, multiplies by y split in two, and
 * evaluates 2^z by range reduction and the exp polynomial.  Within 1 ulp of
 * the C library's results (tests/test_rope_tables.py). */
static double with_lo(double d, uint32_t lo) { return bits2d((d2bits(d) & 0xFFFFFFFF00000000ULL) | lo); }
static double with_hi(double d, uint32_t hi) { return bits2d((d2bits(d) & 0xFFFFFFFFULL) | ((uint64_t)hi << 32)); }
static uint32_t lo32(double d) { return (uint32_t)d2bits(d); }
static int32_t hi32(double d) { return (int32_t)(d2bits(d) >> 32); }

static double fdl_ksin(double x, double y, int iy) {
  const double S1 = bits2d(0xBFC5555555555549ULL), S2 = bits2d(0x3F8111111110F8A6ULL),
               S3 = bits2d(0xBF2A01A019C161D5ULL), S4 = bits2d(0x3EC71DE357B1FE7DULL),
               S5 = bits2d(0xBE5AE5E68A2B9CEBULL), S6 = bits2d(0x3DE5D93A5ACFD57CULL);
  int32_t ix = hi32(x) & 0x7fffffff;
  if (ix < 0x3e400000 && (int)x == 0) return x;
  double z = x * x, v = z * x;
  double r = S2 + z * (S3 + z * (S4 + z * (S5 + z * S6)));
  if (iy == 0) return x + v * (S1 + z * r);
  return x - ((z * (0.5 * y - v * r) - y) - v * S1);
}
static double fdl_kcos(double x, double y) {
  const double C1 = bits2d(0x3FA555555555554CULL), C2 = bits2d(0xBF56C16C16C15177ULL),
               C3 = bits2d(0x3EFA01A019CB1590ULL), C4 = bits2d(0xBE927E4F809C52ADULL),
               C5 = bits2d(0x3E21EE9EBDB4B1C4ULL), C6 = bits2d(0xBDA8FAE9BE8838D4ULL);
  int32_t ix = hi32(x) & 0x7fffffff;
  if (ix < 0x3e400000 && (int)x == 0) return 1.0;
  double z = x * x;
  double r = z * (C1 + z * (C2 + z * (C3 + z * (C4 + z * (C5 + z * C6)))));
  if (ix < 0x3FD33333) return 1.0 - (0.5 * z - (z * r - x * y));
  double qx = ix > 0x3fe90000 ? 0.28125 : bits2d((uint64_t)(uint32_t)(ix - 0x00200000) << 32);
  double hz = 0.5 * z - qx, a = 1.0 - qx;
  return a - (hz - (z * r - x * y));
}
static const int32_t npio2_hw[32] = {
  0x3FF921FB, 0x400921FB, 0x4012D97C, 0x401921FB, 0x401F6A7A, 0x4022D97C, 0x4025FDBB, 0x402921FB,
  0x402C463A, 0x402F6A7A, 0x4031475C, 0x4032D97C, 0x40346B9C, 0x4035FDBB, 0x40378FDB, 0x403921FB,
  0x403AB41B, 0x403C463A, 0x403DD85A, 0x403F6A7A, 0x40407E4C, 0x4041475C, 0x4042106C, 0x4042D97C,
  0x4043A28C, 0x40446B9C, 0x404534AC, 0x4045FDBB, 0x4046C6CB, 0x40478FDB, 0x404858EB, 0x404921FB};
/* |x| <= 2^19 pi/2 only; returns n, y[0]+y[1] = x - n pi/2 */
static int fdl_rem_pio2(double x, double* y) {
  const double invpio2 = bits2d(0x3FE45F306DC9C883ULL), pio2_1 = bits2d(0x3FF921FB54400000ULL),
               pio2_1t = bits2d(0x3DD0B4611A626331ULL), pio2_2 = bits2d(0x3DD0B4611A600000ULL),
               pio2_2t = bits2d(0x3BA3198A2E037073ULL), pio2_3 = bits2d(0x3BA3198A2E000000ULL),
               pio2_3t = bits2d(0x397B839A252049C1ULL);
  int32_t hx = hi32(x), ix = hx & 0x7fffffff;
  if (ix <= 0x3fe921fb) { y[0] = x; y[1] = 0; return 0; }
  if (ix < 0x4002d97c) {
    if (hx > 0) {
      double z = x - pio2_1;
      if (ix != 0x3ff921fb) { y[0] = z - pio2_1t; y[1] = (z - y[0]) - pio2_1t; }
      else { z -= pio2_2; y[0] = z - pio2_2t; y[1] = (z - y[0]) - pio2_2t; }
      return 1;
    } else {
      double z = x + pio2_1;
      if (ix != 0x3ff921fb) { y[0] = z + pio2_1t; y[1] = (z - y[0]) + pio2_1t; }
      else { z += pio2_2; y[0] = z + pio2_2t; y[1] = (z - y[0]) + pio2_2t; }
      return -1;
    }
  }
  if (ix <= 0x413921fb) {
    double t = fabs(x);
    int n = (int)(t * invpio2 + 0.5);
    double fn = (double)n, r = t - fn * pio2_1, w = fn * pio2_1t;
    if (n < 32 && ix != npio2_hw[n - 1]) {
      y[0] = r - w;
    } else {
      int32_t j = ix >> 20;
      y[0] = r - w;
      int32_t i = j - ((hi32(y[0]) >> 20) & 0x7ff);
      if (i > 16) {
        t = r; w = fn * pio2_2; r = t - w; w = fn * pio2_2t - ((t - r) - w); y[0] = r - w;
        i = j - ((hi32(y[0]) >> 20) & 0x7ff);
        if (i > 49) { t = r; w = fn * pio2_3; r = t - w; w = fn * pio2_3t - ((t - r) - w); y[0] = r - w; }
      }
    }
    y[1] = (r - y[0]) - w;
    if (hx < 0) { y[0] = -y[0]; y[1] = -y[1]; return -n; }
    return n;
  }
  y[0] = y[1] = NAN; /* beyond 2^19 pi/2: not needed by the RoPE tables */
  return 0;
}
double orc_fdl_sin(double x) {
  int32_t ix = hi32(x) & 0x7fffffff; double y[2];
  if (ix <= 0x3fe921fb) return fdl_ksin(x, 0.0, 0);
  if (ix >= 0x7ff00000) return x - x;
  int n = fdl_rem_pio2(x, y);
  if (isnan(y[0])) return NAN;
  switch (n & 3) { case 0: return fdl_ksin(y[0], y[1], 1); case 1: return fdl_kcos(y[0], y[1]);
    case 2: return -fdl_ksin(y[0], y[1], 1); default: return -fdl_kcos(y[0], y[1]); }
}
double orc_fdl_cos(double x) {
  int32_t ix = hi32(x) & 0x7fffffff; double y[2];
  if (ix <= 0x3fe921fb) return fdl_kcos(x, 0.0);
  if (ix >= 0x7ff00000) return x - x;
  int n = fdl_rem_pio2(x, y);
  if (isnan(y[0])) return NAN;
  switch (n & 3) { case 0: return fdl_kcos(y[0], y[1]); case 1: return -fdl_ksin(y[0], y[1], 1);
    case 2: return -fdl_kcos(y[0], y[1]); default: return fdl_ksin(y[0], y[1], 1); }
}
/* x > 0 finite, y finite */
double orc_fdl_pow(double x, double y) {
  const double bp[2] = {1.0, 1.5}, dp_h[2] = {0.0, bits2d(0x3FE2B80340000000ULL)},
               dp_l[2] = {0.0, bits2d(0x3E4CFDEB43CFD006ULL)}, two53 = bits2d(0x4340000000000000ULL),
               huge = 1.0e300, tiny = 1.0e-300,
               L1 = bits2d(0x3FE3333333333303ULL), L2 = bits2d(0x3FDB6DB6DB6FABFFULL), L3 = bits2d(0x3FD55555518F264DULL),
               L4 = bits2d(0x3FD17460A91D4101ULL), L5 = bits2d(0x3FCD864A93C9DB65ULL), L6 = bits2d(0x3FCA7E284A454EEFULL),
               P1 = bits2d(0x3FC555555555553EULL), P2 = bits2d(0xBF66C16C16BEBD93ULL), P3 = bits2d(0x3F11566AAF25DE2CULL),
               P4 = bits2d(0xBEBBBD41C5D26BF1ULL), P5 = bits2d(0x3E66376972BEA4D0ULL),
               lg2 = bits2d(0x3FE62E42FEFA39EFULL), lg2_h = bits2d(0x3FE62E4300000000ULL),
               lg2_l = bits2d(0xBE205C610CA86C39ULL), ovt = 8.0085662595372944372e-17,
               cp = bits2d(0x3FEEC709DC3A03FDULL), cp_h = bits2d(0x3FEEC709E0000000ULL), cp_l = bits2d(0xBE3E2FE0145B01F5ULL),
               ivln2 = bits2d(0x3FF71547652B82FEULL), ivln2_h = bits2d(0x3FF7154760000000ULL),
               ivln2_l = bits2d(0x3E54AE0BF85DDF44ULL);
  int32_t hx = hi32(x), hy = hi32(y), ix = hx & 0x7fffffff, iy = hy & 0x7fffffff;
  uint32_t lx = lo32(x), ly = lo32(y);
  if ((iy | ly) == 0) return 1.0;
  double ax = fabs(x);
  if (lx == 0 && (ix == 0x7ff00000 || ix == 0 || ix == 0x3ff00000)) {
    double z = ax; if (hy < 0) z = 1.0 / z; return z;
  }
  double t1, t2;
  if (iy > 0x41e00000) {
    if (iy > 0x43f00000) {
      if (ix <= 0x3fefffff) return hy < 0 ? huge * huge : tiny * tiny;
      if (ix >= 0x3ff00000) return hy > 0 ? huge * huge : tiny * tiny;
    }
    if (ix < 0x3fefffff) return hy < 0 ? huge * huge : tiny * tiny;
    if (ix > 0x3ff00000) return hy > 0 ? huge * huge : tiny * tiny;
    double t = ax - 1.0;
    double w = (t * t) * (0.5 - t * (0.3333333333333333333333 - t * 0.25));
    double u = ivln2_h * t, v = t * ivln2_l - w * ivln2;
    t1 = with_lo(u + v, 0);
    t2 = v - (t1 - u);
  } else {
    int32_t n = 0, k;
    if (ix < 0x00100000) { ax *= two53; n -= 53; ix = hi32(ax); }
    n += (ix >> 20) - 0x3ff;
    int32_t j = ix & 0x000fffff;
    ix = j | 0x3ff00000;
    if (j <= 0x3988E) k = 0;
    else if (j < 0xBB67A) k = 1;
    else { k = 0; n += 1; ix -= 0x00100000; }
    ax = with_hi(ax, (uint32_t)ix);
    double u = ax - bp[k], v = 1.0 / (ax + bp[k]);
    double ss = u * v, s_h = with_lo(ss, 0);
    double t_h = bits2d((uint64_t)(uint32_t)(((ix >> 1) | 0x20000000) + 0x00080000 + (k << 18)) << 32);
    double t_l = ax - (t_h - bp[k]);
    double s_l = v * ((u - s_h * t_h) - s_h * t_l);
    double s2 = ss * ss;
    double r = s2 * s2 * (L1 + s2 * (L2 + s2 * (L3 + s2 * (L4 + s2 * (L5 + s2 * L6)))));
    r += s_l * (s_h + ss);
    s2 = s_h * s_h;
    t_h = with_lo(3.0 + s2 + r, 0);
    t_l = r - ((t_h - 3.0) - s2);
    u = s_h * t_h;
    v = s_l * t_h + t_l * ss;
    double p_h = with_lo(u + v, 0), p_l = v - (p_h - u);
    double z_h = cp_h * p_h, z_l = cp_l * p_h + p_l * cp + dp_l[k];
    double t = (double)n;
    t1 = with_lo(((z_h + z_l) + dp_h[k]) + t, 0);
    t2 = z_l - (((t1 - t) - dp_h[k]) - z_h);
  }
  double s = 1.0;
  double y1 = with_lo(y, 0);
  double p_l = (y - y1) * t1 + y * t2, p_h = y1 * t1, z = p_l + p_h;
  int32_t j = hi32(z), i = (int32_t)lo32(z);
  if (j >= 0x40900000) {
    if (((j - 0x40900000) | i) != 0) return s * huge * huge;
    if (p_l + ovt > z - p_h) return s * huge * huge;
  } else if ((j & 0x7fffffff) >= 0x4090cc00) {
    if (((j - (int32_t)0xc090cc00) | i) != 0) return s * tiny * tiny;
    if (p_l <= z - p_h) return s * tiny * tiny;
  }
  i = j & 0x7fffffff;
  int32_t k = (i >> 20) - 0x3ff, n = 0;
  if (i > 0x3fe00000) {
    n = j + (0x00100000 >> (k + 1));
    k = ((n & 0x7fffffff) >> 20) - 0x3ff;
    double t = bits2d((uint64_t)(uint32_t)(n & ~(0x000fffff >> k)) << 32);
    n = ((n & 0x000fffff) | 0x00100000) >> (20 - k);
    if (j < 0) n = -n;
    p_h -= t;
  }
  double t = with_lo(p_l + p_h, 0);
  double u = t * lg2_h, v = (p_l - (t - p_h)) * lg2 + t * lg2_l;
  z = u + v;
  double w = v - (z - u);
  t = z * z;
  t1 = z - t * (P1 + t * (P2 + t * (P3 + t * (P4 + t * P5))));
  double r = (z * t1) / (t1 - 2.0) - (w + z * w);
  z = 1.0 - (r - z);
  j = hi32(z);
  j += (n << 20);
  if ((j >> 20) <= 0) z = scalbn(z, n);
  else z = with_hi(z, (uint32_t)j);
  return s * z;
}

/* ---- elementwise pieces of layerForward ----------------------------------- */
/* infer.js:30-39: s accumulates v*v in double, sequentially from j = 0.  Rows
 * are independent; each row's sum runs serially on one thread. */
void orc_rmsnorm(const float* x, int rows, int C, const float* w, double eps, float* y) {
#pragma omp parallel for schedule(static) if ((int64_t)rows * C >= PAR_MIN)
  for (int r = 0; r < rows; r++) {
    const float* xr = x + (int64_t)r * C;
    double s = 0.0;
    for (int j = 0; j < C; j++) {
      double v = xr[j];
      s += v * v;
    }
    double inv = 1.0 / sqrt(s / (double)C + eps);
    for (int j = 0; j < C; j++) y[(int64_t)r * C + j] = (float)((double)xr[j] * inv * (double)w[j]);
  }
}

/* infer.js:71-81: f = p / theta^(2i/hd), tables stored f32; Math.pow, cos and
 * sin by the fdlibm method above. */
void orc_rope_tables(int hd, double theta, int maxT, float* cos_t, float* sin_t) {
  int half = hd >> 1;
  for (int p = 0; p < maxT; p++)
    for (int i = 0; i < half; i++) {
      double f = (double)p / orc_fdl_pow(theta, (2.0 * i) / (double)hd);
      cos_t[(int64_t)p * half + i] = (float)orc_fdl_cos(f);
      sin_t[(int64_t)p * half + i] = (float)orc_fdl_sin(f);
    }
}

/* infer.js:83-97: half-split rotation, products and sum in double, stored f32. */
void orc_apply_rope(float* x, int T, int nHeads, int hd, const float* cos_t, const float* sin_t, int pos0) {
  int half = hd >> 1, stride = nHeads * hd;
  for (int t = 0; t < T; t++) {
    int p = pos0 + t;
    for (int h = 0; h < nHeads; h++) {
      float* o = x + (int64_t)t * stride + h * hd;
      for (int i = 0; i < half; i++) {
        double c = cos_t[(int64_t)p * half + i], s = sin_t[(int64_t)p * half + i];
        double a = o[i], b = o[half + i];
        o[i] = (float)(a * c - b * s);
        o[half + i] = (float)(b * c + a * s);
      }
    }
  }
}

/* infer.js:182-194 for one head: causal softmax over columns oldest..see of
 * each row (oldest = 0, no sliding window); masked entries stay 0. */
void orc_softmax_causal(const float* scores, int T, int N, int n0, double scale, float* a) {
  for (int64_t i = 0; i < (int64_t)T * N; i++) a[i] = 0.0f;
  for (int i = 0; i < T; i++) {
    int see = n0 + i;
    double mx = -INFINITY;
    for (int j = 0; j <= see; j++) {
      double v = (double)scores[(int64_t)i * N + j] * scale;
      if (v > mx) mx = v;
    }
    double z = 0.0;
    for (int j = 0; j <= see; j++) {
      double e = orc_exp((double)scores[(int64_t)i * N + j] * scale - mx);
      a[(int64_t)i * N + j] = (float)e;
      z += e;
    }
    for (int j = 0; j <= see; j++) a[(int64_t)i * N + j] = (float)((double)a[(int64_t)i * N + j] / z);
  }
}

/* infer.js:59 + :212: f32(silu(g) * u), silu(v) = v / (1 + exp(-v)) in double. */
void orc_swiglu(const float* g, const float* u, int64_t n, float* out) {
#pragma omp parallel for schedule(static) if (n >= PAR_MIN)
  for (int64_t i = 0; i < n; i++) {
    double v = g[i];
    double s = v / (1.0 + orc_exp(-v));
    out[i] = (float)(s * (double)u[i]);
  }
}

/* ---- vgemmBlock (verified_core.js:425-449), batch 1 ------------------------ */
static int16_t g_mul[65536];
static int8_t g_requant[65536], g_relu[256];
static int g_luts_ready = 0;
static void luts_init(void) {
  if (!g_luts_ready) {
    orc_make_luts(g_mul, g_requant, g_relu);
    g_luts_ready = 1;
  }
}

typedef struct {
  int k, n;
  int8_t* q;  /* k x n row-major, as quantizeCols returns it (LUT path) */
  int8_t* qt; /* n x k: the same values transposed (exact-product path) */
  float* s;   /* n */
} orc_wq;

static int wq_build(orc_wq* w, const float* Wf, int k, int n) {
  w->k = k;
  w->n = n;
  w->qt = NULL;
  w->q = (int8_t*)malloc((size_t)k * n + 1);
  w->s = (float*)malloc(sizeof(float) * (size_t)n + 4);
  if (!w->q || !w->s) return ORC_E_NOMEM;
  return orc_quantize_cols(Wf, k, n, w->q, w->s);
}
static void wq_free(orc_wq* w) {
  free(w->q);
  free(w->qt);
  free(w->s);
  w->q = NULL;
  w->qt = NULL;
  w->s = NULL;
}

/* ---- the exact-product path (golden fixtures at full model size) ------------
 * bgemmJS adds mul-LUT entries in int32.  The mul unit is the exact product of
 * its two int8 indices (its sha256 equals the reference's LFS object id), and
 * k <= 131071 keeps every partial sum inside int32, so the accumulator is the
 * exact integer dot product whatever the order of its terms.  This path forms
 * that dot product directly, over a weight held transposed (n x k), with
 * AVX-512 where the CPU has it.  The quantisers and the epilogue are the
 * functions above, unchanged; tests check this path against the LUT path. */

/* quantizeCols (verified_core.js:122-136) writing qt = the quantised Wᵀ (cols x
 * rows).  Same arithmetic as orc_quantize_cols: absmax in double, f32 scale,
 * quotient by the f32-rounded scale. */
int orc_quantize_cols_t(const float* W, int64_t rows, int64_t cols, int8_t* qt, float* s) {
  if (orc_first_nonfinite(W, rows * cols) >= 0) return ORC_E_NONFINITE;
#pragma omp parallel for schedule(static) if (rows * cols >= PAR_MIN)
  for (int64_t cb = 0; cb < cols; cb += 256) {
    const int64_t ce = cb + 256 < cols ? cb + 256 : cols;
    double mx[256];
    for (int64_t c = cb; c < ce; c++) mx[c - cb] = 0.0;
    for (int64_t r = 0; r < rows; r++) {
      const float* wr = W + r * cols;
      for (int64_t c = cb; c < ce; c++) {
        double a = fabs((double)wr[c]);
        if (a > mx[c - cb]) mx[c - cb] = a;
      }
    }
    for (int64_t c = cb; c < ce; c++) {
      double sc = mx[c - cb] / 127.0;
      if (!(sc > 1e-8)) sc = 1e-8;
      s[c] = (float)sc;
    }
  }
  const int64_t nrb = (rows + 63) / 64, ncb = (cols + 63) / 64;
#pragma omp parallel for schedule(static) if (rows * cols >= PAR_MIN)
  for (int64_t t = 0; t < nrb * ncb; t++) {
    const int64_t r0 = (t % nrb) * 64, c0 = (t / nrb) * 64;
    const int64_t r1 = r0 + 64 < rows ? r0 + 64 : rows, c1 = c0 + 64 < cols ? c0 + 64 : cols;
    for (int64_t c = c0; c < c1; c++) {
      const double sc = (double)s[c];
      for (int64_t r = r0; r < r1; r++) qt[c * rows + r] = clamp8(js_round((double)W[r * cols + c] / sc));
    }
  }
  return ORC_OK;
}

static int cpu_avx512(void) {
#ifdef ORC_X86
  static int v = -1;
  if (v < 0) {
    __builtin_cpu_init();
    v = __builtin_cpu_supports("avx512f") && __builtin_cpu_supports("avx512bw") &&
        __builtin_cpu_supports("avx512vl");
  }
  return v;
#else
  return 0;
#endif
}

/* acc[i*n + j] = sum_p X16[i*kp + p] * Wt[j*k + p] for columns [j0, j1).  X16
 * is the activation widened to int16 and zero-padded to kp (a multiple of 32). */
static void idot_cols_generic(const int16_t* X16, int m, int kp, int k, const int8_t* Wt, int j0, int j1,
                              int32_t* acc, int n) {
  (void)kp;
  for (int j = j0; j < j1; j++) {
    const int8_t* w = Wt + (int64_t)j * k;
    for (int i = 0; i < m; i++) {
      const int16_t* x = X16 + (int64_t)i * kp;
      int32_t t = 0;
      for (int p = 0; p < k; p++) t += (int32_t)x[p] * (int32_t)w[p];
      acc[(int64_t)i * n + j] = t;
    }
  }
}

#ifdef ORC_X86
#define ORC_AVX512 __attribute__((target("avx512f,avx512bw,avx512vl")))
ORC_AVX512 static inline __m512i wload(const int8_t* p, int left) {
  const __mmask32 mk = left >= 32 ? (__mmask32)0xFFFFFFFFu : (__mmask32)((1u << left) - 1u);
  return _mm512_cvtepi8_epi16(_mm256_maskz_loadu_epi8(mk, p));
}
#define MADD(a, x, w) a = _mm512_add_epi32(a, _mm512_madd_epi16(x, w))
ORC_AVX512 static void idot_cols_avx512(const int16_t* X16, int m, int kp, int k, const int8_t* Wt, int j0, int j1,
                                        int32_t* acc, int n) {
  int j = j0;
  for (; j + 4 <= j1; j += 4) {
    const int8_t* w0 = Wt + (int64_t)j * k;
    const int8_t *w1 = w0 + k, *w2 = w1 + k, *w3 = w2 + k;
    int i = 0;
    for (; i + 4 <= m; i += 4) {
      const int16_t* x0 = X16 + (int64_t)i * kp;
      const int16_t *x1 = x0 + kp, *x2 = x1 + kp, *x3 = x2 + kp;
      __m512i a00 = _mm512_setzero_si512(), a01 = a00, a02 = a00, a03 = a00, a10 = a00, a11 = a00, a12 = a00,
              a13 = a00, a20 = a00, a21 = a00, a22 = a00, a23 = a00, a30 = a00, a31 = a00, a32 = a00, a33 = a00;
      for (int p = 0; p < k; p += 32) {
        const __m512i b0 = wload(w0 + p, k - p), b1 = wload(w1 + p, k - p), b2 = wload(w2 + p, k - p),
                      b3 = wload(w3 + p, k - p);
        __m512i x = _mm512_loadu_si512((const void*)(x0 + p));
        MADD(a00, x, b0); MADD(a01, x, b1); MADD(a02, x, b2); MADD(a03, x, b3);
        x = _mm512_loadu_si512((const void*)(x1 + p));
        MADD(a10, x, b0); MADD(a11, x, b1); MADD(a12, x, b2); MADD(a13, x, b3);
        x = _mm512_loadu_si512((const void*)(x2 + p));
        MADD(a20, x, b0); MADD(a21, x, b1); MADD(a22, x, b2); MADD(a23, x, b3);
        x = _mm512_loadu_si512((const void*)(x3 + p));
        MADD(a30, x, b0); MADD(a31, x, b1); MADD(a32, x, b2); MADD(a33, x, b3);
      }
      int32_t* o = acc + (int64_t)i * n + j;
      o[0] = _mm512_reduce_add_epi32(a00); o[1] = _mm512_reduce_add_epi32(a01);
      o[2] = _mm512_reduce_add_epi32(a02); o[3] = _mm512_reduce_add_epi32(a03);
      o += n;
      o[0] = _mm512_reduce_add_epi32(a10); o[1] = _mm512_reduce_add_epi32(a11);
      o[2] = _mm512_reduce_add_epi32(a12); o[3] = _mm512_reduce_add_epi32(a13);
      o += n;
      o[0] = _mm512_reduce_add_epi32(a20); o[1] = _mm512_reduce_add_epi32(a21);
      o[2] = _mm512_reduce_add_epi32(a22); o[3] = _mm512_reduce_add_epi32(a23);
      o += n;
      o[0] = _mm512_reduce_add_epi32(a30); o[1] = _mm512_reduce_add_epi32(a31);
      o[2] = _mm512_reduce_add_epi32(a32); o[3] = _mm512_reduce_add_epi32(a33);
    }
    for (; i < m; i++) {
      const int16_t* x0 = X16 + (int64_t)i * kp;
      __m512i a0 = _mm512_setzero_si512(), a1 = a0, a2 = a0, a3 = a0;
      for (int p = 0; p < k; p += 32) {
        const __m512i x = _mm512_loadu_si512((const void*)(x0 + p));
        MADD(a0, x, wload(w0 + p, k - p)); MADD(a1, x, wload(w1 + p, k - p));
        MADD(a2, x, wload(w2 + p, k - p)); MADD(a3, x, wload(w3 + p, k - p));
      }
      int32_t* o = acc + (int64_t)i * n + j;
      o[0] = _mm512_reduce_add_epi32(a0); o[1] = _mm512_reduce_add_epi32(a1);
      o[2] = _mm512_reduce_add_epi32(a2); o[3] = _mm512_reduce_add_epi32(a3);
    }
  }
  for (; j < j1; j++) {
    const int8_t* w0 = Wt + (int64_t)j * k;
    for (int i = 0; i < m; i++) {
      const int16_t* x0 = X16 + (int64_t)i * kp;
      __m512i a0 = _mm512_setzero_si512();
      for (int p = 0; p < k; p += 32) MADD(a0, _mm512_loadu_si512((const void*)(x0 + p)), wload(w0 + p, k - p));
      acc[(int64_t)i * n + j] = _mm512_reduce_add_epi32(a0);
    }
  }
}
#undef MADD
#endif

/* bgemmJS (batch 1) over a transposed weight Wt (n x k), exact products; the
 * output rules (f32 epilogue, ReLU, int32, declared requant) are orc_bgemm's. */
int orc_bgemm_t(const int8_t* Xq, const int8_t* Wt, const float* rs, const float* cs, int m, int k, int n,
                unsigned flags, void* out) {
  if (m < 0 || k < 0 || n < 0) return ORC_E_INVAL;
  if (orc_acc_bound(k)) return ORC_E_ACCBOUND;
  const int kp = ((k + 31) / 32) * 32;
  int16_t* X16 = (int16_t*)calloc((size_t)m * kp + 32, sizeof(int16_t));
  int32_t* acc = (flags & ORC_ACC) ? (int32_t*)out : (int32_t*)malloc(sizeof(int32_t) * ((size_t)m * n + 1));
  if (!X16 || !acc) { free(X16); if (!(flags & ORC_ACC)) free(acc); return ORC_E_NOMEM; }
  for (int64_t i = 0; i < m; i++)
    for (int64_t p = 0; p < k; p++) X16[i * kp + p] = Xq[i * k + p];
  const int simd = cpu_avx512();
  const int JB = 64;
  const int nb = (n + JB - 1) / JB;
  const int64_t work = (int64_t)m * k * n;
#pragma omp parallel for schedule(dynamic, 1) if (work >= PAR_MIN)
  for (int b = 0; b < nb; b++) {
    const int j0 = b * JB, j1 = j0 + JB < n ? j0 + JB : n;
#ifdef ORC_X86
    if (simd) { idot_cols_avx512(X16, m, kp, k, Wt, j0, j1, acc, n); continue; }
#endif
    idot_cols_generic(X16, m, kp, k, Wt, j0, j1, acc, n);
  }
  (void)simd;
  if (!(flags & ORC_ACC)) {
    luts_init();
    for (int64_t i = 0; i < m; i++)
      for (int64_t j = 0; j < n; j++) {
        const int32_t a = acc[i * n + j];
        if (flags & ORC_REQUANT) {
          const int32_t c = a < -32768 ? -32768 : a > 32767 ? 32767 : a;
          int8_t v = g_requant[(uint16_t)(int16_t)c];
          if (flags & ORC_RELU) v = g_relu[(uint8_t)v];
          ((int8_t*)out)[i * n + j] = v;
        } else {
          const float v = orc_epi(a, rs[i], cs[j]);
          ((float*)out)[i * n + j] = ((flags & ORC_RELU) && v < 0.0f) ? 0.0f : v;
        }
      }
    free(acc);
  }
  free(X16);
  return ORC_OK;
}

/* qt built directly (the model's exact-product path keeps no k x n copy). */
static int wq_build_t(orc_wq* w, const float* Wf, int k, int n) {
  w->k = k;
  w->n = n;
  w->q = NULL;
  w->qt = (int8_t*)malloc((size_t)k * n + 1);
  w->s = (float*)malloc(sizeof(float) * (size_t)n + 4);
  if (!w->qt || !w->s) return ORC_E_NOMEM;
  return orc_quantize_cols_t(Wf, k, n, w->qt, w->s);
}

/* X (m x k f32) times a quantised weight -> out (m x n f32). */
static int vgemm_wq(const float* X, int m, const orc_wq* w, float* out) {
  luts_init();
  int k = w->k, n = w->n;
  int8_t* xq = (int8_t*)malloc((size_t)m * k + 1);
  float* rs = (float*)malloc(sizeof(float) * (size_t)m + 4);
  if (!xq || !rs) { free(xq); free(rs); return ORC_E_NOMEM; }
  int rc = orc_quantize_rows(X, m, k, xq, rs);
  if (rc == ORC_OK)
    rc = w->qt ? orc_bgemm_t(xq, w->qt, rs, w->s, m, k, n, 0, out)
               : orc_bgemm(xq, w->q, rs, w->s, m, k, n, 1, 0, g_mul, g_requant, g_relu, out);
  free(xq);
  free(rs);
  return rc;
}
/* The full per-call vgemmBlock: both operands quantised on every call. */
int orc_vgemm(const float* X, const float* Wf, int m, int k, int n, float* out) {
  orc_wq w;
  int rc = wq_build(&w, Wf, k, n);
  if (rc == ORC_OK) rc = vgemm_wq(X, m, &w, out);
  wq_free(&w);
  return rc;
}
/* The same per-call vgemmBlock through the exact-product path. */
static int vgemm_fast(const float* X, const float* Wf, int m, int k, int n, float* out) {
  orc_wq w;
  int rc = wq_build_t(&w, Wf, k, n);
  if (rc == ORC_OK) rc = vgemm_wq(X, m, &w, out);
  wq_free(&w);
  return rc;
}

/* ---- model ------------------------------------------------------------------ */
typedef struct {
  const float *nrm1, *nrm2, *Wq, *Wk, *Wv, *Wo, *Wgate, *Wup, *Wdown; /* k x n f32 */
  orc_wq q, k, v, o, gate, up, down;
  int quantized;
} orc_layer;

typedef struct orc_model {
  int hidden, layers, heads, kv_heads, head_dim, inter, vocab;
  double eps, theta;
  const float* emb;  /* vocab x hidden */
  const float* nrmF; /* hidden */
  float* lm_kn;      /* hidden x vocab f32 (own copy; embᵀ when tied) */
  orc_wq lm;
  int lm_quantized;
  orc_layer* L;
  int per_call_quant; /* 1: re-quantise weights on every GEMM, as vgemmBlock does */
  int fast;           /* 1: the exact-product path, weights held transposed */
  float *rope_cos, *rope_sin;
  int rope_max;
  float* own_ones;    /* synthetic models: the norm weights (all 1) */
  float* own_emb;     /* synthetic models: the embedding */
} orc_model;

typedef struct {
  int n, max_pos, kv_dim;
  float *k, *v;
} orc_kv_layer;
typedef struct orc_kv {
  int lo, hi;
  orc_kv_layer* L;
} orc_kv;

orc_model* orc_model_new(int hidden, int layers, int heads, int kv_heads, int head_dim, int inter, int vocab,
                         double eps, double theta) {
  if (hidden <= 0 || layers < 0 || heads <= 0 || kv_heads <= 0 || heads % kv_heads || head_dim <= 0 ||
      (head_dim & 1) || inter <= 0 || vocab <= 0)
    return NULL;
  orc_model* m = (orc_model*)calloc(1, sizeof(orc_model));
  if (!m) return NULL;
  m->hidden = hidden; m->layers = layers; m->heads = heads; m->kv_heads = kv_heads;
  m->head_dim = head_dim; m->inter = inter; m->vocab = vocab; m->eps = eps; m->theta = theta;
  m->L = (orc_layer*)calloc((size_t)(layers > 0 ? layers : 1), sizeof(orc_layer));
  return m;
}

void orc_model_free(orc_model* m) {
  if (!m) return;
  for (int l = 0; l < m->layers; l++) {
    orc_layer* y = &m->L[l];
    if (y->quantized) {
      wq_free(&y->q); wq_free(&y->k); wq_free(&y->v); wq_free(&y->o);
      wq_free(&y->gate); wq_free(&y->up); wq_free(&y->down);
    }
  }
  if (m->lm_quantized) wq_free(&m->lm);
  free(m->lm_kn);
  free(m->L);
  free(m->rope_cos);
  free(m->rope_sin);
  free(m->own_ones);
  free(m->own_emb);
  free(m);
}

void orc_model_set_per_call_quant(orc_model* m, int on) { m->per_call_quant = on; }
/* Weights quantised from now on go through the exact-product path. */
void orc_model_set_fast(orc_model* m, int on) { m->fast = on; }

/* Head tensors.  lm_kn == NULL means tied: lm_head = embᵀ (shard.js:92, 123-128). */
int orc_model_set_head(orc_model* m, const float* emb, const float* nrmF, const float* lm_kn) {
  int C = m->hidden, V = m->vocab;
  m->emb = emb;
  m->nrmF = nrmF;
  free(m->lm_kn);
  m->lm_kn = (float*)malloc(sizeof(float) * (size_t)C * V);
  if (!m->lm_kn) return ORC_E_NOMEM;
  if (lm_kn) memcpy(m->lm_kn, lm_kn, sizeof(float) * (size_t)C * V);
  else
    for (int v = 0; v < V; v++)
      for (int c = 0; c < C; c++) m->lm_kn[(int64_t)c * V + v] = emb[(int64_t)v * C + c];
  if (m->lm_quantized) wq_free(&m->lm);
  m->lm_quantized = 0;
  return ORC_OK;
}

int orc_model_set_layer(orc_model* m, int l, const float* nrm1, const float* nrm2, const float* Wq, const float* Wk,
                        const float* Wv, const float* Wo, const float* Wgate, const float* Wup, const float* Wdown) {
  if (l < 0 || l >= m->layers) return ORC_E_INVAL;
  orc_layer* y = &m->L[l];
  y->nrm1 = nrm1; y->nrm2 = nrm2; y->Wq = Wq; y->Wk = Wk; y->Wv = Wv; y->Wo = Wo;
  y->Wgate = Wgate; y->Wup = Wup; y->Wdown = Wdown;
  return ORC_OK;
}

/* Weight quantisation is deterministic, so quantising once and reusing the
 * result is bit-identical to vgemmBlock's per-call quantizeCols. */
static int layer_quantize(orc_model* m, orc_layer* y) {
  if (y->quantized) return ORC_OK;
  int C = m->hidden, q = m->heads * m->head_dim, kv = m->kv_heads * m->head_dim, I = m->inter;
  int rc = ORC_OK;
  int (*build)(orc_wq*, const float*, int, int) = m->fast ? wq_build_t : wq_build;
  rc |= build(&y->q, y->Wq, C, q);
  rc |= build(&y->k, y->Wk, C, kv);
  rc |= build(&y->v, y->Wv, C, kv);
  rc |= build(&y->o, y->Wo, q, C);
  rc |= build(&y->gate, y->Wgate, C, I);
  rc |= build(&y->up, y->Wup, C, I);
  rc |= build(&y->down, y->Wdown, I, C);
  y->quantized = 1;
  return rc ? ORC_E_NONFINITE : ORC_OK;
}

static int proj(orc_model* m, const float* X, int T, const float* Wf, const orc_wq* w, int k, int n, float* out) {
  if (m->per_call_quant) return orc_vgemm(X, Wf, T, k, n, out);
  (void)k; (void)n;
  return vgemm_wq(X, T, w, out);
}

static int rope_ensure(orc_model* m, int need) {
  if (m->rope_max >= need) return ORC_OK;
  int half = m->head_dim >> 1;
  free(m->rope_cos);
  free(m->rope_sin);
  m->rope_cos = (float*)malloc(sizeof(float) * (size_t)need * half + 4);
  m->rope_sin = (float*)malloc(sizeof(float) * (size_t)need * half + 4);
  if (!m->rope_cos || !m->rope_sin) return ORC_E_NOMEM;
  orc_rope_tables(m->head_dim, m->theta, need, m->rope_cos, m->rope_sin);
  m->rope_max = need;
  return ORC_OK;
}

orc_kv* orc_kv_new(orc_model* m, int lo, int hi, int max_pos) {
  if (lo < 0 || hi > m->layers || hi < lo || max_pos < 1) return NULL;
  orc_kv* c = (orc_kv*)calloc(1, sizeof(orc_kv));
  if (!c) return NULL;
  c->lo = lo; c->hi = hi;
  c->L = (orc_kv_layer*)calloc((size_t)(hi - lo + 1), sizeof(orc_kv_layer));
  int kvd = m->kv_heads * m->head_dim;
  for (int l = 0; l < hi - lo; l++) {
    c->L[l].max_pos = max_pos;
    c->L[l].kv_dim = kvd;
    c->L[l].k = (float*)malloc(sizeof(float) * (size_t)max_pos * kvd);
    c->L[l].v = (float*)malloc(sizeof(float) * (size_t)max_pos * kvd);
  }
  return c;
}
void orc_kv_free(orc_kv* c) {
  if (!c) return;
  for (int l = 0; l < c->hi - c->lo; l++) { free(c->L[l].k); free(c->L[l].v); }
  free(c->L);
  free(c);
}
int orc_kv_len(const orc_kv* c, int layer) { return c->L[layer - c->lo].n; }
void orc_kv_read(const orc_kv* c, int layer, float* k, float* v) {
  const orc_kv_layer* y = &c->L[layer - c->lo];
  memcpy(k, y->k, sizeof(float) * (size_t)y->n * y->kv_dim);
  memcpy(v, y->v, sizeof(float) * (size_t)y->n * y->kv_dim);
}

/* One head of infer.js:171-197: the scores vgemmBlock (q_h x k_hᵀ), the causal
 * softmax and the context vgemmBlock (a x v_h), written into the head's
 * columns of ctxOut.  The buffers are the head's own, so heads may run on
 * separate threads. */
static int attn_head(int fast, int h, int group, const float* q, int qDim, const float* K, const float* Vv,
                     int kvDim, int T, int N, int n0, int hd, double scale, float* ctxOut) {
  int rc = ORC_OK;
  const int kvh = h / group;
  float* qh = (float*)malloc(sizeof(float) * (size_t)T * hd);
  float* khT = (float*)malloc(sizeof(float) * (size_t)hd * N);
  float* vh = (float*)malloc(sizeof(float) * (size_t)N * hd);
  float* scores = (float*)malloc(sizeof(float) * (size_t)T * N);
  float* a = (float*)malloc(sizeof(float) * (size_t)T * N);
  float* oh = (float*)malloc(sizeof(float) * (size_t)T * hd);
  int (*vg)(const float*, const float*, int, int, int, float*) = fast ? vgemm_fast : orc_vgemm;
  if (!qh || !khT || !vh || !scores || !a || !oh) { rc = ORC_E_NOMEM; goto out; }
  for (int t = 0; t < T; t++) memcpy(qh + (int64_t)t * hd, q + (int64_t)t * qDim + h * hd, sizeof(float) * hd);
  for (int t = 0; t < N; t++)
    for (int c = 0; c < hd; c++) {
      khT[(int64_t)c * N + t] = K[(int64_t)t * kvDim + kvh * hd + c];
      vh[(int64_t)t * hd + c] = Vv[(int64_t)t * kvDim + kvh * hd + c];
    }
  if ((rc = vg(qh, khT, T, hd, N, scores))) goto out;
  orc_softmax_causal(scores, T, N, n0, scale, a);
  if ((rc = vg(a, vh, T, N, hd, oh))) goto out;
  for (int t = 0; t < T; t++) memcpy(ctxOut + (int64_t)t * qDim + h * hd, oh + (int64_t)t * hd, sizeof(float) * hd);
out:
  free(qh); free(khT); free(vh); free(scores); free(a); free(oh);
  return rc;
}

/* infer.js:114-221, Llama block.  kvl == NULL is the full-window path. */
static int layer_forward(orc_model* m, int li, float* x, int T, orc_kv_layer* kvl, int pos0) {
  orc_layer* y = &m->L[li];
  int rc = ORC_OK;
  if (!m->per_call_quant && (rc = layer_quantize(m, y))) return rc;
  const int C = m->hidden, hd = m->head_dim, nH = m->heads, nKV = m->kv_heads;
  const int qDim = nH * hd, kvDim = nKV * hd, I = m->inter;
  float* h1 = (float*)malloc(sizeof(float) * (size_t)T * C);
  float* q = (float*)malloc(sizeof(float) * (size_t)T * qDim);
  float* k = (float*)malloc(sizeof(float) * (size_t)T * kvDim);
  float* v = (float*)malloc(sizeof(float) * (size_t)T * kvDim);
  float* ctxOut = (float*)calloc((size_t)T * qDim, sizeof(float));
  float* x2 = (float*)malloc(sizeof(float) * (size_t)T * C);
  float* g = (float*)malloc(sizeof(float) * (size_t)T * I);
  float* u = (float*)malloc(sizeof(float) * (size_t)T * I);
  float* tmpC = (float*)malloc(sizeof(float) * (size_t)T * C);
  if (!h1 || !q || !k || !v || !ctxOut || !x2 || !g || !u || !tmpC) { rc = ORC_E_NOMEM; goto done; }

  orc_rmsnorm(x, T, C, y->nrm1, m->eps, h1);
  if ((rc = proj(m, h1, T, y->Wq, &y->q, C, qDim, q))) goto done;
  if ((rc = proj(m, h1, T, y->Wk, &y->k, C, kvDim, k))) goto done;
  if ((rc = proj(m, h1, T, y->Wv, &y->v, C, kvDim, v))) goto done;
  if ((rc = rope_ensure(m, pos0 + T + 1))) goto done;
  orc_apply_rope(q, T, nH, hd, m->rope_cos, m->rope_sin, pos0);
  orc_apply_rope(k, T, nKV, hd, m->rope_cos, m->rope_sin, pos0);

  int n0 = 0, N = T;
  const float *K = k, *Vv = v;
  if (kvl) {
    n0 = kvl->n;
    N = n0 + T;
    if (N > kvl->max_pos) { rc = ORC_E_INVAL; goto done; }
    memcpy(kvl->k + (int64_t)n0 * kvDim, k, sizeof(float) * (size_t)T * kvDim);
    memcpy(kvl->v + (int64_t)n0 * kvDim, v, sizeof(float) * (size_t)T * kvDim);
    kvl->n = N;
    K = kvl->k;
    Vv = kvl->v;
  }
  const int group = nH / nKV;
  const double scale = 1.0 / sqrt((double)hd);
  if (m->fast) {
    /* heads are independent: one head per task, each with its own buffers */
    int* hrc = (int*)calloc((size_t)nH, sizeof(int));
    if (!hrc) { rc = ORC_E_NOMEM; goto done; }
#pragma omp parallel for schedule(dynamic, 1)
    for (int h = 0; h < nH; h++)
      hrc[h] = attn_head(1, h, group, q, qDim, K, Vv, kvDim, T, N, n0, hd, scale, ctxOut);
    for (int h = 0; h < nH && !rc; h++) rc = hrc[h];
    free(hrc);
    if (rc) goto done;
  } else {
    for (int h = 0; h < nH; h++)
      if ((rc = attn_head(0, h, group, q, qDim, K, Vv, kvDim, T, N, n0, hd, scale, ctxOut))) goto done;
  }
  if ((rc = proj(m, ctxOut, T, y->Wo, &y->o, qDim, C, tmpC))) goto done;
  for (int64_t i = 0; i < (int64_t)T * C; i++) x2[i] = x[i] + tmpC[i];
  orc_rmsnorm(x2, T, C, y->nrm2, m->eps, h1);
  if ((rc = proj(m, h1, T, y->Wgate, &y->gate, C, I, g))) goto done;
  if ((rc = proj(m, h1, T, y->Wup, &y->up, C, I, u))) goto done;
  orc_swiglu(g, u, (int64_t)T * I, g);
  if ((rc = proj(m, g, T, y->Wdown, &y->down, I, C, tmpC))) goto done;
  for (int64_t i = 0; i < (int64_t)T * C; i++) x[i] = x2[i] + tmpC[i];
done:
  free(h1); free(q); free(k); free(v); free(ctxOut); free(x2); free(g); free(u); free(tmpC);
  return rc;
}

/* runLayers / runLayersChunk (infer.js:275-296): layers [lo, hi) in place on x
 * (T x hidden).  kv == NULL runs the full-window path. */
int orc_run_layers(orc_model* m, int lo, int hi, float* x, int T, orc_kv* kv, int pos0) {
  if (lo < 0 || hi > m->layers || hi < lo || T < 1) return ORC_E_INVAL;
  if (orc_first_nonfinite(x, (int64_t)T * m->hidden) >= 0) return ORC_E_NONFINITE;
  for (int l = lo; l < hi; l++) {
    orc_kv_layer* kvl = NULL;
    if (kv) {
      if (l < kv->lo || l >= kv->hi) return ORC_E_INVAL;
      kvl = &kv->L[l - kv->lo];
    }
    int rc = layer_forward(m, l, x, T, kvl, pos0);
    if (rc) return rc;
  }
  if (orc_first_nonfinite(x, (int64_t)T * m->hidden) >= 0) return ORC_E_NONFINITE;
  return ORC_OK;
}

/* embedRows (infer.js:298-310), Llama family (no learned positions). */
void orc_embed_rows(const orc_model* m, const int32_t* ids, int T, float* x) {
  for (int i = 0; i < T; i++)
    memcpy(x + (int64_t)i * m->hidden, m->emb + (int64_t)ids[i] * m->hidden, sizeof(float) * m->hidden);
}

/* logitsAt (infer.js:324-334): final RMSNorm over all T rows, then one M=1
 * verified GEMM per requested row against lm_head. */
int orc_logits_rows(orc_model* m, const float* x, int T, const int32_t* rows, int nrows, float* out) {
  int C = m->hidden, V = m->vocab;
  if (!m->lm_kn && !m->lm_quantized) return ORC_E_INVAL;
  if (!m->per_call_quant && !m->lm_quantized) {
    if ((m->fast ? wq_build_t : wq_build)(&m->lm, m->lm_kn, C, V)) return ORC_E_NONFINITE;
    m->lm_quantized = 1;
  }
  float* y = (float*)malloc(sizeof(float) * (size_t)T * C);
  if (!y) return ORC_E_NOMEM;
  orc_rmsnorm(x, T, C, m->nrmF, m->eps, y);
  int rc = ORC_OK;
  for (int r = 0; r < nrows && rc == ORC_OK; r++) {
    if (rows[r] < 0 || rows[r] >= T) { rc = ORC_E_INVAL; break; }
    rc = proj(m, y + (int64_t)rows[r] * C, 1, m->lm_kn, &m->lm, C, V, out + (int64_t)r * V);
  }
  free(y);
  return rc;
}

/* pickToken greedy (infer.js:393-395): strict '>' so the first maximum wins. */
int orc_argmax(const float* logits, int n) {
  int best = 0;
  float bv = -INFINITY;
  for (int j = 0; j < n; j++)
    if (logits[j] > bv) { bv = logits[j]; best = j; }
  return best;
}

/* ---- hashes, probes and fixtures ------------------------------------------ */
/* shard.js:195-200 */
uint32_t orc_fnv1a(const uint8_t* b, int64_t n) {
  uint32_t h = 0x811c9dc5u;
  for (int64_t i = 0; i < n; i++) { h ^= b[i]; h *= 0x01000193u; }
  return h;
}

/* webgpu.js:998-1009: LCG seeded 0x5EED, m=24 k=96 n=24 batch=2, rs = cs = 1. */
void orc_probe_inputs(int8_t* Xq, int8_t* Wq) {
  uint32_t seed = 0x5EED;
  const int nx = 2 * 24 * 96, nw = 2 * 96 * 24;
  for (int i = 0; i < nx + nw; i++) {
    seed = (seed * 1103515245u + 12345u) & 0x7fffffffu;
    double r = (double)seed / (double)0x7fffffff;
    int8_t v = (int8_t)js_round(r * 254.0 - 127.0);
    if (i < nx) Xq[i] = v; else Wq[i - nx] = v;
  }
}

/* test_pipeline.js:32-37: mulberry32(seed), o[i] = f32((r*2 - 1) * scale). */
void orc_mulberry_fill(uint32_t seed, int64_t n, double scale, float* out) {
  uint32_t a = seed;
  for (int64_t i = 0; i < n; i++) {
    a = a + 0x6D2B79F5u;
    uint32_t t = (a ^ (a >> 15)) * (1u | a);
    t = (t + ((t ^ (t >> 7)) * (61u | t))) ^ t;
    double r = (double)(t ^ (t >> 14)) / 4294967296.0;
    out[i] = (float)((r * 2.0 - 1.0) * scale);
  }
}

/* Synthetic random-init weights for the benchmark-size models.  Counter based,
 * so any element can be produced independently (the CUDA model builder uses
 * the same formula): four splitmix64 outputs are summed as 32-bit integers
 * (Irwin-Hall, an approximately normal variable), centred exactly in int64
 * and scaled once in double, then rounded to f32.  Every step is exact or
 * correctly rounded, so CPU and GPU agree bit for bit. */
static uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
  return z ^ (z >> 31);
}
void orc_synth_fill(uint64_t seed, int64_t start, int64_t n, double factor, float* out) {
#pragma omp parallel for schedule(static) if (n >= PAR_MIN)
  for (int64_t i = 0; i < n; i++) {
    uint64_t base = (seed * 0x9E3779B97F4A7C15ULL) + (uint64_t)(start + i) * 4u;
    int64_t s = 0;
    for (int j = 0; j < 4; j++) s += (int64_t)(mix64(base + (uint64_t)j) >> 32);
    s -= (int64_t)2 * 4294967295LL;
    out[i] = (float)((double)s * factor);
  }
}

/* A synthetic benchmark model built in place, through the exact-product path:
 * every weight of layers [lo, hi) (and, with head, the embedding and lm_head)
 * is generated by orc_synth_fill, quantised once (quantizeCols, kept
 * transposed) and its f32 copy dropped, so a Llama-3-8B-sized model needs
 * ~8 GB here instead of ~32 GB.  Tensor seed = model_seed * 1000003 +
 * (layer + 1) * 64 + role; roles emb 1, lm 2, Wq 3, Wk 4, Wv 5, Wo 6,
 * Wgate 7, Wup 8, Wdown 9; norm weights are 1.  tie: lm_head = embᵀ. */
static int synth_wq(uint64_t model_seed, int layer, int role, int k, int n, double factor, orc_wq* w) {
  float* f = (float*)malloc(sizeof(float) * (size_t)k * n + 4);
  if (!f) return ORC_E_NOMEM;
  orc_synth_fill(model_seed * 1000003ULL + (uint64_t)(layer + 1) * 64u + (uint64_t)role, 0, (int64_t)k * n, factor,
                 f);
  int rc = wq_build_t(w, f, k, n);
  free(f);
  return rc;
}

int orc_model_synth(orc_model* m, uint64_t model_seed, double factor, int tie, int lo, int hi, int head) {
  if (lo < 0 || hi > m->layers || hi < lo) return ORC_E_INVAL;
  const int C = m->hidden, q = m->heads * m->head_dim, kv = m->kv_heads * m->head_dim, I = m->inter, V = m->vocab;
  m->fast = 1;
  m->per_call_quant = 0;
  if (!m->own_ones) {
    m->own_ones = (float*)malloc(sizeof(float) * (size_t)C);
    if (!m->own_ones) return ORC_E_NOMEM;
    for (int i = 0; i < C; i++) m->own_ones[i] = 1.0f;
  }
  int rc = ORC_OK;
  for (int l = lo; l < hi && !rc; l++) {
    orc_layer* y = &m->L[l];
    if (y->quantized) continue;
    y->nrm1 = y->nrm2 = m->own_ones;
    y->Wq = y->Wk = y->Wv = y->Wo = y->Wgate = y->Wup = y->Wdown = NULL;
    rc |= synth_wq(model_seed, l, 3, C, q, factor, &y->q);
    rc |= synth_wq(model_seed, l, 4, C, kv, factor, &y->k);
    rc |= synth_wq(model_seed, l, 5, C, kv, factor, &y->v);
    rc |= synth_wq(model_seed, l, 6, q, C, factor, &y->o);
    rc |= synth_wq(model_seed, l, 7, C, I, factor, &y->gate);
    rc |= synth_wq(model_seed, l, 8, C, I, factor, &y->up);
    rc |= synth_wq(model_seed, l, 9, I, C, factor, &y->down);
    y->quantized = 1;
  }
  if (rc || !head) return rc ? ORC_E_NOMEM : ORC_OK;
  free(m->own_emb);
  m->own_emb = (float*)malloc(sizeof(float) * (size_t)V * C);
  if (!m->own_emb) return ORC_E_NOMEM;
  orc_synth_fill(model_seed * 1000003ULL + 1u, 0, (int64_t)V * C, factor, m->own_emb);
  m->emb = m->own_emb;
  m->nrmF = m->own_ones;
  free(m->lm_kn);
  m->lm_kn = NULL;
  if (m->lm_quantized) wq_free(&m->lm);
  m->lm_quantized = 0;
  if (tie) {
    float* t = (float*)malloc(sizeof(float) * (size_t)C * V);
    if (!t) return ORC_E_NOMEM;
#pragma omp parallel for schedule(static)
    for (int64_t c = 0; c < C; c++)
      for (int64_t v = 0; v < V; v++) t[c * V + v] = m->own_emb[v * C + c];
    rc = wq_build_t(&m->lm, t, C, V);
    free(t);
  } else {
    rc = synth_wq(model_seed, -1, 2, C, V, factor, &m->lm);
  }
  if (rc) return rc;
  m->lm_quantized = 1;
  return ORC_OK;
}
