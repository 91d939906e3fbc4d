// dc_osum.cuh -- the reference's serial f64 sums, computed by a whole block.
//
// RMSNorm's sum of squares (infer.js:73-76: `s += v * v`, j = 0..C-1) and the
// softmax denominator (infer.js:100-104: `z += e`, keys in order) are chains of
// rounded double additions.  A single thread replays such a chain at the add
// latency (thousands of dependent adds per row); this file gets the identical
// result from all threads of the block, using the structure of a sum of
// non-negative terms:
//
// * the running sum never decreases, so it leaves each binade [2^E, 2^(E+1))
//   once.  While it stays inside one binade every representable value there
//   is a multiple of u = 2^(E-52); with the sum written as A*u (A an integer
//   below 2^53), `acc + t` is (A + RN(t/u))*u when t/u is not a half-integer,
//   and when t/u = k + 1/2 the tie goes to the even neighbour: the new A is
//   A + k rounded up to even.  Each term is thus one of two integer maps,
//   A -> A + r or A -> roundup_even(A + k), and the family
//   {A -> A + c} u {A -> roundup_even(A + c1) + c2} is closed under
//   composition, so the terms of a stretch compose in parallel (a scan);
// * where the binade may change (predicted from an approximate prefix sum in
//   any order, with a 2^-36 relative margin) and at term 0 the term is made
//   explicit: one thread applies it with a real __dadd_rn step, then applies
//   the composed map of the stretch that follows it.
//
// Every stretch is checked on that chain -- its terms must have been rounded
// in the binade the running sum actually has, and A must stay below 2^53 --
// and a failed check (or more explicit terms than fit, or a negative or
// non-finite term) sends the row to the plain serial loop.  The result is
// therefore always the serial chain's, bit for bit; the parallel path only
// changes how long it takes.
#pragma once
#include <stdint.h>

#include <climits>

namespace dco {

constexpr int MAXSEG = 96;                     // explicit terms per row (else serial)
constexpr double DELTA = 1.0 / 68719476736.0;  // 2^-36 margin around binade edges
constexpr unsigned long long CAP = 1ull << 54; // saturation of the composed constants

// A -> t ? roundup_even(A + c1) + c2 : A + c2
struct Fn {
  unsigned long long c1, c2;
  int t;
};

struct Smem {
  unsigned long long c1[MAXSEG], c2[MAXSEG];  // composed map of stretch s (after explicit term s)
  int ft[MAXSEG];
  int expl[MAXSEG];                           // index of explicit term s
  int emin[MAXSEG], emax[MAXSEG];             // binades its terms were rounded in (must agree)
  unsigned long long wc1[32], wc2[32];
  int wt[32], wr[32];
  double wtot[32];
  int wcnt[32];
  int wbad[32];
  int nseg;
  double tv[MAXSEG];                           // value of explicit term s
  double result;
};

__device__ __forceinline__ unsigned long long sat(unsigned long long x) { return x < CAP ? x : CAP; }

// f, then g
__device__ __forceinline__ Fn then(const Fn& f, const Fn& g) {
  Fn h;
  if (!g.t) {
    h.t = f.t;
    h.c1 = f.c1;
    h.c2 = sat(f.c2 + g.c2);
  } else if (!f.t) {
    h.t = 1;
    h.c1 = sat(f.c2 + g.c1);
    h.c2 = g.c2;
  } else {  // roundup_even(2m + f.c2 + g.c1) = 2m + roundup_even(f.c2 + g.c1), 2m even
    h.t = 1;
    h.c1 = f.c1;
    h.c2 = sat(((f.c2 + g.c1 + 1ull) & ~1ull) + g.c2);
  }
  return h;
}

__device__ __forceinline__ unsigned long long apply(int t, unsigned long long c1, unsigned long long c2,
                                                    unsigned long long A) {
  return t ? sat(((A + c1 + 1ull) & ~1ull) + c2) : sat(A + c2);
}

// E of the binade holding x >= 0, with subnormals (and 0) in the first normal
// binade: both have spacing 2^-1074.
__device__ __forceinline__ int binade(double x) {
  const int f = (int)((unsigned long long)__double_as_longlong(x) >> 52) & 0x7ff;
  return (f ? f : 1) - 1023;
}

// t >= 0 over u = 2^(E-52): r = RN(t/u) with a half-integer reported as a tie
// (r then holds its floor).  t/u >= 2^53 only happens for a term that moves
// the sum out of the binade, which is explicit; r then saturates and the
// stretch check fails.
__device__ __forceinline__ void units(double t, int E, unsigned long long& r, bool& tie) {
  constexpr double MAGIC = 6755399441055744.0;  // 1.5 * 2^52: MAGIC + q lands on an integer grid
  if (E > -900) {
    // q = t * 2^(52-E) is exact (a power-of-two scale that neither overflows
    // nor loses bits, except for q far below 1/2 where only r = 0 matters)
    const double q = __dmul_rn(t, __longlong_as_double((long long)(1075 - E) << 52));
    if (q < 2251799813685248.0) {  // q < 2^51: RN-even(q) from the grid, d = q - RN-even(q)
      const double y = __dadd_rn(q, MAGIC);
      const double d = __dsub_rn(q, __dsub_rn(y, MAGIC));
      const unsigned long long rne = ((unsigned long long)__double_as_longlong(y) & 0xFFFFFFFFFFFFFull) - (1ull << 51);
      tie = d == 0.5 || d == -0.5;
      r = rne - (d < 0.0 && tie ? 1ull : 0ull);  // a tie keeps its floor
      return;
    }
    const double fl = floor(q);
    const double fr = __dsub_rn(q, fl);
    tie = fr == 0.5;
    r = fl < 18014398509481984.0 ? (unsigned long long)fl + (fr > 0.5 ? 1ull : 0ull) : CAP;
    return;
  }
  const unsigned long long b = (unsigned long long)__double_as_longlong(t);
  const int f = (int)(b >> 52) & 0x7ff;
  const unsigned long long M = (b & 0xFFFFFFFFFFFFFull) | (f ? (1ull << 52) : 0ull);
  const int et = (f ? f : 1) - 1075;  // t = M * 2^et
  const int d = (E - 52) - et;
  tie = false;
  if (d < 0) {
    r = M ? CAP : 0ull;
  } else if (d == 0) {
    r = M;
  } else if (d < 64) {
    const unsigned long long rem = M & ((1ull << d) - 1), half = 1ull << (d - 1);
    r = (M >> d) + (rem > half ? 1ull : 0ull);
    tie = rem == half;
  } else {
    r = 0;
  }
}

template <typename T>
__device__ __forceinline__ T warp_incl(T v, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const T y = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += y;
  }
  return v;
}

// Segmented composition: (reset, f) then (reset', g) = reset' ? (1, g) : (reset, f then g).
struct SegFn {
  Fn f;
  int reset;
};
__device__ __forceinline__ SegFn seg_then(const SegFn& a, const SegFn& b) {
  if (b.reset) return b;
  SegFn c;
  c.reset = a.reset;
  c.f = then(a.f, b.f);
  return c;
}
__device__ __forceinline__ SegFn shfl_up_seg(const SegFn& v, int o) {
  SegFn r;
  r.f.c1 = __shfl_up_sync(0xffffffffu, v.f.c1, o);
  r.f.c2 = __shfl_up_sync(0xffffffffu, v.f.c2, o);
  r.f.t = __shfl_up_sync(0xffffffffu, v.f.t, o);
  r.reset = __shfl_up_sync(0xffffffffu, v.reset, o);
  return r;
}

// The reference's loop, one thread: acc = 0; acc = acc + t[j] for j < n.
__device__ __forceinline__ double serial(const double* t, int n) {
  double a = 0.0;
  for (int j = 0; j < n; j++) a = __dadd_rn(a, t[j]);
  return a;
}

// Term j is explicit when it is term 0 of a chunk, when the approximate sums
// before and after it lie in different binades, or when one of them lies
// within 2^-36 of a binade edge (the approximation could be on the wrong side).
__device__ __forceinline__ bool explicit_term(double before, double after, int j, int& Eb) {
  constexpr unsigned long long MANT = 0xFFFFFFFFFFFFFull, EDGE = 1ull << 16;
  const unsigned long long bb = (unsigned long long)__double_as_longlong(before);
  const unsigned long long ba = (unsigned long long)__double_as_longlong(after);
  const int fb = (int)(bb >> 52), fa = (int)(ba >> 52);
  Eb = (fb ? fb : 1) - 1023;
  const int Ea = (fa ? fa : 1) - 1023;
  return j == 0 || Eb != Ea || (fb > 1 && (bb & MANT) < EDGE) || (ba & MANT) > MANT - EDGE;
}
__device__ __forceinline__ Fn term_map(double v, int E) {
  unsigned long long r;
  bool tie;
  units(v, E, r, tie);
  Fn fn;
  fn.t = tie ? 1 : 0;
  fn.c1 = tie ? r : 0ull;
  fn.c2 = tie ? 0ull : r;
  return fn;
}

// One chunk of at most PER * blockDim.x terms, continuing the chain from
// acc_in (the exact running sum before the chunk).  Thread i owns terms
// [i*PER, i*PER + PER); PER is odd, so that consecutive lanes reading shared
// memory 8*PER bytes apart hit distinct banks.  The per-term loops stay
// rolled: the kernel's code then fits the instruction cache.
template <int PER>
__device__ __forceinline__ double osum_chunk(const double* t, int len, double acc_in, Smem& S) {
  const int tid = threadIdx.x, nt = blockDim.x, lane = tid & 31, wid = tid >> 5, nw = nt >> 5;
  const int lo = min(len, tid * PER), hi = min(len, lo + PER);
  // 1. approximate sums (only used to predict binades)
  double loc = 0.0;
  bool bad = !(acc_in >= 0.0) || isinf(acc_in);
#pragma unroll 1
  for (int j = lo; j < hi; j++) {
    const double v = t[j];
    bad |= !(v >= 0.0) || isinf(v);
    loc += v;
  }
  const double inc = warp_incl(loc, lane);
  if (lane == 31) S.wtot[wid] = inc;
  for (int i = tid; i < MAXSEG; i += nt) {
    S.emin[i] = INT_MAX;
    S.emax[i] = INT_MIN;
    S.ft[i] = 0;
    S.c1[i] = 0ull;
    S.c2[i] = 0ull;
  }
  // per-warp votes read back after a plain barrier (a block vote,
  // __syncthreads_or, takes microseconds to deliver its result)
  const bool wbad = __any_sync(0xffffffffu, bad);
  if (lane == 0) S.wbad[wid] = wbad ? 1 : 0;
  __syncthreads();
  bad = false;
  for (int w = 0; w < nw; w++) bad |= S.wbad[w] != 0;
  bool fits = false;
  if (!bad) {
    if (wid == 0) {
      const double w = lane < nw ? S.wtot[lane] : 0.0;
      const double wi = warp_incl(w, lane);
      double ex = __shfl_up_sync(0xffffffffu, wi, 1);
      if (lane == 0) ex = 0.0;
      if (lane < nw) S.wtot[lane] = ex;
    }
    __syncthreads();
    double exl = __shfl_up_sync(0xffffffffu, inc, 1);
    if (lane == 0) exl = 0.0;
    const double P = acc_in + (S.wtot[wid] + exl);  // ~ the sum before this run
    // 2. explicit terms of the run (bit k of exmask: term lo + k), and their ordinals
    unsigned exmask = 0u;
    {
      double before = P;
#pragma unroll 1
      for (int j = lo; j < hi; j++) {
        const double after = before + t[j];
        int Eb;
        if (explicit_term(before, after, j, Eb)) exmask |= 1u << (j - lo);
        before = after;
      }
    }
    const int cnt = __popc(exmask);
    const int cinc = warp_incl(cnt, lane);
    if (lane == 31) S.wcnt[wid] = cinc;
    __syncthreads();
    if (wid == 0) {
      const int w = lane < nw ? S.wcnt[lane] : 0;
      const int wi = warp_incl(w, lane);
      int ex = __shfl_up_sync(0xffffffffu, wi, 1);
      if (lane == 0) ex = 0;
      if (lane < nw) S.wcnt[lane] = ex;
      if (lane == 31) S.nseg = wi;  // total explicit terms
    }
    __syncthreads();
    const int nseg = S.nseg;
    const int base = S.wcnt[wid] + cinc - cnt;  // explicit terms before this run
    fits = nseg <= MAXSEG;
    // 3. compose the run's terms: the head piece (up to its first explicit
    //    term), inner pieces (stored at once) and the tail piece.  Between
    //    explicit terms the predicted binade cannot change, so a piece's
    //    binade is read once, at its start, and recorded for the check.
    Fn head = {0ull, 0ull, 0}, cur = {0ull, 0ull, 0};
    if (fits && hi > lo) {
      int ord = base - 1;
      double before = P;
      int E = binade(P);
      bool open = false;  // the current piece holds a term
#pragma unroll 1
      for (int j = lo; j < hi; j++) {
        const double v = t[j];
        if ((exmask >> (j - lo)) & 1u) {
          if (ord >= 0 && open) {
            atomicMin(&S.emin[ord], E);
            atomicMax(&S.emax[ord], E);
          }
          if (ord >= base) {  // an inner piece: both ends in this run
            S.c1[ord] = cur.c1;
            S.c2[ord] = cur.c2;
            S.ft[ord] = cur.t;
          } else {
            head = cur;
          }
          ord++;
          S.expl[ord] = j;
          S.tv[ord] = v;
          cur = Fn{0ull, 0ull, 0};
          open = false;
          before = before + v;
          E = binade(before);
        } else {
          // A -> A + r, or for a tie A -> roundup_even(A + r); pieces stay
          // below 2^59 inside a run, so no saturation is needed here
          unsigned long long r;
          bool tie;
          units(v, E, r, tie);
          if (!tie) {
            cur.c2 += r;
          } else if (!cur.t) {
            cur.t = 1;
            cur.c1 = cur.c2 + r;
            cur.c2 = 0ull;
          } else {
            cur.c2 = (cur.c2 + r + 1ull) & ~1ull;
          }
          open = true;
          before = before + v;
        }
      }
      if (ord >= 0 && open) {
        atomicMin(&S.emin[ord], E);
        atomicMax(&S.emax[ord], E);
      }
      cur.c1 = sat(cur.c1);
      cur.c2 = sat(cur.c2);
      head.c1 = sat(head.c1);
      head.c2 = sat(head.c2);
    }
    // 4. chain the pieces across runs: segmented scan of (has explicit, tail
    //    or whole-run map) over the threads in order
    const bool seen = exmask != 0u;
    SegFn mine;
    mine.reset = seen ? 1 : 0;
    mine.f = cur;  // seen: the tail piece; else the whole run
    SegFn incl = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const SegFn y = shfl_up_seg(incl, o);
      if (lane >= o) incl = seg_then(y, incl);
    }
    SegFn lexc = shfl_up_seg(incl, 1);
    if (lane == 0) lexc = SegFn{Fn{0ull, 0ull, 0}, 0};
    if (lane == 31) {
      S.wc1[wid] = incl.f.c1;
      S.wc2[wid] = incl.f.c2;
      S.wt[wid] = incl.f.t;
      S.wr[wid] = incl.reset;
    }
    __syncthreads();
    if (wid == 0) {
      SegFn w = {Fn{0ull, 0ull, 0}, 0};
      if (lane < nw) w = SegFn{Fn{S.wc1[lane], S.wc2[lane], S.wt[lane]}, S.wr[lane]};
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const SegFn y = shfl_up_seg(w, o);
        if (lane >= o) w = seg_then(y, w);
      }
      SegFn ex = shfl_up_seg(w, 1);
      if (lane == 0) ex = SegFn{Fn{0ull, 0ull, 0}, 0};
      if (lane < nw) {
        S.wc1[lane] = ex.f.c1;
        S.wc2[lane] = ex.f.c2;
        S.wt[lane] = ex.f.t;
        S.wr[lane] = ex.reset;
      }
    }
    __syncthreads();
    if (fits) {
      const SegFn wex = {Fn{S.wc1[wid], S.wc2[wid], S.wt[wid]}, S.wr[wid]};
      const SegFn exc = seg_then(wex, lexc);  // everything before this run
      if (seen && base >= 1) {                // the stretch ending at this run's first explicit term
        const Fn f = then(exc.f, head);
        S.c1[base - 1] = f.c1;
        S.c2[base - 1] = f.c2;
        S.ft[base - 1] = f.t;
      }
      if (tid == nt - 1 && nseg >= 1) {  // the last stretch runs to the end
        const SegFn all = seg_then(exc, mine);
        S.c1[nseg - 1] = all.f.c1;
        S.c2[nseg - 1] = all.f.c2;
        S.ft[nseg - 1] = all.f.t;
      }
    }
    __syncthreads();
  }
  // 5. the chain itself (one thread): explicit terms by __dadd_rn, stretches
  //    by their composed maps, each checked
  if (tid == 0) {
    double a = acc_in;
    bool ok = fits;
    if (ok) {
      const int nseg = S.nseg;
#pragma unroll 1
      for (int s = 0; s < nseg; s++) {
        a = __dadd_rn(a, S.tv[s]);
        const int E = S.emin[s], E2 = S.emax[s];
        if (E > E2) continue;  // no term between this explicit one and the next
        const unsigned long long bits = (unsigned long long)__double_as_longlong(a);
        const int f = (int)(bits >> 52);
        if (E2 != E || (f ? f : 1) - 1023 != E) { ok = false; break; }
        const unsigned long long A = (bits & 0xFFFFFFFFFFFFFull) | (f ? (1ull << 52) : 0ull);
        const unsigned long long A2 = apply(S.ft[s], S.c1[s], S.c2[s], A);
        if (A2 > (1ull << 53) - 1ull) { ok = false; break; }
        a = __longlong_as_double((long long)(((unsigned long long)(E + 1022) << 52) + A2));
      }
    }
    if (!ok) {
      a = acc_in;
      for (int j = 0; j < len; j++) a = __dadd_rn(a, t[j]);
    }
    S.result = a;
  }
  __syncthreads();
  return S.result;
}

// Same value as serial(t, n), computed by the whole block (blockDim.x a
// multiple of 32, at most 1024) in chunks of 17 * blockDim.x terms.  Every
// thread must call it; every thread gets the sum.  `t` may be in shared or
// global memory.
__device__ __forceinline__ double ordered_sum(const double* t, int n, Smem& S) {
  constexpr int PER = 17;
  const int chunk = PER * (int)blockDim.x;
  double acc = 0.0;
  for (int c0 = 0; c0 < n; c0 += chunk) acc = osum_chunk<PER>(t + c0, min(chunk, n - c0), acc, S);
  return acc;
}

}  // namespace dco
