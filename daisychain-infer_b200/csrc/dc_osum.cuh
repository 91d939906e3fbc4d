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

constexpr int MAXW = 24;                       // explicit terms per warp and chunk (else serial)
constexpr double DELTA = 1.0 / 68719476736.0;  // 2^-36 margin around binade edges
constexpr unsigned long long CAP = 1ull << 54; // saturation of the composed constants

// A -> t ? roundup_even(A + c1) + c2 : A + c2
struct Fn {
  unsigned long long c1, c2;
  int t;
};

// Per warp: its explicit terms (value, and the map of the stretch that
// follows each up to the next explicit term of the warp), the map of its terms
// before the first explicit one (head) and after the last (tail), or of all
// its terms when it has none (kept in tail).
struct Entry {
  double v;
  unsigned long long c1, c2;
  int t, emin, emax;
};
template <int NW>  // warps of the block
struct SmemT {
  Entry ent[NW][MAXW];
  Entry whead[NW], wtail[NW];  // v unused
  int wn[NW];                  // explicit terms of warp w
  int wbad[NW];
  double wtot[NW];
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
// The general case of units(): integer arithmetic on the term's bits.
__device__ __noinline__ unsigned long long units_bits(double t, int E, bool* tie) {
  const unsigned long long b = (unsigned long long)__double_as_longlong(t);
  const int f = (int)(b >> 52) & 0x7ff;
  const unsigned long long M = (b & 0xFFFFFFFFFFFFFull) | (f ? (1ull << 52) : 0ull);
  const int et = (f ? f : 1) - 1075;  // t = M * 2^et
  const int d = (E - 52) - et;
  *tie = false;
  if (d < 0) return M ? CAP : 0ull;
  if (d == 0) return M;
  if (d >= 64) return 0ull;
  const unsigned long long rem = M & ((1ull << d) - 1), half = 1ull << (d - 1);
  *tie = rem == half;
  return (M >> d) + (rem > half ? 1ull : 0ull);
}
__device__ __forceinline__ void units(double t, int E, unsigned long long& r, bool& tie) {
  constexpr double MAGIC = 6755399441055744.0;  // 1.5 * 2^52: MAGIC + q lands on an integer grid
  // q = t * 2^(52-E) is exact (a power-of-two scale that neither overflows
  // nor loses bits, except for q far below 1/2 where only r = 0 matters)
  const double q = __dmul_rn(t, __longlong_as_double((long long)(1075 - max(E, -900)) << 52));
  if (E > -900 && q < 2251799813685248.0) {  // q < 2^51: RN-even(q) from the grid
    const double y = __dadd_rn(q, MAGIC);
    const double d = __dsub_rn(q, __dsub_rn(y, MAGIC));
    const unsigned long long rne = ((unsigned long long)__double_as_longlong(y) & 0xFFFFFFFFFFFFFull) - (1ull << 51);
    tie = d == 0.5 || d == -0.5;
    r = rne - (d < 0.0 && tie ? 1ull : 0ull);  // a tie keeps its floor
    return;
  }
  r = units_bits(t, E, &tie);
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

// A stretch map with the binades its terms were rounded in (empty: emin > emax)
// and whether an explicit term precedes it inside the scanned range.
struct SegFn {
  Fn f;
  int emin, emax;
  int reset;
};
__device__ __forceinline__ SegFn seg_empty() { return SegFn{Fn{0ull, 0ull, 0}, INT_MAX, INT_MIN, 0}; }
__device__ __forceinline__ SegFn seg_cat(const SegFn& a, const SegFn& b) {  // a, then b
  if (b.reset) return b;
  SegFn c;
  c.f = then(a.f, b.f);
  c.emin = min(a.emin, b.emin);
  c.emax = max(a.emax, b.emax);
  c.reset = a.reset;
  return c;
}
__device__ __forceinline__ SegFn shfl_up_seg(const SegFn& v, int o) {
  SegFn r;
  r.f.c1 = __shfl_up_sync(0xffffffffu, v.f.c1, o);
  r.f.c2 = __shfl_up_sync(0xffffffffu, v.f.c2, o);
  r.f.t = __shfl_up_sync(0xffffffffu, v.f.t, o);
  r.emin = __shfl_up_sync(0xffffffffu, v.emin, o);
  r.emax = __shfl_up_sync(0xffffffffu, v.emax, o);
  r.reset = __shfl_up_sync(0xffffffffu, v.reset, o);
  return r;
}
__device__ __forceinline__ void put(Entry& e, const SegFn& s) {
  e.c1 = sat(s.f.c1);
  e.c2 = sat(s.f.c2);
  e.t = s.f.t;
  e.emin = s.emin;
  e.emax = s.emax;
}
__device__ __forceinline__ SegFn get(const Entry& e) { return SegFn{Fn{e.c1, e.c2, e.t}, e.emin, e.emax, 0}; }

// The reference's loop, one thread: acc = 0; acc = acc + t[j] for j < n.
__device__ __forceinline__ double serial(const double* t, int n) {
  double a = 0.0;
#pragma unroll 1
  for (int j = 0; j < n; j++) a = __dadd_rn(a, t[j]);
  return a;
}

// Binade tracking along a lane's run of approximate sums.  A term is explicit
// when it is term 0 of the chunk, when the piece it would join started within
// the margin above its binade's lower edge, or when the approximate sum after
// it reaches the margin below the binade's upper edge.
struct Track {
  int E;
  double top;  // 2^(E+1) * (1 - 2^-36)
  bool low;    // the piece starts within 2^-36 above 2^E
  __device__ __forceinline__ void start(double x) {
    E = binade(x);
    top = __longlong_as_double((long long)(E + 1024) << 52) * (1.0 - DELTA);
    const int f = (int)((unsigned long long)__double_as_longlong(x) >> 52);
    low = f > 1 && x < __longlong_as_double((long long)(E + 1023) << 52) * (1.0 + DELTA);
  }
};

// Finish a stretch on the serial chain: apply its map to the exact running sum
// a (checked: every term rounded in a's binade, result below 2^53 units).
__device__ __forceinline__ bool finish(double& a, const SegFn& st) {
  if (st.emin > st.emax) return true;  // no term
  const int E = st.emin;
  const unsigned long long bits = (unsigned long long)__double_as_longlong(a);
  const int f = (int)(bits >> 52);
  if (st.emax != E || (f ? f : 1) - 1023 != E) return false;
  const unsigned long long A = (bits & 0xFFFFFFFFFFFFFull) | (f ? (1ull << 52) : 0ull);
  const unsigned long long A2 = apply(st.f.t, st.f.c1, st.f.c2, A);
  if (A2 > (1ull << 53) - 1ull) return false;
  a = __longlong_as_double((long long)(((unsigned long long)(E + 1022) << 52) + A2));
  return true;
}

// One chunk of at most PER * 32 * NW terms (blockDim.x == 32 * NW), continuing the
// chain from acc_in (the exact running sum before the chunk).  Lane l of warp
// w owns terms [(32w + l) * PER, ... + PER); PER is odd, so that consecutive
// lanes reading shared memory 8*PER bytes apart hit distinct banks.  Two block
// barriers; the rest is warp-local.  The per-term loops stay rolled: this code
// runs once per row on one SM, where instruction fetch, not arithmetic, sets
// the pace of long straight-line code.
template <int PER, int NW>
__device__ __forceinline__ double osum_chunk(const double* t, int len, double acc_in, SmemT<NW>& S) {
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int lo = min(len, tid * PER), hi = min(len, lo + PER);
  // 1. the run's approximate sum, warp prefix sums
  double loc = 0.0;
  bool bad = !(acc_in >= 0.0) || isinf(acc_in);
#pragma unroll 1
  for (int j = lo; j < hi; j++) {
    const double v = t[j];
    bad |= !(v >= 0.0) || isinf(v);
    loc += v;
  }
  const double inc = warp_incl(loc, lane);
  const bool wbad = __any_sync(0xffffffffu, bad);
  if (lane == 31) {
    S.wtot[wid] = inc;
    S.wbad[wid] = wbad ? 1 : 0;
  }
  __syncthreads();
  bool any_bad = false;
  double P = acc_in;
#pragma unroll 1
  for (int w = 0; w < NW; w++) {
    any_bad |= S.wbad[w] != 0;
    if (w < wid) P += S.wtot[w];
  }
  if (!any_bad) {
    double exl = __shfl_up_sync(0xffffffffu, inc, 1);
    if (lane == 0) exl = 0.0;
    P += exl;  // ~ the exact sum before this run
    // 2a. explicit terms of the run (bit k: term lo + k)
    unsigned exmask = 0u;
    {
      Track tr;
      tr.start(P);
      double before = P;
#pragma unroll 1
      for (int j = lo; j < hi; j++) {
        const double after = before + t[j];
        if (j == 0 || tr.low || after >= tr.top) {
          exmask |= 1u << (j - lo);
          tr.start(after);
        }
        before = after;
      }
    }
    const int cnt = __popc(exmask);
    const int cinc = warp_incl(cnt, lane);
    const int wn = __shfl_sync(0xffffffffu, cinc, 31);
    const bool fits = wn <= MAXW;
    // 2b. compose: head piece (before the first explicit term), inner pieces
    //     (stored at once) and the tail piece, each with its binade
    SegFn head = seg_empty(), cur = seg_empty();
    if (fits) {
      const int base = cinc - cnt;  // explicit terms of this warp before this run
      int ord = base - 1;
      Track tr;
      tr.start(P);
      double before = P;
#pragma unroll 1
      for (int j = lo; j < hi; j++) {
        const double v = t[j], after = before + v;
        if ((exmask >> (j - lo)) & 1u) {
          if (ord >= base) put(S.ent[wid][ord], cur);
          else head = cur;
          ord++;
          S.ent[wid][ord].v = v;
          cur = seg_empty();
          tr.start(after);
        } else {
          unsigned long long r;
          bool tie;
          units(v, tr.E, r, tie);
          if (!tie) {
            cur.f.c2 += r;
          } else if (!cur.f.t) {
            cur.f.t = 1;
            cur.f.c1 = cur.f.c2 + r;
            cur.f.c2 = 0ull;
          } else {
            cur.f.c2 = (cur.f.c2 + r + 1ull) & ~1ull;
          }
          cur.emin = min(cur.emin, tr.E);
          cur.emax = max(cur.emax, tr.E);
        }
        before = after;
      }
      // a run's constants stay below 2^59 (17 terms of < 2^55): saturate once
      cur.f.c1 = sat(cur.f.c1);
      cur.f.c2 = sat(cur.f.c2);
      head.f.c1 = sat(head.f.c1);
      head.f.c2 = sat(head.f.c2);
    }
    // 2c. chain the runs of the warp: segmented scan of (has explicit,
    //     tail or whole-run map)
    SegFn incl = cur;
    incl.reset = exmask ? 1 : 0;
#pragma unroll 1
    for (int o = 1; o < 32; o <<= 1) {
      const SegFn y = shfl_up_seg(incl, o);
      if (lane >= o) incl = seg_cat(y, incl);
    }
    SegFn lexc = shfl_up_seg(incl, 1);
    if (lane == 0) lexc = seg_empty();
    if (fits) {
      if (exmask) {  // the stretch ending at this run's first explicit term
        const SegFn h = seg_cat(lexc, head);
        if (lexc.reset) put(S.ent[wid][cinc - cnt - 1], h);
        else put(S.whead[wid], h);
      }
      if (lane == 31) put(S.wtail[wid], incl);
    }
    if (lane == 31) S.wn[wid] = wn;
  }
  __syncthreads();
  // 3a. the map after each warp's last explicit term runs through the
  //     following warps up to the next explicit term (or the chunk's end):
  //     composed by one lane per warp, in parallel
  if (wid == 0 && !any_bad && lane < NW) {
    const int n = S.wn[lane];
    if (n > 0 && n <= MAXW) {
      SegFn m = get(S.wtail[lane]);
#pragma unroll 1
      for (int x = lane + 1; x < NW; x++) {
        if (S.wn[x] > 0) {
          m = seg_cat(m, get(S.whead[x]));
          break;
        }
        m = seg_cat(m, get(S.wtail[x]));
      }
      put(S.ent[lane][n - 1], m);
    }
  }
  __syncwarp();
  // 3b. the chain itself (one thread): explicit terms by __dadd_rn, the
  //     stretch after each by its composed map, each checked
  if (tid == 0) {
    double a = acc_in;
    bool ok = !any_bad && (len == 0 || S.wn[0] > 0);  // term 0 is explicit
    if (ok) {
#pragma unroll 1
      for (int w = 0; w < NW; w++) ok &= S.wn[w] <= MAXW;
    }
    if (ok) {
#pragma unroll 1
      for (int w = 0; w < NW; w++) {
        const int n = S.wn[w];
#pragma unroll 1
        for (int i = 0; i < n; i++) {
          const Entry& e = S.ent[w][i];
          a = __dadd_rn(a, e.v);
          ok &= finish(a, get(e));
        }
      }
    }
    if (!ok) {
      a = acc_in;
#pragma unroll 1
      for (int j = 0; j < len; j++) a = __dadd_rn(a, t[j]);
    }
    S.result = a;
  }
  __syncthreads();
  return S.result;
}

// Same value as serial(t, n), computed by the whole block (NW warps) in
// chunks of 17 * 32 * NW terms.  Every thread must call it; every thread gets
// the sum.  `t` may be in shared or global memory.  A block of another size
// than 32 * NW threads takes the serial loop.
template <int NW>
__device__ __forceinline__ double ordered_sum(const double* t, int n, SmemT<NW>& S) {
  constexpr int PER = 17;
  if (blockDim.x != 32 * NW) {
    if (threadIdx.x == 0) S.result = serial(t, n);
    __syncthreads();
    const double r = S.result;
    __syncthreads();
    return r;
  }
  double acc = 0.0;
#pragma unroll 1
  for (int c0 = 0; c0 < n; c0 += PER * 32 * NW)
    acc = osum_chunk<PER, NW>(t + c0, min(PER * 32 * NW, n - c0), acc, S);
  return acc;
}
using Smem = SmemT<8>;    // 256-thread blocks
using Smem16 = SmemT<16>; // 512-thread blocks

}  // namespace dco
