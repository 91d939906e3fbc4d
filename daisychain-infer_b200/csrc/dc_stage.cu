// dc_stage.cu -- one pipeline stage of the verified forward pass, resident on one B200.
//
// Restates public/infer.js for the Llama family (RMSNorm, RoPE, GQA, SwiGLU):
// layerForward :114-221, runLayers :275-283, runLayersChunk :288-296,
// embedRows :298-310, logitsAt :324-334, greedy pickToken :390-396.  A stage
// owns a contiguous layer range [lo, hi) (shard.js planStages :32-52); the
// head stage also owns the embedding, the final norm and lm_head.
//
// Bit-exactness rules kept here (every f32/f64 step is an explicitly rounded
// operation; the library is built with --fmad=false):
//  * RMSNorm: s += v*v in double, sequentially from j = 0 (one thread walks
//    the row), inv = 1/sqrt(s/C + eps), y = f32((x*inv)*w)           (:30-39)
//  * every GEMM input is quantised per row (double scale) and every weight per
//    column (f32 scale), as vgemmBlock does (verified_core.js:425-449); the
//    weights are quantised once at load, which is bit-identical;
//  * Q/K/V share the row quantisation of h1, so their weights are concatenated
//    column-wise into one GEMM; gate/up likewise (exact: column scales are
//    per column, row scales are shared);
//  * RoPE: f32(a*c - b*s) with the products and the difference in double
//    (:83-97); tables f = p / theta^(2i/hd) built on the host once;
//  * attention per head (:171-197): scores = vgemm(q_h, k_hᵀ) with the row
//    scale per (query token, head) and the column scale per (key token, kv
//    head) -- stable as the cache grows, so int8 K and its scale are cached
//    at append; causal softmax: mx = max(s*scale) in double, e = exp(s*scale -
//    mx) (fdlibm method), a = f32(e), z += e sequentially in key order,
//    a = f32(a / z); ctx = vgemm(a, v_h) with the row scale per query row and
//    the column scale per (kv head, channel) over all N cached tokens -- the
//    V cache stays f32 and its int8 copy is re-quantised whenever a channel's
//    scale moves (the running absmax only grows, so unchanged channels keep
//    their int8 values);
//  * SwiGLU: f32(silu(g) * u) with silu(v) = v / (1 + exp(-v)) in double;
//  * residuals: f32 adds.
#include <math.h>

#include <algorithm>
#include <vector>

#include "dc_fdlibm.cuh"
#include "dc_internal.cuh"
#include "dc_math.cuh"
#include "dc_osum.cuh"
#include "dc_ptx.cuh"

#include <cooperative_groups.h>

struct dc_mat {
  int k = 0, n = 0, ldk = 0;
  int8_t* qt = nullptr;  // n x ldk, quantised Wᵀ (zero past k)
  float* cs = nullptr;   // n column scales
};

struct dc_kv {
  int8_t* k8 = nullptr;   // [kvh][max_pos][hd] int8 keys (rotated)
  float* ks = nullptr;    // [kvh][max_pos] key scales (f32, quantizeCols rule)
  float* v = nullptr;     // [max_pos][kvDim] f32 values
  float* vt = nullptr;    // [kvDim][ldvt] the same values channel-major (a channel's column re-quantises from it)
  int8_t* v8t = nullptr;  // [kvh][hd][ldp] int8 values (channel-major) under the current channel scales
  float* vs = nullptr;    // [kvDim] channel scales
  uint32_t* vmax = nullptr;  // [kvDim] running |v| maximum (float bits)
  int* vchg = nullptr;    // [kvDim] channel scale changed on this step
};

struct dc_layer {
  float* nrm1 = nullptr;
  float* nrm2 = nullptr;
  dc_mat qkv, o, gu, down;
  dc_kv kv;
};

struct dc_stage {
  dc_ctx* ctx = nullptr;
  dc_spec spec;
  int lo = 0, hi = 0, head = 0, max_rows = 0, max_pos = 0;
  int C = 0, hd = 0, nH = 0, nKV = 0, qDim = 0, kvDim = 0, I = 0, V = 0, nqkv = 0;
  int ldC = 0, ldQ = 0, ldI = 0, ldp = 0;  // ldp: positions per channel row of the int8 V cache
  int ldvt = 0;  // positions per channel row of the f32 channel-major V copy (ldp + 8: no power-of-two stride)
  std::vector<dc_layer> L;
  float* emb = nullptr;  // V x C
  float* nrmF = nullptr;
  dc_mat lm;
  float* rope_cos = nullptr;  // max_pos x hd/2
  float* rope_sin = nullptr;
  int kv_len = 0;  // tokens in the KV cache (chunk path)
  // activation scratch
  float* hbuf = nullptr;   // max_rows x max(nqkv, 2I, C)
  float* hmid = nullptr;   // max_rows x I: the SwiGLU output (the down projection's input)
  float* ctxo = nullptr;   // max_rows x qDim
  int8_t* xq = nullptr;    // max_rows x max(ldC, ldQ, ldI)
  float* rs = nullptr;     // max_rows
  float* lx = nullptr;     // logits rows x C gathered
  uint32_t* rowmax = nullptr;  // max_rows running row maxima (float bits)
  // device-side positions (read by the kernels, so decode laps can be replayed as a graph)
  int* d_pos = nullptr;     // cached tokens of this stage
  int* d_zero = nullptr;    // constant 0 (the full window)
  int* d_step = nullptr;    // head: decode lap counter (index into the picks buffer)
  float* xlap = nullptr;    // head: the one hidden row a decode lap carries
  float* logits1 = nullptr; // head: logits of the lap's row
  unsigned long long* amax_keys = nullptr;  // head: greedy-pick keys (8 rows), kept at zero between uses
  int* att_done = nullptr;  // decode attention: CTAs finished (kept at zero between launches)
  int8_t* a8g = nullptr;    // chunk attention: probability rows [head][row][ldp] (max_rows rows)
  float* asg = nullptr;     // and their scales [head][row]
  // a pass of several chunks (dc_stage_forward_chunks): chunk g's value channel
  // scales, their change flags, and (every chunk but the last, whose values go
  // to the cache) its int8 values [g][kv head][channel][ldp]
  float* vsg = nullptr;     // [DC_MAX_CHUNKS][kvDim]
  int* vchgg = nullptr;     // [DC_MAX_CHUNKS][kvDim]
  int8_t* v8s = nullptr;    // [max_chunks - 1][kvDim][ldp]
  int max_chunks = 1;       // chunks one pass may hold (min(max_rows, DC_MAX_CHUNKS))
  uint32_t* vstage = nullptr;  // [2][kvDim] decode row: the attention's new value channel maxima, then scales
                               // (float bits), committed to the layer's cache by the O projection
  cudaGraphExec_t lap_exec = nullptr;
  unsigned long long lap_nk = 0;  // kernels in one replay of lap_exec
  float* xrow = nullptr;              // one-row graph: the row, in place
  cudaGraphExec_t row_exec = nullptr;  // one-row graph of this stage's layers
  unsigned long long row_nk = 0;
  bool row_graph = true;
  bool row_fused = false;  // decode rows: GEMVs with the norm / SwiGLU / row quantisation fused
  int pass_attn = 0;       // a pass's attention: 0 k_attn_chunk when the CTAs fill the SMs, 1 always, 2 never
  bool o_rowq = true;      // decode rows: the O projection quantises the context row itself (not the attention's last CTA)
  std::vector<dc_stage*> lap_key;
  int32_t* lap_picks = nullptr;
  std::vector<void*> allocs;
};

namespace {

constexpr int NORM_THREADS = 256;
constexpr int ATT_THREADS = 256;

__device__ __forceinline__ float block_max_f(float v, float* red) {
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    float w = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
    for (int o = 16; o; o >>= 1) w = fmaxf(w, __shfl_xor_sync(0xffffffffu, w, o));
    if (threadIdx.x == 0) red[0] = w;
  }
  __syncthreads();
  float r = red[0];
  __syncthreads();
  return r;
}

__device__ __forceinline__ double block_max_d(double v, double* red) {
  for (int o = 16; o; o >>= 1) v = fmax(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    double w = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : -INFINITY;
    for (int o = 16; o; o >>= 1) w = fmax(w, __shfl_xor_sync(0xffffffffu, w, o));
    if (threadIdx.x == 0) red[0] = w;
  }
  __syncthreads();
  double r = red[0];
  __syncthreads();
  return r;
}

// max(mx/127, 1e-8) in double (verified_core.js:114, :128).
__device__ __forceinline__ double quant_scale(float mx) {
  double sc = __ddiv_rn((double)mx, 127.0);  // (inline: an out-of-line call is an instruction fetch away)
  return sc > 1e-8 ? sc : 1e-8;
}

// The serial-order sum of dc_osum.cuh, out of line: only ambiguous rows reach
// it, so its code stays out of the callers' instruction stream.  Every thread
// of the block calls it.
__device__ __noinline__ double ordered_sum_cold(const double* t, int n, dco::Smem& osm) {
  return dco::ordered_sum(t, n, osm);
}
__device__ __noinline__ double ordered_sum_cold16(const double* t, int n, dco::Smem16& osm) {
  return dco::ordered_sum(t, n, osm);
}
template <int NW> struct OsumCold;
template <> struct OsumCold<8> {
  static __device__ __forceinline__ double sum(const double* t, int n, dco::SmemT<8>& s) { return ordered_sum_cold(t, n, s); }
};
template <> struct OsumCold<16> {
  static __device__ __forceinline__ double sum(const double* t, int n, dco::SmemT<16>& s) {
    return ordered_sum_cold16(t, n, s);
  }
};

// Dynamic shared memory of k_rmsnorm_quant: squares (double) and the row
// (float), plus the weight row (float) when that still fits.

// 1 / sqrt(s / C + eps) with every step correctly rounded (infer.js:77-78);
// monotone non-increasing in s.
__device__ __noinline__ double rms_inv(double s, int C, double eps) {
  return __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(s, (double)C), eps)));
}
// Block sums of two doubles in any order (used only to bracket serial sums).
__device__ __forceinline__ double2 block_sum_d2(double a, double b, double2* red) {
  for (int o = 16; o; o >>= 1) {
    a += __shfl_xor_sync(0xffffffffu, a, o);
    b += __shfl_xor_sync(0xffffffffu, b, o);
  }
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = make_double2(a, b);
  __syncthreads();
  if (threadIdx.x < 32) {
    double2 w = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : make_double2(0.0, 0.0);
    for (int o = 16; o; o >>= 1) {
      w.x += __shfl_xor_sync(0xffffffffu, w.x, o);
      w.y += __shfl_xor_sync(0xffffffffu, w.y, o);
    }
    if (threadIdx.x == 0) red[0] = w;
  }
  __syncthreads();
  const double2 r = red[0];
  __syncthreads();
  return r;
}

// Radius of an interval around s that holds the serial sum t_0 + t_1 + ... +
// t_(n-1) of non-negative doubles (each add rounded to nearest), where s is
// the same terms summed in any order with every term passing through at most
// `depth` rounded adds, and w is the sum of (n - j) * t_j (any order).  The
// serial sum errs by at most u times the sum of its exact prefix sums, i.e.
// u * sum (n - j) t_j (each add errs by at most u times its result, and the
// running sum stays within a factor 1 + gamma_n of the exact prefix); s errs
// by at most gamma_depth times the total.  u = 2^-53; the constants absorb
// the rounding of w, of this radius and of s -/+ radius.
__device__ __forceinline__ double serial_sum_radius(double s, double w, int depth) {
  return 1.1102230246251565e-16 * (1.001 * w + (double)(depth + 8) * s);
}

// RMSNorm of one row (infer.js:30-39) fused with quantizeRows of its output,
// computed by the whole block (NW warps); every thread calls it after
// griddepcontrol.wait.  xr: the row (C floats; float4 access when `vec`),
// wr: the weight row (in shared memory when the caller copied it there with
// cp.async, `wpend` then says the copies are still in flight).  Shared
// scratch: sq (C doubles), ys (C floats).  Output: yo (the normalised f32 row,
// no quantisation) when not null, else q (ldq bytes, zero past C) and *s
// (thread 0).  A non-finite input sets DC_ST_NONFINITE in *status.
template <int NW>
__device__ __forceinline__ void rmsnorm_quant_block(const float* xr, int C, const float* wr, bool wpend, bool vec,
                                                    double eps, double* sq, float* ys, int8_t* q, int ldq,
                                                    float* s, int* status, float* yo, int exact_sum,
                                                    dco::SmemT<NW>& osm, float* red, double2* redd2, int* vote) {
  bool bad = false;
  if (vec) {
#pragma unroll 4
    for (int i = threadIdx.x; i < (C >> 2); i += blockDim.x) {
      const float4 v = reinterpret_cast<const float4*>(xr)[i];
      bad |= !isfinite(v.x) || !isfinite(v.y) || !isfinite(v.z) || !isfinite(v.w);
      reinterpret_cast<float4*>(ys)[i] = v;
      sq[4 * i + 0] = __dmul_rn((double)v.x, (double)v.x);  // exact: a float square fits in a double
      sq[4 * i + 1] = __dmul_rn((double)v.y, (double)v.y);
      sq[4 * i + 2] = __dmul_rn((double)v.z, (double)v.z);
      sq[4 * i + 3] = __dmul_rn((double)v.w, (double)v.w);
    }
    if (wpend) asm volatile("cp.async.wait_all;" ::: "memory");  // this thread's copies (the barrier below publishes them)
  } else {
    for (int j = threadIdx.x; j < C; j += blockDim.x) {
      const float v = xr[j];
      bad |= !isfinite(v);
      ys[j] = v;
      sq[j] = __dmul_rn((double)v, (double)v);
    }
  }
  // warp votes and a plain barrier: a block vote (__syncthreads_or) costs microseconds here
  if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) atomicOr(status, DC_ST_NONFINITE);
  __syncthreads();
  // The reference sums s += v*v for j = 0 .. C-1, each step rounded.  That
  // serial value is bracketed first: an any-order sum S' and the error bound
  // of serial_sum_radius give an interval that holds it, inv = 1/sqrt(s/C +
  // eps) is monotone in s, and each y_j = f32(x_j*inv*w_j) is monotone in inv.
  // When every y_j is the same at both ends of the bracket, it is the serial
  // sum's y_j; otherwise (rare: some y_j within ~1e-13 of an f32 rounding
  // boundary) the block computes the serial-order sum itself.
  float mx = 0.0f;
  bool any = false;
  {
    double part = 0.0, wpart = 0.0;
    for (int j = threadIdx.x; j < C; j += blockDim.x) {
      part += sq[j];
      wpart += (double)(C - j) * sq[j];
    }
    const double2 sw = block_sum_d2(part, wpart, redd2);
    const double h = serial_sum_radius(sw.x, sw.y, (C + (int)blockDim.x - 1) / (int)blockDim.x + 10);
    // (both ends inline, so their division and square-root chains overlap)
    const double inv_hi = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(sw.x - h, (double)C), eps)));
    const double inv_lo = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(sw.x + h, (double)C), eps)));
    // Both ends of the bracket in one pass: the value at the lower end is kept
    // (the serial sum's whenever no output is ambiguous), with its |y| maximum.
    bool amb = exact_sum != 0;
    if (vec) {
#pragma unroll 2
      for (int i = threadIdx.x; i < (C >> 2); i += blockDim.x) {
        const float4 wv = reinterpret_cast<const float4*>(wr)[i];
        float4 y = reinterpret_cast<const float4*>(ys)[i];
        const float4 x = y;
        y.x = __double2float_rn(__dmul_rn(__dmul_rn((double)x.x, inv_lo), (double)wv.x));
        y.y = __double2float_rn(__dmul_rn(__dmul_rn((double)x.y, inv_lo), (double)wv.y));
        y.z = __double2float_rn(__dmul_rn(__dmul_rn((double)x.z, inv_lo), (double)wv.z));
        y.w = __double2float_rn(__dmul_rn(__dmul_rn((double)x.w, inv_lo), (double)wv.w));
        amb |= y.x != __double2float_rn(__dmul_rn(__dmul_rn((double)x.x, inv_hi), (double)wv.x)) ||
               y.y != __double2float_rn(__dmul_rn(__dmul_rn((double)x.y, inv_hi), (double)wv.y)) ||
               y.z != __double2float_rn(__dmul_rn(__dmul_rn((double)x.z, inv_hi), (double)wv.z)) ||
               y.w != __double2float_rn(__dmul_rn(__dmul_rn((double)x.w, inv_hi), (double)wv.w));
        reinterpret_cast<float4*>(ys)[i] = y;
        mx = fmaxf(mx, fmaxf(fmaxf(fabsf(y.x), fabsf(y.y)), fmaxf(fabsf(y.z), fabsf(y.w))));
      }
    } else {
      for (int j = threadIdx.x; j < C; j += blockDim.x) {
        const double xw = (double)ys[j], wj = (double)wr[j];
        const float y = __double2float_rn(__dmul_rn(__dmul_rn(xw, inv_lo), wj));
        amb |= y != __double2float_rn(__dmul_rn(__dmul_rn(xw, inv_hi), wj));
        ys[j] = y;
        mx = fmaxf(mx, fabsf(y));
      }
    }
    // one exchange carries the ambiguity vote and the row maximum
    const bool wamb = __any_sync(0xffffffffu, amb);
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) {
      vote[threadIdx.x >> 5] = wamb ? 1 : 0;
      red[threadIdx.x >> 5] = mx;
    }
    __syncthreads();
    for (int wv = 0; wv < (int)(blockDim.x >> 5); wv++) {
      any |= vote[wv] != 0;
      mx = fmaxf(mx, red[wv]);
    }
  }
  if (any) {  // rare: the serial-order sum, then the outputs again from the input row
    const double inv = rms_inv(OsumCold<NW>::sum(sq, C, osm), C, eps);
    mx = 0.0f;
    for (int j = threadIdx.x; j < C; j += blockDim.x) {
      const float y = __double2float_rn(__dmul_rn(__dmul_rn((double)xr[j], inv), (double)wr[j]));
      ys[j] = y;
      mx = fmaxf(mx, fabsf(y));
    }
    mx = block_max_f(mx, red);  // (its barriers also publish ys)
  }
  if (yo) {  // the normalised row itself (infer.js rmsnorm), no quantisation
    __syncthreads();
    for (int j = threadIdx.x; j < C; j += blockDim.x) yo[j] = ys[j];
    return;
  }
  const double sc = quant_scale(mx), rsc = __drcp_rn(sc);
  const float rscf = __double2float_rn(rsc);
  if (threadIdx.x == 0) s[0] = __double2float_rn(sc);
  if (vec && (ldq & 3) == 0 && (reinterpret_cast<uintptr_t>(q) & 3) == 0) {
#pragma unroll 1
    for (int i = threadIdx.x; i < (ldq >> 2); i += blockDim.x) {
      char4 o = make_char4(0, 0, 0, 0);
      if (4 * i < C) {
        const float4 y = reinterpret_cast<const float4*>(ys)[i];
        o.x = dc_quant_div_f(y.x, sc, rsc, rscf);
        o.y = dc_quant_div_f(y.y, sc, rsc, rscf);
        o.z = dc_quant_div_f(y.z, sc, rsc, rscf);
        o.w = dc_quant_div_f(y.w, sc, rsc, rscf);
      }
      reinterpret_cast<char4*>(q)[i] = o;
    }
  } else {
#pragma unroll 1
    for (int j = threadIdx.x; j < ldq; j += blockDim.x) q[j] = j < C ? dc_quant_div_f(ys[j], sc, rsc, rscf) : (int8_t)0;
  }
}

// RMSNorm of one row fused with quantizeRows of its output, one block of NT
// threads per row (NORM_WIDE for rows that run alone or in a single wave: a
// one-row norm is a chain of dependent phases, and wider blocks shorten each).
// x rows x C f32 -> q rows x ldq int8 (+ s[row]); the f32 norm output is not kept.
// Dynamic shared memory: C doubles (v*v) and C floats (x, then y); then,
// when the launch leaves room for it, C floats (the weight row); then the
// exact ordered sum's scratch, unless it fits over the y row (which that rare
// path rewrites afterwards).  Without the weight row a 256-thread block takes
// about 12 bytes per column, so four blocks share an SM at C = 4096.
constexpr int NORM_WIDE = 512;
template <int NT>
__host__ __device__ constexpr bool rms_osm_alias(int C) {
  return 4 * (size_t)C >= sizeof(dco::SmemT<NT / 32>);
}
__host__ __device__ constexpr size_t rms_osm_at(int C, bool with_w) {  // byte offset of the scratch
  return ((with_w ? 16 : 12) * (size_t)C + 15) & ~(size_t)15;
}
template <int NT>
static size_t rms_smem_t(int C, bool with_w) {
  return rms_osm_at(C, with_w) + (rms_osm_alias<NT>(C) ? 0 : sizeof(dco::SmemT<NT / 32>));
}
// with_w: keep the weight row on chip when that still leaves 20 KB of the SM
static size_t rms_smem(int C, int nt, bool with_w = true) {
  const bool w = with_w && (nt == NORM_WIDE ? rms_smem_t<NORM_WIDE>(C, true) : rms_smem_t<NORM_THREADS>(C, true)) +
                                   20 * 1024 <= 232448;
  return nt == NORM_WIDE ? rms_smem_t<NORM_WIDE>(C, w) : rms_smem_t<NORM_THREADS>(C, w);
}
template <int NT>
__global__ void __launch_bounds__(NT, NT == NORM_THREADS ? 4 : 1) k_rmsnorm_quant(const float* x, int C,
                                                               const float* w, double eps,
                                                               int8_t* q, int ldq,
                                                               float* s, int* status,
                                                               float* yo = nullptr,
                                                               uint32_t* zrow = nullptr,
                                                               int exact_sum = 0) {
  extern __shared__ __align__(16) double sq[];
  float* ys = (float*)(sq + C);
  uint32_t dsm;
  asm("mov.u32 %0, %%dynamic_smem_size;" : "=r"(dsm));
  using Osm = dco::SmemT<NT / 32>;
  const bool alias = rms_osm_alias<NT>(C);
  const bool with_w = dsm >= rms_osm_at(C, true) + (alias ? 0 : sizeof(Osm));
  float* wsm = with_w ? ys + C : nullptr;
  Osm& osm = alias ? *reinterpret_cast<Osm*>(ys) : *reinterpret_cast<Osm*>((uint8_t*)sq + rms_osm_at(C, with_w));
  __shared__ float red[32];
  __shared__ double2 redd2[32];
  __shared__ int vote[32];
  // the GEMV that consumes q may launch now: it streams its weights meanwhile
  asm volatile("griddepcontrol.launch_dependents;");
  const int row = blockIdx.x;
  const float* xr = x + (int64_t)row * C;
  // float4 access when the row allows it (all loads of a thread in flight at once)
  const bool vec = (C & 3) == 0 && ((reinterpret_cast<uintptr_t>(xr) | reinterpret_cast<uintptr_t>(w)) & 15) == 0;
  // The weight row is constant: its copy into shared memory (asynchronous,
  // awaited after the input row's loads) starts before the grid-dependency
  // wait.  Everything else this kernel reads or writes comes after it.
  bool wpend = false;
  if (vec && wsm) {
    for (int i = threadIdx.x; i < (C >> 2); i += blockDim.x)
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dcp::smem_u32(wsm + 4 * i)), "l"(w + 4 * i)
                   : "memory");
    asm volatile("cp.async.commit_group;" ::: "memory");
    wpend = true;
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (zrow && threadIdx.x == 0) zrow[row] = 0;  // the row maximum the next row quantisation collects
  if (!vec && wsm)
    for (int j = threadIdx.x; j < C; j += blockDim.x) wsm[j] = w[j];  // published by the block's first barrier
  rmsnorm_quant_block<NT / 32>(xr, C, wsm ? wsm : w, wpend, vec, eps, sq, ys, q + (int64_t)row * ldq, ldq,
                                          s + row, status, yo ? yo + (int64_t)row * C : nullptr, exact_sum, osm, red,
                                          redd2, vote);
}

// quantizeRows of the f32 row x (n values; zero past n up to ldq) by one
// block with the scale sc (rsc = 1/sc), x read through L2 (another CTA wrote
// it): each thread's 16 loads are in flight before its first conversion.
__device__ __forceinline__ void quant_row_block(const float* x, int n, int ldq, double sc, double rsc, int8_t* q) {
  constexpr int U = 16;
  const float rscf = __double2float_rn(rsc);
#pragma unroll 1
  for (int j0 = threadIdx.x; j0 < ldq; j0 += U * (int)blockDim.x) {
    float v[U];
#pragma unroll
    for (int u = 0; u < U; u++) {
      const int j = j0 + u * (int)blockDim.x;
      v[u] = j < n ? __ldcg(x + j) : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < U; u++) {
      const int j = j0 + u * (int)blockDim.x;
      if (j < ldq) q[j] = j < n ? dc_quant_div_f(v[u], sc, rsc, rscf) : (int8_t)0;
    }
  }
}

// quant_row_block with the scale from the row maximum *rowmax (float bits,
// written by other CTAs): the maximum is loaded together with the row's first
// values, and thread 0 stores the scale f32(sc) in *s.
__device__ __forceinline__ void quant_row_block_max(const float* x, int n, int ldq, const uint32_t* rowmax,
                                                    int8_t* q, float* s) {
  constexpr int U = 16;
  const uint32_t mb = __ldcg(rowmax);
  double sc = 1.0, rsc = 1.0;
  float rscf = 1.0f;
#pragma unroll 1
  for (int j0 = threadIdx.x, it = 0; j0 < ldq; j0 += U * (int)blockDim.x, it++) {
    float v[U];
#pragma unroll
    for (int u = 0; u < U; u++) {
      const int j = j0 + u * (int)blockDim.x;
      v[u] = j < n ? __ldcg(x + j) : 0.0f;
    }
    if (it == 0) {
      sc = quant_scale(__uint_as_float(mb));
      rsc = __drcp_rn(sc);
      rscf = __double2float_rn(rsc);
      if (threadIdx.x == 0) s[0] = __double2float_rn(sc);
    }
#pragma unroll
    for (int u = 0; u < U; u++) {
      const int j = j0 + u * (int)blockDim.x;
      if (j < ldq) q[j] = j < n ? dc_quant_div_f(v[u], sc, rsc, rscf) : (int8_t)0;
    }
  }
}

// The softmax denominator z (infer.js:100-104: z += e_j in key order, each
// add rounded) as far as the probabilities a_j = f32(f32(e_j) / z) can tell:
// an any-order sum and serial_sum_radius bracket the serial z (non-negative
// terms), each a_j is monotone in z, so when every a_j is the same at both
// ends of the bracket the lower end gives the serial z's a_j; otherwise the
// block computes the serial-order sum.  `af` holds f32(e_j).
__device__ __forceinline__ double softmax_z(const double* e, const float* af, int n, dco::Smem& osm, double2* redd2,
                                            int* vote) {
  double part = 0.0, wpart = 0.0;
  for (int j = threadIdx.x; j < n; j += blockDim.x) {
    part += e[j];
    wpart += (double)(n - j) * e[j];
  }
  const double2 zw = block_sum_d2(part, wpart, redd2);
  const double h = serial_sum_radius(zw.x, zw.y, (n + (int)blockDim.x - 1) / (int)blockDim.x + 10);
  const double zp = zw.x, zlo = zp - h, zhi = zp + h;
  const double rlo = __drcp_rn(zlo), rhi = __drcp_rn(zhi);
  bool amb = false;
  for (int j = threadIdx.x; j < n && !amb; j += blockDim.x)
    amb |= dc_div_to_f32((double)af[j], zlo, rlo) != dc_div_to_f32((double)af[j], zhi, rhi);
  const bool wamb = __any_sync(0xffffffffu, amb);
  if ((threadIdx.x & 31) == 0) vote[threadIdx.x >> 5] = wamb ? 1 : 0;
  __syncthreads();
  bool any = false;
  for (int w = 0; w < (int)(blockDim.x >> 5); w++) any |= vote[w] != 0;
  __syncthreads();
  return any ? ordered_sum_cold(e, n, osm) : zlo;
}

// RoPE on the q and k parts of the fused QKV output row, quantisation of each
// rotated key (per kv head, quantizeCols rule), append of keys and values to
// the cache at row n0 + t, and the running per-channel |v| maximum.
// grid (ceil(T / R), nH + nKV + kvDim / 64), block 64, R rows per block:
// block y < nH rotates query head y in place;
// nH <= y < nH + nKV rotates key head y - nH, quantises it and appends it;
// the last block appends the value row and folds |v| into the channel maxima
// (vmax null: only appends).
template <int R>
__global__ void __launch_bounds__(64) k_rope_append(float* h, int nqkv, int nH, int nKV, int hd,
                                                    const float* rc, const float* rsn,
                                                    const int* n0p, int max_pos,
                                                    int8_t* k8, float* ks,
                                                    float* vcache, uint32_t* vmax,
                                                    float* vs, int* vchg,
                                                    int8_t* v8t, int ldp, int* status, float* vt, int ldvt,
                                                    int T) {
  // The decode attention after this kernel reads the cache's older keys and
  // int8 values before its own grid-dependency wait.  Its launch is released
  // only once this kernel has passed its wait, so every earlier kernel -- the
  // previous step's attention, which rewrites the rows of moved value channels,
  // among them -- has completed by then (each kernel of the chain waits for its
  // predecessor before it completes).
  // The position counter is set before the step's first kernel and the RoPE
  // tables are constant: this thread's first table entries (one per row of
  // the block) are read before the wait, so their round trips overlap the
  // kernel in front.  A block takes rows t0 .. t0 + R - 1 (below T).
  const int n0 = *n0p;  // cached tokens before this chunk = its first position
  const int t0 = blockIdx.x * R, hh = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int half = hd >> 1, qDim = nH * hd, kvDim = nKV * hd;
  const bool rot = hh < nH + nKV && tid < half;
  double c_first[R], s_first[R];
#pragma unroll
  for (int rr = 0; rr < R; rr++) {
    const bool ok = rot && t0 + rr < T;
    const int64_t p = n0 + t0 + rr;
    c_first[rr] = ok ? (double)rc[p * half + tid] : 0.0;
    s_first[rr] = ok ? (double)rsn[p * half + tid] : 0.0;
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");  // launched as a programmatic dependent
  asm volatile("griddepcontrol.launch_dependents;");
  __shared__ float kr[R][128];
  __shared__ float red[R][2];
  bool bad = false;
  if (hh >= nH + nKV) {
    // values, 64 channels per block: copy and fold into the running channel
    // maximum; with one row (vs != null) also the channel scales, their change
    // flags and the row's int8 values, which otherwise k_vscale and k_vquant*
    // compute once every row is in
    const int c = (hh - nH - nKV) * 64 + tid;
    if (c < kvDim) {
#pragma unroll
      for (int rr = 0; rr < R; rr++) {
        const int t = t0 + rr;
        if (t >= T) break;
        const float v = h[(int64_t)t * nqkv + qDim + kvDim + c];
        bad |= !isfinite(v);
        vcache[(int64_t)(n0 + t) * kvDim + c] = v;
        vt[(int64_t)c * ldvt + n0 + t] = v;
        if (vs) {  // (one row)
          const uint32_t m = max(vmax[c], __float_as_uint(fabsf(v)));
          vmax[c] = m;
          const float ns = __double2float_rn(quant_scale(__uint_as_float(m)));
          vchg[c] = n0 == 0 || ns != vs[c];
          vs[c] = ns;
          // the new row's int8 value (channel-major); older rows move only when
          // the channel's scale did (k_vquant_dev)
          v8t[(int64_t)c * ldp + n0] = dc_clamp8(dc_js_round(dc_ddiv_slow((double)v, (double)ns)));
        } else if (vmax) {  // (a pass of several chunks: k_vscale_chunks folds them per chunk)
          atomicMax(vmax + c, __float_as_uint(fabsf(v)));
        }
      }
    }
    if (bad) atomicOr(status, DC_ST_NONFINITE);
    return;
  }
  const bool isq = hh < nH;
#pragma unroll
  for (int rr = 0; rr < R; rr++) {
    const int t = t0 + rr;
    if (t >= T) break;
    const int64_t p = n0 + t;
    float* row = h + (int64_t)t * nqkv;
    float* o = isq ? row + hh * hd : row + qDim + (hh - nH) * hd;
    for (int i = tid; i < half; i += 64) {
      const bool first = i == tid;
      const double c = first ? c_first[rr] : (double)rc[p * half + i];
      const double s = first ? s_first[rr] : (double)rsn[p * half + i];
      const double a = o[i], b = o[half + i];
      const float na = __double2float_rn(__dsub_rn(__dmul_rn(a, c), __dmul_rn(b, s)));
      const float nb = __double2float_rn(__dadd_rn(__dmul_rn(b, c), __dmul_rn(a, s)));
      if (isq) {
        o[i] = na;
        o[half + i] = nb;
      } else {
        kr[rr][i] = na;
        kr[rr][half + i] = nb;
      }
    }
  }
  if (isq) return;
  __syncthreads();
  // each rotated key: absmax over hd (all the block's rows in one exchange), f32
  // scale (quantizeCols rule), int8 row
  float mx[R];
#pragma unroll
  for (int rr = 0; rr < R; rr++) {
    mx[rr] = 0.0f;
    if (t0 + rr < T)
      for (int c = tid; c < hd; c += 64) {
        const float v = kr[rr][c];
        bad |= !isfinite(v);
        mx[rr] = fmaxf(mx[rr], fabsf(v));
      }
#pragma unroll
    for (int o = 16; o; o >>= 1) mx[rr] = fmaxf(mx[rr], __shfl_xor_sync(0xffffffffu, mx[rr], o));
    if (lane == 0) red[rr][warp] = mx[rr];
  }
  __syncthreads();
  const int g = hh - nH;
#pragma unroll
  for (int rr = 0; rr < R; rr++) {
    const int t = t0 + rr;
    if (t >= T) break;
    const float sc = __double2float_rn(quant_scale(fmaxf(red[rr][0], red[rr][1])));
    const int64_t slot = (int64_t)g * max_pos + n0 + t;
    if (tid == 0) ks[slot] = sc;
    const double rsc = __drcp_rn((double)sc);
    for (int c = tid; c < hd; c += 64) k8[slot * hd + c] = dc_quant_div((double)kr[rr][c], (double)sc, rsc);
  }
  if (bad) atomicOr(status, DC_ST_NONFINITE);
}

// Channel scales of V over all cached tokens; flags the channels whose scale moved.
__global__ void k_vscale(const uint32_t* vmax, float* vs, int* vchg,
                         int kvDim, const int* n0p) {
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");  // launched as a programmatic dependent
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= kvDim) return;
  const int fresh = *n0p == 0;
  const float ns = __double2float_rn(quant_scale(__uint_as_float(vmax[c])));
  vchg[c] = fresh || ns != vs[c];
  vs[c] = ns;
}

// int8 V under the channel scales, stored channel-major ([kv head][channel][ldp]
// so a context dot product streams contiguous bytes): rows >= n0 always, older
// rows only in channels whose scale moved.  One tile of 64 rows (from jb) x 32
// channels (from cb) on 256 threads (32 channels x 8 rows), transposed through
// shared memory.
__device__ __forceinline__ void vquant_tile(const float* vcache, const float* vs, const int* vchg, int8_t* v8t,
                                            int N, int n0, int kvDim, int hd, int ldp, int jb, int cb) {
  __shared__ int8_t tile[32][65];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int c = cb + tx;
  const bool cval = c < kvDim;
  const bool chg = cval && vchg[c] != 0;
  const double sc = cval ? (double)vs[c] : 1.0, rsc = __drcp_rn(sc);
  const float rscf = __double2float_rn(rsc);
  for (int r = ty; r < 64; r += 8) {
    const int j = jb + r;
    int8_t v = 0;
    if (cval && j < N && (j >= n0 || chg)) v = dc_quant_div_f(vcache[(int64_t)j * kvDim + c], sc, rsc, rscf);
    tile[tx][r] = v;
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < 32 * 64; idx += blockDim.x) {
    const int cl = idx >> 6, r = idx & 63;
    const int cc = cb + cl, j = jb + r;
    if (cc >= kvDim || j >= N) continue;
    if (j < n0 && !vchg[cc]) continue;  // an unchanged channel keeps its int8 rows
    const int g = cc / hd, ch = cc - g * hd;
    v8t[((int64_t)g * hd + ch) * ldp + j] = tile[cl][r];
  }
}

// grid (ceil(N/64), ceil(kvDim/32)), block 256: vquant_tile over rows 0..N-1.
__global__ void __launch_bounds__(256) k_vquant(const float* vcache, const float* vs,
                                                const int* vchg, int8_t* v8t, int N, int n0,
                                                int kvDim, int hd, int ldp) {
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");  // launched as a programmatic dependent
  vquant_tile(vcache, vs, vchg, v8t, N, n0, kvDim, hd, ldp, blockIdx.x * 64, blockIdx.y * 32);
}

// A pass of several consecutive chunks (dc_stage_forward_chunks): G chunks,
// chunk g holding rows [end[g-1], end[g]) of the pass (end[-1] = 0).
struct ChunkSet {
  int G;
  int end[DC_MAX_CHUNKS];
};

// The value channel scales as of each chunk's last row (the per-column scales
// of vh in infer.js:186-196 are taken over the cache as it stands after that
// chunk's append): per channel, the running |v| maximum folded over the pass's
// rows one chunk at a time; chunk g's scale and its change flag against the
// cache's current scale go to vsg/vchgg[g], and the last chunk's become the
// cache's (vmax, vs, vchg).  grid ceil(kvDim/32), block 32 x DC_MAX_CHUNKS:
// warp g takes chunk g's rows for the block's 32 channels (lane = channel).
__global__ void __launch_bounds__(32 * DC_MAX_CHUNKS) k_vscale_chunks(const float* vcache, uint32_t* vmax,
                                                                     float* vs, int* vchg, int kvDim,
                                                                     const int* n0p, ChunkSet cks, float* vsg,
                                                                     int* vchgg) {
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");  // launched as a programmatic dependent
  __shared__ uint32_t cm[DC_MAX_CHUNKS][32];  // [chunk][channel]: |v| maxima of the chunk's rows
  const int lane = threadIdx.x & 31, gw = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + lane;
  const int n0 = *n0p;
  if (gw < cks.G) {
    uint32_t m = 0;
    const int rb = gw ? cks.end[gw - 1] : 0, re = cks.end[gw];
    if (c < kvDim) {
      const float* vc = vcache + (int64_t)(n0 + rb) * kvDim + c;
#pragma unroll 4
      for (int r = 0; r < re - rb; r++) m = max(m, __float_as_uint(fabsf(__ldcg(vc + (int64_t)r * kvDim))));
    }
    cm[gw][lane] = m;
  }
  __syncthreads();
  if (gw != 0 || c >= kvDim) return;
  const int fresh = n0 == 0;
  const float prior = vs[c];
  uint32_t m = vmax[c];
  float ns = prior;
  int chg = 0;
  for (int g = 0; g < cks.G; g++) {
    m = max(m, cm[g][lane]);
    ns = __double2float_rn(quant_scale(__uint_as_float(m)));
    chg = fresh || ns != prior;
    vsg[g * kvDim + c] = ns;
    vchgg[g * kvDim + c] = chg;
  }
  vmax[c] = m;
  vs[c] = ns;
  vchg[c] = chg;
}

// The int8 values each chunk of a pass attends with.  Blocks below `ntiles`:
// the last chunk's into the cache (its new rows, and older rows in channels
// whose scale moved), one 64-row x 32-channel tile each, as k_vquant.  The
// blocks after them: chunk g < G-1 (blockIdx / 8 ... ) for 8 channels, one
// warp per channel: a channel whose scale at chunk g's end is not the final
// one gets chunk g's int8 row (every position up to the chunk's end) in the
// pass buffer v8s[g]; every other channel of chunk g reads the cache's rows,
// so its warp returns at once.  grid ntiles + (G - 1) * ceil(kvDim / 8), 256
// threads.  The moved rows read the channel-major f32 copy (contiguous).
__global__ void __launch_bounds__(256) k_vquant_chunks(const float* vcache, const float* vs, const int* vchg,
                                                       int8_t* v8t, int n0, int kvDim, int hd, int ldp,
                                                       ChunkSet cks, const float* vsg, int8_t* v8s, int ntiles,
                                                       const float* vt, int ldvt) {
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");  // launched as a programmatic dependent
  const int N = n0 + cks.end[cks.G - 1];
  const int b = blockIdx.x;
  if (b < ntiles) {
    const int nrt = (N + 63) / 64;
    vquant_tile(vcache, vs, vchg, v8t, N, n0, kvDim, hd, ldp, (b % nrt) * 64, (b / nrt) * 32);
    return;
  }
  const int cgroups = (kvDim + 7) / 8;
  const int g = (b - ntiles) / cgroups;
  const int c = ((b - ntiles) % cgroups) * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (c >= kvDim) return;
  const float sg = vsg[(int64_t)g * kvDim + c];
  if (sg == vs[c]) return;  // (warp-uniform)
  const int Ng = n0 + cks.end[g];
  const double sc = (double)sg, rsc = __drcp_rn(sc);
  const float rscf = __double2float_rn(rsc);
  int8_t* dst = v8s + ((int64_t)g * kvDim + c) * ldp;
#pragma unroll 4
  for (int j = lane; j < Ng; j += 32) dst[j] = dc_quant_div_f(__ldcg(vt + (int64_t)c * ldvt + j), sc, rsc, rscf);
}

// The tiled quantisation for short chunks and decode steps, reading the cache
// length from device memory: grid (ceil(max_pos/128), ceil(kvDim/32)) tiles of
// 128 rows x 32 channels.  A tile with no channel whose scale moved and no new
// row to write exits at once (for one-row steps, fresh_done = 1, the append
// already wrote the new row); the others quantise and transpose like k_vquant.
__global__ void __launch_bounds__(256) k_vquant_dev(const float* vcache, const float* vs,
                                                    const int* vchg, int8_t* v8t, int T,
                                                    const int* n0p, int kvDim, int hd, int ldp,
                                                    int fresh_done) {
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");  // launched as a programmatic dependent
  __shared__ int8_t tile[32][129];
  const int n0 = *n0p, N = n0 + T;
  const int cb = blockIdx.y * 32, jb = blockIdx.x * 128;
  if (jb >= N) return;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int c = cb + tx;
  const bool cval = c < kvDim;
  const bool chg = cval && vchg[c] != 0;
  // rows >= n0 still to write in this tile (unless the one-row append wrote them)
  const bool fresh_rows = !fresh_done && jb + 128 > n0;
  // every warp holds the same 32 channels, so this warp vote is block-uniform
  if (!fresh_rows && !__any_sync(0xffffffffu, chg)) return;
  const double sc = cval ? (double)vs[c] : 1.0, rsc = __drcp_rn(sc);
#pragma unroll
  for (int r = ty; r < 128; r += 8) {  // 16 rows per thread, loads in flight together
    const int j = jb + r;
    int8_t v = 0;
    if (cval && j < N && (chg || (!fresh_done && j >= n0)))
      v = dc_quant_div((double)vcache[(int64_t)j * kvDim + c], sc, rsc);
    tile[tx][r] = v;
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < 32 * 128; idx += blockDim.x) {
    const int cl = idx >> 7, r = idx & 127;
    const int cc = cb + cl, j = jb + r;
    if (cc >= kvDim || j >= N) continue;
    if (!vchg[cc] && (fresh_done || j < n0)) continue;
    v8t[(int64_t)cc * ldp + j] = tile[cl][r];
  }
}

__global__ void k_setpos(int* p, int v) { *p = v; }
__global__ void k_addpos(int* p, int v) { *p += v; }

__device__ __forceinline__ int dp4a16(const int4 a, const int4 b, int acc) {
  acc = __dp4a(a.x, b.x, acc);
  acc = __dp4a(a.y, b.y, acc);
  acc = __dp4a(a.z, b.z, acc);
  return __dp4a(a.w, b.w, acc);
}

// One (query head, query row): scores, causal softmax, context.  N = n0 + T.
// Scores: hd/16 lanes per key, 16-byte loads of the int8 key row, shuffle sum.
// Context: one warp per output channel, lanes stream 16-byte chunks of that
// channel's int8 values (channel-major cache) against the int8 probabilities.
__global__ void __launch_bounds__(ATT_THREADS, 4) k_attention(const float* h, int nqkv, int nH, int nKV,
                                                           int hd, const int8_t* k8,
                                                           const float* ks,
                                                           const int8_t* v8t,
                                                           const float* vs, int T,
                                                           const int* n0p, int max_pos,
                                                           int ldp, double scale, float* out,
                                                           uint32_t* rowmax, int qDim,
                                                           int* status, int8_t* a8g = nullptr,
                                                           float* asg = nullptr) {
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");  // launched as a programmatic dependent
  extern __shared__ __align__(16) uint8_t sm[];
  double* ed = (double*)sm;                                 // max_pos doubles: e_j
  float* af = (float*)(ed + max_pos);                       // max_pos floats: scores, then a_j
  int8_t* a8 = (int8_t*)(sm + ((12 * (size_t)max_pos + 15) & ~(size_t)15));  // ldp int8, 16-byte aligned
  __shared__ __align__(16) int8_t q8[128];
  __shared__ float red[32];
  __shared__ double2 redd2[32];  // also the 32 doubles of block_max_d / block_sum_d
  double* redd = reinterpret_cast<double*>(redd2);
  __shared__ int vote[32];
  __shared__ dco::Smem osm;
  const int hq = blockIdx.x, i = blockIdx.y;
  const int group = nH / nKV, g = hq / group;
  const int n0 = *n0p;
  const int see = n0 + i;  // this query's own position in the cache (keys 0..see are visible)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  // 1. quantise the query row of this head (row scale per (token, head), double)
  const float* qrow = h + (int64_t)i * nqkv + hq * hd;
  float mx = 0.0f;
  bool bad = false;
  for (int c = threadIdx.x; c < hd; c += blockDim.x) {
    float v = qrow[c];
    bad |= !isfinite(v);
    mx = fmaxf(mx, fabsf(v));
  }
  mx = block_max_f(mx, red);
  const double qsc = quant_scale(mx);
  const float qs = __double2float_rn(qsc);
  const double rqsc = __drcp_rn(qsc);
  for (int c = threadIdx.x; c < hd; c += blockDim.x) q8[c] = dc_quant_div((double)qrow[c], qsc, rqsc);
  __syncthreads();
  // 2. scores for keys 0..see: one key per thread (its 128-byte row in one
  //    line), int32 dot over hd, verified epilogue
  {
    const int8_t* kb = k8 + (int64_t)g * max_pos * hd;
    const float* ksg = ks + (int64_t)g * max_pos;
    const int nchk = hd >> 4;
    const int4* q4 = (const int4*)q8;
    for (int j = threadIdx.x; j <= see; j += blockDim.x) {
      const int4* kr = (const int4*)(kb + (int64_t)j * hd);
      const float kscale = ksg[j];
      int acc = 0;
#pragma unroll 8
      for (int c = 0; c < nchk; c++) acc = dp4a16(kr[c], q4[c], acc);
      af[j] = dc_epi(acc, qs, kscale);
    }
  }
  __syncthreads();
  // 3. row maximum of s*scale (double, exact)
  double m = -INFINITY;
  for (int j = threadIdx.x; j <= see; j += blockDim.x) m = fmax(m, __dmul_rn((double)af[j], scale));
  m = block_max_d(m, redd);
  // 4. e_j and its f32 copy
  for (int j = threadIdx.x; j <= see; j += blockDim.x) {
    const double e = dcm::fdlibm_exp_sel(__dsub_rn(__dmul_rn((double)af[j], scale), m));
    ed[j] = e;
    af[j] = __double2float_rn(e);
  }
  __syncthreads();
  // 5. z: the serial key-order sum, as far as the probabilities can tell
  const double z = softmax_z(ed, af, see + 1, osm, redd2, vote);
  // 6. a_j = f32(a_j / z); 7. quantise the probability row over all N columns
  float amx = 0.0f;
  const double rz = __drcp_rn(z);
  for (int j = threadIdx.x; j <= see; j += blockDim.x) {
    const float a = dc_div_to_f32((double)af[j], z, rz);
    af[j] = a;
    amx = fmaxf(amx, fabsf(a));
  }
  amx = block_max_f(amx, red);
  const double asc = quant_scale(amx), rasc = __drcp_rn(asc);
  const float as = __double2float_rn(asc);
  if (a8g) {
    // split form: the probability row (zero past `see`, up to the chunk's last
    // key) and its scale go to global memory; k_attn_ctx forms the context
    const int nfill = (n0 + T + 15) & ~15;
    int8_t* dst = a8g + ((int64_t)hq * T + i) * ldp;
    for (int j = threadIdx.x; j < nfill; j += blockDim.x) dst[j] = j <= see ? dc_quant_div((double)af[j], asc, rasc) : (int8_t)0;
    if (threadIdx.x == 0) asg[hq * T + i] = as;
    if (bad) atomicOr(status, DC_ST_NONFINITE);
    return;
  }
  const int nchunk = (see + 16) >> 4;  // 16-byte chunks covering keys 0..see
  for (int j = threadIdx.x; j < nchunk * 16; j += blockDim.x)
    a8[j] = j <= see ? dc_quant_div((double)af[j], asc, rasc) : (int8_t)0;
  __syncthreads();
  // 8. ctx[c] = sum_j a8[j] * v8[c][j] over j <= see (a8 is zero past `see`)
  const int4* a4 = (const int4*)a8;
  const int8_t* vg = v8t + (int64_t)g * hd * ldp;
  for (int c0 = warp * 4; c0 < hd; c0 += nwarps * 4) {
    const int4* r0 = (const int4*)(vg + (int64_t)(c0 + 0) * ldp);
    const int4* r1 = (const int4*)(vg + (int64_t)(c0 + 1) * ldp);
    const int4* r2 = (const int4*)(vg + (int64_t)(c0 + 2) * ldp);
    const int4* r3 = (const int4*)(vg + (int64_t)(c0 + 3) * ldp);
    int s0 = 0, s1 = 0, s2 = 0, s3 = 0;
    int q = lane;
    for (; q + 32 < nchunk; q += 64) {  // two chunks of four channels: 8 loads in flight
      const int4 a0 = a4[q], a1 = a4[q + 32];
      const int4 v00 = r0[q], v10 = r1[q], v20 = r2[q], v30 = r3[q];
      const int4 v01 = r0[q + 32], v11 = r1[q + 32], v21 = r2[q + 32], v31 = r3[q + 32];
      s0 = dp4a16(v01, a1, dp4a16(v00, a0, s0));
      s1 = dp4a16(v11, a1, dp4a16(v10, a0, s1));
      s2 = dp4a16(v21, a1, dp4a16(v20, a0, s2));
      s3 = dp4a16(v31, a1, dp4a16(v30, a0, s3));
    }
    for (; q < nchunk; q += 32) {
      const int4 av = a4[q];
      s0 = dp4a16(r0[q], av, s0);
      s1 = dp4a16(r1[q], av, s1);
      s2 = dp4a16(r2[q], av, s2);
      s3 = dp4a16(r3[q], av, s3);
    }
    for (int o = 16; o; o >>= 1) {
      s0 += __shfl_xor_sync(0xffffffffu, s0, o);
      s1 += __shfl_xor_sync(0xffffffffu, s1, o);
      s2 += __shfl_xor_sync(0xffffffffu, s2, o);
      s3 += __shfl_xor_sync(0xffffffffu, s3, o);
    }
    if (lane < 4) {
      const int c = c0 + lane;
      const int acc = lane == 0 ? s0 : lane == 1 ? s1 : lane == 2 ? s2 : s3;
      const float o = dc_epi(acc, as, vs[g * hd + c]);
      out[(int64_t)i * qDim + hq * hd + c] = o;
      bad |= !isfinite(o);
      atomicMax(rowmax + i, __float_as_uint(fabsf(o)));  // for the next GEMM's row quantisation
    }
  }
  if (bad) atomicOr(status, DC_ST_NONFINITE);
}

// The attention of one chunk's query rows (at most 16) for one head, the
// whole of infer.js:174-196 for those rows in one CTA: grid (nH, G) (G chunks
// of a pass, 1 otherwise), AR_THREADS threads, HD the head dim (64, 128 or
// 256).  The rows share every key and value load, and the per-row reductions
// are warp-level:
//  1. warp w quantises query row w (quantizeRows of the head's HD values);
//  2. scores s_ij = epi(q_i . k_j, qs_i, ks_j) by 16-row x 8-key int8
//     tensor-core tiles (mma.sync m16n8k32, int32 accumulators: the dot
//     products are exact), each warp taking every 16th tile, keys read
//     straight from the cache (16 bytes per thread; the bytes a thread gives
//     the A and B fragments are the same physical head-dim positions, so the
//     sum over them is the dot product); s into shared memory, the exact row
//     maximum of s * scale (double) on the way;
//  3. warp w: e_j = exp(s_j * scale - m) (fdlibm method, double) for keys
//     0..see, f32(e_j) kept in place, the bracket of the serial sum z;
//     a_j = f32(f32(e_j) / z) at the lower end of the bracket, checked
//     against the upper end; the row's |a| maximum;
//  4. a row whose a_j depend on where z falls in the bracket (rare) gets the
//     serial key-order z from the whole block (dco::ordered_sum over e_j
//     recomputed in double);
//  5. warp w quantises its a row (quantizeRows over the row's keys; zero past
//     `see`) into shared memory;
//  6. the context ctx_ic = sum_j a8_ij v8_cj by 16-row x 8-channel int8 tiles
//     over the keys (value rows channel-major from the cache, or for a chunk
//     before a pass's last, from the pass buffer in channels whose scale moved
//     after it), verified epilogue with the row's probability scale and the
//     channel's value scale; |ctx| folded into the row maxima.
// Dynamic shared memory: 16 * ldp floats (scores / e / a) + 16 * ldp bytes
// (the int8 probability rows; before them, one row of doubles for step 4).
constexpr int AR_THREADS = 512;
__device__ __forceinline__ void mma_s8_16832(int& c0, int& c1, int& c2, int& c3, unsigned a0, unsigned a1,
                                             unsigned a2, unsigned a3, unsigned b0, unsigned b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(c0), "+r"(c1), "+r"(c2), "+r"(c3)
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// Two m16n8k32 steps over 64 k positions: A rows gi / gi + 8 and the B column
// each give the same 16 physical bytes (64p + 16 ti ..) of their rows.
__device__ __forceinline__ void mma_s8_pair(int* c, const int4& ra, const int4& rb, const int4& kb) {
  mma_s8_16832(c[0], c[1], c[2], c[3], ra.x, rb.x, ra.y, rb.y, kb.x, kb.y);
  mma_s8_16832(c[0], c[1], c[2], c[3], ra.z, rb.z, ra.w, rb.w, kb.z, kb.w);
}

template <int HD>
__global__ void __launch_bounds__(AR_THREADS, 1) k_attn_chunk(const float* h, int nqkv, int nH, int nKV,
                                                             const int8_t* k8, const float* ks,
                                                             const int8_t* v8t, const float* vs, int T,
                                                             const int* n0p, int max_pos, int ldp, double scale,
                                                             float* out, int qDim, uint32_t* rowmax, int* status,
                                                             ChunkSet cks, const int8_t* v8s, const float* vsg) {
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");  // launched as a programmatic dependent
  constexpr int NP = HD / 64;  // pairs of 32-byte k-steps
  constexpr int QLD = HD + 16;
  extern __shared__ __align__(16) uint8_t sm[];
  float* S = (float*)sm;                                  // [16][ldp]
  int8_t* A8 = (int8_t*)(S + (size_t)16 * ldp);           // [16][ldp]
  double* eb = (double*)A8;                               // [ldp] (step 4, before A8 is written)
  __shared__ __align__(16) int8_t q8s[16 * QLD];
  __shared__ float qsf[16], asf[16];
  __shared__ double wm[16][16];  // [warp][row] maxima
  __shared__ float amxs[16];
  __shared__ int ambs[16];
  __shared__ dco::Smem16 osm;
  __shared__ double2 etab[64];  // 2^(j/64) for the table-driven exp (published by the first barrier)
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int hq = blockIdx.x, g = hq / (nH / nKV);
  dcm::exp2_tab_load(etab);
  int r0 = 0, r1 = T;
  const int8_t* vz = nullptr;  // chunk z < G-1 of a pass: its buffer, and its value scales
  const float* vsz = vs;
  if (cks.G > 1) {
    const int z = blockIdx.y;
    r0 = z ? cks.end[z - 1] : 0;
    r1 = cks.end[z];
    if (z < cks.G - 1) {
      vz = v8s + (int64_t)z * nKV * HD * ldp;
      vsz = vsg + (int64_t)z * nKV * HD;
    }
  }
  const int Tc = r1 - r0, n0 = *n0p;
  const int Nc = n0 + r1;  // keys the chunk's last row sees
  // 1. the query rows, quantised (warp w: row w); rows past the chunk are zero
  {
    bool bad = false;
    float v[HD / 32];
    float mx = 0.0f;
    if (warp < Tc) {
      const float* qrow = h + (int64_t)(r0 + warp) * nqkv + hq * HD;
#pragma unroll
      for (int u = 0; u < HD / 32; u++) {
        v[u] = qrow[lane + 32 * u];
        bad |= !isfinite(v[u]);
        mx = fmaxf(mx, fabsf(v[u]));
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const double qsc = quant_scale(mx), rqsc = __drcp_rn(qsc);
#pragma unroll
    for (int u = 0; u < HD / 32; u++)
      q8s[warp * QLD + lane + 32 * u] = warp < Tc ? dc_quant_div((double)v[u], qsc, rqsc) : (int8_t)0;
    if (lane == 0) qsf[warp] = __double2float_rn(qsc);
    if (bad) atomicOr(status, DC_ST_NONFINITE);
  }
  __syncthreads();
  // 2. scores by 16 x 8 tiles
  const int gi = lane >> 2, ti = lane & 3;
  const int see0 = n0 + r0 + gi, see1 = see0 + 8;  // rows gi and gi + 8 see keys 0..see
  int4 QA[NP], QB[NP];
#pragma unroll
  for (int p = 0; p < NP; p++) {
    QA[p] = *(const int4*)(q8s + gi * QLD + 64 * p + 16 * ti);
    QB[p] = *(const int4*)(q8s + (gi + 8) * QLD + 64 * p + 16 * ti);
  }
  const float qs0 = gi < Tc ? qsf[gi] : 0.0f, qs1 = gi + 8 < Tc ? qsf[gi + 8] : 0.0f;
  double m0 = -INFINITY, m1 = -INFINITY;
  const int8_t* kb = k8 + (int64_t)g * max_pos * HD;
  const float* ksg = ks + (int64_t)g * max_pos;
  const int ntile = (Nc + 7) >> 3;
#pragma unroll 2
  for (int tile = warp; tile < ntile; tile += AR_THREADS / 32) {
    const int key = min(tile * 8 + gi, max_pos - 1);
    const int4* kr = (const int4*)(kb + (int64_t)key * HD) + ti;
    int4 kv[NP];
#pragma unroll
    for (int p = 0; p < NP; p++) kv[p] = __ldcg(kr + 4 * p);
    const int j0 = tile * 8 + 2 * ti;
    const float ks0 = ksg[min(j0, max_pos - 1)], ks1 = ksg[min(j0 + 1, max_pos - 1)];
    int c[4] = {0, 0, 0, 0};
#pragma unroll
    for (int p = 0; p < NP; p++) mma_s8_pair(c, QA[p], QB[p], kv[p]);
    const float s00 = dc_epi(c[0], qs0, ks0), s01 = dc_epi(c[1], qs0, ks1);
    const float s10 = dc_epi(c[2], qs1, ks0), s11 = dc_epi(c[3], qs1, ks1);
    *(float2*)(S + (size_t)gi * ldp + j0) = make_float2(s00, s01);
    *(float2*)(S + (size_t)(gi + 8) * ldp + j0) = make_float2(s10, s11);
    if (j0 <= see0) m0 = fmax(m0, __dmul_rn((double)s00, scale));
    if (j0 + 1 <= see0) m0 = fmax(m0, __dmul_rn((double)s01, scale));
    if (j0 <= see1) m1 = fmax(m1, __dmul_rn((double)s10, scale));
    if (j0 + 1 <= see1) m1 = fmax(m1, __dmul_rn((double)s11, scale));
  }
#pragma unroll
  for (int o = 1; o <= 2; o <<= 1) {
    m0 = fmax(m0, __shfl_xor_sync(0xffffffffu, m0, o));
    m1 = fmax(m1, __shfl_xor_sync(0xffffffffu, m1, o));
  }
  if (ti == 0) {
    wm[warp][gi] = m0;
    wm[warp][gi + 8] = m1;
  }
  __syncthreads();
  // 3. warp w: row w's softmax over keys 0..see
  const int row = warp, see = n0 + r0 + row, n = see + 1;
  float* Sr = S + (size_t)row * ldp;
  if (row < Tc) {
    double m = wm[0][row];
#pragma unroll
    for (int w = 1; w < 16; w++) m = fmax(m, wm[w][row]);
    double part = 0.0;
    float wpart = 0.0f;  // sum of (n - j) e_j: only the radius needs it, to well within its 1e-3 slack
    // f32(e_j) as the fdlibm exp rounds it, and e_j within 2^-51 relative of
    // fdlibm's for the sum, from the table-driven exp with no branch in the
    // loop (exp_settle's test, inline).  Below x = -700 both are zero to far
    // within the bracket's radius.  A key whose f32 rounding the bound cannot
    // settle (about one in 2^24) sends its row to the exact path below, which
    // recomputes the whole row with fdlibm.
    bool unsettled = false;
#pragma unroll 4
    for (int j = lane; j < n; j += 32) {
      const double x = __dsub_rn(__dmul_rn((double)Sr[j], scale), m);
      const double t = x >= -700.0 ? dcm::exp_tang(x, etab) : 0.0;
      const float ef = __double2float_rn(__dmul_rn(t, 1.0 - 0x1p-49));
      unsettled |= ef != __double2float_rn(__dmul_rn(t, 1.0 + 0x1p-49));
      Sr[j] = ef;
      part += t;
      wpart = __fadd_rn(wpart, __fmul_rn((float)(n - j), ef));
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      part += __shfl_xor_sync(0xffffffffu, part, o);
      wpart += __shfl_xor_sync(0xffffffffu, wpart, o);
    }
    // a term passes through at most ceil(n / 32) adds in its lane and 5 in the
    // warp; the radius also covers the terms' distance from fdlibm's (2^-51
    // relative each, taken as 2^-48 of the sum)
    const double hr = __dadd_rn(serial_sum_radius(part, (double)wpart, (n + 31) / 32 + 10), __dmul_rn(0x1p-48, part));
    const double zlo = part - hr, zhi = part + hr;
    const double rlo = __drcp_rn(zlo), rhi = __drcp_rn(zhi);
    const bool narrow = __dsub_rn(zhi, zlo) < 5e-13 * zlo;
    bool amb = false;
    float amx = 0.0f;
#pragma unroll 4
    for (int j = lane; j < n; j += 32) {
      const float a = dc_div_bracket((double)Sr[j], zlo, rlo, zhi, rhi, narrow, &amb);
      Sr[j] = a;
      amx = fmaxf(amx, a);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) amx = fmaxf(amx, __shfl_xor_sync(0xffffffffu, amx, o));
    const bool wamb = __any_sync(0xffffffffu, amb || unsettled);
    if (lane == 0) {
      amxs[row] = amx;
      ambs[row] = wamb ? 1 : 0;
      wm[0][row] = m;  // (kept for the exact path)
    }
  } else if (lane == 0) {
    ambs[row] = 0;
  }
  __syncthreads();
  // 4. rows whose probabilities the bracket cannot settle: the serial z
#pragma unroll 1
  for (int i = 0; i < Tc; i++) {
    if (!ambs[i]) continue;  // (block-uniform)
    const int ni = n0 + r0 + i + 1;
    const double m = wm[0][i];
    const int4* q4 = (const int4*)(q8s + i * QLD);
    for (int j = tid; j < ni; j += AR_THREADS) {
      const int4* kr = (const int4*)(kb + (int64_t)j * HD);
      int acc = 0;
#pragma unroll
      for (int cc = 0; cc < HD / 16; cc++) acc = dp4a16(kr[cc], q4[cc], acc);
      eb[j] = dcm::fdlibm_exp_sel(__dsub_rn(__dmul_rn((double)dc_epi(acc, qsf[i], ksg[j]), scale), m));
    }
    __syncthreads();
    const double z = ordered_sum_cold16(eb, ni, osm);
    const double rz = __drcp_rn(z);
    float amx = 0.0f;
    float* Si = S + (size_t)i * ldp;
    for (int j = tid; j < ni; j += AR_THREADS) {
      const float a = dc_div_to_f32((double)__double2float_rn(eb[j]), z, rz);
      Si[j] = a;
      amx = fmaxf(amx, fabsf(a));
    }
    amx = block_max_f(amx, (float*)wm[1]);  // (32 floats of scratch)
    if (tid == 0) amxs[i] = amx;
    __syncthreads();
  }
  // 5. each probability row quantised into A8 (zero past `see`, up to Kc)
  const int Kc = (Nc + 63) & ~63;  // keys of the context's k-steps (ldp is a multiple of 64)
  if (row < Tc) {
    const double asc = quant_scale(amxs[row]), rasc = __drcp_rn(asc);
    const float rascf = __double2float_rn(rasc);
    uint32_t* dst = (uint32_t*)(A8 + (size_t)row * ldp);
    for (int j4 = lane; j4 < (Kc >> 2); j4 += 32) {
      const float4 a = *(const float4*)(Sr + 4 * j4);
      const int j = 4 * j4;
      const uint32_t b0 = j <= see ? (uint8_t)dc_quant_div_f(a.x, asc, rasc, rascf) : 0u;
      const uint32_t b1 = j + 1 <= see ? (uint8_t)dc_quant_div_f(a.y, asc, rasc, rascf) : 0u;
      const uint32_t b2 = j + 2 <= see ? (uint8_t)dc_quant_div_f(a.z, asc, rasc, rascf) : 0u;
      const uint32_t b3 = j + 3 <= see ? (uint8_t)dc_quant_div_f(a.w, asc, rasc, rascf) : 0u;
      dst[j4] = b0 | (b1 << 8) | (b2 << 16) | (b3 << 24);
    }
    if (lane == 0) asf[row] = __double2float_rn(asc);
  } else {
    uint32_t* dst = (uint32_t*)(A8 + (size_t)row * ldp);
    for (int j4 = lane; j4 < (Kc >> 2); j4 += 32) dst[j4] = 0u;
  }
  __syncthreads();
  // 6. the context by 16 x 8 tiles over the keys (64 per step pair)
  constexpr int NT = HD / 8;                     // channel tiles
  constexpr int TPW = NT > 16 ? NT / 16 : 1;      // tiles per warp
  constexpr int KS = NT < 16 ? 16 / NT : 1;       // key splits (warps sharing a tile)
  const int tile0 = warp % (16 / KS), sp = warp / (16 / KS);
  const int npair = Kc >> 6, per = (npair + KS - 1) / KS;
  const int p0 = sp * per, p1 = min(npair, p0 + per);
  int acc[TPW][4];
  const int4* vrow[TPW];
#pragma unroll
  for (int u = 0; u < TPW; u++) {
    acc[u][0] = acc[u][1] = acc[u][2] = acc[u][3] = 0;
    const int cc = g * HD + (tile0 + 16 * u) * 8 + gi;  // this lane's B channel
    const int8_t* src = (vz && vsz[cc] != vs[cc]) ? vz : v8t;
    vrow[u] = (const int4*)(src + (int64_t)cc * ldp) + ti;
  }
  const int4* ar = (const int4*)(A8 + (size_t)gi * ldp) + ti;
  const int4* br = (const int4*)(A8 + (size_t)(gi + 8) * ldp) + ti;
#pragma unroll 2
  for (int p = p0; p < p1; p++) {
    const int4 ra = ar[4 * p], rb = br[4 * p];
#pragma unroll
    for (int u = 0; u < TPW; u++) mma_s8_pair(acc[u], ra, rb, __ldcg(vrow[u] + 4 * p));
  }
  if (KS > 1) {  // the other key splits' partial sums into split 0 (exact int32)
    int* red = (int*)S;  // [split][tile][lane][4] (the score rows are free now)
    if (sp > 0)
      *(int4*)(red + (((sp - 1) * 16 + tile0) * 32 + lane) * 4) = make_int4(acc[0][0], acc[0][1], acc[0][2], acc[0][3]);
    __syncthreads();
    if (sp == 0) {
      for (int q = 1; q < KS; q++) {
        const int4 o = *(const int4*)(red + (((q - 1) * 16 + tile0) * 32 + lane) * 4);
        acc[0][0] += o.x;
        acc[0][1] += o.y;
        acc[0][2] += o.z;
        acc[0][3] += o.w;
      }
    }
  }
  if (sp == 0) {
    bool bad = false;
    float x0 = 0.0f, x1 = 0.0f;  // |ctx| maxima of rows gi, gi + 8
    const float as0 = gi < Tc ? asf[gi] : 0.0f, as1 = gi + 8 < Tc ? asf[gi + 8] : 0.0f;
#pragma unroll
    for (int u = 0; u < TPW; u++) {
      const int c = (tile0 + 16 * u) * 8 + 2 * ti;
      const float vc0 = vsz[g * HD + c], vc1 = vsz[g * HD + c + 1];
      if (gi < Tc) {
        const float o0 = dc_epi(acc[u][0], as0, vc0), o1 = dc_epi(acc[u][1], as0, vc1);
        *(float2*)(out + (int64_t)(r0 + gi) * qDim + hq * HD + c) = make_float2(o0, o1);
        bad |= !isfinite(o0) || !isfinite(o1);
        x0 = fmaxf(x0, fmaxf(fabsf(o0), fabsf(o1)));
      }
      if (gi + 8 < Tc) {
        const float o0 = dc_epi(acc[u][2], as1, vc0), o1 = dc_epi(acc[u][3], as1, vc1);
        *(float2*)(out + (int64_t)(r0 + gi + 8) * qDim + hq * HD + c) = make_float2(o0, o1);
        bad |= !isfinite(o0) || !isfinite(o1);
        x1 = fmaxf(x1, fmaxf(fabsf(o0), fabsf(o1)));
      }
    }
#pragma unroll
    for (int o = 1; o <= 2; o <<= 1) {
      x0 = fmaxf(x0, __shfl_xor_sync(0xffffffffu, x0, o));
      x1 = fmaxf(x1, __shfl_xor_sync(0xffffffffu, x1, o));
    }
    if (ti == 0 && gi < Tc) atomicMax(rowmax + r0 + gi, __float_as_uint(x0));
    if (ti == 0 && gi + 8 < Tc) atomicMax(rowmax + r0 + gi + 8, __float_as_uint(x1));
    if (bad) atomicOr(status, DC_ST_NONFINITE);
  }
}

// The context of a chunk's T rows for 32 channels of one head, from the
// probability rows k_attention wrote (split form): grid (nH, hd / 32, G), 256
// threads; ctx[t][c] = sum_j a8[t][j] * v8[c][j] (exact int32), verified
// epilogue with the row's probability scale and the channel's value scale.
// The 32 value rows and the chunk's probability rows land in shared memory by
// 1-D bulk copies.  Dynamic shared memory: (32 + 16) * ldp.  In a pass of
// several chunks (cks.G > 1) CTA z forms chunk z's rows (at most 16) with the
// values and scales of that chunk (v8s/vsg, the cache's for the last chunk).
__global__ void __launch_bounds__(256) k_attn_ctx(const int8_t* a8g, const float* asg,
                                                  const int8_t* v8t, const float* vs,
                                                  int nH, int nKV, int hd, int T, const int* n0p,
                                                  int ldp, float* out, int qDim,
                                                  uint32_t* rowmax, int* status,
                                                  ChunkSet cks, const int8_t* v8s, const float* vsg) {
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");  // launched as a programmatic dependent
  extern __shared__ __align__(16) uint8_t sm[];
  int8_t* sV = (int8_t*)sm;              // 32 x ldp
  int8_t* sA = sV + (size_t)32 * ldp;     // Tc x ldp
  __shared__ __align__(8) uint64_t bar;
  __shared__ float sas[16];
  const int hq = blockIdx.x, c0 = blockIdx.y * 32;
  const int g = hq / (nH / nKV);
  const int tid = threadIdx.x;
  int r0 = 0, r1 = T;  // this CTA's rows
  const int8_t* vsrc = v8t;  // this thread's value row (tid < 32: channel c0 + tid)
  if (cks.G > 1) {
    const int z = blockIdx.z;
    r0 = z ? cks.end[z - 1] : 0;
    r1 = cks.end[z];
    if (z < cks.G - 1) {
      const float* vz = vsg + (int64_t)z * nKV * hd;
      const int cc = g * hd + c0 + (tid & 31);
      if (vz[cc] != vs[cc]) vsrc = v8s + (int64_t)z * nKV * hd * ldp;  // a channel whose scale moved later
      vs = vz;
    }
  }
  const int Tc = r1 - r0;
  const int nfill = (*n0p + r1 + 15) & ~15;  // bytes of each row in use
  if (tid == 0) {
    dcp::mbar_init(&bar, 1);
    dcp::mbar_fence_init();
  }
  __syncthreads();
  if (tid < 32) {
    if (tid == 0) dcp::mbar_expect_tx(&bar, (uint32_t)((32 + Tc) * nfill));
    __syncwarp();
    dcp::bulk_load(sV + (size_t)tid * ldp, vsrc + ((int64_t)g * hd + c0 + tid) * ldp, (uint32_t)nfill, &bar);
    if (tid < Tc)
      dcp::bulk_load(sA + (size_t)tid * ldp, a8g + ((int64_t)hq * T + r0 + tid) * ldp, (uint32_t)nfill, &bar);
  }
  if (tid < Tc) sas[tid] = asg[hq * T + r0 + tid];
  const bool ok = dcp::mbar_wait(&bar, 0, status);
  __syncthreads();
  if (!ok) return;
  const int cl = tid >> 3, tg = tid & 7;  // channel c0 + cl; rows tg and tg + 8 of the chunk
  const int t0 = tg, t1 = tg + 8;
  const int4* vr = (const int4*)(sV + (size_t)cl * ldp);
  const int4* ar0 = (const int4*)(sA + (size_t)(t0 < Tc ? t0 : 0) * ldp);
  const int4* ar1 = (const int4*)(sA + (size_t)(t1 < Tc ? t1 : 0) * ldp);
  int s0 = 0, s1 = 0;
  for (int q = 0; q < (nfill >> 4); q++) {
    const int4 v = vr[q];
    s0 = dp4a16(v, ar0[q], s0);
    s1 = dp4a16(v, ar1[q], s1);
  }
  const int c = c0 + cl;
  const float vsc = vs[g * hd + c];
  bool bad = false;
  if (t0 < Tc) {
    const float o = dc_epi(s0, sas[t0], vsc);
    out[(int64_t)(r0 + t0) * qDim + hq * hd + c] = o;
    bad |= !isfinite(o);
    atomicMax(rowmax + r0 + t0, __float_as_uint(fabsf(o)));
  }
  if (t1 < Tc) {
    const float o = dc_epi(s1, sas[t1], vsc);
    out[(int64_t)(r0 + t1) * qDim + hq * hd + c] = o;
    bad |= !isfinite(o);
    atomicMax(rowmax + r0 + t1, __float_as_uint(fabsf(o)));
  }
  if (bad) atomicOr(status, DC_ST_NONFINITE);
}

// Attention of one decode row (T = 1) against the whole cache, split over
// channel groups: grid (nH, hd / CH), 256 threads.  Every CTA of a head
// computes the head's scores and probabilities (the same numbers as
// k_attention: scores, exact max, fdlibm exp, the serial softmax sum,
// quantizeRows of the probabilities) and then CH channels of the context.
// The keys stream through a three-slot shared-memory ring of 256-key blocks,
// and the CTA's CH value rows (channel-major) land in shared memory once, all
// by 1-D bulk async copies, so the loads are in flight while the softmax runs.
// Dynamic shared memory: 3 * 256 * hd (keys) + CH * ldp (values) + 13 * ldp.
// hd is 32, 64, 128 or 256; CH divides hd.
constexpr int ATTD_KB = 256;  // keys per ring slot
constexpr int ATTD_NS = 3;    // ring slots (two blocks in flight while one is consumed)
__global__ void __launch_bounds__(256) k_attention_dec(const float* h, int nqkv, int nH, int nKV, int hd,
                                                       const int8_t* k8, const float* ks,
                                                       const int8_t* v8t, const float* vs,
                                                       const int* n0p, int max_pos, int ldp, int CH,
                                                       double scale, float* out,
                                                       uint32_t* rowmax, int* done,
                                                       int8_t* xq, int ldq, float* rsq,
                                                       int* status) {
  extern __shared__ __align__(16) uint8_t sm[];
  asm volatile("griddepcontrol.launch_dependents;");  // the O projection may start streaming its weights
  asm volatile("griddepcontrol.wait;" ::: "memory");  // launched as a programmatic dependent
  const int ldpv = ldp;                                        // bytes per value row in shared memory
  int8_t* sK = (int8_t*)sm;                                    // ATTD_NS slots x ATTD_KB x hd
  int8_t* sV = sK + ATTD_NS * ATTD_KB * hd;                    // CH x ldpv
  double* xs = (double*)(sV + (size_t)CH * ldpv);              // ldp doubles: s*scale, then e
  float* af = (float*)(xs + ldp);                              // ldp floats: key scales, then f32(e), then a
  int8_t* a8 = (int8_t*)(af + ldp);                            // ldp bytes
  __shared__ __align__(8) uint64_t full[ATTD_NS], vbar;
  __shared__ __align__(16) int8_t q8[256];
  __shared__ float red[32];
  __shared__ double2 redd2[32];  // also the 32 doubles of block_max_d / block_sum_d
  double* redd = reinterpret_cast<double*>(redd2);
  __shared__ int vote[32];
  __shared__ int abort_flag;
  __shared__ dco::Smem osm;
  const int hq = blockIdx.x, c0 = blockIdx.y * CH;
  const int g = hq / (nH / nKV);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n0 = *n0p, N = n0 + 1;            // keys 0..n0 are visible
  const int ldpN = (N + 15) & ~15;            // 16-byte chunks covering the keys
  const int nb = (N + ATTD_KB - 1) / ATTD_KB;  // key blocks
  const int8_t* kg = k8 + (int64_t)g * max_pos * hd;
  if (tid == 0) {
    for (int i = 0; i < ATTD_NS; i++) dcp::mbar_init(&full[i], 1);
    dcp::mbar_init(&vbar, 1);
    abort_flag = 0;
    dcp::mbar_fence_init();
  }
  __syncthreads();
  int issued[ATTD_NS];  // thread 0: last key block issued into each slot
  for (int i = 0; i < ATTD_NS; i++) issued[i] = -1;
  if (warp == 0) {  // issue: the CH value rows, then the first ATTD_NS key blocks
    if (lane == 0) dcp::mbar_expect_tx(&vbar, (uint32_t)(CH * ldpN));
    __syncwarp();
    for (int c = lane; c < CH; c += 32)
      dcp::bulk_load(sV + (size_t)c * ldpv, v8t + ((int64_t)g * hd + c0 + c) * ldp, (uint32_t)ldpN, &vbar);
    if (lane == 0)
      for (int b = 0; b < ATTD_NS && b < nb; b++) {
        issued[b] = b;
        const int kn = min(ATTD_KB, N - b * ATTD_KB);
        const uint32_t bytes = (uint32_t)(((kn * hd) + 15) & ~15);
        // the first block also brings the key scales (max_pos is a multiple of 16)
        const uint32_t sbytes = b == 0 ? (uint32_t)(((N + 3) & ~3) * 4) : 0u;
        dcp::mbar_expect_tx(&full[b], bytes + sbytes);
        dcp::bulk_load(sK + (size_t)b * ATTD_KB * hd, kg + (int64_t)b * ATTD_KB * hd, bytes, &full[b]);
        if (sbytes) dcp::bulk_load(af, ks + (int64_t)g * max_pos, sbytes, &full[b]);
      }
  }
  // 1. the query row of this head, quantised (row scale per (token, head), double)
  const float* qrow = h + hq * hd;
  float mx = 0.0f;
  bool bad = false;
  for (int c = tid; c < hd; c += 256) {
    const float v = qrow[c];
    bad |= !isfinite(v);
    mx = fmaxf(mx, fabsf(v));
  }
  mx = block_max_f(mx, red);
  const double qsc = quant_scale(mx), rqsc = __drcp_rn(qsc);
  const float qs = __double2float_rn(qsc);
  for (int c = tid; c < hd; c += 256) q8[c] = dc_quant_div((double)qrow[c], qsc, rqsc);
  __syncthreads();
  // 2. scores block by block from the ring: one key per thread (256 keys per
  //    block), the int32 dot over hd from 16-byte chunks taken in a rotated
  //    order (lanes 4l..4l+3 start at chunk l: at most 4-way bank conflicts),
  //    then the verified epilogue; no shuffles
  const int nchk = hd >> 4;  // a power of two: hd is 32, 64, 128 or 256
  const int rot = lane >> 2;
  double m = -INFINITY;
  for (int b = 0; b < nb; b++) {
    const int slot = b % ATTD_NS;
    if (!dcp::mbar_wait(&full[slot], (uint32_t)(b / ATTD_NS) & 1u, status)) abort_flag = 1;
    __syncthreads();
    if (abort_flag) break;
    const int kb = b * ATTD_KB, kn = min(ATTD_KB, N - kb);
    const int k = tid;  // ATTD_KB == blockDim.x
    if (k < kn) {
      const int8_t* kr = sK + (size_t)slot * ATTD_KB * hd + (size_t)k * hd;
      int acc = 0;
#pragma unroll 4
      for (int c = 0; c < nchk; c++) {
        const int cc = (c + rot) & (nchk - 1);
        acc = dp4a16(*(const int4*)(kr + cc * 16), ((const int4*)q8)[cc], acc);
      }
      const double x = __dmul_rn((double)dc_epi(acc, qs, af[kb + k]), scale);
      xs[kb + k] = x;
      m = fmax(m, x);
    }
    __syncthreads();  // slot consumed
    if (tid == 0 && b + ATTD_NS < nb) {
      issued[slot] = b + ATTD_NS;
      const int kn2 = min(ATTD_KB, N - (b + ATTD_NS) * ATTD_KB);
      const uint32_t bytes = (uint32_t)(((kn2 * hd) + 15) & ~15);
      dcp::mbar_expect_tx(&full[slot], bytes);
      dcp::bulk_load(sK + (size_t)slot * ATTD_KB * hd, kg + (int64_t)(b + ATTD_NS) * ATTD_KB * hd, bytes,
                     &full[slot]);
    }
  }
  const bool aborted = abort_flag != 0;
  if (!aborted) {
    // 3. row maximum (exact); 4. e_j and its f32 copy
    m = block_max_d(m, redd);
#pragma unroll 1
    for (int j = tid; j < N; j += 256) {
      const double e = dcm::fdlibm_exp_sel(__dsub_rn(xs[j], m));
      xs[j] = e;
      af[j] = __double2float_rn(e);
    }
    __syncthreads();
    // 5. z: the serial key-order sum, as far as the probabilities can tell
    const double z = softmax_z(xs, af, N, osm, redd2, vote);
    // 6. a_j = f32(f32(e_j) / z); 7. quantizeRows of the probability row
    const double rz = __drcp_rn(z);
    float amx = 0.0f;
    for (int j = tid; j < N; j += 256) {
      const float a = dc_div_to_f32((double)af[j], z, rz);
      af[j] = a;
      amx = fmaxf(amx, a);
    }
    amx = block_max_f(amx, red);
    const double asc = quant_scale(amx), rasc = __drcp_rn(asc);
    const float as = __double2float_rn(asc);
    for (int j = tid; j < ldpN; j += 256) a8[j] = j < N ? dc_quant_div((double)af[j], asc, rasc) : (int8_t)0;
    __syncthreads();
    // 8. ctx[c] = sum_j a8[j] * v[c][j] for this CTA's CH channels
    if (!dcp::mbar_wait(&vbar, 0, status)) abort_flag = 1;
    __syncthreads();
    if (!abort_flag) {
      const int nch = ldpN >> 4;
      const int4* a4 = (const int4*)a8;
      for (int cl = warp * 4; cl < CH; cl += 32) {
        int sacc[4] = {0, 0, 0, 0};
        for (int q = lane; q < nch; q += 32) {
          const int4 av = a4[q];
#pragma unroll
          for (int u = 0; u < 4; u++) sacc[u] = dp4a16(((const int4*)(sV + (size_t)(cl + u) * ldpv))[q], av, sacc[u]);
        }
#pragma unroll
        for (int u = 0; u < 4; u++)
          for (int o = 16; o; o >>= 1) sacc[u] += __shfl_xor_sync(0xffffffffu, sacc[u], o);
        if (lane < 4) {
          const int c = c0 + cl + lane;
          const int acc = lane == 0 ? sacc[0] : lane == 1 ? sacc[1] : lane == 2 ? sacc[2] : sacc[3];
          const float o = dc_epi(acc, as, vs[g * hd + c]);
          out[hq * hd + c] = o;
          bad |= !isfinite(o);
          atomicMax(rowmax, __float_as_uint(fabsf(o)));
        }
      }
    }
  }
  if (abort_flag && tid == 0) {  // let copies still in flight land before the CTA goes away (bounded)
    dcp::mbar_wait(&vbar, 0, status);
    for (int sl = 0; sl < ATTD_NS; sl++)
      if (issued[sl] >= 0) dcp::mbar_wait(&full[sl], (uint32_t)(issued[sl] / ATTD_NS) & 1u, status);
  }
  if (bad) atomicOr(status, DC_ST_NONFINITE);
  // the last CTA to finish quantises the whole context row (quantizeRows) for
  // the O projection, then re-arms the counter
  __shared__ int is_last;
  __threadfence();
  __syncthreads();
  if (tid == 0) is_last = atomicAdd(done, 1) == (int)(gridDim.x * gridDim.y) - 1;
  __syncthreads();
  if (is_last) {
    __threadfence();
    const double sc = quant_scale(__uint_as_float(__ldcg(rowmax))), rsc = __drcp_rn(sc);
    const int qDim = nH * hd;
    if (tid == 0) {
      rsq[0] = __double2float_rn(sc);
      *done = 0;
    }
    quant_row_block(out, qDim, ldq, sc, rsc, xq);
  }
}

// The rare path of k_attention_dcl, out of line: the serial key-order z
// itself.  Every CTA of the cluster gathers all e_j (and f32(e_j)) from their
// owners, sums them in key order (the same value in each), and publishes in
// *xf the largest probability of its own keys under that z.  Every thread of
// every CTA of the cluster calls it.
__device__ __noinline__ double dcl_exact_z(double* xs, float* af, int N, int S, int r, int nmine, dco::Smem& osm,
                                           float* red, float* xf) {
  namespace cg = cooperative_groups;
  cg::cluster_group cl = cg::this_cluster();
  const int tid = threadIdx.x;
  for (int j = tid; j < N; j += 256) {
    const int owner = (j / ATTD_KB) % S;
    if (owner != r) {
      xs[j] = *cl.map_shared_rank(&xs[j], owner);
      af[j] = *cl.map_shared_rank(&af[j], owner);
    }
  }
  __syncthreads();
  const double z = dco::ordered_sum(xs, N, osm);
  const double rz = __drcp_rn(z);
  float a2 = 0.0f;
  for (int i = 0; i < nmine; i++) {
    const int j = (r + i * S) * ATTD_KB + tid;
    if (j < N) a2 = fmaxf(a2, dc_div_to_f32((double)af[j], z, rz));
  }
  a2 = block_max_f(a2, red);
  cl.sync();  // everyone has read the published values before they change
  if (tid == 0) *xf = a2;
  return z;
}

// The decode attention of k_attention_dec with the head's S = hd / CH CTAs
// forming a thread-block cluster: CTA r computes the scores, exps and
// probabilities of key blocks r, r + S, r + 2S, ... only, and the CTAs
// exchange through distributed shared memory what the softmax needs across
// blocks (the maximum, the partial sums of e, the probability maximum, and
// finally the int8 probability rows for the context).  Each CTA then forms the
// context of its CH channels over all keys.  The numbers are k_attention_dec's
// after k_rope_append, whose one-row work (RoPE, the query and key
// quantisation, the value append and channel scales) each CTA does itself for
// its head and channels.  Every CTA takes every cluster barrier on every path.
__global__ void __launch_bounds__(256) k_attention_dcl(const float* h, int nqkv, int nH, int nKV, int hd,
                                                       int8_t* k8, float* ks,
                                                       int8_t* v8t, const float* vs,
                                                       const int* n0p, int max_pos, int ldp, int CH,
                                                       double scale, float* out,
                                                       uint32_t* rowmax, int* done,
                                                       int8_t* xq, int ldq, float* rsq,
                                                       int* status, float* vt, int ldvt, const float* rc,
                                                       const float* rsn, float* vcache, const uint32_t* vmax,
                                                       uint32_t* vmax_next, float* vs_next) {
  namespace cg = cooperative_groups;
  cg::cluster_group cl = cg::this_cluster();
  extern __shared__ __align__(16) uint8_t sm[];
  asm volatile("griddepcontrol.launch_dependents;");  // the O projection may start streaming its weights
  const int ldpv = ldp;
  int8_t* sK = (int8_t*)sm;                                    // ATTD_NS slots x ATTD_KB x hd
  int8_t* sV = sK + ATTD_NS * ATTD_KB * hd;                    // CH x ldpv
  double* xs = (double*)(sV + (size_t)CH * ldpv);              // ldp doubles: s*scale, then e
  float* af = (float*)(xs + ldp);                              // ldp floats: key scales, then f32(e), then a
  int8_t* a8 = (int8_t*)(af + ldp);                            // ldp bytes
  __shared__ __align__(8) uint64_t full[ATTD_NS], vbar, mvbar;
  __shared__ __align__(16) int8_t q8[256];
  __shared__ __align__(16) int8_t knew[256];  // this step's key, rotated and quantised
  __shared__ float ch_ns[32];                 // this CTA's value channels: their scales after this step,
  __shared__ int8_t ch_q[32];                 //   their int8 values at position n0
  __shared__ unsigned chg_mask;               //   and which of them moved (bit per channel):
  __shared__ int mlist[32];                   //   the moved ones in order, their new scales
  __shared__ double msc[32], mrs[32];         //   and the scales' reciprocals
  __shared__ float red[32];
  __shared__ double2 redd2[32];  // also the 32 doubles of block_max_d / block_sum_d
  double* redd = reinterpret_cast<double*>(redd2);
  __shared__ int vote[32];
  __shared__ int abort_flag;
  // The cluster's exchanges: every warp stores its partial result into slot
  // [rank * 8 + warp] of every CTA of the cluster (remote stores, ordered by
  // the cluster barrier that follows), and each thread then reduces the S * 8
  // slots from its own shared memory, in slot order (the same value in every
  // CTA).
  __shared__ double x_max[64];    // score maxima
  __shared__ double2 x_sum[64];   // (sum of e, sum of (N - j) e_j)
  __shared__ int x_amb[64];       // 1: some probability is ambiguous under the bracket
  __shared__ float x_cmax[8];     // the context maxima of this CTA's warps
  __shared__ float xf;            // (the exact path) this CTA's probability maximum
  __shared__ dco::Smem osm;
  const int S = (int)gridDim.y, r = (int)blockIdx.y;
  const int hq = blockIdx.x, c0 = r * CH;
  const int g = hq / (nH / nKV);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // The position counter is set before the step's first kernel runs, and the
  // keys, key scales and int8 values of positions below n0 were written by
  // earlier steps: they are read before the grid-dependency wait, so their
  // copies overlap the kernels in front of this one.  Position n0 (this
  // step's key and value, formed here in step 1) and the value channels whose
  // scale moved this step come after it.
  const int n0 = *n0p, N = n0 + 1;
  const int ldpN = (N + 15) & ~15;
  const int nb = (N + ATTD_KB - 1) / ATTD_KB;
  const int nmine = r < nb ? (nb - r + S - 1) / S : 0;  // this CTA's key blocks: r, r + S, ...
  const int8_t* kg = k8 + (int64_t)g * max_pos * hd;
  if (tid == 0) {
    for (int i = 0; i < ATTD_NS; i++) dcp::mbar_init(&full[i], 1);
    dcp::mbar_init(&vbar, 1);
    dcp::mbar_init(&mvbar, 1);
    abort_flag = 0;
    dcp::mbar_fence_init();
  }
  __syncthreads();
  int issued[ATTD_NS];
  for (int i = 0; i < ATTD_NS; i++) issued[i] = -1;
  // Every key and key scale this CTA reads from the cache is older than n0:
  // the CTA's first ATTD_NS key blocks (without position n0, which step 1
  // forms) and the scales below n0 are copied before the grid-dependency wait,
  // the scales on the first block's barrier (all but the last n0 % 4, which
  // lanes 1-3 load).  Blocks past the ring's slots follow as slots free up.
  const uint32_t s_old = (uint32_t)((n0 & ~3) * 4);
  auto key_block = [&](int i, int rows, uint32_t sc_bytes) {  // lane 0 of warp 0: key block i into ring slot i
    issued[i] = i;
    const int b = r + i * S;
    const uint32_t bytes = (uint32_t)(rows * hd);  // (hd is a multiple of 16)
    dcp::mbar_expect_tx(&full[i], bytes + sc_bytes);
    if (bytes) dcp::bulk_load(sK + (size_t)i * ATTD_KB * hd, kg + (int64_t)b * ATTD_KB * hd, bytes, &full[i]);
  };
  const bool last_mine = (nb - 1) % S == r;  // this CTA owns the block with position n0
  if (warp == 0) {
    if (lane == 0) dcp::mbar_expect_tx(&vbar, (uint32_t)(CH * ldpN));
    __syncwarp();
    #pragma unroll 1
    for (int c = lane; c < CH; c += 32)
      dcp::bulk_load(sV + (size_t)c * ldpv, v8t + ((int64_t)g * hd + c0 + c) * ldp, (uint32_t)ldpN, &vbar);
    if (lane == 0 && nmine > 0) {
      #pragma unroll 1
      for (int i = 0; i < ATTD_NS && i < nmine; i++)
        key_block(i, min(ATTD_KB, n0 - (r + i * S) * ATTD_KB), i == 0 ? s_old : 0u);
      if (s_old) dcp::bulk_load(af, ks + (int64_t)g * max_pos, s_old, &full[0]);
    }
    if (nmine > 0 && lane >= 1 && lane <= (n0 & 3)) {
      const int j = (n0 & ~3) + lane - 1;
      af[j] = ks[(int64_t)g * max_pos + j];
    }
  }
  // 1. this step's row (infer.js:139-165), computed alike by every head of the
  // KV group; the group's first head writes the key and this CTA's value
  // channels to the cache (no CTA reads them there during this step):
  //  - the query head and the kv head's new key rotated (f32(a c - b s),
  //    f32(b c + a s) in double) and quantised (the query per row, double
  //    scale; the key by the quantizeCols rule, f32 scale);
  //  - this CTA's value channels: appended, their running |v| maximum and the
  //    scale it gives, the change flag against the current scale, and the
  //    int8 value of the new position.  The new maxima and scales go to
  //    vmax_next / vs_next: every cluster of the KV group reads the current
  //    ones during this kernel, and the O projection commits them.
  // The rotation tables, the channel maxima and scales are read before the
  // grid-dependency wait (the kernel before this one releases it only after its
  // own wait, so every earlier kernel has completed); the row after it.
  const int qDim = nH * hd, kvDim = nKV * hd, half = hd >> 1;
  const bool writer = hq % (nH / nKV) == 0;
  bool bad = false;
  // thread i < hd / 2 rotates the pairs (i, i + hd/2) of the query head and the
  // key; warp 0's lanes < CH hold this CTA's value channels
  const bool rt = tid < half;
  float qa = 0.0f, qb = 0.0f, ka = 0.0f, kb = 0.0f;
  {
    const double c = rt ? (double)rc[(int64_t)n0 * half + tid] : 0.0;
    const double s = rt ? (double)rsn[(int64_t)n0 * half + tid] : 0.0;
    const int cc = g * hd + c0 + lane;
    const bool vl = warp == 7 && lane < CH;  // (the rotation takes threads below hd / 2 <= 128)
    const uint32_t vm0 = vl ? vmax[cc] : 0u;
    const float vs0 = vl ? vs[cc] : 0.0f;
    asm volatile("griddepcontrol.wait;" ::: "memory");  // launched as a programmatic dependent
    if (rt) {
      const double a = h[hq * hd + tid], b = h[hq * hd + half + tid];
      const double e = h[qDim + g * hd + tid], f = h[qDim + g * hd + half + tid];
      qa = __double2float_rn(__dsub_rn(__dmul_rn(a, c), __dmul_rn(b, s)));
      qb = __double2float_rn(__dadd_rn(__dmul_rn(b, c), __dmul_rn(a, s)));
      ka = __double2float_rn(__dsub_rn(__dmul_rn(e, c), __dmul_rn(f, s)));
      kb = __double2float_rn(__dadd_rn(__dmul_rn(f, c), __dmul_rn(e, s)));
      bad |= !isfinite(qa) || !isfinite(qb) || !isfinite(ka) || !isfinite(kb);
    }
    if (warp == 7) {
      bool mv = false;
      if (vl) {
        const float v = h[qDim + kvDim + cc];
        bad |= !isfinite(v);
        const uint32_t mx = max(vm0, __float_as_uint(fabsf(v)));
        const float ns = __double2float_rn(quant_scale(__uint_as_float(mx)));
        mv = n0 == 0 || ns != vs0;
        const double rns = __drcp_rn((double)ns);
        const int8_t qv = dc_quant_div_f(v, (double)ns, rns, __double2float_rn(rns));
        ch_ns[lane] = ns;
        ch_q[lane] = qv;
        if (writer) {
          vcache[(int64_t)n0 * kvDim + cc] = v;
          vt[(int64_t)cc * ldvt + n0] = v;
          v8t[(int64_t)cc * ldp + n0] = qv;
          vmax_next[cc] = mx;
          vs_next[cc] = ns;
        }
      }
      const unsigned vm = __ballot_sync(0xffffffffu, mv);
      if (lane == 0) chg_mask = vm;
      if (mv) {  // the moved channels in order, with their new scales
        const int slot = __popc(vm & ((1u << lane) - 1u));
        mlist[slot] = lane;
        msc[slot] = (double)ch_ns[lane];
        mrs[slot] = __drcp_rn(msc[slot]);
      }
    }
  }
  {
    float mq = fmaxf(fabsf(qa), fabsf(qb)), mk = fmaxf(fabsf(ka), fabsf(kb));
    for (int o = 16; o; o >>= 1) {
      mq = fmaxf(mq, __shfl_xor_sync(0xffffffffu, mq, o));
      mk = fmaxf(mk, __shfl_xor_sync(0xffffffffu, mk, o));
    }
    if (lane == 0) {
      red[warp] = mq;
      red[8 + warp] = mk;
    }
  }
  __syncthreads();
  float mq = red[0], mk = red[8];
  for (int w = 1; w < 8; w++) {
    mq = fmaxf(mq, red[w]);
    mk = fmaxf(mk, red[8 + w]);
  }
  const double qsc = quant_scale(mq);
  const float qs = __double2float_rn(qsc);
  const float ksc = __double2float_rn(quant_scale(mk));
  if (rt) {
    const double rqsc = __drcp_rn(qsc), rksc = __drcp_rn((double)ksc);
    const float rqf = __double2float_rn(rqsc), rkf = __double2float_rn(rksc);
    q8[tid] = dc_quant_div_f(qa, qsc, rqsc, rqf);
    q8[half + tid] = dc_quant_div_f(qb, qsc, rqsc, rqf);
    knew[tid] = dc_quant_div_f(ka, (double)ksc, rksc, rkf);
    knew[half + tid] = dc_quant_div_f(kb, (double)ksc, rksc, rkf);
  }
  __syncthreads();
  const int nmv = __popc(chg_mask);  // moved value channels of this CTA
  if (writer && last_mine) {  // the group's copy of the new key
    if (tid < (hd >> 4)) ((int4*)(k8 + ((int64_t)g * max_pos + n0) * hd))[tid] = ((const int4*)knew)[tid];
    if (tid == 0) ks[(int64_t)g * max_pos + n0] = ksc;
  }
  // 2. scores of this CTA's key blocks (one key per thread)
  const int nchk = hd >> 4;
  const int rot = lane >> 2;
  double m = -INFINITY;
  auto score_block = [&](int i, int slot) {
    const int kb = (r + i * S) * ATTD_KB, kn = min(ATTD_KB, N - kb);
    const int k = tid;
    if (k < kn) {
      const int8_t* kr = sK + (size_t)slot * ATTD_KB * hd + (size_t)k * hd;
      int acc = 0;
#pragma unroll 4
      for (int c = 0; c < nchk; c++) {
        const int cc = (c + rot) & (nchk - 1);
        acc = dp4a16(*(const int4*)(kr + cc * 16), ((const int4*)q8)[cc], acc);
      }
      const double x = __dmul_rn((double)dc_epi(acc, qs, af[kb + k]), scale);
      xs[kb + k] = x;
      m = fmax(m, x);
    }
  };
  if (nmine <= ATTD_NS) {
    // every key block of this CTA has a ring slot of its own: one barrier for all
    bool ok = true;
    for (int i = 0; i < nmine; i++) ok &= dcp::mbar_wait(&full[i], 0u, status);
    if (!ok) abort_flag = 1;
    if (last_mine) {  // the block holding position n0: its key and scale from step 1
      const int i = (nb - 1 - r) / S;
      if (tid < (hd >> 4))
        ((int4*)(sK + (size_t)i * ATTD_KB * hd + (size_t)(n0 - (nb - 1) * ATTD_KB) * hd))[tid] = ((const int4*)knew)[tid];
      if (tid == 0) af[n0] = ksc;
    }
    __syncthreads();
    if (!abort_flag) {
#pragma unroll
      for (int i = 0; i < ATTD_NS; i++)
        if (i < nmine) score_block(i, i);
    }
  } else {
    _Pragma("unroll 1") for (int i = 0; i < nmine; i++) {
      const int slot = i % ATTD_NS, b = r + i * S;
      if (!dcp::mbar_wait(&full[slot], (uint32_t)(i / ATTD_NS) & 1u, status)) abort_flag = 1;
      if (b == nb - 1) {  // the block holding position n0: its key and scale from step 1
        if (tid < (hd >> 4))
          ((int4*)(sK + (size_t)slot * ATTD_KB * hd + (size_t)(n0 - b * ATTD_KB) * hd))[tid] = ((const int4*)knew)[tid];
        if (tid == 0) af[n0] = ksc;
      }
      __syncthreads();
      if (abort_flag) break;
      score_block(i, slot);
      __syncthreads();
      if (tid == 0 && i + ATTD_NS < nmine) {
        issued[slot] = i + ATTD_NS;
        const int b2 = r + (i + ATTD_NS) * S;
        const int kn2 = min(ATTD_KB, N - b2 * ATTD_KB);
        const uint32_t bytes = (uint32_t)(((kn2 * hd) + 15) & ~15);
        dcp::mbar_expect_tx(&full[slot], bytes);
        dcp::bulk_load(sK + (size_t)slot * ATTD_KB * hd, kg + (int64_t)b2 * ATTD_KB * hd, bytes, &full[slot]);
      }
    }
  }
  // The key ring is free from here on: the moved channels' f32 rows (as many
  // as it holds) are copied into it now, so that the copies overlap the
  // softmax; step 8 re-quantises them from shared memory.
  const uint32_t mrow = (uint32_t)((n0 * 4 + 15) & ~15);
  const int ring_rows = mrow ? min(nmv, (int)((size_t)ATTD_NS * ATTD_KB * hd / mrow)) : 0;
  bool mv_issued = false;  // (thread 0)
  if (ring_rows > 0) __syncthreads();  // every thread's reads of the ring are done
  if (tid == 0 && ring_rows > 0 && !abort_flag) {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // after the scores' reads of the ring
    dcp::mbar_expect_tx(&mvbar, (uint32_t)ring_rows * mrow);
    for (int m = 0; m < ring_rows; m++)
      dcp::bulk_load(sK + (size_t)m * mrow, vt + (int64_t)(g * hd + c0 + mlist[m]) * ldvt, mrow, &mvbar);
    mv_issued = true;
  }
  // 3. the exact maximum over the cluster
  for (int o = 16; o; o >>= 1) m = fmax(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane < S) *cl.map_shared_rank(&x_max[r * 8 + warp], lane) = m;
  cl.sync();
  m = -INFINITY;
#pragma unroll 8
  for (int i = 0; i < S * 8; i++) m = fmax(m, x_max[i]);
  // 4. e_j of this CTA's keys; the cluster's any-order sum brackets z
  double part = 0.0, wpart = 0.0;
  // (the loops over this CTA's keys are unrolled: a thread's keys are independent
  // chains of double-precision work, so their latencies overlap)
#pragma unroll 4
  for (int i = 0; i < nmine; i++) {
    const int j = (r + i * S) * ATTD_KB + tid;
    if (j < N) {
      const double e = dcm::fdlibm_exp_sel(__dsub_rn(xs[j], m));
      xs[j] = e;
      af[j] = __double2float_rn(e);
      part += e;
      wpart += (double)(N - j) * e;
    }
  }
  for (int o = 16; o; o >>= 1) {
    part += __shfl_xor_sync(0xffffffffu, part, o);
    wpart += __shfl_xor_sync(0xffffffffu, wpart, o);
  }
  if (lane < S) *cl.map_shared_rank(&x_sum[r * 8 + warp], lane) = make_double2(part, wpart);
  cl.sync();
  double zp = 0.0, zw = 0.0;
#pragma unroll 8
  for (int i = 0; i < S * 8; i++) {
    const double2 v = x_sum[i];
    zp += v.x;
    zw += v.y;
  }
  // a term passes through at most nmine adds in its thread, 5 in its warp and
  // S * 8 - 1 <= 63 over the warps of the cluster
  const double zr = serial_sum_radius(zp, zw, (N + ATTD_KB - 1) / ATTD_KB + 72);
  const double zlo = zp - zr, zhi = zp + zr;
  const double rlo = __drcp_rn(zlo), rhi = __drcp_rn(zhi);
  const bool narrow = __dsub_rn(zhi, zlo) < 5e-13 * zlo;
  // 6-7. a_j = f32(f32(e_j) / z) of this CTA's keys at the lower end of z's
  // bracket, quantised with the row's scale.  The row's largest probability is
  // that of its largest score (e = 1 there, and f32(f32(e) / z) grows with e),
  // so the scale needs no exchange: only the ambiguity flags travel, with the
  // probability bytes, before one cluster barrier.
  float amx = dc_div_to_f32(1.0, zlo, rlo);
  double asc = quant_scale(amx), rasc = __drcp_rn(asc);
  float rascf = __double2float_rn(rasc);
  bool amb = false;
#pragma unroll 4
  for (int i = 0; i < nmine; i++) {
    const int j = (r + i * S) * ATTD_KB + tid;
    if (j < ldpN)
      a8[j] = j < N ? dc_quant_div_f(dc_div_bracket((double)af[j], zlo, rlo, zhi, rhi, narrow, &amb), asc, rasc, rascf)
                    : (int8_t)0;
  }
  // this CTA's probability bytes to the other CTAs, 16 at a time (remote
  // stores, ordered by the barrier after them); no CTA touches another's
  // shared memory after the last one, so none has to wait before it exits
  auto send_a8 = [&]() {
    __syncthreads();
    #pragma unroll 1
    for (int q16 = tid; q16 < (ldpN >> 4); q16 += 256) {
      if (((q16 << 4) / ATTD_KB) % S != r) continue;
      const int4 v = ((const int4*)a8)[q16];
#pragma unroll 1
      for (int p = 0; p < S; p++)
        if (p != r) *cl.map_shared_rank(&((int4*)a8)[q16], p) = v;
    }
  };
  {
    const int wamb = __any_sync(0xffffffffu, amb) ? 1 : 0;
    if (lane < S) *cl.map_shared_rank(&x_amb[r * 8 + warp], lane) = wamb;
  }
  send_a8();
  cl.sync();
  int any_amb = 0;
#pragma unroll 8
  for (int i = 0; i < S * 8; i++) any_amb |= x_amb[i];
  if (any_amb) {
    // the rare exact path (cluster-uniform): the serial z, then every CTA's
    // probability bytes again under it
    const double z = dcl_exact_z(xs, af, N, S, r, nmine, osm, red, &xf);
    const double rz = __drcp_rn(z);
    amx = dc_div_to_f32(1.0, z, rz);
    asc = quant_scale(amx);
    rasc = __drcp_rn(asc);
    rascf = __double2float_rn(rasc);
#pragma unroll 4
    for (int i = 0; i < nmine; i++) {
      const int j = (r + i * S) * ATTD_KB + tid;
      if (j < ldpN) a8[j] = j < N ? dc_quant_div_f(dc_div_to_f32((double)af[j], z, rz), asc, rasc, rascf) : (int8_t)0;
    }
    send_a8();
    cl.sync();
  }
  const float as = __double2float_rn(asc);
  // 8. the context of this CTA's CH channels over all keys
  const bool vok = dcp::mbar_wait(&vbar, 0, status) && (ring_rows == 0 || abort_flag || dcp::mbar_wait(&mvbar, 0, status));
  if (!vok) abort_flag = 1;
  __syncthreads();
  if (!abort_flag) {
    // The value rows came in before the grid-dependency wait.  This step's
    // column n0 is taken from step 1, and a channel whose scale moved this step
    // is re-quantised here from the f32 cache (k_vquant_dev's arithmetic); the
    // first head of the KV group writes those rows back for the next steps
    // (another head reading them meanwhile re-quantises the same channel
    // itself).
    // the moved channels' rows: from the ring, then any rest from global
    // memory (eight loads in flight per thread)
    for (int m = 0; m < nmv; m++) {
      const int c = mlist[m];
      const double sc = msc[m], rsc = mrs[m];
      const float rscf = (float)rsc;
      int8_t* dq = sV + (size_t)c * ldpv;
      int8_t* gq = v8t + (int64_t)(g * hd + c0 + c) * ldp;
      if (m < ring_rows) {
        const float* src = (const float*)(sK + (size_t)m * mrow);
        for (int j = tid; j < n0; j += 256) {
          const int8_t q = dc_quant_div_f(src[j], sc, rsc, rscf);
          dq[j] = q;
          if (writer) gq[j] = q;
        }
        continue;
      }
      const float* src = vt + (int64_t)(g * hd + c0 + c) * ldvt;
      #pragma unroll 1
      for (int j0 = tid; j0 < n0; j0 += 8 * 256) {
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; u++) v[u] = j0 + 256 * u < n0 ? __ldcg(src + j0 + 256 * u) : 0.0f;
#pragma unroll
        for (int u = 0; u < 8; u++) {
          const int j = j0 + 256 * u;
          if (j < n0) {
            const int8_t q = dc_quant_div_f(v[u], sc, rsc, rscf);
            dq[j] = q;
            if (writer) gq[j] = q;
          }
        }
      }
    }
    for (int c = tid; c < CH; c += 256) sV[(size_t)c * ldpv + n0] = ch_q[c];
    __syncthreads();
  }
  float cmx = 0.0f;  // this thread's |context| maximum
  if (!abort_flag) {
    const int nch = ldpN >> 4;
    const int4* a4 = (const int4*)a8;
    #pragma unroll 1
    for (int cl4 = warp * 4; cl4 < CH; cl4 += 32) {
      int sacc[4] = {0, 0, 0, 0};
      #pragma unroll 1
      for (int q = lane; q < nch; q += 32) {
        const int4 av = a4[q];
#pragma unroll
        for (int u = 0; u < 4; u++) sacc[u] = dp4a16(((const int4*)(sV + (size_t)(cl4 + u) * ldpv))[q], av, sacc[u]);
      }
#pragma unroll
      for (int u = 0; u < 4; u++)
        for (int o = 16; o; o >>= 1) sacc[u] += __shfl_xor_sync(0xffffffffu, sacc[u], o);
      if (lane < 4) {
        const int c = c0 + cl4 + lane;
        const int acc = lane == 0 ? sacc[0] : lane == 1 ? sacc[1] : lane == 2 ? sacc[2] : sacc[3];
        const float o = dc_epi(acc, as, ch_ns[c - c0]);
        out[hq * hd + c] = o;
        bad |= !isfinite(o);
        cmx = fmaxf(cmx, fabsf(o));
      }
    }
  }
  if (abort_flag && tid == 0) {
    dcp::mbar_wait(&vbar, 0, status);
    if (mv_issued) dcp::mbar_wait(&mvbar, 0, status);
    for (int sl = 0; sl < ATTD_NS; sl++)
      if (issued[sl] >= 0) dcp::mbar_wait(&full[sl], (uint32_t)(issued[sl] / ATTD_NS) & 1u, status);
  }
  if (bad) atomicOr(status, DC_ST_NONFINITE);
  // one |context| maximum per CTA into the row maximum
  for (int o = 16; o; o >>= 1) cmx = fmaxf(cmx, __shfl_xor_sync(0xffffffffu, cmx, o));
  if (lane == 0) x_cmax[warp] = cmx;
  __syncthreads();
  if (tid == 0) {
    float v = x_cmax[0];
    for (int w = 1; w < 8; w++) v = fmaxf(v, x_cmax[w]);
    atomicMax(rowmax, __float_as_uint(v));
  }
  // without xq the O projection quantises the context row from the row
  // maximum itself; otherwise the last CTA to finish quantises it
  // (quantizeRows), then re-arms the counter
  if (!xq) return;
  __shared__ int is_last;
  __threadfence();
  __syncthreads();
  if (tid == 0) is_last = atomicAdd(done, 1) == (int)(gridDim.x * gridDim.y) - 1;
  __syncthreads();
  if (is_last) {
    __threadfence();
    const int qDim = nH * hd;
    if (tid == 0) *done = 0;
    quant_row_block_max(out, qDim, ldq, rowmax, xq, rsq);
  }
}

using dcm::swiglu_f32;

// the exact SwiGLU chain out of line, for the rare calls of a branch-free loop
static __device__ __noinline__ float swiglu_f32_cold(float gf, float uf) { return swiglu_f32(gf, uf); }

// Blocks per row of an element-parallel row kernel (256 threads, grid-stride
// over the row): enough for about four blocks per SM over all rows.
static int ew_blocks(const dc_ctx* ctx, int cols, int rows) {
  const int need = (4 * ctx->sm_count + rows - 1) / rows;
  return std::max(1, std::min((cols + 255) / 256, need));
}

// SwiGLU, element-parallel over grid (ew_blocks, rows): hid = f32(silu(g)*u)
// with silu(v) = v / (1 + exp(-v)) in double, from the fused gate/up GEMM's
// interleaved output row (g_j at 2j, u_j at 2j + 1) into hout (I per row), and
// |hid| folded into the row maximum (rowmax must start at 0).  The row's
// quantisation follows in k_rowquant once every block has contributed.
__global__ void __launch_bounds__(256) k_swiglu(const float* h, int I, float* hout, uint32_t* rowmax,
                                               int* status) {
  asm volatile("griddepcontrol.launch_dependents;");
  __shared__ double2 etab[64];
  dcm::exp2_tab_load(etab);  // (constant: before the wait)
  asm volatile("griddepcontrol.wait;" ::: "memory");  // launched as a programmatic dependent
  __syncthreads();
  __shared__ float red[32];
  const int row = blockIdx.y;
  const float2* g = (const float2*)(h + (int64_t)row * 2 * I);
  float mx = 0.0f;
  bool bad = false;
  // eight elements per thread at a time: their loads in flight together, then
  // their (independent) double-precision chains side by side
  const int stride = gridDim.x * blockDim.x;
  for (int j0 = blockIdx.x * blockDim.x + threadIdx.x; j0 < I; j0 += 8 * stride) {
    float2 gu[8];
#pragma unroll
    for (int u = 0; u < 8; u++) gu[u] = j0 + u * stride < I ? g[j0 + u * stride] : make_float2(0.0f, 0.0f);
    // the eight values with no branch, then (rarely) the exact chain for those
    // the error bound cannot settle
    float y[8];
    bool ok[8], all = true;
#pragma unroll
    for (int u = 0; u < 8; u++) {
      y[u] = dcm::swiglu_fast(gu[u].x, gu[u].y, etab, &ok[u]);
      all &= ok[u] || j0 + u * stride >= I;
    }
    if (!__all_sync(__activemask(), all)) {
#pragma unroll
      for (int u = 0; u < 8; u++)
        if (!ok[u] && j0 + u * stride < I) y[u] = swiglu_f32_cold(gu[u].x, gu[u].y);
    }
#pragma unroll
    for (int u = 0; u < 8; u++) {
      const int j = j0 + u * stride;
      if (j < I) {
        bad |= !isfinite(y[u]);
        hout[(int64_t)row * I + j] = y[u];
        mx = fmaxf(mx, fabsf(y[u]));
      }
    }
  }
  mx = block_max_f(mx, red);
  if (threadIdx.x == 0) atomicMax(rowmax + row, __float_as_uint(mx));
  if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) atomicOr(status, DC_ST_NONFINITE);
}

// quantizeRows from a finished row maximum, element-parallel over grid
// (ew_blocks of a quarter of the row, rows): s[row] = f32(max(mx/127, 1e-8)) in
// double, q = clamp(round(x/sc)); any grid covers the row (grid-stride).
__global__ void __launch_bounds__(256) k_rowquant(const float* x, int64_t ldx, int cols,
                                                 const uint32_t* rowmax, int8_t* q,
                                                 int ldq, float* s) {
  asm volatile("griddepcontrol.launch_dependents;");  // the next GEMV may start streaming weights
  asm volatile("griddepcontrol.wait;" ::: "memory");  // launched as a programmatic dependent
  const int row = blockIdx.y;
  const double sc = quant_scale(__uint_as_float(rowmax[row])), rsc = __drcp_rn(sc);
  const float rscf = __double2float_rn(rsc);
  if (blockIdx.x == 0 && threadIdx.x == 0) s[row] = __double2float_rn(sc);
  const float* xr = x + row * ldx;
  int8_t* qr = q + (int64_t)row * ldq;
  if (((reinterpret_cast<uintptr_t>(xr) & 15) | (cols & 3) | (ldq & 3)) == 0) {
    // four values per thread and step (16-byte loads, 4-byte stores), four steps in flight
    const int n4 = ldq >> 2, c4 = cols >> 2;
#pragma unroll 4
    for (int j4 = blockIdx.x * blockDim.x + threadIdx.x; j4 < n4; j4 += gridDim.x * blockDim.x) {
      char4 o = make_char4(0, 0, 0, 0);
      if (j4 < c4) {
        const float4 v = reinterpret_cast<const float4*>(xr)[j4];
        o.x = dc_quant_div_f(v.x, sc, rsc, rscf);
        o.y = dc_quant_div_f(v.y, sc, rsc, rscf);
        o.z = dc_quant_div_f(v.z, sc, rsc, rscf);
        o.w = dc_quant_div_f(v.w, sc, rsc, rscf);
      }
      reinterpret_cast<char4*>(qr)[j4] = o;
    }
    return;
  }
#pragma unroll 4
  for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < ldq; j += gridDim.x * blockDim.x)
    qr[j] = j < cols ? dc_quant_div_f(xr[j], sc, rsc, rscf) : (int8_t)0;
}


// ---- the decode row's GEMVs with their neighbours fused ---------------------
// A one-row GEMV (M = 1: the decode step of infer.js:353-365) whose int8
// activation row each block forms on chip from the previous kernel's f32
// output, so that no normalisation or quantisation kernel runs between two
// GEMVs of a decode layer:
//   FG_NORM   x (K floats) -> RMSNorm with weight nw (infer.js:30-39) ->
//             quantizeRows (rmsnorm_quant_block: k_rmsnorm_quant's arithmetic);
//   FG_ROWQ   x (K floats) whose |x| maximum the previous kernel folded into
//             *rmax -> quantizeRows (k_rowquant's arithmetic);
// and whose epilogue is the verified store (f32 epilogue, added to `out` with
// DC_F_ADDTO: the residual) or
//   FG_SWIGLU the weight rows interleaved (gate_j, up_j), so the warp holding
//             both accumulators forms h_j = f32(silu(g_j) * u_j) (infer.js:59,
//             212), writes it to out[j] and folds |h_j| into *rmax_out (zeroed
//             by an earlier kernel of the step).
// zero2, when not null, is set to {0, 0} by one thread after the wait (the row
// maxima the step's later kernels collect).  512 threads, one block per SM;
// each warp streams two weight rows at a time (16-byte non-allocating loads, 8
// per lane in flight per row).  Before griddepcontrol.wait every warp asks L2
// for its first two rows, so the weight stream is under way while the prologue
// runs.  Dynamic shared memory: FG_NORM: 16*K bytes (squares, row, weight) +
// ldK; FG_ROWQ: ldK (the int8 row).
constexpr int FG_THREADS = 512;
constexpr int FG_SEG = 8;
// A copy the fused GEMV makes after its wait (n 0: none): src[i] -> vmax[i] and
// the float bits src[n + i] -> vs[i], i < n.
struct VCommit {
  const uint32_t* src;
  uint32_t* vmax;
  float* vs;
  int n;
};
enum { FG_NORM = 1, FG_ROWQ = 2, FG_SWIGLU = 4 };
static size_t fg_smem(int mode, int K) {
  return ((mode & FG_NORM) ? 16 * (size_t)K : 0) + (size_t)round_up(K, 16) + 16;
}
__device__ __forceinline__ int4 ld_weights16(const int4* p, uint64_t pol) {
  int4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.s32 {%0,%1,%2,%3}, [%4], %5;"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p), "l"(pol));
  return v;
}
template <int MODE>
__global__ void __launch_bounds__(FG_THREADS, 1) k_gemv_fused(const float* x, int K, const float* nw, double eps,
                                                              const uint32_t* rmax, const int8_t* __restrict__ Wt,
                                                              int ldw, const float* __restrict__ cs, int n,
                                                              unsigned flags, float* out, uint32_t* rmax_out,
                                                              uint32_t* zero2, int* status, VCommit vc) {
  extern __shared__ __align__(16) uint8_t fsm[];
  __shared__ float red[32];
  __shared__ double2 redd2[32];
  __shared__ int vote[32];
  __shared__ float s_row;
  __shared__ dco::Smem16 osm;
  if (!(flags & DC_F_LATE_RELEASE)) asm volatile("griddepcontrol.launch_dependents;");
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int gw = blockIdx.x * (FG_THREADS / 32) + warp, nwarps = gridDim.x * (FG_THREADS / 32);
  const int ldK = (K + 15) & ~15;
  double* sq = (double*)fsm;
  float* ys = (float*)(fsm + 8 * (size_t)K);
  float* wsm = ys + K;
  int8_t* x8 = (int8_t*)(fsm + ((MODE & FG_NORM) ? 16 * (size_t)K : 0));
  // constant data first: L2 requests for this warp's first two weight rows,
  // and (FG_NORM) the norm weight into shared memory
  if (gw * 2 < n) {
    const char* r0 = (const char*)(Wt + (int64_t)(gw * 2) * ldw);
    const char* r1 = (const char*)(Wt + (int64_t)min(gw * 2 + 1, n - 1) * ldw);
    for (int c = lane * 128; c < K; c += 32 * 128) {
      asm volatile("prefetch.global.L2 [%0];" ::"l"(r0 + c));
      asm volatile("prefetch.global.L2 [%0];" ::"l"(r1 + c));
    }
  }
  const bool vec = (K & 3) == 0 && ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(nw)) & 15) == 0;
  bool wpend = false;
  if ((MODE & FG_NORM) && vec) {
    for (int i = threadIdx.x; i < (K >> 2); i += blockDim.x)
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dcp::smem_u32(wsm + 4 * i)), "l"(nw + 4 * i)
                   : "memory");
    asm volatile("cp.async.commit_group;" ::: "memory");
    wpend = true;
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (flags & DC_F_LATE_RELEASE) asm volatile("griddepcontrol.launch_dependents;");
  // (residual adds) this lane's output value of the warp's first pair, loaded
  // now so that its round trip overlaps the prologue
  const bool addto = (flags & DC_F_ADDTO) && !(MODE & FG_SWIGLU);
  const float res0 = addto && lane < 2 && gw * 2 + lane < n ? out[gw * 2 + lane] : 0.0f;
  if (zero2 && blockIdx.x == 0 && threadIdx.x == 0) {
    zero2[0] = 0;
    zero2[1] = 0;
  }
  // the decode attention's new value channel maxima and scales into the cache's
  for (int i = blockIdx.x * FG_THREADS + threadIdx.x; i < vc.n; i += gridDim.x * FG_THREADS) {
    vc.vmax[i] = vc.src[i];
    vc.vs[i] = __uint_as_float(vc.src[vc.n + i]);
  }
  // ---- prologue: the int8 activation row in shared memory
  if (MODE & FG_NORM) {
    if (!vec)
      for (int j = threadIdx.x; j < K; j += blockDim.x) wsm[j] = nw[j];  // published by the block's first barrier
    rmsnorm_quant_block<FG_THREADS / 32>(x, K, wsm, wpend, vec, eps, sq, ys, x8, ldK, &s_row, status, nullptr, 0, osm,
                                         red, redd2, vote);
  } else {
    // the row's loads eight at a time in flight, then their quotients
    constexpr int U = 8;
    const double sc = quant_scale(__uint_as_float(*rmax)), rsc = __drcp_rn(sc);
    const float rscf = __double2float_rn(rsc);
    if (threadIdx.x == 0) s_row = __double2float_rn(sc);
#pragma unroll 1
    for (int j0 = threadIdx.x; j0 < ldK; j0 += U * FG_THREADS) {
      float v[U];
#pragma unroll
      for (int u = 0; u < U; u++) {
        const int j = j0 + u * FG_THREADS;
        v[u] = j < K ? __ldcg(x + j) : 0.0f;
      }
#pragma unroll
      for (int u = 0; u < U; u++) {
        const int j = j0 + u * FG_THREADS;
        if (j < ldK) x8[j] = j < K ? dc_quant_div_f(v[u], sc, rsc, rscf) : (int8_t)0;
      }
    }
  }
  __syncthreads();
  const float rsv = s_row;
  // ---- the GEMV: two weight rows per warp at a time
  const int nch = ldK >> 4;
  const int4* X4 = (const int4*)x8;
  const uint64_t pol = dcp::l2_evict_first();
  bool bad = false;
  float hmax = 0.0f;
  for (int j0 = gw * 2; j0 < n; j0 += nwarps * 2) {
    const int j1 = min(j0 + 1, n - 1);
    const int4* w0 = (const int4*)(Wt + (int64_t)j0 * ldw);
    const int4* w1 = (const int4*)(Wt + (int64_t)j1 * ldw);
    int a0 = 0, a1 = 0;
#pragma unroll 1
    for (int c0 = 0; c0 < nch; c0 += 32 * FG_SEG) {
      int4 wa[FG_SEG], wb[FG_SEG];
#pragma unroll
      for (int u = 0; u < FG_SEG; u++) {
        const int c = c0 + u * 32 + lane;
        wa[u] = c < nch ? ld_weights16(w0 + c, pol) : make_int4(0, 0, 0, 0);
        wb[u] = c < nch ? ld_weights16(w1 + c, pol) : make_int4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < FG_SEG; u++) {
        const int c = c0 + u * 32 + lane;
        const int4 xv = c < nch ? X4[c] : make_int4(0, 0, 0, 0);
        a0 = dp4a16(wa[u], xv, a0);
        a1 = dp4a16(wb[u], xv, a1);
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      a0 += __shfl_xor_sync(0xffffffffu, a0, o);
      a1 += __shfl_xor_sync(0xffffffffu, a1, o);
    }
    if (MODE & FG_SWIGLU) {
      if (lane == 0) {
        const float h = swiglu_f32(dc_epi(a0, rsv, cs[j0]), dc_epi(a1, rsv, cs[j1]));
        bad |= !isfinite(h);
        out[j0 >> 1] = h;
        hmax = fmaxf(hmax, fabsf(h));
      }
    } else if (lane < 2 && (lane == 0 || j0 + 1 < n)) {
      const int j = lane == 0 ? j0 : j1;
      float v = dc_epi(lane == 0 ? a0 : a1, rsv, cs[j]);
      if (flags & DC_F_ADDTO) v = __fadd_rn(j0 == gw * 2 ? res0 : out[j], v);  // residual: out = out + v (f32 add)
      out[j] = v;
    }
  }
  if (MODE & FG_SWIGLU) {
    if (lane == 0 && hmax > 0.0f) atomicMax(rmax_out, __float_as_uint(hmax));
    if (bad) atomicOr(status, DC_ST_NONFINITE);
  }
}

// One embedding row (C floats) copied by the block with every load in flight
// before the first store (the table is cold in HBM).
__device__ __forceinline__ void embed_row(const float* __restrict__ src, int C, float* __restrict__ dst) {
  constexpr int U = 8;
  for (int j0 = threadIdx.x; j0 < C; j0 += U * (int)blockDim.x) {
    float v[U];
#pragma unroll
    for (int u = 0; u < U; u++) {
      const int j = j0 + u * (int)blockDim.x;
      v[u] = j < C ? src[j] : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < U; u++) {
      const int j = j0 + u * (int)blockDim.x;
      if (j < C) dst[j] = v[u];
    }
  }
}

__global__ void k_embed(const int32_t* __restrict__ ids, int T, const float* __restrict__ emb, int C, int V,
                        float* __restrict__ x, int* status) {
  const int t = blockIdx.x;
  const int id = ids[t];
  if (id < 0 || id >= V) {
    if (threadIdx.x == 0) atomicOr(status, DC_ST_BOUNDS);
    return;
  }
  embed_row(emb + (int64_t)id * C, C, x + (int64_t)t * C);
}

// One id per decode lap: ids[*stepp] (the previous lap's greedy pick).
__global__ void k_embed_at(const int32_t* __restrict__ ids, const int* __restrict__ stepp,
                           const float* __restrict__ emb, int C, int V, float* __restrict__ x, int* status) {
  const int id = ids[*stepp];
  if (id < 0 || id >= V) {
    if (threadIdx.x == 0) atomicOr(status, DC_ST_BOUNDS);
    return;
  }
  embed_row(emb + (int64_t)id * C, C, x);
}

__global__ void k_gather_rows(const float* __restrict__ x, int C, const int32_t* __restrict__ rows, int nrows,
                              float* __restrict__ y) {
  const int r = blockIdx.x;
  for (int j = threadIdx.x; j < C; j += blockDim.x) y[(int64_t)r * C + j] = x[(int64_t)rows[r] * C + j];
}

// Greedy pick over a grid: the key (orderable value bits, then the complement
// of the index) is maximal for the largest value and, among equal values, the
// smallest index -- the first maximum that pickToken's strict '>' scan keeps
// (infer.js:393-395).  -0 is folded to +0 first, since -0 > +0 is false there.
__device__ __forceinline__ unsigned long long argmax_key(float v, int j) {
  if (v == 0.0f) v = 0.0f;
  const uint32_t b = __float_as_uint(v);
  const uint32_t ord = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((unsigned long long)ord << 32) | (0xFFFFFFFFu - (uint32_t)j);
}
// grid (blocks, rows): each block folds a slice of its row into keys[row] (zero beforehand).
__global__ void __launch_bounds__(256) k_argmax_part(const float* __restrict__ logits, int V,
                                                    unsigned long long* __restrict__ keys) {
  const float* l = logits + (int64_t)blockIdx.y * V;
  unsigned long long best = 0;
  for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < V; j += gridDim.x * blockDim.x) {
    const unsigned long long kk = argmax_key(l[j], j);
    best = kk > best ? kk : best;
  }
  for (int o = 16; o; o >>= 1) {
    const unsigned long long ob = __shfl_xor_sync(0xffffffffu, best, o);
    best = ob > best ? ob : best;
  }
  if ((threadIdx.x & 31) == 0 && best) atomicMax(keys + blockIdx.y, best);
}
// picks[(*stepp) + row] = index of keys[row]; resets the keys for the next use.
__global__ void k_argmax_fin(unsigned long long* __restrict__ keys, int rows, int32_t* __restrict__ out,
                             const int* __restrict__ stepp) {
  const int r = threadIdx.x;
  if (r >= rows) return;
  const unsigned long long kk = keys[r];
  out[(stepp ? *stepp : 0) + r] = (int32_t)(0xFFFFFFFFu - (uint32_t)(kk & 0xFFFFFFFFu));
  keys[r] = 0;
}

// ---- weight loading ----------------------------------------------------------
// Element (r, c) of a k x n weight, from an f32 buffer or from the synthetic
// random-init generator (counter based; the CPU oracle restates it).
struct WSrc {
  const float* W = nullptr;  // k x n f32 row-major, or null for synthetic
  uint64_t seed = 0;
  int64_t n = 0;             // columns of the source matrix
  int transposed = 0;        // synthetic only: element (r, c) is index c * k + r (embᵀ)
  int64_t k = 0;
  double factor = 0.0;
};
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
  return z ^ (z >> 31);
}
__device__ __forceinline__ float wsrc_at(const WSrc& s, int64_t r, int64_t c) {
  if (s.W) return s.W[r * s.n + c];
  const int64_t idx = s.transposed ? c * s.k + r : r * s.n + c;
  const uint64_t base = s.seed * 0x9E3779B97F4A7C15ULL + (uint64_t)idx * 4u;
  int64_t acc = 0;
  for (int j = 0; j < 4; j++) acc += (int64_t)(mix64(base + (uint64_t)j) >> 32);
  acc -= (int64_t)2 * 4294967295LL;
  return __double2float_rn(__dmul_rn((double)acc, s.factor));
}

// Source column c lands in destination column c * cstride (cstride 2
// interleaves the gate and up projections: gate_j, up_j, gate_j+1, ...).
__global__ void __launch_bounds__(256) k_wscale(WSrc src, int k, int n, int cstride, float* __restrict__ s,
                                                int* status) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= n) return;
  float mx = 0.0f;
  bool bad = false;
  for (int r = 0; r < k; r++) {
    const float v = wsrc_at(src, r, c);
    bad |= !isfinite(v);
    mx = fmaxf(mx, fabsf(v));
  }
  if (bad) atomicOr(status, DC_ST_NONFINITE);
  s[(int64_t)c * cstride] = __double2float_rn(quant_scale(mx));
}

__global__ void __launch_bounds__(256) k_wquant_t(WSrc src, int k, int n, int cstride, const float* __restrict__ s,
                                                  int8_t* __restrict__ qt, int ldq) {
  __shared__ int8_t tile[32][33];
  const int r0 = blockIdx.y * 32, c0 = blockIdx.x * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  for (int i = ty; i < 32; i += 8) {
    const int r = r0 + i, c = c0 + tx;
    int8_t v = 0;
    if (r < k && c < n)
      v = dc_clamp8(dc_js_round(__ddiv_rn((double)wsrc_at(src, r, c), (double)s[(int64_t)c * cstride])));
    tile[i][tx] = v;
  }
  __syncthreads();
  for (int i = ty; i < 32; i += 8) {
    const int c = c0 + i, r = r0 + tx;
    if (c < n && r < ldq) qt[(int64_t)c * cstride * ldq + r] = r < k ? tile[tx][i] : (int8_t)0;
  }
}

__global__ void k_synth_f32(WSrc src, int64_t rows, int64_t cols, float* __restrict__ out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < rows * cols;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = wsrc_at(src, i / cols, i % cols);
}

__global__ void k_fill_f32(float* p, int64_t n, float v) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    p[i] = v;
}

}  // namespace

// ---- host side ------------------------------------------------------------------
static int st_alloc(dc_stage* S, void** p, size_t bytes) {
  if (cudaMalloc(p, bytes ? bytes : 16) != cudaSuccess) {
    cudaGetLastError();
    return dc_fail(S->ctx, DC_E_NOMEM, "stage: device allocation of %zu bytes failed", bytes);
  }
  S->allocs.push_back(*p);
  return DC_OK;
}
#define ST_ALLOC(S, ptr, bytes)                               \
  do {                                                        \
    int _rc = st_alloc((S), (void**)&(ptr), (size_t)(bytes)); \
    if (_rc) return _rc;                                      \
  } while (0)

static int mat_alloc(dc_stage* S, dc_mat& m, int k, int n) {
  m.k = k;
  m.n = n;
  m.ldk = round_up(k, 16);
  ST_ALLOC(S, m.qt, (size_t)n * m.ldk);
  ST_ALLOC(S, m.cs, 4 * (size_t)n);
  return DC_OK;
}

// Quantise one source matrix (k x n_src) into columns [col0, col0 + n_src) of m.
// Quantise a k x n_src source into columns col0, col0 + cstride, ... of m.
static int mat_load(dc_stage* S, dc_mat& m, int col0, const WSrc& src, int n_src, int cstride = 1) {
  cudaStream_t st = S->ctx->stream;
  float* s = m.cs + col0;
  int8_t* qt = m.qt + (int64_t)col0 * m.ldk;
  k_wscale<<<(n_src + 255) / 256, 256, 0, st>>>(src, m.k, n_src, cstride, s, S->ctx->d_status); dc_count_launch();
  DC_CUDA(S->ctx, cudaGetLastError());
  dim3 grid((n_src + 31) / 32, (m.ldk + 31) / 32);
  k_wquant_t<<<grid, 256, 0, st>>>(src, m.k, n_src, cstride, s, qt, m.ldk); dc_count_launch();
  DC_CUDA(S->ctx, cudaGetLastError());
  return DC_OK;
}

static int upload(dc_stage* S, const float* h, size_t n, float** d) {
  ST_ALLOC(S, *d, 4 * n);
  DC_CUDA(S->ctx, cudaMemcpyAsync(*d, h, 4 * n, cudaMemcpyHostToDevice, S->ctx->stream));
  return DC_OK;
}

// The shared-memory carve-out of every kernel a layer launches (dc_set_smem).
static int stage_kernel_attrs(dc_ctx* ctx) {
  const void* fns[] = {(const void*)k_rope_append<1>, (const void*)k_rope_append<4>, (const void*)k_vscale,
                       (const void*)k_vquant,
                       (const void*)k_vquant_dev,  (const void*)k_setpos,      (const void*)k_addpos,
                       (const void*)k_swiglu,      (const void*)k_rowquant,    (const void*)k_embed,
                       (const void*)k_embed_at,    (const void*)k_argmax_part, (const void*)k_argmax_fin};
  for (const void* f : fns)
    if (int rc = dc_set_smem(ctx, f, 0)) return rc;
  return DC_OK;
}

extern "C" int dc_stage_create(dc_ctx* ctx, const dc_spec* spec, int lo, int hi, int head, int max_rows,
                               int max_pos, dc_stage** out) {
  if (!ctx || !spec || !out) return DC_E_INVAL;
  if (int rc = stage_kernel_attrs(ctx)) return rc;
  if (max_pos > 0) max_pos = round_up(max_pos, 16);  // whole 16-byte rows of key scales and int8 values
  const dc_spec& s = *spec;
  if (s.hidden <= 0 || s.heads <= 0 || s.kv_heads <= 0 || s.heads % s.kv_heads || s.head_dim <= 0 ||
      (s.head_dim % 16) || s.head_dim > 128 || s.inter <= 0 || s.vocab <= 0 || lo < 0 || hi > s.layers || hi < lo ||
      max_rows < 1 || max_pos < 1 || s.hidden > 16384 || s.inter > 32768)
    return dc_fail(ctx, DC_E_INVAL, "stage: unsupported spec (head_dim must be a multiple of 16, at most 128)");
  if (s.hidden > DC_MAX_INT32_K || s.inter > DC_MAX_INT32_K || s.heads * s.head_dim > DC_MAX_INT32_K ||
      max_pos > DC_MAX_INT32_K)
    return dc_fail(ctx, DC_E_ACCBOUND, "stage: a contraction would exceed %d", DC_MAX_INT32_K);
  dc_stage* S = new dc_stage();
  S->ctx = ctx;
  S->spec = s;
  S->lo = lo;
  S->hi = hi;
  S->head = head;
  S->max_rows = max_rows;
  S->max_chunks = std::min(max_rows, DC_MAX_CHUNKS);
  S->max_pos = max_pos;
  S->C = s.hidden;
  S->hd = s.head_dim;
  S->nH = s.heads;
  S->nKV = s.kv_heads;
  S->qDim = s.heads * s.head_dim;
  S->kvDim = s.kv_heads * s.head_dim;
  S->I = s.inter;
  S->V = s.vocab;
  S->nqkv = S->qDim + 2 * S->kvDim;
  S->ldC = round_up(S->C, 16);
  S->ldQ = round_up(S->qDim, 16);
  S->ldI = round_up(S->I, 16);
  S->ldp = round_up(max_pos, 64);
  S->ldvt = S->ldp + 8;
  int rc = DC_OK;
  auto fail = [&](int r) {
    dc_stage_free(S);
    return r;
  };
  S->L.resize(hi - lo);
  for (auto& ly : S->L) {
    if ((rc = st_alloc(S, (void**)&ly.nrm1, 4 * (size_t)S->C)) || (rc = st_alloc(S, (void**)&ly.nrm2, 4 * (size_t)S->C)))
      return fail(rc);
    if ((rc = mat_alloc(S, ly.qkv, S->C, S->nqkv)) || (rc = mat_alloc(S, ly.o, S->qDim, S->C)) ||
        (rc = mat_alloc(S, ly.gu, S->C, 2 * S->I)) || (rc = mat_alloc(S, ly.down, S->I, S->C)))
      return fail(rc);
    dc_kv& kv = ly.kv;
    if ((rc = st_alloc(S, (void**)&kv.k8, (size_t)S->nKV * max_pos * S->hd)) ||
        (rc = st_alloc(S, (void**)&kv.ks, 4 * (size_t)S->nKV * max_pos)) ||
        (rc = st_alloc(S, (void**)&kv.v, 4 * (size_t)max_pos * S->kvDim)) ||
        (rc = st_alloc(S, (void**)&kv.vt, 4 * (size_t)S->ldvt * S->kvDim)) ||
        (rc = st_alloc(S, (void**)&kv.v8t, (size_t)S->kvDim * S->ldp)) ||
        (rc = st_alloc(S, (void**)&kv.vs, 4 * (size_t)S->kvDim)) ||
        (rc = st_alloc(S, (void**)&kv.vmax, 4 * (size_t)S->kvDim)) ||
        (rc = st_alloc(S, (void**)&kv.vchg, 4 * (size_t)S->kvDim)))
      return fail(rc);
  }
  if (head) {
    if ((rc = st_alloc(S, (void**)&S->emb, 4 * (size_t)S->V * S->C)) ||
        (rc = st_alloc(S, (void**)&S->nrmF, 4 * (size_t)S->C)) || (rc = mat_alloc(S, S->lm, S->C, S->V)))
      return fail(rc);
  }
  const int wide = std::max(std::max(S->nqkv, 2 * S->I), S->C);
  if ((rc = st_alloc(S, (void**)&S->hbuf, 4 * (size_t)max_rows * wide)) ||
      (rc = st_alloc(S, (void**)&S->hmid, 4 * (size_t)max_rows * S->I)) ||
      (rc = st_alloc(S, (void**)&S->ctxo, 4 * (size_t)max_rows * S->qDim)) ||
      (rc = st_alloc(S, (void**)&S->xq, (size_t)max_rows * std::max(std::max(S->ldC, S->ldQ), S->ldI))) ||
      (rc = st_alloc(S, (void**)&S->rs, 4 * (size_t)max_rows)) ||
      (rc = st_alloc(S, (void**)&S->rowmax, 4 * (size_t)std::max(max_rows, 2))) ||
      (rc = st_alloc(S, (void**)&S->d_pos, 16)) || (rc = st_alloc(S, (void**)&S->d_zero, 16)) ||
      (rc = st_alloc(S, (void**)&S->d_step, 16)) || (rc = st_alloc(S, (void**)&S->xlap, 4 * (size_t)S->C)) ||
      (rc = st_alloc(S, (void**)&S->logits1, 4 * (size_t)(head ? S->V : 1))) ||
      (rc = st_alloc(S, (void**)&S->amax_keys, 64)) ||
      (rc = st_alloc(S, (void**)&S->att_done, 16)) ||
      (rc = st_alloc(S, (void**)&S->xrow, 4 * (size_t)S->C)) ||
      (rc = st_alloc(S, (void**)&S->a8g, (size_t)S->max_rows * S->nH * S->ldp)) ||
      (rc = st_alloc(S, (void**)&S->vstage, 8 * (size_t)S->kvDim)) ||
      (rc = st_alloc(S, (void**)&S->asg, 4 * (size_t)S->max_rows * S->nH)) ||
      (rc = st_alloc(S, (void**)&S->vsg, 4 * (size_t)DC_MAX_CHUNKS * S->kvDim)) ||
      (rc = st_alloc(S, (void**)&S->vchgg, 4 * (size_t)DC_MAX_CHUNKS * S->kvDim)) ||
      (S->max_chunks > 1 &&
       (rc = st_alloc(S, (void**)&S->v8s, (size_t)(S->max_chunks - 1) * S->kvDim * S->ldp))) ||
      (rc = st_alloc(S, (void**)&S->lx, 4 * (size_t)8 * S->C)))
    return fail(rc);
  // RoPE tables (infer.js:71-81), positions 0 .. max_pos-1, with the fdlibm
  // method of Math.pow / Math.cos / Math.sin (dc_fdlibm.cuh)
  const int half = S->hd / 2;
  std::vector<float> c((size_t)max_pos * half), sn((size_t)max_pos * half);
  bool ok = true;
  for (int i = 0; i < half && ok; i++) {
    bool okp = true;
    const double den = dcf::pow(s.rope_theta, (2.0 * i) / (double)S->hd, &okp);
    ok = okp;
    for (int p = 0; p < max_pos && ok; p++) {
      const double f = (double)p / den;
      bool okc = true, oks = true;
      c[(size_t)p * half + i] = (float)dcf::cos(f, &okc);
      sn[(size_t)p * half + i] = (float)dcf::sin(f, &oks);
      ok = okc && oks;
    }
  }
  if (!ok) {
    dc_fail(ctx, DC_E_INVAL, "stage_create: rope_theta %g gives RoPE angles outside the table builder's range",
            s.rope_theta);
    return fail(DC_E_INVAL);
  }
  if ((rc = upload(S, c.data(), c.size(), &S->rope_cos)) || (rc = upload(S, sn.data(), sn.size(), &S->rope_sin)))
    return fail(rc);
  if (cudaMemsetAsync(S->amax_keys, 0, 64, ctx->stream) != cudaSuccess ||
      cudaMemsetAsync(S->att_done, 0, 16, ctx->stream) != cudaSuccess ||
      cudaMemsetAsync(S->d_zero, 0, 16, ctx->stream) != cudaSuccess ||
      cudaMemsetAsync(S->d_pos, 0, 16, ctx->stream) != cudaSuccess)
    return fail(dc_fail(ctx, DC_E_CUDA, "stage: position init failed"));
  if ((rc = dc_stage_kv_reset(S)) || (rc = dc_sync(ctx))) return fail(rc);
  *out = S;
  return DC_OK;
}

extern "C" void dc_stage_free(dc_stage* S) {
  if (!S) return;
  if (S->ctx) cudaStreamSynchronize(S->ctx->stream);
  if (S->lap_exec) cudaGraphExecDestroy(S->lap_exec);
  if (S->row_exec) cudaGraphExecDestroy(S->row_exec);
  for (void* p : S->allocs) cudaFree(p);
  delete S;
}

static WSrc f32src(const float* dW, int k, int n) {
  WSrc s;
  s.W = dW;
  s.n = n;
  s.k = k;
  return s;
}

// Upload one host k x n matrix and quantise it into columns col0, col0 + cstride, ... of m.
static int load_host(dc_stage* S, dc_mat& m, int col0, const float* W, int k, int n, float* tmp, int cstride = 1) {
  DC_CUDA(S->ctx, cudaMemcpyAsync(tmp, W, 4 * (size_t)k * n, cudaMemcpyHostToDevice, S->ctx->stream));
  return mat_load(S, m, col0, f32src(tmp, k, n), n, cstride);
}

extern "C" int dc_stage_set_layer(dc_stage* S, int layer, const float* nrm1, const float* nrm2, const float* Wq,
                                  const float* Wk, const float* Wv, const float* Wo, const float* Wgate,
                                  const float* Wup, const float* Wdown) {
  if (!S || layer < S->lo || layer >= S->hi || !nrm1 || !nrm2 || !Wq || !Wk || !Wv || !Wo || !Wgate || !Wup ||
      !Wdown)
    return dc_fail(S ? S->ctx : nullptr, DC_E_INVAL, "stage_set_layer: bad arguments");
  dc_layer& ly = S->L[layer - S->lo];
  dc_ctx* ctx = S->ctx;
  float* tmp = nullptr;
  const size_t big = std::max((size_t)S->C * std::max(S->qDim, S->I), (size_t)S->I * S->C);
  if (cudaMalloc(&tmp, 4 * big) != cudaSuccess) {
    cudaGetLastError();
    return dc_fail(ctx, DC_E_NOMEM, "stage_set_layer: staging allocation failed");
  }
  int rc = DC_OK;
  cudaError_t e = cudaMemcpyAsync(ly.nrm1, nrm1, 4 * (size_t)S->C, cudaMemcpyHostToDevice, ctx->stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(ly.nrm2, nrm2, 4 * (size_t)S->C, cudaMemcpyHostToDevice, ctx->stream);
  if (e != cudaSuccess) rc = dc_cuda_fail(ctx, e, "norm upload");
  if (!rc) rc = load_host(S, ly.qkv, 0, Wq, S->C, S->qDim, tmp);
  if (!rc) rc = dc_sync(ctx);
  if (!rc) rc = load_host(S, ly.qkv, S->qDim, Wk, S->C, S->kvDim, tmp);
  if (!rc) rc = dc_sync(ctx);
  if (!rc) rc = load_host(S, ly.qkv, S->qDim + S->kvDim, Wv, S->C, S->kvDim, tmp);
  if (!rc) rc = dc_sync(ctx);
  if (!rc) rc = load_host(S, ly.o, 0, Wo, S->qDim, S->C, tmp);
  if (!rc) rc = dc_sync(ctx);
  if (!rc) rc = load_host(S, ly.gu, 0, Wgate, S->C, S->I, tmp, 2);  // gate_j in column 2j
  if (!rc) rc = dc_sync(ctx);
  if (!rc) rc = load_host(S, ly.gu, 1, Wup, S->C, S->I, tmp, 2);    // up_j in column 2j + 1
  if (!rc) rc = dc_sync(ctx);
  if (!rc) rc = load_host(S, ly.down, 0, Wdown, S->I, S->C, tmp);
  if (!rc) rc = dc_sync(ctx);
  cudaFree(tmp);
  return rc;
}

extern "C" int dc_stage_set_head(dc_stage* S, const float* emb, const float* nrmF, const float* lm_kn) {
  if (!S || !S->head || !emb || !nrmF) return dc_fail(S ? S->ctx : nullptr, DC_E_INVAL, "stage_set_head: bad arguments");
  dc_ctx* ctx = S->ctx;
  DC_CUDA(ctx, cudaMemcpyAsync(S->emb, emb, 4 * (size_t)S->V * S->C, cudaMemcpyHostToDevice, ctx->stream));
  DC_CUDA(ctx, cudaMemcpyAsync(S->nrmF, nrmF, 4 * (size_t)S->C, cudaMemcpyHostToDevice, ctx->stream));
  int rc;
  if (lm_kn) {
    float* tmp = nullptr;
    if (cudaMalloc(&tmp, 4 * (size_t)S->C * S->V) != cudaSuccess) {
      cudaGetLastError();
      return dc_fail(ctx, DC_E_NOMEM, "stage_set_head: staging allocation failed");
    }
    rc = load_host(S, S->lm, 0, lm_kn, S->C, S->V, tmp);
    if (!rc) rc = dc_sync(ctx);
    cudaFree(tmp);
  } else {
    // tied: lm_head = embᵀ (shard.js:92, 123-128): element (c, v) = emb[v][c]
    float* tmp = nullptr;
    if (cudaMalloc(&tmp, 4 * (size_t)S->C * S->V) != cudaSuccess) {
      cudaGetLastError();
      return dc_fail(ctx, DC_E_NOMEM, "stage_set_head: staging allocation failed");
    }
    std::vector<float> t((size_t)S->C * S->V);
    for (int v = 0; v < S->V; v++)
      for (int c = 0; c < S->C; c++) t[(size_t)c * S->V + v] = emb[(size_t)v * S->C + c];
    rc = load_host(S, S->lm, 0, t.data(), S->C, S->V, tmp);
    if (!rc) rc = dc_sync(ctx);
    cudaFree(tmp);
  }
  return rc;
}

// Synthetic random-init weights, generated on the device from the counter-based
// formula (norm weights 1).  Tensor seed = model_seed * 1000003 + (layer+1)*64 + role
// with roles emb 1, lm 2, Wq 3, Wk 4, Wv 5, Wo 6, Wgate 7, Wup 8, Wdown 9.
extern "C" int dc_stage_synth(dc_stage* S, uint64_t model_seed, double factor) {
  if (!S) return DC_E_INVAL;
  dc_ctx* ctx = S->ctx;
  auto seed_of = [&](int layer, int role) { return model_seed * 1000003ull + (uint64_t)(layer + 1) * 64u + role; };
  auto src = [&](int layer, int role, int k, int n) {
    WSrc s;
    s.seed = seed_of(layer, role);
    s.n = n;
    s.k = k;
    s.factor = factor;
    return s;
  };
  int rc = DC_OK;
  for (int l = S->lo; l < S->hi && !rc; l++) {
    dc_layer& ly = S->L[l - S->lo];
    k_fill_f32<<<8, 256, 0, ctx->stream>>>(ly.nrm1, S->C, 1.0f); dc_count_launch();
    k_fill_f32<<<8, 256, 0, ctx->stream>>>(ly.nrm2, S->C, 1.0f); dc_count_launch();
    rc = mat_load(S, ly.qkv, 0, src(l, 3, S->C, S->qDim), S->qDim);
    if (!rc) rc = mat_load(S, ly.qkv, S->qDim, src(l, 4, S->C, S->kvDim), S->kvDim);
    if (!rc) rc = mat_load(S, ly.qkv, S->qDim + S->kvDim, src(l, 5, S->C, S->kvDim), S->kvDim);
    if (!rc) rc = mat_load(S, ly.o, 0, src(l, 6, S->qDim, S->C), S->C);
    if (!rc) rc = mat_load(S, ly.gu, 0, src(l, 7, S->C, S->I), S->I, 2);  // gate_j in column 2j
    if (!rc) rc = mat_load(S, ly.gu, 1, src(l, 8, S->C, S->I), S->I, 2);  // up_j in column 2j + 1
    if (!rc) rc = mat_load(S, ly.down, 0, src(l, 9, S->I, S->C), S->C);
  }
  if (!rc && S->head) {
    WSrc e = src(-1, 1, S->V, S->C);
    k_synth_f32<<<1024, 256, 0, ctx->stream>>>(e, S->V, S->C, S->emb); dc_count_launch();
    k_fill_f32<<<8, 256, 0, ctx->stream>>>(S->nrmF, S->C, 1.0f); dc_count_launch();
    if (S->spec.tie) {
      WSrc t = e;  // embᵀ: element (c, v) = emb index v*C + c
      t.transposed = 1;
      t.k = S->C;
      t.n = S->V;
      rc = mat_load(S, S->lm, 0, t, S->V);
    } else {
      rc = mat_load(S, S->lm, 0, src(-1, 2, S->C, S->V), S->V);
    }
  }
  if (!rc) rc = dc_sync(ctx);
  return rc;
}

extern "C" int dc_stage_kv_reset(dc_stage* S) {
  if (!S) return DC_E_INVAL;
  S->kv_len = 0;
  for (auto& ly : S->L) DC_CUDA(S->ctx, cudaMemsetAsync(ly.kv.vmax, 0, 4 * (size_t)S->kvDim, S->ctx->stream));
  return DC_OK;
}

extern "C" int dc_stage_kv_len(const dc_stage* S) { return S ? S->kv_len : -1; }

// The activation hop from one stage to the next (app.js:705-765, wire.js
// :106-138): T rows of hidden floats from x_src (on the source stage's
// device) to x_dst (on the destination's), after the source stage's work and
// before any later work of the destination: the copy runs on the source
// context's stream, and the destination's stream waits for it through an
// event.  Stages on different devices copy peer to peer; on one device it is
// a device copy.
extern "C" int dc_stage_handoff(dc_stage* src, dc_stage* dst, const float* x_src, float* x_dst, int T) {
  if (!src || !dst) return DC_E_INVAL;
  if (!x_src || !x_dst || T < 1 || T > dst->max_rows || src->C != dst->C)
    return dc_fail(src->ctx, DC_E_INVAL, "stage_handoff: bad arguments");
  dc_ctx* a = src->ctx;
  dc_ctx* b = dst->ctx;
  const size_t bytes = 4 * (size_t)T * src->C;
  if (a->device == b->device)
    DC_CUDA(a, cudaMemcpyAsync(x_dst, x_src, bytes, cudaMemcpyDeviceToDevice, a->stream));
  else
    DC_CUDA(a, cudaMemcpyPeerAsync(x_dst, b->device, x_src, a->device, bytes, a->stream));
  if (a != b) {
    DC_CUDA(a, cudaEventRecord(a->ev_hop, a->stream));
    DC_CUDA(b, cudaStreamWaitEvent(b->stream, a->ev_hop, 0));
  }
  return DC_OK;
}

extern "C" int dc_stage_embed(dc_stage* S, const int32_t* ids, int T, float* x) {
  if (!S || !S->head || T < 1 || T > S->max_rows || !ids || !x)
    return dc_fail(S ? S->ctx : nullptr, DC_E_INVAL, "stage_embed: bad arguments");
  k_embed<<<T, 256, 0, S->ctx->stream>>>(ids, T, S->emb, S->C, S->V, x, S->ctx->d_status); dc_count_launch();
  DC_CUDA(S->ctx, cudaGetLastError());
  return DC_OK;
}

static int launch_argmax(dc_stage* S, const float* logits, int rows, int32_t* picks, const int* stepp) {
  cudaStream_t st = S->ctx->stream;
  const int blocks = std::max(1, std::min(2 * S->ctx->sm_count, (S->V + 255) / 256));
  k_argmax_part<<<dim3(blocks, rows), 256, 0, st>>>(logits, S->V, S->amax_keys);
  dc_count_launch();
  k_argmax_fin<<<1, 32, 0, st>>>(S->amax_keys, rows, picks, stepp);
  dc_count_launch();
  DC_CUDA(S->ctx, cudaGetLastError());
  return DC_OK;
}

static int gemm(dc_stage* S, const dc_mat& m, int T, const int8_t* xq, int ldx, float* out, unsigned flags) {
  return dc_gemm_dispatch(S->ctx, xq, ldx, m.qt, m.ldk, S->rs, m.cs, T, m.k, m.n, 1, flags, out, S->ctx->stream, 0);
}

// Launch as a programmatic dependent of the previous kernel on the stream: the
// CTAs may be scheduled while that kernel finishes.  Every kernel launched so
// executes griddepcontrol.wait before it touches memory that earlier work on
// the stream writes or reads (only constant data may be read before it), and
// none of their pointer parameters to such memory is __restrict__: the
// compiler may move a load through a restrict pointer above the wait's inline
// assembly (a loop-invariant load hoisted out of a loop did exactly that).
template <typename... KArgs, typename... Args>
static cudaError_t launch_dep(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// The fused one-row GEMV fits on chip when its norm row does (16 bytes per
// column plus the int8 row, below the 227 KB a block may have).
static bool fg_fits(const dc_stage* S) {
  return fg_smem(FG_NORM, S->C) + 24 * 1024 <= 232448 && fg_smem(FG_ROWQ, S->I) + 24 * 1024 <= 232448;
}

// k_gemv_fused<mode> over the weight m (out = epilogue of m's n columns; with
// FG_SWIGLU the n/2 SwiGLU values), launched as a programmatic dependent.
static cudaError_t launch_fused(dc_stage* S, int mode, const float* x, int K, const float* nw, const uint32_t* rmax,
                                const dc_mat& m, unsigned flags, float* out, uint32_t* rmax_out, uint32_t* zero2,
                                VCommit vc = {nullptr, nullptr, nullptr, 0}) {
  dc_ctx* ctx = S->ctx;
  const int blocks = std::max(1, std::min(ctx->sm_count, (m.n + 31) / 32));
  const size_t smem = fg_smem(mode, K);
  cudaError_t e;
  switch (mode) {
    case FG_NORM:
      e = launch_dep(k_gemv_fused<FG_NORM>, dim3(blocks), dim3(FG_THREADS), smem, ctx->stream, x, K, nw,
                     S->spec.norm_eps, rmax, (const int8_t*)m.qt, m.ldk, (const float*)m.cs, m.n, flags, out, rmax_out,
                     zero2, ctx->d_status, vc);
      break;
    case FG_NORM | FG_SWIGLU:
      e = launch_dep(k_gemv_fused<FG_NORM | FG_SWIGLU>, dim3(blocks), dim3(FG_THREADS), smem, ctx->stream, x, K, nw,
                     S->spec.norm_eps, rmax, (const int8_t*)m.qt, m.ldk, (const float*)m.cs, m.n, flags, out, rmax_out,
                     zero2, ctx->d_status, vc);
      break;
    default:
      e = launch_dep(k_gemv_fused<FG_ROWQ>, dim3(blocks), dim3(FG_THREADS), smem, ctx->stream, x, K, nw,
                     S->spec.norm_eps, rmax, (const int8_t*)m.qt, m.ldk, (const float*)m.cs, m.n, flags, out, rmax_out,
                     zero2, ctx->d_status, vc);
      break;
  }
  dc_count_launch();
  return e;
}

// The layer loop of one stage on T rows of x (in place).  Every position the
// kernels need is read from *n0p (the cached tokens before this call; 0 for the
// full window), so the same launches can be captured once in a CUDA graph and
// replayed lap after lap.  n0 is the host's copy, used only to size the tiled
// V quantisation of chunk/window calls (T > 8), which are never captured.
// The chunk attention's split form (k_attention, then k_attn_ctx per 32
// channels) fits this stage's geometry.
static bool split_ctx_ok(const dc_stage* S) {
  return S->a8g && S->hd % 32 == 0 && (size_t)(32 + 16) * S->ldp + 1024 <= 232448;
}

static int forward_layers(dc_stage* S, float* x, int T, int n0, int use_kv, const int* n0p,
                          const ChunkSet* cks = nullptr) {
  dc_ctx* ctx = S->ctx;
  const bool multi = cks && cks->G > 1;  // several chunks in this pass (split context path, checked by the caller)
  const ChunkSet one = {0, {}};
  cudaStream_t st = ctx->stream;
  const int N = n0 + T;
  const double scale = 1.0 / sqrt((double)S->hd);
  const size_t att_smem = ((12 * (size_t)S->max_pos + 15) & ~(size_t)15) + (size_t)S->ldp + 16;
  if (int rc0 = dc_set_smem(ctx, (const void*)k_attention, (int)att_smem)) return rc0;
  // the decode attention (one row): the widest channel group whose buffers fit on chip
  int dec_ch = 0;
  size_t dec_smem = 0;
  if (S->hd == 32 || S->hd == 64 || S->hd == 128 || S->hd == 256) {
    for (int ch = 32; ch >= 8 && !dec_ch; ch >>= 1) {
      if (S->hd % ch) continue;
      const size_t need = (size_t)ATTD_NS * ATTD_KB * S->hd + (size_t)(ch + 13) * S->ldp;
      if (need + 12 * 1024 <= 232448) {
        dec_ch = ch;
        dec_smem = need;
      }
    }
    if (dec_ch) {
      if (int rc0 = dc_set_smem(ctx, (const void*)k_attention_dec, (int)dec_smem)) return rc0;
      if (int rc0 = dc_set_smem(ctx, (const void*)k_attention_dcl, (int)dec_smem)) return rc0;
    }
  }
  // chunk rows (T <= 16): probabilities per (head, row), then the context per
  // (head, 32 channels) from shared-memory copies of the value and probability rows
  const size_t ctx_smem = (size_t)(32 + 16) * S->ldp;
  const bool split_ctx = split_ctx_ok(S);
  // a pass of several chunks: each chunk's attention by k_attn_chunk (a chunk's
  // rows of one head per CTA) when there are CTAs enough for the SMs and its
  // shared memory fits (16 score rows and 16 probability rows, beside ~24 KB of
  // static shared memory)
  auto ar_kernel = S->hd == 64 ? k_attn_chunk<64> : S->hd == 128 ? k_attn_chunk<128> : k_attn_chunk<256>;
  const size_t ar_smem = 80 * (size_t)S->ldp;
  const bool use_ar = multi && split_ctx && (S->hd == 64 || S->hd == 128 || S->hd == 256) &&
                      ar_smem + 24 * 1024 <= 232448 && S->pass_attn != 2 &&
                      (S->pass_attn == 1 || S->nH * cks->G >= ctx->sm_count / 2);
  if (use_ar)
    if (int rc0 = dc_set_smem(ctx, (const void*)ar_kernel, (int)ar_smem)) return rc0;
  if (split_ctx)
    if (int rc0 = dc_set_smem(ctx, (const void*)k_attn_ctx, (int)ctx_smem)) return rc0;
  // rows that fit in one wave get the wide norm block; more than three waves'
  // worth of rows leave the weight row in L2 (four blocks per SM)
  const bool nwide = T <= ctx->sm_count;
  auto norm_k = nwide ? k_rmsnorm_quant<NORM_WIDE> : k_rmsnorm_quant<NORM_THREADS>;
  const int norm_nt = nwide ? NORM_WIDE : NORM_THREADS;
  // always raised: the kernel's static shared memory counts against the 48 KB default too
  const size_t nrm_smem = rms_smem(S->C, norm_nt, T <= 3 * ctx->sm_count);
  if (int rc0 = dc_set_smem(ctx, (const void*)norm_k, (int)nrm_smem)) return rc0;
  // a decode row: GEMVs with the norms, the SwiGLU and the row quantisation fused
  const bool fuse = T == 1 && use_kv && dec_ch && S->row_fused && fg_fits(S);
  // a decode row's O projection through the fused GEMV that quantises its input row
  const bool o_rowq = T == 1 && use_kv && dec_ch && S->o_rowq && fg_smem(FG_ROWQ, S->qDim) + 24 * 1024 <= 232448;
  if (o_rowq)
    if (int rc0 = dc_set_smem(ctx, (const void*)k_gemv_fused<FG_ROWQ>, (int)fg_smem(FG_ROWQ, S->qDim))) return rc0;
  if (fuse) {
    if (int rc0 = dc_set_smem(ctx, (const void*)k_gemv_fused<FG_NORM>, (int)fg_smem(FG_NORM, S->C))) return rc0;
    if (int rc0 = dc_set_smem(ctx, (const void*)k_gemv_fused<FG_NORM | FG_SWIGLU>, (int)fg_smem(FG_NORM, S->C)))
      return rc0;
    if (int rc0 = dc_set_smem(ctx, (const void*)k_gemv_fused<FG_ROWQ>, (int)fg_smem(FG_ROWQ, S->I))) return rc0;
  }
  // the decode row's cluster attention: it rotates, quantises and appends the
  // step's row itself (no k_rope_append), re-quantises moved value channels,
  // and leaves the new channel maxima and scales for the O projection to commit
  const bool dcl = T == 1 && use_kv && dec_ch && o_rowq && S->hd / dec_ch > 1 && S->hd / dec_ch <= 8;
  // its kernel before releases it only after that kernel's own wait
  const unsigned qkv_flags = dcl ? DC_F_LATE_RELEASE : 0u;
  int rc;
  for (auto& ly : S->L) {
    dc_kv& kv = ly.kv;
    // attention block
    if (fuse) {  // RMSNorm + QKV; zeroes the row maxima the attention and the SwiGLU collect
      DC_CUDA(ctx, launch_fused(S, FG_NORM, x, S->C, ly.nrm1, nullptr, ly.qkv, qkv_flags, S->hbuf, nullptr,
                                S->rowmax));
    } else {
      DC_CUDA(ctx, launch_dep(norm_k, dim3(T), dim3(norm_nt), nrm_smem, st, x, S->C, ly.nrm1,
                              S->spec.norm_eps, S->xq, S->ldC, S->rs, ctx->d_status, nullptr, S->rowmax, 0));
      dc_count_launch();
      if ((rc = gemm(S, ly.qkv, T, S->xq, S->ldC, S->hbuf, qkv_flags))) return rc;
    }
    if (!use_kv) DC_CUDA(ctx, cudaMemsetAsync(kv.vmax, 0, 4 * (size_t)S->kvDim, st));
    if (!dcl) {
      // four rows per block for long chunk passes (short ones keep a block per
      // row, so that they still fill the SMs; one row: the scale path of a decode row)
      const int vblocks = (S->kvDim + 63) / 64;
      if (T >= 128) {
        DC_CUDA(ctx, launch_dep(k_rope_append<4>, dim3((T + 3) / 4, S->nH + S->nKV + vblocks), dim3(64), 0, st,
                                S->hbuf, S->nqkv, S->nH, S->nKV, S->hd, S->rope_cos, S->rope_sin, n0p, S->max_pos,
                                kv.k8, kv.ks, kv.v, multi ? nullptr : kv.vmax, (float*)nullptr, kv.vchg, kv.v8t,
                                S->ldp, ctx->d_status, kv.vt, S->ldvt, T));
      } else {
        DC_CUDA(ctx, launch_dep(k_rope_append<1>, dim3(T, S->nH + S->nKV + vblocks), dim3(64), 0, st, S->hbuf,
                                S->nqkv, S->nH, S->nKV, S->hd, S->rope_cos, S->rope_sin, n0p, S->max_pos, kv.k8,
                                kv.ks, kv.v, multi ? nullptr : kv.vmax, T == 1 ? kv.vs : nullptr, kv.vchg, kv.v8t,
                                S->ldp, ctx->d_status, kv.vt, S->ldvt, T));
      }
      dc_count_launch();
    }
    if (multi) {
      DC_CUDA(ctx, launch_dep(k_vscale_chunks, dim3((S->kvDim + 31) / 32), dim3(32 * DC_MAX_CHUNKS), 0, st,
                              (const float*)kv.v,
                              kv.vmax, kv.vs, kv.vchg, S->kvDim, n0p, *cks, S->vsg, S->vchgg));
      dc_count_launch();
    } else if (T > 1) {
      DC_CUDA(ctx, launch_dep(k_vscale, dim3((S->kvDim + 127) / 128), dim3(128), 0, st, kv.vmax, kv.vs, kv.vchg,
                              S->kvDim, n0p));
      dc_count_launch();
    }
    if (dcl) {
    } else if (multi) {
      const int ntiles = ((N + 63) / 64) * ((S->kvDim + 31) / 32);
      DC_CUDA(ctx, launch_dep(k_vquant_chunks, dim3(ntiles + (cks->G - 1) * ((S->kvDim + 7) / 8)), dim3(256), 0, st,
                              (const float*)kv.v, (const float*)kv.vs, (const int*)kv.vchg, kv.v8t, n0, S->kvDim, S->hd,
                              S->ldp, *cks, (const float*)S->vsg, S->v8s, ntiles, (const float*)kv.vt, S->ldvt));
    } else if (T <= 8) {
      DC_CUDA(ctx, launch_dep(k_vquant_dev, dim3((S->max_pos + 127) / 128, (S->kvDim + 31) / 32), dim3(256), 0, st,
                              kv.v, kv.vs, kv.vchg, kv.v8t, T, n0p, S->kvDim, S->hd, S->ldp, T == 1 ? 1 : 0));
    } else {
      DC_CUDA(ctx, launch_dep(k_vquant, dim3((N + 63) / 64, (S->kvDim + 31) / 32), dim3(256), 0, st, kv.v, kv.vs,
                              kv.vchg, kv.v8t, N, n0, S->kvDim, S->hd, S->ldp));
    }
    if (!dcl) dc_count_launch();
    if (dcl) {
      // the channel-group CTAs of a head as one cluster: the key work is split among them
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(S->nH, S->hd / dec_ch);
      cfg.blockDim = dim3(256);
      cfg.dynamicSmemBytes = dec_smem;
      cfg.stream = st;
      cudaLaunchAttribute attr[2];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 1;
      attr[0].val.clusterDim.y = S->hd / dec_ch;
      attr[0].val.clusterDim.z = 1;
      attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // a programmatic dependent too
      attr[1].val.programmaticStreamSerializationAllowed = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 2;
      DC_CUDA(ctx, cudaLaunchKernelEx(&cfg, k_attention_dcl, (const float*)S->hbuf, S->nqkv, S->nH, S->nKV, S->hd,
                                      kv.k8, kv.ks, kv.v8t, (const float*)kv.vs, n0p, S->max_pos, S->ldp, dec_ch,
                                      scale, S->ctxo, S->rowmax, S->att_done, (int8_t*)nullptr, S->ldQ, S->rs,
                                      ctx->d_status, kv.vt, S->ldvt, (const float*)S->rope_cos,
                                      (const float*)S->rope_sin, kv.v, (const uint32_t*)kv.vmax, S->vstage,
                                      (float*)(S->vstage + S->kvDim)));
      dc_count_launch();
    } else if (T == 1 && use_kv && dec_ch) {
      DC_CUDA(ctx, launch_dep(k_attention_dec, dim3(S->nH, S->hd / dec_ch), dim3(256), dec_smem, st, S->hbuf, S->nqkv,
                              S->nH, S->nKV, S->hd, kv.k8, kv.ks, kv.v8t, kv.vs, n0p, S->max_pos, S->ldp, dec_ch,
                              scale, S->ctxo, S->rowmax, S->att_done, S->xq, S->ldQ, S->rs, ctx->d_status));
      dc_count_launch();
    } else if (use_ar) {
      DC_CUDA(ctx, launch_dep(ar_kernel, dim3(S->nH, cks->G), dim3(AR_THREADS), ar_smem, st, (const float*)S->hbuf,
                              S->nqkv, S->nH, S->nKV, (const int8_t*)kv.k8, (const float*)kv.ks,
                              (const int8_t*)kv.v8t, (const float*)kv.vs, T, n0p, S->max_pos, S->ldp, scale,
                              S->ctxo, S->qDim, S->rowmax, ctx->d_status, *cks, (const int8_t*)S->v8s,
                              (const float*)S->vsg));
      dc_count_launch();
      DC_CUDA(ctx, launch_dep(k_rowquant, dim3(ew_blocks(ctx, (S->ldQ + 3) / 4, T), T), dim3(256), 0, st, S->ctxo,
                              (int64_t)S->qDim, S->qDim, S->rowmax, S->xq, S->ldQ, S->rs));
      dc_count_launch();
    } else if (split_ctx && (T <= 16 || multi)) {
      DC_CUDA(ctx, launch_dep(k_attention, dim3(S->nH, T), dim3(ATT_THREADS), att_smem, st, S->hbuf, S->nqkv,
                              S->nH, S->nKV, S->hd, kv.k8, kv.ks, kv.v8t, kv.vs, T, n0p, S->max_pos, S->ldp, scale,
                              S->ctxo, S->rowmax, S->qDim, ctx->d_status, S->a8g, S->asg));
      dc_count_launch();
      DC_CUDA(ctx, launch_dep(k_attn_ctx, dim3(S->nH, S->hd / 32, multi ? cks->G : 1), dim3(256), ctx_smem, st,
                              (const int8_t*)S->a8g, (const float*)S->asg, (const int8_t*)kv.v8t,
                              (const float*)kv.vs, S->nH, S->nKV, S->hd, T, n0p, S->ldp, S->ctxo, S->qDim,
                              S->rowmax, ctx->d_status, multi ? *cks : one, (const int8_t*)S->v8s,
                              (const float*)S->vsg));
      dc_count_launch();
      DC_CUDA(ctx, launch_dep(k_rowquant, dim3(ew_blocks(ctx, (S->ldQ + 3) / 4, T), T), dim3(256), 0, st, S->ctxo,
                              (int64_t)S->qDim, S->qDim, S->rowmax, S->xq, S->ldQ, S->rs));
      dc_count_launch();
    } else {
      k_attention<<<dim3(S->nH, T), ATT_THREADS, att_smem, st>>>(S->hbuf, S->nqkv, S->nH, S->nKV, S->hd, kv.k8, kv.ks,
                                                                kv.v8t, kv.vs, T, n0p, S->max_pos, S->ldp, scale,
                                                                S->ctxo, S->rowmax, S->qDim, ctx->d_status);
      dc_count_launch();
      k_rowquant<<<dim3(ew_blocks(ctx, (S->ldQ + 3) / 4, T), T), 256, 0, st>>>(S->ctxo, S->qDim, S->qDim, S->rowmax, S->xq, S->ldQ,
                                                                S->rs);
      dc_count_launch();
    }
    if (dcl) {  // x2 = x + attn, the context row quantised by the GEMV's blocks; the value scales committed
      DC_CUDA(ctx, launch_fused(S, FG_ROWQ, S->ctxo, S->qDim, nullptr, S->rowmax, ly.o, DC_F_ADDTO, x, nullptr,
                                nullptr, VCommit{S->vstage, kv.vmax, kv.vs, S->kvDim}));
    } else if ((rc = gemm(S, ly.o, T, S->xq, S->ldQ, x, DC_F_ADDTO))) {  // x2 = x + attn
      return rc;
    }
    // MLP block
    if (fuse) {  // RMSNorm + gate/up + SwiGLU; then the down projection quantises its own input
      DC_CUDA(ctx, launch_fused(S, FG_NORM | FG_SWIGLU, x, S->C, ly.nrm2, nullptr, ly.gu, 0, S->hmid, S->rowmax + 1,
                                nullptr));
      DC_CUDA(ctx, launch_fused(S, FG_ROWQ, S->hmid, S->I, nullptr, S->rowmax + 1, ly.down, DC_F_ADDTO, x, nullptr,
                                nullptr));
      continue;
    }
    DC_CUDA(ctx, launch_dep(norm_k, dim3(T), dim3(norm_nt), nrm_smem, st, x, S->C, ly.nrm2,
                            S->spec.norm_eps, S->xq, S->ldC, S->rs, ctx->d_status, nullptr, S->rowmax, 0));
    dc_count_launch();
    // a decode row: SwiGLU in the gate/up GEMV's epilogue (the interleaved rows
    // gate_j, up_j are one warp's pair); otherwise its own kernel
    int swg = DC_E_INVAL;
    if (T == 1) {
      swg = dc_gemv_swiglu(ctx, S->xq, ly.gu.qt, ly.gu.ldk, S->rs, ly.gu.cs, ly.gu.k, ly.gu.n, S->hmid, S->rowmax, st);
      if (swg != DC_OK && swg != DC_E_INVAL) return swg;
    }
    if (swg == DC_E_INVAL) {
      if ((rc = gemm(S, ly.gu, T, S->xq, S->ldC, S->hbuf, 0))) return rc;
      DC_CUDA(ctx, launch_dep(k_swiglu, dim3(ew_blocks(ctx, S->I, T), T), dim3(256), 0, st, S->hbuf, S->I, S->hmid,
                              S->rowmax, ctx->d_status));
      dc_count_launch();
    }
    DC_CUDA(ctx, launch_dep(k_rowquant, dim3(ew_blocks(ctx, (S->ldI + 3) / 4, T), T), dim3(256), 0, st, S->hmid, (int64_t)S->I,
                            S->I, S->rowmax, S->xq, S->ldI, S->rs));
    dc_count_launch();
    if ((rc = gemm(S, ly.down, T, S->xq, S->ldI, x, DC_F_ADDTO))) return rc;  // out = x2 + down
    DC_CUDA(ctx, cudaGetLastError());
  }
  return DC_OK;
}

// runLayers (use_kv = 0: full window, positions 0..T-1) or runLayersChunk
// (use_kv = 1: positions pos0.., keys/values appended to this stage's cache).
// Moves the context onto its own (capturable) stream for the scope: the own
// stream waits for the caller's, and the caller's waits for the own stream at
// the end of the scope.
struct StreamSwap {
  dc_ctx* c;
  cudaStream_t user;
  bool on;
  explicit StreamSwap(dc_ctx* c_) : c(c_), user(c_->stream), on(false) {}
  int fork() {
    if (c->stream == c->own_stream) return DC_OK;
    DC_CUDA(c, cudaEventRecord(c->ev_fork, c->stream));
    DC_CUDA(c, cudaStreamWaitEvent(c->own_stream, c->ev_fork, 0));
    c->stream = c->own_stream;
    on = true;
    return DC_OK;
  }
  ~StreamSwap() {
    if (on) {
      cudaEventRecord(c->ev_join, c->own_stream);
      cudaStreamWaitEvent(user, c->ev_join, 0);
      c->stream = user;
    }
  }
};

// One cached row (T = 1) through the stage's layers as a CUDA graph: the row is
// copied into the stage's own buffer, the graph (captured on first use; every
// position-dependent kernel reads the position from d_pos) runs in place, and
// the row is copied back.  Used for decode steps of a multi-GPU pipeline, where
// each stage runs one row per token.
static int forward_row_graph(dc_stage* S, float* x, int n0) {
  dc_ctx* ctx = S->ctx;
  StreamSwap swap(ctx);
  if (int rc = swap.fork()) return rc;
  cudaStream_t s = ctx->stream;
  DC_CUDA(ctx, cudaMemcpyAsync(S->xrow, x, 4 * (size_t)S->C, cudaMemcpyDeviceToDevice, s));
  k_setpos<<<1, 1, 0, s>>>(S->d_pos, n0);
  dc_count_launch();
  if (!S->row_exec) {
    cudaGraph_t g = nullptr;
    const unsigned long long nk0 = dc_launch_count();
    DC_CUDA(ctx, cudaStreamBeginCapture(s, cudaStreamCaptureModeRelaxed));
    int rc = forward_layers(S, S->xrow, 1, n0, 1, S->d_pos);
    cudaError_t e = cudaStreamEndCapture(s, &g);
    S->row_nk = dc_launch_count() - nk0;
    dc_count_launches(-(long long)S->row_nk);  // captured, not launched
    if (rc) {
      if (g) cudaGraphDestroy(g);
      return rc;
    }
    if (e != cudaSuccess) return dc_cuda_fail(ctx, e, "cudaStreamEndCapture");
    e = cudaGraphInstantiate(&S->row_exec, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return dc_cuda_fail(ctx, e, "cudaGraphInstantiate");
  }
  DC_CUDA(ctx, cudaGraphLaunch(S->row_exec, s));
  dc_count_launches((long long)S->row_nk);
  DC_CUDA(ctx, cudaMemcpyAsync(x, S->xrow, 4 * (size_t)S->C, cudaMemcpyDeviceToDevice, s));
  return DC_OK;
}

extern "C" int dc_stage_set_row_graph(dc_stage* S, int on) {
  if (!S) return DC_E_INVAL;
  S->row_graph = on != 0;
  return DC_OK;
}

extern "C" int dc_stage_set_timeline(dc_stage* S, unsigned long long* buf, int per_lap, int laps) {
  if (!S || per_lap < 0 || laps < 0 || (per_lap && laps && !buf))
    return dc_fail(S ? S->ctx : nullptr, DC_E_INVAL, "stage_set_timeline: bad arguments");
  dc_ctx* ctx = S->ctx;
  const bool on = per_lap > 0 && laps > 0;
  ctx->tl_buf = on ? buf : nullptr;
  ctx->tl_per_lap = on ? per_lap : 0;
  ctx->tl_laps = on ? laps : 0;
  ctx->tl_kind.clear();
  ctx->tl_bytes.clear();
  if (S->lap_exec) cudaGraphExecDestroy(S->lap_exec);  // a captured lap holds the other kernel sequence
  S->lap_exec = nullptr;
  S->lap_key.clear();
  return DC_OK;
}

extern "C" int dc_stage_timeline_info(const dc_stage* S, int* kinds, double* bytes, int cap) {
  if (!S) return -1;
  const dc_ctx* ctx = S->ctx;
  const int n = (int)ctx->tl_kind.size();
  for (int i = 0; i < n && i < cap; i++) {
    if (kinds) kinds[i] = ctx->tl_kind[i];
    if (bytes) bytes[i] = ctx->tl_bytes[i];
  }
  return n;
}

extern "C" int dc_stage_set_pass_attention(dc_stage* S, int mode) {
  if (!S || mode < 0 || mode > 2) return DC_E_INVAL;
  S->pass_attn = mode;
  return DC_OK;
}

extern "C" int dc_stage_set_row_fusion(dc_stage* S, int on) {
  if (!S) return DC_E_INVAL;
  if ((on != 0) != S->row_fused) {  // captured graphs hold the other kernel sequence
    if (S->row_exec) cudaGraphExecDestroy(S->row_exec);
    S->row_exec = nullptr;
    if (S->lap_exec) cudaGraphExecDestroy(S->lap_exec);
    S->lap_exec = nullptr;
    S->lap_key.clear();
  }
  S->row_fused = on != 0;
  return DC_OK;
}

extern "C" int dc_stage_forward(dc_stage* S, float* x, int T, int pos0, int use_kv) {
  if (!S || !x || T < 1 || T > S->max_rows) return dc_fail(S ? S->ctx : nullptr, DC_E_INVAL, "stage_forward: bad T");
  dc_ctx* ctx = S->ctx;
  const int n0 = use_kv ? S->kv_len : 0;
  const int N = n0 + T;
  if (use_kv && pos0 != n0)
    return dc_fail(ctx, DC_E_INVAL, "stage_forward: chunk position %d does not follow the cached %d tokens", pos0, n0);
  if (N > S->max_pos || pos0 + T > S->max_pos)
    return dc_fail(ctx, DC_E_INVAL, "stage_forward: %d positions exceed max_pos %d", N, S->max_pos);
  if (S->L.empty()) return DC_OK;
  if (use_kv && T == 1 && S->row_graph && !ctx->timing) {
    if (int rc = forward_row_graph(S, x, n0)) return rc;
    S->kv_len = N;
    return DC_OK;
  }
  const int* n0p = S->d_zero;
  if (use_kv) {
    k_setpos<<<1, 1, 0, ctx->stream>>>(S->d_pos, n0);
    dc_count_launch();
    n0p = S->d_pos;
  }
  int rc = forward_layers(S, x, T, n0, use_kv, n0p);
  if (rc) return rc;
  if (use_kv) S->kv_len = N;
  return DC_OK;
}

// runLayersChunk on several consecutive chunks in one pass over the weights
// (infer.js:288-296 called once per chunk, as generateChunked does, :339-367):
// every row-wise step is the same at any row count, and the only quantity that
// depends on where a chunk ends -- the value channel scales its context is
// formed with (the per-column scales of vh over the cache as it stands after
// the chunk's append, :154-165, :186-196) -- is computed per chunk
// (k_vscale_chunks, k_vquant_chunks, k_attn_ctx per chunk).  So the rows and
// the cache come out bit-identical to one dc_stage_forward per chunk.  Where
// the split context path does not fit (head_dim not a multiple of 32, or a
// chunk of more than 16 rows), the chunks run one by one.
extern "C" int dc_stage_forward_chunks(dc_stage* S, float* x, int T, int pos0, const int* rows, int nchunks) {
  if (!S || !x || !rows || nchunks < 1 || nchunks > DC_MAX_CHUNKS || T < 1 || T > S->max_rows)
    return dc_fail(S ? S->ctx : nullptr, DC_E_INVAL, "stage_forward_chunks: bad arguments");
  dc_ctx* ctx = S->ctx;
  ChunkSet cks = {nchunks, {}};
  int sum = 0, widest = 0;
  for (int g = 0; g < nchunks; g++) {
    if (rows[g] < 1) return dc_fail(ctx, DC_E_INVAL, "stage_forward_chunks: chunk %d has %d rows", g, rows[g]);
    sum += rows[g];
    widest = std::max(widest, rows[g]);
    cks.end[g] = sum;
  }
  if (sum != T) return dc_fail(ctx, DC_E_INVAL, "stage_forward_chunks: chunks hold %d rows, not %d", sum, T);
  if (nchunks == 1) return dc_stage_forward(S, x, T, pos0, 1);
  const int n0 = S->kv_len;
  if (pos0 != n0)
    return dc_fail(ctx, DC_E_INVAL, "stage_forward_chunks: position %d does not follow the cached %d tokens", pos0, n0);
  if (n0 + T > S->max_pos)
    return dc_fail(ctx, DC_E_INVAL, "stage_forward_chunks: %d positions exceed max_pos %d", n0 + T, S->max_pos);
  if (S->L.empty()) return DC_OK;
  if (!split_ctx_ok(S) || widest > 16 || nchunks > S->max_chunks) {
    for (int g = 0, r = 0; g < nchunks; r += rows[g], g++)
      if (int rc = dc_stage_forward(S, x + (size_t)r * S->C, rows[g], pos0 + r, 1)) return rc;
    return DC_OK;
  }
  k_setpos<<<1, 1, 0, ctx->stream>>>(S->d_pos, n0);
  dc_count_launch();
  if (int rc = forward_layers(S, x, T, n0, 1, S->d_pos, &cks)) return rc;
  S->kv_len = n0 + T;
  return DC_OK;
}

// One decode lap of the whole ring on one device: greedy pick from the
// previous lap's hidden row (logitsAt, infer.js:324-334 + pickToken :393-395)
// into picks[step], embedRows of that id (:298-310), runLayersChunk on every
// stage (:288-296), step + 1 -- the chunked decode loop of infer.js:353-365
// (app.js:907-921) with the token id never leaving the device.
static int decode_lap(dc_stage** st, int ns, int32_t* picks) {
  dc_stage* H = st[0];
  dc_ctx* ctx = H->ctx;
  cudaStream_t s = ctx->stream;
  int rc = DC_OK;
  dc_timeline_begin(ctx, H->d_step);
  struct TimelineEnd {  // (an early error return ends the lap's stamping too)
    dc_ctx* c;
    ~TimelineEnd() { dc_timeline_end(c); }
  } tl_end{ctx};
  if (H->row_fused && fg_fits(H)) {  // final RMSNorm fused into the lm_head GEMV
    if (int rc0 = dc_set_smem(ctx, (const void*)k_gemv_fused<FG_NORM>, (int)fg_smem(FG_NORM, H->C))) return rc0;
    DC_CUDA(ctx, launch_fused(H, FG_NORM, H->xlap, H->C, H->nrmF, nullptr, H->lm, 0, H->logits1, nullptr, nullptr));
  } else {
    const size_t nrm_smem = rms_smem(H->C, NORM_WIDE);
    // always raised: the kernel's static shared memory counts against the 48 KB default too
    if (int rc0 = dc_set_smem(ctx, (const void*)k_rmsnorm_quant<NORM_WIDE>, (int)nrm_smem)) return rc0;
    k_rmsnorm_quant<NORM_WIDE><<<1, NORM_WIDE, nrm_smem, s>>>(H->xlap, H->C, H->nrmF, H->spec.norm_eps, H->xq, H->ldC, H->rs,
                                                       ctx->d_status);
    dc_count_launch();
    rc = dc_gemm_dispatch(ctx, H->xq, H->ldC, H->lm.qt, H->lm.ldk, H->rs, H->lm.cs, 1, H->C, H->V, 1, 0, H->logits1, s,
                          0);
    if (rc) return rc;
  }
  if ((rc = launch_argmax(H, H->logits1, 1, picks, H->d_step))) return rc;
  k_embed_at<<<1, 512, 0, s>>>(picks, H->d_step, H->emb, H->C, H->V, H->xlap, ctx->d_status);
  dc_count_launch();
  for (int i = 0; i < ns; i++) {
    dc_stage* S = st[i];
    if (S->L.empty()) continue;
    if ((rc = forward_layers(S, H->xlap, 1, S->kv_len, 1, S->d_pos))) return rc;
    k_addpos<<<1, 1, 0, s>>>(S->d_pos, 1);
    dc_count_launch();
  }
  dc_timeline_end(ctx);  // (the stamps of a lap end before its counter moves)
  k_addpos<<<1, 1, 0, s>>>(H->d_step, 1);
  dc_count_launch();
  DC_CUDA(ctx, cudaGetLastError());
  return DC_OK;
}

// n_new decode laps over stages[0..ns) (all on the context's device, stage 0
// the head), starting from `x_last` (device, one hidden row: the last row of
// the prefill's output).  picks (device int32, n_new) receive the greedy ids.
// With use_graph, lap 0 runs as ordinary launches and one lap is captured as a
// CUDA graph (cached on the head for this stage list) and replayed for the rest.
extern "C" int dc_decode_run(dc_stage** stages, int ns, const float* x_last, int n_new, int32_t* picks,
                             int use_graph) {
  if (!stages || ns < 1 || !stages[0] || !stages[0]->head || !x_last || !picks || n_new < 0)
    return dc_fail(stages && stages[0] ? stages[0]->ctx : nullptr, DC_E_INVAL, "decode_run: bad arguments");
  dc_stage* H = stages[0];
  dc_ctx* ctx = H->ctx;
  cudaStream_t s = ctx->stream;
  for (int i = 0; i < ns; i++) {
    if (!stages[i] || stages[i]->ctx != ctx) return dc_fail(ctx, DC_E_INVAL, "decode_run: stages must share a context");
    if (stages[i]->kv_len + n_new > stages[i]->max_pos)
      return dc_fail(ctx, DC_E_INVAL, "decode_run: %d + %d positions exceed max_pos %d", stages[i]->kv_len, n_new,
                     stages[i]->max_pos);
  }
  if (n_new == 0) return DC_OK;
  // Work on the context's own stream (the legacy default stream cannot be
  // captured): it waits for the caller's stream, and the caller's stream waits
  // for it when the laps are enqueued.
  StreamSwap swap(ctx);
  if (int rc0 = swap.fork()) return rc0;
  s = ctx->stream;
  DC_CUDA(ctx, cudaMemcpyAsync(H->xlap, x_last, 4 * (size_t)H->C, cudaMemcpyDeviceToDevice, s));
  k_setpos<<<1, 1, 0, s>>>(H->d_step, 0);
  dc_count_launch();
  for (int i = 0; i < ns; i++) {
    k_setpos<<<1, 1, 0, s>>>(stages[i]->d_pos, stages[i]->kv_len);
    dc_count_launch();
  }
  int rc = decode_lap(stages, ns, picks);
  if (rc) return rc;
  if (n_new > 1) {
    if (use_graph) {
      std::vector<dc_stage*> key(stages, stages + ns);
      if (!H->lap_exec || H->lap_key != key || H->lap_picks != picks) {
        if (H->lap_exec) cudaGraphExecDestroy(H->lap_exec);
        H->lap_exec = nullptr;
        const bool timing = ctx->timing;
        ctx->timing = false;  // no per-GEMM timing events inside the captured lap
        cudaGraph_t g = nullptr;
        const unsigned long long nk0 = dc_launch_count();
        DC_CUDA(ctx, cudaStreamBeginCapture(s, cudaStreamCaptureModeRelaxed));
        rc = decode_lap(stages, ns, picks);
        cudaError_t e = cudaStreamEndCapture(s, &g);
        H->lap_nk = dc_launch_count() - nk0;
        dc_count_launches(-(long long)H->lap_nk);  // captured, not launched
        ctx->timing = timing;
        if (rc) {
          if (g) cudaGraphDestroy(g);
          return rc;
        }
        if (e != cudaSuccess) return dc_cuda_fail(ctx, e, "cudaStreamEndCapture");
        e = cudaGraphInstantiate(&H->lap_exec, g, 0);
        cudaGraphDestroy(g);
        if (e != cudaSuccess) return dc_cuda_fail(ctx, e, "cudaGraphInstantiate");
        H->lap_key = key;
        H->lap_picks = picks;
      }
      for (int n = 1; n < n_new; n++) {
        DC_CUDA(ctx, cudaGraphLaunch(H->lap_exec, s));
        dc_count_launches(H->lap_nk);
      }
    } else {
      for (int n = 1; n < n_new; n++)
        if ((rc = decode_lap(stages, ns, picks))) return rc;
    }
  }
  for (int i = 0; i < ns; i++) stages[i]->kv_len += n_new;
  return DC_OK;
}

// logitsAt (infer.js:324-334): final RMSNorm of the requested rows, lm_head
// GEMV (one row of M per requested row; rows are independent), greedy pick.
extern "C" int dc_stage_logits(dc_stage* S, const float* x, int T, const int32_t* rows, int nrows, float* logits,
                               int32_t* picks) {
  if (!S || !S->head || !x || !rows || nrows < 1 || nrows > 8 || T < 1)
    return dc_fail(S ? S->ctx : nullptr, DC_E_INVAL, "stage_logits: bad arguments");
  dc_ctx* ctx = S->ctx;
  cudaStream_t st = ctx->stream;
  for (int r = 0; r < nrows; r++)
    if (rows[r] < 0 || rows[r] >= T) return dc_fail(ctx, DC_E_INVAL, "readout row outside the window");
  for (int r = 0; r < nrows; r++)
    DC_CUDA(ctx, cudaMemcpyAsync(S->lx + (size_t)r * S->C, x + (size_t)rows[r] * S->C, 4 * (size_t)S->C,
                                 cudaMemcpyDeviceToDevice, st));
  const size_t nrm_smem = rms_smem(S->C, NORM_WIDE);
  // always raised: the kernel's static shared memory counts against the 48 KB default too
  if (int rc0 = dc_set_smem(ctx, (const void*)k_rmsnorm_quant<NORM_WIDE>, (int)nrm_smem)) return rc0;
  k_rmsnorm_quant<NORM_WIDE><<<nrows, NORM_WIDE, nrm_smem, st>>>(S->lx, S->C, S->nrmF, S->spec.norm_eps, S->xq, S->ldC, S->rs,
                                                          ctx->d_status); dc_count_launch();
  int rc = dc_gemm_dispatch(ctx, S->xq, S->ldC, S->lm.qt, S->lm.ldk, S->rs, S->lm.cs, nrows, S->C, S->V, 1, 0,
                            logits, st, 0);
  if (rc) return rc;
  if (picks && (rc = launch_argmax(S, logits, nrows, picks, nullptr))) return rc;
  DC_CUDA(ctx, cudaGetLastError());
  return DC_OK;
}

// Test access to one layer's cache: keys as int8 + scales and values as f32.
extern "C" int dc_stage_kv_read(dc_stage* S, int layer, int8_t* k8, float* ks, float* v) {
  if (!S || layer < S->lo || layer >= S->hi) return DC_E_INVAL;
  const dc_kv& kv = S->L[layer - S->lo].kv;
  const int n = S->kv_len;
  for (int g = 0; g < S->nKV; g++) {
    if (k8)
      DC_CUDA(S->ctx, cudaMemcpy(k8 + (size_t)g * n * S->hd, kv.k8 + (size_t)g * S->max_pos * S->hd, (size_t)n * S->hd,
                                 cudaMemcpyDeviceToHost));
    if (ks)
      DC_CUDA(S->ctx, cudaMemcpy(ks + (size_t)g * n, kv.ks + (size_t)g * S->max_pos, 4 * (size_t)n,
                                 cudaMemcpyDeviceToHost));
  }
  if (v) DC_CUDA(S->ctx, cudaMemcpy(v, kv.v, 4 * (size_t)n * S->kvDim, cudaMemcpyDeviceToHost));
  return DC_OK;
}

// ---- standalone row operations (parity access to the fused kernels' math) ----
__global__ void __launch_bounds__(256) k_ordered_sum(const double* __restrict__ t, int n, double* __restrict__ out) {
  __shared__ dco::Smem osm;
  const double v = dco::ordered_sum(t + (int64_t)blockIdx.x * n, n, osm);
  if (threadIdx.x == 0) out[blockIdx.x] = v;
}

extern "C" int dc_ordered_sum_dev(dc_ctx* ctx, const double* terms, int rows, int n, double* out) {
  if (!ctx || rows < 0 || n < 0 || (rows && (!out || (n && !terms)))) return dc_fail(ctx, DC_E_INVAL, "ordered_sum: bad arguments");
  if (!rows) return DC_OK;
  k_ordered_sum<<<rows, 256, 0, ctx->stream>>>(terms, n, out);
  dc_count_launch();
  DC_CUDA(ctx, cudaGetLastError());
  return DC_OK;
}

__global__ void k_exp(const double* __restrict__ x, int n, double* __restrict__ y, int sel) {
  __shared__ double2 tab[64];
  dcm::exp2_tab_load(tab);
  __syncthreads();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  double e = 0.0;
  // (sel 4, 5: the SwiGLU value of g = f32(x), u = f32(x / 2 + 1/4), settled and exact)
  const float g = (float)x[i], u = (float)__dadd_rn(__dmul_rn(x[i], 0.5), 0.25);
  switch (sel) {
    case 0: y[i] = dcm::fdlibm_exp(x[i]); break;
    case 1: y[i] = dcm::fdlibm_exp_sel(x[i]); break;
    case 2: y[i] = dcm::exp_tang(x[i], tab); break;
    case 3: y[i] = (double)dcm::exp_settle(x[i], tab, &e); break;
    case 4: y[i] = (double)dcm::swiglu_settle(g, u, tab); break;
    default: y[i] = (double)dcm::swiglu_f32(g, u); break;
  }
}

extern "C" int dc_exp_dev(dc_ctx* ctx, const double* x, int n, double* y, int sel) {
  if (!ctx || n < 0 || (n && (!x || !y))) return dc_fail(ctx, DC_E_INVAL, "exp: bad arguments");
  if (!n) return DC_OK;
  if (sel < 0 || sel > 5) return dc_fail(ctx, DC_E_INVAL, "exp: sel %d not in 0..5", sel);
  k_exp<<<(n + 255) / 256, 256, 0, ctx->stream>>>(x, n, y, sel);
  dc_count_launch();
  DC_CUDA(ctx, cudaGetLastError());
  return DC_OK;
}

extern "C" int dc_rmsnorm_dev(dc_ctx* ctx, const float* x, int rows, int cols, const float* w, double eps, float* y,
                              int exact_sum) {
  if (!ctx || rows < 0 || cols < 1 || (rows && (!x || !w || !y))) return dc_fail(ctx, DC_E_INVAL, "rmsnorm: bad arguments");
  if ((size_t)cols * 12 > 200 * 1024) return dc_fail(ctx, DC_E_INVAL, "rmsnorm: row of %d does not fit on chip", cols);
  if (!rows) return DC_OK;
  const bool wide = rows <= ctx->sm_count;
  const int smem = (int)rms_smem(cols, wide ? NORM_WIDE : NORM_THREADS);
  auto norm_k = wide ? k_rmsnorm_quant<NORM_WIDE> : k_rmsnorm_quant<NORM_THREADS>;
  if (int rc = dc_set_smem(ctx, (const void*)norm_k, smem)) return rc;
  norm_k<<<rows, wide ? NORM_WIDE : NORM_THREADS, smem, ctx->stream>>>(x, cols, w, eps, nullptr, 0, nullptr, ctx->d_status, y,
                                                           nullptr, exact_sum);
  dc_count_launch();
  DC_CUDA(ctx, cudaGetLastError());
  return DC_OK;
}
