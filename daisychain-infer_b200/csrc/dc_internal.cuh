// dc_internal.cuh -- shared definitions of libdcinfer (not part of the C ABI).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include <string>

#include "../../include/dcinfer.h"

// Internal GEMM flag (beside the public DC_RELU / DC_ACC / DC_REQUANT): add the
// f32 epilogue value to what `out` already holds (the residual connection).
#define DC_F_ADDTO 0x100u
// Internal: the one-row GEMV over interleaved gate/up weight rows (gate_j at
// row 2j, up_j at 2j + 1) stores h_j = f32(silu(g_j) * u_j) instead of the two
// outputs, and folds |h_j| into a row maximum (dc_gemv_swiglu).
#define DC_F_SWIGLU 0x200u
// Internal: the one-row GEMV releases its programmatic dependent only after
// its own grid-dependency wait (the decode attention after the QKV projection
// reads older cache rows before its wait; they must follow the previous step).
#define DC_F_LATE_RELEASE 0x400u

// Device status word bits (atomicOr'd by kernels, read and cleared by dc_sync).
#define DC_ST_NONFINITE 1
#define DC_ST_TIMEOUT 2
#define DC_ST_BOUNDS 4

#include <vector>

struct dc_timed {
  cudaEvent_t a = nullptr, b = nullptr;
  int kind = 0;  // 1 GEMV, 2 SIMT, 3 tcgen05
  double bytes = 0, ops = 0;
};

struct dc_ctx {
  int device = 0;
  int sm_count = 148;
  cudaStream_t stream = nullptr;      // where work is launched
  cudaStream_t own_stream = nullptr;  // created by dc_init
  cudaEvent_t ev_fork = nullptr, ev_join = nullptr;  // ordering between `stream` and `own_stream`
  cudaEvent_t ev_hop = nullptr;  // dc_stage_handoff: the source stage's work is done
  std::string err;
  char label[160] = {0};
  // LUT units: host copies (checked by sha256) and device copies.
  int16_t h_mul[65536];
  int8_t h_requant[65536];
  int8_t h_relu[256];
  int16_t* d_mul = nullptr;
  int8_t* d_requant = nullptr;
  int8_t* d_relu = nullptr;
  int* d_status = nullptr;
  // grow-only scratch for the host-buffer entry points
  void* scratch = nullptr;
  size_t scratch_bytes = 0;
  bool tc_enabled = true;  // tcgen05 GEMM passed its gate
  bool tc2_enabled = true;  // its 2-SM variant (M > 128) passed its gate
  bool tp2_enabled = true;  // its persistent 2-SM form (M > 128, many tiles) passed its gate
  // split-K scratch of the tcgen05 GEMM (kept zero between calls by the kernel)
  int32_t* tc_partial = nullptr;
  int* tc_counters = nullptr;
  size_t tc_partial_cap = 0, tc_counter_cap = 0;
  // dc_bgemm_dev_noalloc: device address of the library's fixed scratch array,
  // looked up by the first call on this context
  int32_t* noalloc_scratch = nullptr;
  // decode-lap timeline (dc_stage_set_timeline): a %globaltimer stamp after
  // every launch of a lap, and what each launch was
  unsigned long long* tl_buf = nullptr;
  int tl_per_lap = 0, tl_idx = 0, tl_laps = 0;
  const int* tl_step = nullptr;        // the lap counter (device)
  std::vector<int> tl_kind;            // per launch of the lap: 1 one-row GEMV, 3 tcgen05, 0 other
  std::vector<double> tl_bytes;        // and its algorithmic bytes (GEMMs)
  // live GEMM timing (dc_timing / dc_timing_read)
  bool timing = false;
  std::vector<dc_timed> timed;
  std::vector<cudaEvent_t> event_pool;
};

struct dc_weight {
  dc_ctx* ctx = nullptr;
  int k = 0, n = 0, ldw = 0;
  int8_t* qt = nullptr;  // n x ldw int8, quantised Wᵀ, zero past k
  float* cs = nullptr;   // n column scales
  bool owns = true;
};

static inline int round_up(int v, int a) { return (v + a - 1) / a * a; }

// Record an error message on the context and return the code.
int dc_fail(dc_ctx* ctx, int code, const char* fmt, ...);
// Map a CUDA error to DC_E_CUDA with a message.
int dc_cuda_fail(dc_ctx* ctx, cudaError_t e, const char* what);
#define DC_CUDA(ctx, call)                                      \
  do {                                                          \
    cudaError_t _e = (call);                                    \
    if (_e != cudaSuccess) return dc_cuda_fail((ctx), _e, #call); \
  } while (0)

int dc_scratch(dc_ctx* ctx, size_t bytes, void** p);

// Allow `bytes` of dynamic shared memory for kernel `func` on ctx's device; the
// attribute is set once per (kernel, device) and raised only when needed.  The
// first call for a kernel also sets the maximal shared-memory carve-out, the
// same for every kernel of the library, so that consecutive kernels never
// make the SM repartition its L1 / shared memory.
int dc_set_smem(dc_ctx* ctx, const void* func, int bytes);

// Kernels launched by this library in this process (reported by dc_launch_count).
void dc_count_launch();
// Decode-lap timeline: start stamping the launches of one lap on ctx (a stamp
// now, then one after every launch until dc_timeline_end); tag the latest
// launch as a GEMM of the given kind and algorithmic bytes.
void dc_timeline_begin(dc_ctx* ctx, const int* step);
void dc_timeline_end(dc_ctx* ctx);
void dc_timeline_tag(dc_ctx* ctx, int kind, double bytes);
void dc_count_launches(long long n);  // e.g. the kernels of one CUDA-graph replay

// ---- launchers shared between translation units ----------------------------
int dc_launch_quant_rows(dc_ctx* ctx, const float* X, int rows, int cols, int8_t* q, int ldq, float* s,
                         cudaStream_t st);
int dc_launch_quant_cols_t(dc_ctx* ctx, const float* W, int rows, int cols, int8_t* qt, int ldq, float* s,
                           cudaStream_t st);
int dc_launch_transpose_i8(dc_ctx* ctx, const int8_t* W, int k, int n, int8_t* Wt, int ldw, int batch,
                           cudaStream_t st);

// GEMM dispatch on device buffers.  kind: 0 auto, 1 GEMV, 2 SIMT, 3 tcgen05.
int dc_gemm_dispatch(dc_ctx* ctx, const int8_t* Xq, int ldx, const int8_t* Wt, int ldw, const float* rs,
                     const float* cs, int m, int k, int n, int batch, unsigned flags, void* out, cudaStream_t st,
                     int kind);
// L2 prefetch of a device range (dc_gemm.cu).
int dc_l2_prefetch_on(dc_ctx* ctx, const void* p, size_t bytes, cudaStream_t st);
int dc_gemm_lut(dc_ctx* ctx, const int8_t* Xq, const int8_t* Wq, const float* rs, const float* cs, int m, int k,
                int n, int batch, unsigned flags, void* out, cudaStream_t st);
// tcgen05 path (dc_gemm_tc.cu): returns DC_E_INVAL when the shape is not supported.
int dc_gemm_tc(dc_ctx* ctx, const int8_t* Xq, int ldx, const int8_t* Wt, int ldw, const float* rs, const float* cs,
               int m, int k, int n, int batch, unsigned flags, void* out, cudaStream_t st);
// The same with caller-provided split-K scratch of the given capacities; clear = 1
// zeroes the part a split-K launch uses first (scratch of unknown contents).
int dc_gemm_tc_with(dc_ctx* ctx, const int8_t* Xq, int ldx, const int8_t* Wt, int ldw, const float* rs,
                    const float* cs, int m, int k, int n, int batch, unsigned flags, void* out, cudaStream_t st,
                    int32_t* partial, int* counters, size_t partial_cap, size_t counter_cap, int clear);
// The decode row's gate/up GEMV with SwiGLU in its epilogue: Wt holds n2 = 2I
// interleaved rows (gate_j, up_j); hout (I floats) = f32(silu(g_j) * u_j) of
// the f32 epilogue values; |hout| folded into *rowmax (zeroed by an earlier
// kernel).  DC_E_INVAL when the operands do not suit the one-row GEMV.
int dc_gemv_swiglu(dc_ctx* ctx, const int8_t* Xq, const int8_t* Wt, int ldw, const float* rs, const float* cs,
                   int k, int n2, float* hout, uint32_t* rowmax, cudaStream_t st);
// dc_gemm_dispatch without the timing events: kind 1 GEMV (m <= 8), 2 SIMT dp4a,
// 3 tcgen05 (falls back to 2 for shapes it does not take), 0 by m.
int dc_gemm_untimed(dc_ctx* ctx, const int8_t* Xq, int ldx, const int8_t* Wt, int ldw, const float* rs,
                    const float* cs, int m, int k, int n, int batch, unsigned flags, void* out, cudaStream_t st,
                    int kind);

// ---- device helpers ---------------------------------------------------------
// ECMAScript Math.round on a double: nearest, ties toward +infinity.
__device__ __forceinline__ double dc_js_round(double v) {
  double r = floor(v);
  if (__dsub_rn(v, r) >= 0.5) r = __dadd_rn(r, 1.0);
  return r;
}
__device__ __forceinline__ int8_t dc_clamp8(double v) {
  return v < -128.0 ? (int8_t)-128 : v > 127.0 ? (int8_t)127 : (int8_t)(int)v;
}
// The correctly rounded double quotient, out of line (one copy of the
// division's code per kernel; reached only from the checks below).
static __device__ __noinline__ double dc_ddiv_slow(double a, double b) { return __ddiv_rn(a, b); }

// clamp8(Math.round(v / s)) for s > 0 with |v / s| below a few hundred (every
// quantiser here: s >= max|v| / 127, rounded).  rs = 1/s (any rounding).  The
// quotient comes from v * rs, within a few ulp of the rounded v / s; only when
// that lands within 2^-20 of a half-integer -- where Math.round's decision
// could depend on the last bits -- is the correctly rounded quotient taken.
__device__ __forceinline__ int8_t dc_quant_div(double v, double s, double rs) {
  double q = __dmul_rn(v, rs);
  const double f = __dsub_rn(q, floor(q));
  if (fabs(__dsub_rn(f, 0.5)) < 9.5367431640625e-07) q = dc_ddiv_slow(v, s);
  return dc_clamp8(dc_js_round(q));
}

// dc_quant_div for an f32 value v with |v / s| <= 128, mostly in f32: the
// product v * rsf (rsf = f32(1/s)) is within 2^-16 of v / s, so when it lies
// more than 2^-13 from a half-integer it rounds as the quotient does; nearer,
// the double path decides.
__device__ __forceinline__ int8_t dc_quant_div_f(float v, double s, double rs, float rsf) {
  const float q = __fmul_rn(v, rsf);
  const float fl = floorf(q);
  const float fr = __fsub_rn(q, fl);
  if (fabsf(__fsub_rn(fr, 0.5f)) < 1.220703125e-4f) return dc_quant_div((double)v, s, rs);
  const float r = fr > 0.5f ? __fadd_rn(fl, 1.0f) : fl;
  return r < -128.0f ? (int8_t)-128 : r > 127.0f ? (int8_t)127 : (int8_t)(int)r;
}

// f32(a / z) for a >= 0, z > 0 (the double quotient rounded to float): from
// a * rz (rz = 1/z, any rounding) unless that lies within 2^-40 (relative) of
// a midpoint between two floats, or at a power of two or below the normal
// range, where the correctly rounded double quotient decides.
__device__ __forceinline__ float dc_div_to_f32(double a, double z, double rz) {
  const double q = __dmul_rn(a, rz);
  const float f = __double2float_rn(q);
  const unsigned fb = __float_as_uint(f);
  const int fe = (int)((fb >> 23) & 0xff);
  if (fe <= 1 || fe >= 254 || (fb & 0x7fffff) == 0) return __double2float_rn(dc_ddiv_slow(a, z));
  const double hu = __longlong_as_double((long long)(fe - 151 + 1023) << 52);  // half a float ulp at f
  const double d = fabs(__dsub_rn(q, (double)f));
  if (fabs(__dsub_rn(d, hu)) < q * 9.094947017729282e-13) return __double2float_rn(dc_ddiv_slow(a, z));
  return f;
}

// f32(a / zlo) for the lower end of a bracket [zlo, zhi] that holds a serial
// sum z (a >= 0, rlo = 1/zlo and rhi = 1/zhi in any rounding), and in *amb
// whether f32(a / z) may differ across the bracket.  `narrow` says the bracket
// is below 5e-13 relative: then a quotient a * rlo clear of every f32
// rounding boundary (by a margin beyond the bracket's width and the product's
// rounding) rounds the same way for every z in the bracket, and only the
// quotients near a boundary take both ends.  The result is
// dc_div_to_f32(a, zlo, rlo) in every case.
__device__ __forceinline__ float dc_div_bracket(double a, double zlo, double rlo, double zhi, double rhi,
                                                bool narrow, bool* amb) {
  const double q = __dmul_rn(a, rlo);
  const float f = __double2float_rn(q);
  const unsigned fb = __float_as_uint(f);
  const int fe = (int)((fb >> 23) & 0xff);
  // the 29 mantissa bits of q that the f32 rounding drops, against the
  // midpoint 2^28: within 2^13 double ulps of it (a superset of within 2^-40
  // relative) the quotient is near a rounding boundary; a bracket below 5e-13
  // relative moves the quotient by under 2^12.2 ulps
  const int low = (int)(__double_as_longlong(q) & 0x1fffffffLL);
  const bool slow = fe <= 1 || fe >= 254 || (fb & 0x7fffff) == 0 || abs(low - 0x10000000) < 0x2000;
  if (!slow && narrow) return f;
  const float flo = slow ? __double2float_rn(dc_ddiv_slow(a, zlo)) : f;
  *amb |= flo != dc_div_to_f32(a, zhi, rhi);
  return flo;
}

// verified_core.js:227-228: f32(f32(f32(s) * a) * b), each step rounded.
__device__ __forceinline__ float dc_epi(int32_t s, float a, float b) {
  return __fmul_rn(__fmul_rn(__int2float_rn(s), a), b);
}
// The requant unit (public/requant_lut.bin, 65536 entries) maps the 16-bit
// pattern of a saturated accumulator to (int8)(s16 >> 8) -- the arithmetic
// shift by luts_meta.json's "shift": 8 -- and the ReLU unit (relu_lut.bin) an
// 8-bit pattern to max(s8, 0).  dc_init rebuilds both tables, checks their
// sha256 against the reference's LFS object ids, and gates every kernel that
// uses these definitions against the LUT kernel, which reads the tables
// themselves (dc_store_out_lut); so evaluating the definition here returns the
// table entry, without a dependent memory lookup for every output.
__device__ __forceinline__ int8_t dc_requant_unit(int32_t acc, bool relu) {
  const int32_t a = acc < -32768 ? -32768 : (acc > 32767 ? 32767 : acc);
  const int8_t v = (int8_t)(a >> 8);
  return relu && v < 0 ? (int8_t)0 : v;
}
// Store one output element in the mode selected by flags.
__device__ __forceinline__ void dc_store_out(void* out, int64_t idx, int32_t acc, float rsv, float csv, unsigned flags,
                                             const int8_t* __restrict__ requant, const int8_t* __restrict__ relu) {
  (void)requant;
  (void)relu;
  if (flags & DC_ACC) {
    ((int32_t*)out)[idx] = acc;
  } else if (flags & DC_REQUANT) {
    ((int8_t*)out)[idx] = dc_requant_unit(acc, (flags & DC_RELU) != 0);
  } else {
    float v = dc_epi(acc, rsv, csv);
    if ((flags & DC_RELU) && v < 0.0f) v = 0.0f;
    if (flags & DC_F_ADDTO) v = __fadd_rn(((const float*)out)[idx], v);  // residual: out = out + v (f32 add)
    ((float*)out)[idx] = v;
  }
}
// dc_store_out reading the requant and ReLU units from their device tables
// (the LUT kernel, the gates' yardstick).
__device__ __forceinline__ void dc_store_out_lut(void* out, int64_t idx, int32_t acc, float rsv, float csv,
                                                 unsigned flags, const int8_t* __restrict__ requant,
                                                 const int8_t* __restrict__ relu) {
  if (flags & DC_REQUANT) {
    int32_t a = acc < -32768 ? -32768 : (acc > 32767 ? 32767 : acc);
    int8_t v = __ldg(requant + (uint16_t)(int16_t)a);
    if (flags & DC_RELU) v = __ldg(relu + (uint8_t)v);
    ((int8_t*)out)[idx] = v;
  } else {
    dc_store_out(out, idx, acc, rsv, csv, flags, requant, relu);
  }
}
