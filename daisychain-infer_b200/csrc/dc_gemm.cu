// dc_gemm.cu -- the verified W8A8 GEMM unit (compute.bgemm, public/webgpu.js:836-857).
//
// out[bz, i, j] = epilogue( sum_p X[bz, i, p] * W[bz, p, j] )  (int8 x int8 -> int32)
//
// The mul LUT is the exact product table s8(a)*s8(b) (its sha256 equals the
// reference's LFS object), so an integer dot product IS the LUT GEMM; the
// int32 sum is exact because k <= 131071 keeps |sum| < 2^31
// (verified_core.js:41-49).  Kernels here:
//   k_lut_gemm   every product looked up in the mul unit (the reference's
//                WGSL_BG_LUT twin, webgpu.js:108-133); the init gate's yardstick
//   k_gemv       M <= 8 rows: HBM-streaming, 128-bit weight loads, dp4a,
//                warp-shuffle reduction (decode, lm_head, lookahead rows)
//   k_gemm_simt  dp4a register-tiled GEMM for shapes the tensor-core path
//                does not take
// and the tcgen05 tensor-core kernel in dc_gemm_tc.cu.
#include <stdarg.h>

#include <algorithm>

#include "dc_internal.cuh"
#include "dc_math.cuh"
#include "dc_ptx.cuh"

namespace {

// ---- the LUT twin: one thread per output, reference layouts ----------------
__global__ void k_lut_gemm(const int8_t* __restrict__ X, const int8_t* __restrict__ W, const float* __restrict__ rs,
                           const float* __restrict__ cs, int m, int k, int n, unsigned flags,
                           const int16_t* __restrict__ mul, const int8_t* __restrict__ requant,
                           const int8_t* __restrict__ relu, void* out) {
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  const int col = blockIdx.y * blockDim.y + threadIdx.y;
  const int bz = blockIdx.z;
  if (row >= m || col >= n) return;
  const int8_t* xr = X + ((int64_t)bz * m + row) * k;
  const int8_t* wc = W + (int64_t)bz * k * n + col;
  uint32_t s = 0;
  for (int p = 0; p < k; p++) s += (uint32_t)(int32_t)__ldg(mul + ((uint8_t)xr[p]) * 256 + (uint8_t)wc[(int64_t)p * n]);
  dc_store_out_lut(out, ((int64_t)bz * m + row) * n + col, (int32_t)s, rs[bz * m + row], cs[bz * n + col], flags, requant,
               relu);
}

// A weight load: read once, so it bypasses L1 and is first out of L2 (`pol`
// from dcp::l2_evict_first()).
__device__ __forceinline__ int4 ld_stream(const int4* p, uint64_t pol) {
  int4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.s32 {%0,%1,%2,%3}, [%4], %5;"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p), "l"(pol));
  return v;
}

// ---- GEMV: M <= MR rows ---------------------------------------------------
// G warps per output column j (G = 1, 2, 4 or 8: more than one when the matrix
// has fewer columns than the GPU has warps), each streaming a contiguous K
// slice of the weight row Wᵀ[j] with 16-byte non-allocating loads, 8 in flight
// per lane (one 4 KB row in a single round trip).  The MR activation rows sit in
// shared memory.  Partial sums are int32 (exact in any order): a butterfly
// shuffle inside the warp, then the G warps of a column add theirs in shared
// memory.  Columns step through the grid; the block's 8 warps move together.
__device__ __forceinline__ int dp4a16g(const int4 a, const int4 b, int acc) {
  acc = __dp4a(a.x, b.x, acc);
  acc = __dp4a(a.y, b.y, acc);
  acc = __dp4a(a.z, b.z, acc);
  return __dp4a(a.w, b.w, acc);
}

template <int MR, int G>
__global__ void __launch_bounds__(256, 3) k_gemv(const int8_t* __restrict__ X, int ldx,
                                                 const int8_t* __restrict__ Wt, int ldw,
                                                 const float* __restrict__ rs, const float* __restrict__ cs, int m,
                                                 int k, int n, unsigned flags, const int8_t* __restrict__ requant,
                                                 const int8_t* __restrict__ relu, void* out) {
  extern __shared__ int4 xs[];
  __shared__ int part[8][MR];
  const int bz = blockIdx.y;
  const int nch = (k + 15) >> 4;  // 16-byte chunks per row (<= ldx/16, ldw/16)
  const int8_t* Xb = X + (int64_t)bz * m * ldx;
  for (int idx = threadIdx.x; idx < MR * nch; idx += blockDim.x) {
    const int r = idx / nch, c = idx - r * nch;
    xs[idx] = (r < m) ? *((const int4*)(Xb + (int64_t)r * ldx) + c) : make_int4(0, 0, 0, 0);
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int SLOTS = 8 / G;  // columns per block step
  const int slot = warp / G, kp = warp - slot * G;
  const int per = (nch + G - 1) / G;
  const int c_lo = kp * per, c_hi = min(nch, c_lo + per);
  const int8_t* Wb = Wt + (int64_t)bz * n * ldw;
  const uint64_t pol = dcp::l2_evict_first();
  for (int jb = blockIdx.x * SLOTS; jb < n; jb += gridDim.x * SLOTS) {
    const int j = jb + slot;
    int acc[MR];
#pragma unroll
    for (int r = 0; r < MR; r++) acc[r] = 0;
    if (j < n) {
      const int4* wrow = (const int4*)(Wb + (int64_t)j * ldw);
      for (int c = c_lo + lane; c < c_hi; c += 256) {
        int4 w[8];
#pragma unroll
        for (int u = 0; u < 8; u++) w[u] = (c + 32 * u < c_hi) ? ld_stream(wrow + c + 32 * u, pol) : make_int4(0, 0, 0, 0);
#pragma unroll
        for (int u = 0; u < 8; u++) {
          if (c + 32 * u < c_hi) {
#pragma unroll
            for (int r = 0; r < MR; r++) acc[r] = dp4a16g(w[u], xs[r * nch + c + 32 * u], acc[r]);
          }
        }
      }
#pragma unroll
      for (int r = 0; r < MR; r++)
#pragma unroll
        for (int o = 16; o; o >>= 1) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], o);
    }
    if (G > 1) {
      if (lane == 0)
#pragma unroll
        for (int r = 0; r < MR; r++) part[warp][r] = acc[r];
      __syncthreads();
      if (kp == 0 && lane < MR && lane < m && j < n) {
        int v = 0;
        for (int q = 0; q < G; q++) v += part[warp + q][lane];
        dc_store_out(out, ((int64_t)bz * m + lane) * n + j, v, rs[bz * m + lane], cs[bz * n + j], flags, requant,
                     relu);
      }
      __syncthreads();
    } else {
      int mine = 0;
#pragma unroll
      for (int r = 0; r < MR; r++)
        if (r == lane) mine = acc[r];
      if (lane < MR && lane < m && j < n)
        dc_store_out(out, ((int64_t)bz * m + lane) * n + j, mine, rs[bz * m + lane], cs[bz * n + j], flags, requant,
                     relu);
    }
  }
}

// ---- L2 prefetch -------------------------------------------------------------
// Bulk prefetches (cp.async.bulk.prefetch.L2) of [p, p + bytes) in 64 KB
// pieces, spread over the grid: the copy engine pulls the bytes into L2 while
// the issuing threads move on.  p and bytes are 16-byte multiples.
__global__ void k_l2_prefetch(const int8_t* __restrict__ p, size_t bytes) {
  constexpr size_t PIECE = 65536;
  const size_t npiece = (bytes + PIECE - 1) / PIECE;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < npiece; i += (size_t)gridDim.x * blockDim.x) {
    const size_t off = i * PIECE;
    const uint32_t len = (uint32_t)((bytes - off) < PIECE ? (bytes - off) : PIECE);
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p + off), "r"(len) : "memory");
  }
}

// ---- one-row GEMV (M = 1), the decode path ---------------------------------
// Each warp takes two weight rows (output columns) at a time and walks K in
// segments of 8 x 32 16-byte chunks: the 16 streaming weight loads of a
// segment (L1 no-allocate) and its 8 activation loads (L1-resident: every warp
// reads the same row) are issued back to back, then consumed by dp4a.  No
// shared memory, no prologue: a CTA starts pulling weights at its first
// instruction, and 4-warp CTAs at 4 per SM keep ~128 KB of loads in flight on
// each SM.  Grid-stride over row pairs; the epilogue is dc_store_out, or with
// DC_F_SWIGLU (interleaved gate/up rows: a warp's pair is gate_j, up_j) the
// SwiGLU of the pair's two f32 epilogue values, stored at j, with the CTA's
// |h| maximum folded into *rowmax by one atomic per CTA.  The SwiGLU (a chain
// of double-precision exp and division) is deferred: lane t % 32 keeps the
// accumulators of the warp's t-th pair, and every 32 pairs (and at the end)
// the lanes evaluate theirs side by side, off the weight stream's path.
constexpr int GV_SEG = 8;
// X and rs are written by the kernel before this one on the stream: they carry
// no __restrict__, so that no load of them is moved above griddepcontrol.wait.
__global__ void __launch_bounds__(128, 4) k_gemv_row(const int8_t* X, const int8_t* __restrict__ Wt,
                                                     int ldw, const float* rs,
                                                     const float* __restrict__ cs, int k, int n, unsigned flags,
                                                     const int8_t* __restrict__ requant,
                                                     const int8_t* __restrict__ relu, void* out,
                                                     uint32_t* rowmax, int* status) {
  // the next kernel (launched as a programmatic dependent) may be scheduled
  // now; it waits for this grid's completion before reading its output
  // (DC_F_LATE_RELEASE: once this grid has passed its own wait)
  if (!(flags & DC_F_LATE_RELEASE)) asm volatile("griddepcontrol.launch_dependents;");
  __shared__ float wmax[4];
  // (DC_F_SWIGLU) the pair this lane keeps, and its |h| maximum
  int sa0 = 0, sa1 = 0, sj = -1;
  float sc0 = 0.0f, sc1 = 0.0f, hmax = 0.0f;
  auto swiglu_flush = [&]() {
    if (sj >= 0) {
      const float r0 = rs[0];
      const float h = dcm::swiglu_f32(dc_epi(sa0, r0, sc0), dc_epi(sa1, r0, sc1));
      ((float*)out)[sj] = h;
      if (!isfinite(h)) atomicOr(status, DC_ST_NONFINITE);
      hmax = fmaxf(hmax, fabsf(h));
      sj = -1;
    }
  };
  int t = 0;  // pairs this warp has taken
  const int lane = threadIdx.x & 31;
  // warps numbered across blocks first: the last, partial round of row pairs
  // falls on one warp in each of many blocks (SMs), not on whole blocks
  const int gw = (threadIdx.x >> 5) * gridDim.x + blockIdx.x, nw = gridDim.x * 4;
  const int nch = (k + 15) >> 4;
  const int4* X4 = (const int4*)X;
  const uint64_t pol = dcp::l2_evict_first();
  bool waited = false;
  // loaded right after the wait, so that their round trips overlap the
  // weight stream: the row scale, and (f32 residual adds) this lane's output
  // value of the warp's first pair
  const bool addto = (flags & DC_F_ADDTO) && !(flags & (DC_ACC | DC_REQUANT | DC_F_SWIGLU));
  float rs0 = 0.0f, res0 = 0.0f;
  for (int j0 = gw * 2; j0 < n; j0 += nw * 2, t++) {
    const int j1 = min(j0 + 1, n - 1);
    const int4* w0 = (const int4*)(Wt + (int64_t)j0 * ldw);
    const int4* w1 = (const int4*)(Wt + (int64_t)j1 * ldw);
    // L2 requests ahead of the register loads: the rest of these two rows past
    // the first segment, and the warp's next two rows, so each later round
    // trip of the warp starts from L2 instead of DRAM
    {
      const int jn = j0 + nw * 2;
      const char* p0 = (const char*)w0;
      const char* p1 = (const char*)w1;
      for (int b = 32 * GV_SEG * 16 + lane * 128; b < k; b += 32 * 128) {
        asm volatile("prefetch.global.L2 [%0];" ::"l"(p0 + b));
        asm volatile("prefetch.global.L2 [%0];" ::"l"(p1 + b));
      }
      if (jn < n) {
        const char* q0 = (const char*)(Wt + (int64_t)jn * ldw);
        const char* q1 = (const char*)(Wt + (int64_t)min(jn + 1, n - 1) * ldw);
        for (int b = lane * 128; b < k; b += 32 * 128) {
          asm volatile("prefetch.global.L2 [%0];" ::"l"(q0 + b));
          asm volatile("prefetch.global.L2 [%0];" ::"l"(q1 + b));
        }
      }
    }
    const float csv = cs[lane == 1 ? j1 : j0];  // the epilogue's column scale, loaded with the weights
    int a0 = 0, a1 = 0;
#pragma unroll 1
    for (int c0 = 0; c0 < nch; c0 += 32 * GV_SEG) {
      int4 wa[GV_SEG], wb[GV_SEG], xv[GV_SEG];
#pragma unroll
      for (int u = 0; u < GV_SEG; u++) {
        const int c = c0 + u * 32 + lane;
        wa[u] = c < nch ? ld_stream(w0 + c, pol) : make_int4(0, 0, 0, 0);
        wb[u] = c < nch ? ld_stream(w1 + c, pol) : make_int4(0, 0, 0, 0);
      }
      if (!waited) {
        // launched as a programmatic dependent: the weights (constant) are
        // already in flight; the activation row is read only after the
        // kernel that writes it has completed
        asm volatile("griddepcontrol.wait;" ::: "memory");
        waited = true;
        if (flags & DC_F_LATE_RELEASE) asm volatile("griddepcontrol.launch_dependents;");
        rs0 = rs[0];
        if (addto && lane < 2 && j0 + lane < n) res0 = ((const float*)out)[j0 + lane];
      }
#pragma unroll
      for (int u = 0; u < GV_SEG; u++) {
        const int c = c0 + u * 32 + lane;
        xv[u] = c < nch ? X4[c] : make_int4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < GV_SEG; u++) {
        a0 = dp4a16g(wa[u], xv[u], a0);
        a1 = dp4a16g(wb[u], xv[u], a1);
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      a0 += __shfl_xor_sync(0xffffffffu, a0, o);
      a1 += __shfl_xor_sync(0xffffffffu, a1, o);
    }
    if (flags & DC_F_SWIGLU) {
      const float c0 = __shfl_sync(0xffffffffu, csv, 0), c1 = __shfl_sync(0xffffffffu, csv, 1);
      if (lane == (t & 31)) {
        sa0 = a0;
        sa1 = a1;
        sc0 = c0;
        sc1 = c1;
        sj = j0 >> 1;
      }
      if ((t & 31) == 31) swiglu_flush();
    } else if (addto && t == 0) {  // the first pair: its residuals are in res0
      if (lane < 2 && j0 + lane < n) {
        float v = dc_epi(lane == 0 ? a0 : a1, rs0, csv);
        if ((flags & DC_RELU) && v < 0.0f) v = 0.0f;
        ((float*)out)[j0 + lane] = __fadd_rn(res0, v);  // residual: out = out + v (f32 add)
      }
    } else {
      if (lane == 0) dc_store_out(out, j0, a0, rs0, csv, flags, requant, relu);
      if (lane == 1 && j0 + 1 < n) dc_store_out(out, j0 + 1, a1, rs0, csv, flags, requant, relu);
    }
  }
  if (!waited) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (flags & DC_F_LATE_RELEASE) asm volatile("griddepcontrol.launch_dependents;");
  }
  if (flags & DC_F_SWIGLU) {
    swiglu_flush();
#pragma unroll
    for (int o = 16; o; o >>= 1) hmax = fmaxf(hmax, __shfl_xor_sync(0xffffffffu, hmax, o));
    if (lane == 0) wmax[threadIdx.x >> 5] = hmax;
    __syncthreads();
    if (threadIdx.x == 0)
      atomicMax(rowmax, __float_as_uint(fmaxf(fmaxf(wmax[0], wmax[1]), fmaxf(wmax[2], wmax[3]))));
  }
}

// ---- bulk-staged GEMV: M <= MR rows, the decode path -----------------------
// One CTA per SM streams a contiguous range of weight rows (rows_per_cta rows
// of Wᵀ, i.e. output columns) through a ring of `stages` shared-memory stages
// of R rows each, filled by 1-D bulk async copies (cp.async.bulk + mbarrier
// transaction counts) issued by one producer thread: several 20-32 KB copies
// are in flight per SM, which is what keeps HBM busy.  Eight consumer warps
// form the dot products from shared memory (16-byte reads, dp4a, butterfly
// shuffle).  When a stage holds fewer than 8 rows, WR = 8/R warps share a row
// and add their int32 partials with shared-memory atomics; the last of them
// applies the epilogue.  Waits are bounded; a timeout aborts the whole CTA.
//
// Launched as a programmatic dependent: the producer starts streaming weights
// (constant) at once; the consumer warps read the activation rows (written by
// the previous kernel: X and rs carry no __restrict__) after
// griddepcontrol.wait and meet on a named barrier.
template <int MR>
__global__ void __launch_bounds__(288, 1) k_gemv_bulk(const int8_t* X, int ldx,
                                                      const int8_t* __restrict__ Wt, int ldw,
                                                      const float* rs, const float* __restrict__ cs,
                                                      int m, int k, int n, unsigned flags,
                                                      const int8_t* __restrict__ requant,
                                                      const int8_t* __restrict__ relu, void* out, int R, int stages,
                                                      int rows_per_cta, int* status) {
  extern __shared__ __align__(128) uint8_t smraw[];
  __shared__ int rowacc[8][8][MR];  // [stage % 8][row in stage][r]
  __shared__ int rowcnt[8][8];
  __shared__ int abort_flag;
  const int nch = (k + 15) >> 4;
  const int stage_bytes = R * ldw;
  uint8_t* sW = smraw;
  int4* xs = (int4*)(smraw + (size_t)stages * stage_bytes);
  uint64_t* full = (uint64_t*)(xs + MR * nch);
  uint64_t* empty = full + stages;
  // DC_F_LATE_RELEASE: the dependent launches when this grid completes
  if (!(flags & DC_F_LATE_RELEASE)) asm volatile("griddepcontrol.launch_dependents;");
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bz = blockIdx.y;
  const int rb = blockIdx.x * rows_per_cta;
  const int nrows = min(n, rb + rows_per_cta) - rb;
  const int nst = nrows > 0 ? (nrows + R - 1) / R : 0;
  if (tid == 0) {
    for (int s = 0; s < stages; s++) {
      dcp::mbar_init(&full[s], 1);
      dcp::mbar_init(&empty[s], 8);
    }
    dcp::mbar_fence_init();
    abort_flag = 0;
  }
  for (int i = tid; i < 8 * 8 * MR; i += blockDim.x) (&rowacc[0][0][0])[i] = 0;
  for (int i = tid; i < 8 * 8; i += blockDim.x) (&rowcnt[0][0])[i] = 0;
  __syncthreads();
  if (nst == 0) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    return;
  }
  if (warp < 8) {
    // consumers: the activation rows, once the kernel that writes them is done
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int8_t* Xb = X + (int64_t)bz * m * ldx;
    for (int idx = tid; idx < MR * nch; idx += 256) {
      const int r = idx / nch, c = idx - r * nch;
      xs[idx] = (r < m) ? *((const int4*)(Xb + (int64_t)r * ldx) + c) : make_int4(0, 0, 0, 0);
    }
    dcp::named_sync(1, 256);
  }
  if (warp == 8) {
    // ---- producer
    if (lane == 0) {
      int issued = 0;
      const int8_t* Wb = Wt + ((int64_t)bz * n + rb) * ldw;
      const uint64_t pol = dcp::l2_evict_first();
      for (int it = 0; it < nst; it++) {
        const int s = it % stages;
        if (it >= stages && !dcp::mbar_wait(&empty[s], (uint32_t)((it / stages) - 1) & 1u, status)) {
          atomicExch(&abort_flag, 1);
          break;
        }
        if (*(volatile int*)&abort_flag) break;
        const int rows_this = min(R, nrows - it * R);
        const uint32_t bytes = (uint32_t)rows_this * (uint32_t)ldw;
        dcp::mbar_expect_tx(&full[s], bytes);
        dcp::bulk_load_hint(sW + (size_t)s * stage_bytes, Wb + (int64_t)it * R * ldw, bytes, &full[s], pol);
        issued++;
      }
      // let every issued copy land before this CTA's shared memory can go away
      for (int it = max(0, issued - stages); it < issued; it++)
        dcp::mbar_wait(&full[it % stages], (uint32_t)(it / stages) & 1u, status);
    }
    return;
  }
  // ---- consumers
  const int WR = R >= 8 ? 1 : 8 / R;
  const int per = (nch + WR - 1) / WR;
  for (int it = 0; it < nst; it++) {
    const int s = it % stages;
    if (*(volatile int*)&abort_flag) break;
    if (!dcp::mbar_wait(&full[s], (uint32_t)(it / stages) & 1u, status)) {
      atomicExch(&abort_flag, 1);
      break;
    }
    const int rows_this = min(R, nrows - it * R);
    const uint8_t* base = sW + (size_t)s * stage_bytes;
    const int j0 = rb + it * R;
    if (WR == 1) {
      for (int rr = warp; rr < rows_this; rr += 8) {
        const int4* wr = (const int4*)(base + (size_t)rr * ldw);
        int acc[MR];
#pragma unroll
        for (int r = 0; r < MR; r++) acc[r] = 0;
        for (int c = lane; c < nch; c += 32) {
          const int4 w = wr[c];
#pragma unroll
          for (int r = 0; r < MR; r++) acc[r] = dp4a16g(w, xs[r * nch + c], acc[r]);
        }
#pragma unroll
        for (int r = 0; r < MR; r++)
#pragma unroll
          for (int o = 16; o; o >>= 1) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], o);
        int mine = 0;
#pragma unroll
        for (int r = 0; r < MR; r++)
          if (r == lane) mine = acc[r];
        if (lane < MR && lane < m) {
          const int j = j0 + rr;
          dc_store_out(out, ((int64_t)bz * m + lane) * n + j, mine, rs[bz * m + lane], cs[bz * n + j], flags, requant,
                       relu);
        }
      }
    } else {
      const int rr = warp / WR, p = warp - rr * WR;
      if (rr < rows_this) {
        const int4* wr = (const int4*)(base + (size_t)rr * ldw);
        const int c1 = min(nch, (p + 1) * per);
        int acc[MR];
#pragma unroll
        for (int r = 0; r < MR; r++) acc[r] = 0;
        for (int c = p * per + lane; c < c1; c += 32) {
          const int4 w = wr[c];
#pragma unroll
          for (int r = 0; r < MR; r++) acc[r] = dp4a16g(w, xs[r * nch + c], acc[r]);
        }
#pragma unroll
        for (int r = 0; r < MR; r++)
#pragma unroll
          for (int o = 16; o; o >>= 1) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], o);
        int* ra = rowacc[s & 7][rr];
        if (lane == 0)
#pragma unroll
          for (int r = 0; r < MR; r++) atomicAdd(&ra[r], acc[r]);
        __threadfence_block();
        __syncwarp();
        int last = 0;
        if (lane == 0) last = (atomicAdd(&rowcnt[s & 7][rr], 1) == WR - 1);
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
          __threadfence_block();
          if (lane < MR && lane < m) {
            const int j = j0 + rr;
            const int v = atomicExch(&ra[lane], 0);
            dc_store_out(out, ((int64_t)bz * m + lane) * n + j, v, rs[bz * m + lane], cs[bz * n + j], flags, requant,
                         relu);
          }
          if (lane == 0) rowcnt[s & 7][rr] = 0;
          __syncwarp();
        }
      }
    }
    __syncwarp();
    if (lane == 0) dcp::mbar_arrive(&empty[s]);
  }
}

// ---- SIMT dp4a GEMM: 64 x 64 output tile, 256 threads, 4 x 4 per thread ---
__global__ void __launch_bounds__(256) k_gemm_simt(const int8_t* __restrict__ X, int ldx,
                                                   const int8_t* __restrict__ Wt, int ldw,
                                                   const float* __restrict__ rs, const float* __restrict__ cs, int m,
                                                   int k, int n, unsigned flags, const int8_t* __restrict__ requant,
                                                   const int8_t* __restrict__ relu, void* out) {
  __shared__ int xs[64][17];
  __shared__ int ws[64][17];
  const int bz = blockIdx.z;
  const int row0 = blockIdx.y * 64, col0 = blockIdx.x * 64;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int8_t* Xb = X + (int64_t)bz * m * ldx;
  const int8_t* Wb = Wt + (int64_t)bz * n * ldw;
  int acc[4][4] = {};
  for (int k0 = 0; k0 < k; k0 += 64) {
    for (int idx = threadIdx.x; idx < 64 * 16; idx += 256) {
      int r = idx >> 4, c = idx & 15;
      int kk = k0 + 4 * c;
      int xv = 0, wv = 0;
      if (row0 + r < m && kk < ldx) xv = *(const int*)(Xb + (int64_t)(row0 + r) * ldx + kk);
      if (col0 + r < n && kk < ldw) wv = *(const int*)(Wb + (int64_t)(col0 + r) * ldw + kk);
      xs[r][c] = xv;
      ws[r][c] = wv;
    }
    __syncthreads();
#pragma unroll
    for (int c = 0; c < 16; c++) {
      int a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; i++) a[i] = xs[ty + 16 * i][c];
#pragma unroll
      for (int j = 0; j < 4; j++) b[j] = ws[tx + 16 * j][c];
#pragma unroll
      for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = __dp4a(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; i++) {
    int row = row0 + ty + 16 * i;
    if (row >= m) continue;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      int col = col0 + tx + 16 * j;
      if (col < n)
        dc_store_out(out, ((int64_t)bz * m + row) * n + col, acc[i][j], rs[bz * m + row], cs[bz * n + col], flags,
                     requant, relu);
    }
  }
}

template <int MR, int G>
int launch_gemv_g(dc_ctx* ctx, const int8_t* Xq, int ldx, const int8_t* Wt, int ldw, const float* rs,
                  const float* cs, int m, int k, int n, int batch, unsigned flags, void* out, cudaStream_t st,
                  size_t smem, int blocks) {
  if (smem > 48 * 1024)
    if (int rc = dc_set_smem(ctx, (const void*)k_gemv<MR, G>, (int)smem)) return rc;
  k_gemv<MR, G><<<dim3(blocks, batch), 256, smem, st>>>(Xq, ldx, Wt, ldw, rs, cs, m, k, n, flags, ctx->d_requant,
                                                        ctx->d_relu, out);
  dc_count_launch();
  DC_CUDA(ctx, cudaGetLastError());
  return DC_OK;
}

// Bulk-staged GEMV launch: ~32 KB stages of whole weight rows, as many stages as
// fit beside the activation rows, one CTA per SM over contiguous row ranges.
// Returns DC_E_INVAL (nothing launched) when the operands are not 16-byte
// aligned or a stage does not fit; the caller then uses k_gemv.
template <int MR>
int launch_gemv_bulk(dc_ctx* ctx, const int8_t* Xq, int ldx, const int8_t* Wt, int ldw, const float* rs,
                     const float* cs, int m, int k, int n, int batch, unsigned flags, void* out, cudaStream_t st) {
  if (((uintptr_t)Wt & 15) || ((uintptr_t)Xq & 15) || (ldw & 15) || (ldx & 15)) return DC_E_INVAL;
  const int nch = (k + 15) >> 4;
  const size_t xbytes = (size_t)MR * nch * 16;
  int R = 32768 / ldw;
  if (R >= 8) R = std::min(64, R / 8 * 8);
  else R = R >= 4 ? 4 : (R >= 2 ? 2 : 1);
  const size_t stage_bytes = (size_t)R * ldw;
  const size_t budget = 216 * 1024;
  if (xbytes + 2 * stage_bytes + 256 > budget) return DC_E_INVAL;
  const int stages = (int)std::min<size_t>(8, (budget - xbytes - 256) / stage_bytes);
  const size_t smem = (size_t)stages * stage_bytes + xbytes + 16 * (size_t)stages + 128;
  int gx = std::min(ctx->sm_count, n);
  const int rows_per_cta = (n + gx - 1) / gx;
  gx = (n + rows_per_cta - 1) / rows_per_cta;
  if (int rc = dc_set_smem(ctx, (const void*)k_gemv_bulk<MR>, (int)smem)) return rc;
  // a programmatic dependent: the weight stream starts while the previous kernel finishes
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(gx, batch);
  cfg.blockDim = dim3(288);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  DC_CUDA(ctx, cudaLaunchKernelEx(&cfg, k_gemv_bulk<MR>, Xq, ldx, Wt, ldw, rs, cs, m, k, n, flags,
                                  (const int8_t*)ctx->d_requant, (const int8_t*)ctx->d_relu, out, R, stages,
                                  rows_per_cta, ctx->d_status));
  dc_count_launch();
  DC_CUDA(ctx, cudaGetLastError());
  return DC_OK;
}

// k_gemv_row on one activation row (16-byte aligned operands), launched as a
// programmatic dependent: the CTAs may start, and issue their weight loads,
// while the previous kernel on the stream finishes.
static int launch_gemv_row(dc_ctx* ctx, const int8_t* Xq, const int8_t* Wt, int ldw, const float* rs,
                           const float* cs, int k, int n, unsigned flags, void* out, cudaStream_t st,
                           uint32_t* rowmax = nullptr) {
  if (int rc = dc_set_smem(ctx, (const void*)k_gemv_row, 0)) return rc;
  const int pairs = (n + 1) / 2;
  const int blocks = std::max(1, std::min(pairs, ctx->sm_count * 4));  // four per SM when there are pairs enough
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(blocks);
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  DC_CUDA(ctx, cudaLaunchKernelEx(&cfg, k_gemv_row, Xq, Wt, ldw, rs, cs, k, n, flags, (const int8_t*)ctx->d_requant,
                                  (const int8_t*)ctx->d_relu, out, rowmax, ctx->d_status));
  dc_count_launch();
  DC_CUDA(ctx, cudaGetLastError());
  return DC_OK;
}

template <int MR>
int launch_gemv(dc_ctx* ctx, const int8_t* Xq, int ldx, const int8_t* Wt, int ldw, const float* rs, const float* cs,
                int m, int k, int n, int batch, unsigned flags, void* out, cudaStream_t st) {
  if (MR == 1 && m == 1 && batch == 1 && !(((uintptr_t)Wt | (uintptr_t)Xq) & 15) && !(ldw & 15))
    return launch_gemv_row(ctx, Xq, Wt, ldw, rs, cs, k, n, flags, out, st);
  {
    const int rc = launch_gemv_bulk<MR>(ctx, Xq, ldx, Wt, ldw, rs, cs, m, k, n, batch, flags, out, st);
    if (rc != DC_E_INVAL) return rc;
  }
  const int nch = (k + 15) >> 4;
  const size_t smem = (size_t)MR * nch * 16;
  if (smem > 200 * 1024) return dc_fail(ctx, DC_E_INVAL, "gemv: k=%d too long for %d rows in shared memory", k, MR);
  const int per_sm = smem > 64 * 1024 ? 1 : 3;
  const int warps = ctx->sm_count * per_sm * 8;
  // warps per column: split K so that the (column, K-slice) units fill whole
  // rounds of the resident warps, keeping each slice at least 128 chunks
  int G = 1;
  double best = 0.0;
  for (int g = 1; g <= 8; g *= 2) {
    if (g > 1 && nch < 128 * g) break;
    const long units = (long)n * batch * g;
    const long rounds = (units + warps - 1) / warps;
    const double eff = (double)units / ((double)rounds * warps);
    if (eff > best + 0.02) {
      best = eff;
      G = g;
    }
  }
  int blocks = (n + 8 / G - 1) / (8 / G);
  if (blocks > ctx->sm_count * per_sm) blocks = ctx->sm_count * per_sm;
  if (blocks < 1) blocks = 1;
  switch (G) {
    case 1: return launch_gemv_g<MR, 1>(ctx, Xq, ldx, Wt, ldw, rs, cs, m, k, n, batch, flags, out, st, smem, blocks);
    case 2: return launch_gemv_g<MR, 2>(ctx, Xq, ldx, Wt, ldw, rs, cs, m, k, n, batch, flags, out, st, smem, blocks);
    case 4: return launch_gemv_g<MR, 4>(ctx, Xq, ldx, Wt, ldw, rs, cs, m, k, n, batch, flags, out, st, smem, blocks);
    default: return launch_gemv_g<MR, 8>(ctx, Xq, ldx, Wt, ldw, rs, cs, m, k, n, batch, flags, out, st, smem, blocks);
  }
}

}  // namespace

int dc_fail(dc_ctx* ctx, int code, const char* fmt, ...) {
  if (ctx) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    ctx->err = buf;
  }
  return code;
}

int dc_cuda_fail(dc_ctx* ctx, cudaError_t e, const char* what) {
  return dc_fail(ctx, DC_E_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

int dc_gemm_lut(dc_ctx* ctx, const int8_t* Xq, const int8_t* Wq, const float* rs, const float* cs, int m, int k,
                int n, int batch, unsigned flags, void* out, cudaStream_t st) {
  if (m == 0 || n == 0) return DC_OK;
  dim3 blk(8, 8);
  dim3 grid((m + 7) / 8, (n + 7) / 8, batch);
  k_lut_gemm<<<grid, blk, 0, st>>>(Xq, Wq, rs, cs, m, k, n, flags, ctx->d_mul, ctx->d_requant, ctx->d_relu, out); dc_count_launch();
  DC_CUDA(ctx, cudaGetLastError());
  return DC_OK;
}

static int gemm_dispatch_impl(dc_ctx* ctx, const int8_t* Xq, int ldx, const int8_t* Wt, int ldw, const float* rs,
                              const float* cs, int m, int k, int n, int batch, unsigned flags, void* out,
                              cudaStream_t st, int kind);

static cudaEvent_t timing_event(dc_ctx* ctx) {
  cudaEvent_t e = nullptr;
  if (!ctx->event_pool.empty()) {
    e = ctx->event_pool.back();
    ctx->event_pool.pop_back();
  } else if (cudaEventCreate(&e) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  return e;
}

// With timing on (dc_timing), every GEMM launch is bracketed by CUDA events on
// its own stream and its algorithmic bytes and ops are recorded.
// One GEMM's launches with its accounting: the timeline tag (kind, algorithmic
// bytes) and, with timing on, CUDA events around it on its stream.
template <typename F>
static int accounted(dc_ctx* ctx, int kind, double bytes, double ops, cudaStream_t st, F&& launch) {
  if (!ctx->timing) {
    const int rc = launch();
    dc_timeline_tag(ctx, kind, bytes);
    return rc;
  }
  dc_timed t;
  t.a = timing_event(ctx);
  t.b = timing_event(ctx);
  t.kind = kind;
  t.bytes = bytes;
  t.ops = ops;
  if (t.a) cudaEventRecord(t.a, st);
  const int rc = launch();
  if (t.b) cudaEventRecord(t.b, st);
  if (t.a && t.b) ctx->timed.push_back(t);
  return rc;
}

int dc_gemm_dispatch(dc_ctx* ctx, const int8_t* Xq, int ldx, const int8_t* Wt, int ldw, const float* rs,
                     const float* cs, int m, int k, int n, int batch, unsigned flags, void* out, cudaStream_t st,
                     int kind) {
  if (m == 0 || n == 0 || batch == 0) return DC_OK;
  const double ob = (flags & DC_ACC) ? 4 : (flags & DC_REQUANT) ? 1 : 4;
  const double bytes = (double)batch * ((double)m * k + (double)k * n + 4.0 * m + 4.0 * n + ob * m * n);
  return accounted(ctx, (kind == 0) ? (m <= 8 ? 1 : 3) : kind, bytes, 2.0 * batch * (double)m * n * k, st,
                   [&] { return gemm_dispatch_impl(ctx, Xq, ldx, Wt, ldw, rs, cs, m, k, n, batch, flags, out, st, kind); });
}

int dc_gemv_swiglu(dc_ctx* ctx, const int8_t* Xq, const int8_t* Wt, int ldw, const float* rs, const float* cs,
                   int k, int n2, float* hout, uint32_t* rowmax, cudaStream_t st) {
  if (n2 < 2 || (n2 & 1) || !rowmax || (((uintptr_t)Wt | (uintptr_t)Xq) & 15) || (ldw & 15)) return DC_E_INVAL;
  if (k > DC_MAX_INT32_K) return dc_fail(ctx, DC_E_ACCBOUND, "gemv_swiglu: k=%d", k);
  const double bytes = (double)k + (double)k * n2 + 4.0 + 4.0 * n2 + 4.0 * (n2 / 2);
  return accounted(ctx, 1, bytes, 2.0 * (double)n2 * k, st,
                   [&] { return launch_gemv_row(ctx, Xq, Wt, ldw, rs, cs, k, n2, DC_F_SWIGLU, hout, st, rowmax); });
}

extern "C" int dc_timing(dc_ctx* ctx, int on) {
  if (!ctx) return DC_E_INVAL;
  for (auto& t : ctx->timed) {
    ctx->event_pool.push_back(t.a);
    ctx->event_pool.push_back(t.b);
  }
  ctx->timed.clear();
  ctx->timing = on != 0;
  return DC_OK;
}

extern "C" int dc_timing_read(dc_ctx* ctx, int kind, double* ms, long long* launches, double* bytes, double* ops) {
  if (!ctx) return DC_E_INVAL;
  DC_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  double tms = 0, tb = 0, to = 0;
  long long n = 0;
  for (auto& t : ctx->timed) {
    if (t.kind != kind) continue;
    float e = 0;
    DC_CUDA(ctx, cudaEventSynchronize(t.b));
    DC_CUDA(ctx, cudaEventElapsedTime(&e, t.a, t.b));
    tms += e;
    tb += t.bytes;
    to += t.ops;
    n++;
  }
  if (ms) *ms = tms;
  if (launches) *launches = n;
  if (bytes) *bytes = tb;
  if (ops) *ops = to;
  return DC_OK;
}

static int gemm_dispatch_impl(dc_ctx* ctx, const int8_t* Xq, int ldx, const int8_t* Wt, int ldw, const float* rs,
                              const float* cs, int m, int k, int n, int batch, unsigned flags, void* out,
                              cudaStream_t st, int kind) {
  if (kind == 0) kind = (m <= 8) ? 1 : 3;
  if (kind == 3) {
    if (ctx->tc_enabled) {
      int rc = dc_gemm_tc(ctx, Xq, ldx, Wt, ldw, rs, cs, m, k, n, batch, flags, out, st);
      if (rc != DC_E_INVAL) return rc;
    }
    kind = 2;  // shape the tensor-core kernel does not take: the SIMT kernel
  }
  if (kind == 1) {
    if (m <= 1) return launch_gemv<1>(ctx, Xq, ldx, Wt, ldw, rs, cs, m, k, n, batch, flags, out, st);
    if (m <= 2) return launch_gemv<2>(ctx, Xq, ldx, Wt, ldw, rs, cs, m, k, n, batch, flags, out, st);
    if (m <= 4) return launch_gemv<4>(ctx, Xq, ldx, Wt, ldw, rs, cs, m, k, n, batch, flags, out, st);
    if (m <= 8) return launch_gemv<8>(ctx, Xq, ldx, Wt, ldw, rs, cs, m, k, n, batch, flags, out, st);
    kind = 2;
  }
  dim3 grid((n + 63) / 64, (m + 63) / 64, batch);
  k_gemm_simt<<<grid, 256, 0, st>>>(Xq, ldx, Wt, ldw, rs, cs, m, k, n, flags, ctx->d_requant, ctx->d_relu, out); dc_count_launch();
  DC_CUDA(ctx, cudaGetLastError());
  return DC_OK;
}

int dc_gemm_untimed(dc_ctx* ctx, const int8_t* Xq, int ldx, const int8_t* Wt, int ldw, const float* rs,
                    const float* cs, int m, int k, int n, int batch, unsigned flags, void* out, cudaStream_t st,
                    int kind) {
  if (m == 0 || n == 0 || batch == 0) return DC_OK;
  return gemm_dispatch_impl(ctx, Xq, ldx, Wt, ldw, rs, cs, m, k, n, batch, flags, out, st, kind);
}

int dc_scratch(dc_ctx* ctx, size_t bytes, void** p) {
  if (bytes > ctx->scratch_bytes) {
    DC_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
    if (ctx->scratch) cudaFree(ctx->scratch);
    ctx->scratch = nullptr;
    ctx->scratch_bytes = 0;
    size_t want = bytes + (bytes >> 2) + 4096;
    if (cudaMalloc(&ctx->scratch, want) != cudaSuccess) {
      cudaGetLastError();
      return dc_fail(ctx, DC_E_NOMEM, "scratch allocation of %zu bytes failed", want);
    }
    ctx->scratch_bytes = want;
  }
  *p = ctx->scratch;
  return DC_OK;
}

static size_t al256(size_t v) { return (v + 255) & ~(size_t)255; }

static int out_elem_bytes(unsigned flags) { return (flags & DC_ACC) ? 4 : (flags & DC_REQUANT) ? 1 : 4; }

extern "C" int dc_bgemm(dc_ctx* ctx, const int8_t* Xq, const int8_t* Wq, const float* rs, const float* cs, int m,
                        int k, int n, int batch, unsigned flags, void* out) {
  if (!ctx) return DC_E_INVAL;
  if (m < 0 || k < 0 || n < 0 || batch < 1) return dc_fail(ctx, DC_E_INVAL, "bgemm: bad shape");
  if (k > DC_MAX_INT32_K)
    return dc_fail(ctx, DC_E_ACCBOUND,
                   "bgemm: contraction length %d exceeds the int32 accumulator headroom %d (the sum would wrap)", k,
                   DC_MAX_INT32_K);
  if ((int64_t)m * n * batch == 0) return DC_OK;
  if (!Xq || !Wq || !rs || !cs || !out) return dc_fail(ctx, DC_E_INVAL, "bgemm: null buffer");
  const int ld = round_up(k > 0 ? k : 1, 16);
  const size_t bx = al256((size_t)batch * m * ld), bw = al256((size_t)batch * k * n),
               bwt = al256((size_t)batch * n * ld), brs = al256(4 * (size_t)batch * m),
               bcs = al256(4 * (size_t)batch * n),
               bo = al256((size_t)out_elem_bytes(flags) * batch * m * n);
  void* base;
  int rc = dc_scratch(ctx, bx + bw + bwt + brs + bcs + bo, &base);
  if (rc) return rc;
  char* p = (char*)base;
  int8_t* dx = (int8_t*)p; p += bx;
  int8_t* dw = (int8_t*)p; p += bw;
  int8_t* dwt = (int8_t*)p; p += bwt;
  float* drs = (float*)p; p += brs;
  float* dcs = (float*)p; p += bcs;
  void* dout = p;
  cudaStream_t st = ctx->stream;
  DC_CUDA(ctx, cudaMemsetAsync(dx, 0, bx, st));
  if (k > 0) {
    DC_CUDA(ctx, cudaMemcpy2DAsync(dx, ld, Xq, k, k, (size_t)batch * m, cudaMemcpyHostToDevice, st));
    DC_CUDA(ctx, cudaMemcpyAsync(dw, Wq, (size_t)batch * k * n, cudaMemcpyHostToDevice, st));
  }
  DC_CUDA(ctx, cudaMemcpyAsync(drs, rs, 4 * (size_t)batch * m, cudaMemcpyHostToDevice, st));
  DC_CUDA(ctx, cudaMemcpyAsync(dcs, cs, 4 * (size_t)batch * n, cudaMemcpyHostToDevice, st));
  if ((rc = dc_launch_transpose_i8(ctx, dw, k, n, dwt, ld, batch, st))) return rc;
  if ((rc = dc_gemm_dispatch(ctx, dx, ld, dwt, ld, drs, dcs, m, k, n, batch, flags, dout, st, 0))) return rc;
  DC_CUDA(ctx, cudaMemcpyAsync(out, dout, (size_t)out_elem_bytes(flags) * batch * m * n, cudaMemcpyDeviceToHost, st));
  return dc_sync(ctx);
}

extern "C" int dc_bgemm_dev(dc_ctx* ctx, const int8_t* Xq, int ldx, const int8_t* Wt, int ldw, const float* rs,
                            const float* cs, int m, int k, int n, int batch, unsigned flags, void* out) {
  if (!ctx) return DC_E_INVAL;
  if (m < 0 || k < 0 || n < 0 || batch < 1 || ldx < k || ldw < k || (ldx & 15) || (ldw & 15))
    return dc_fail(ctx, DC_E_INVAL, "bgemm_dev: bad shape or leading dimension");
  if (k > DC_MAX_INT32_K)
    return dc_fail(ctx, DC_E_ACCBOUND, "bgemm_dev: contraction length %d exceeds %d", k, DC_MAX_INT32_K);
  return dc_gemm_dispatch(ctx, Xq, ldx, Wt, ldw, rs, cs, m, k, n, batch, flags, out, ctx->stream, 0);
}

// Internal entry for tests: force one kernel (1 GEMV, 2 SIMT, 3 tcgen05).
extern "C" int dc_bgemm_dev_kind(dc_ctx* ctx, const int8_t* Xq, int ldx, const int8_t* Wt, int ldw, const float* rs,
                                 const float* cs, int m, int k, int n, int batch, unsigned flags, void* out,
                                 int kind) {
  if (!ctx) return DC_E_INVAL;
  if (m < 0 || k < 0 || n < 0 || batch < 1 || ldx < k || ldw < k || (ldx & 15) || (ldw & 15))
    return dc_fail(ctx, DC_E_INVAL, "bgemm_dev: bad shape or leading dimension");
  if (k > DC_MAX_INT32_K) return dc_fail(ctx, DC_E_ACCBOUND, "bgemm_dev: k=%d too long", k);
  if (kind == 3) {
    if (m == 0 || n == 0) return DC_OK;
    return dc_gemm_tc(ctx, Xq, ldx, Wt, ldw, rs, cs, m, k, n, batch, flags, out, ctx->stream);
  }
  return dc_gemm_dispatch(ctx, Xq, ldx, Wt, ldw, rs, cs, m, k, n, batch, flags, out, ctx->stream, kind);
}

extern "C" int dc_bgemm_lut_dev(dc_ctx* ctx, const int8_t* Xq, const int8_t* Wq, const float* rs, const float* cs,
                                int m, int k, int n, int batch, unsigned flags, void* out) {
  if (!ctx) return DC_E_INVAL;
  if (m < 0 || k < 0 || n < 0 || batch < 1) return dc_fail(ctx, DC_E_INVAL, "bgemm_lut: bad shape");
  if (k > DC_MAX_INT32_K) return dc_fail(ctx, DC_E_ACCBOUND, "bgemm_lut: k=%d too long", k);
  return dc_gemm_lut(ctx, Xq, Wq, rs, cs, m, k, n, batch, flags, out, ctx->stream);
}

// ---- resident weights -------------------------------------------------------
extern "C" int dc_weight_register(dc_ctx* ctx, const float* W, int k, int n, dc_weight** out) {
  if (!ctx || !W || !out || k <= 0 || n <= 0) return dc_fail(ctx, DC_E_INVAL, "weight_register: bad arguments");
  if (k > DC_MAX_INT32_K) return dc_fail(ctx, DC_E_ACCBOUND, "weight_register: k=%d exceeds %d", k, DC_MAX_INT32_K);
  dc_weight* w = new dc_weight();
  w->ctx = ctx;
  w->k = k;
  w->n = n;
  w->ldw = round_up(k, 16);
  float* dW = nullptr;
  cudaError_t e = cudaMalloc(&w->qt, (size_t)n * w->ldw);
  if (e == cudaSuccess) e = cudaMalloc(&w->cs, 4 * (size_t)n);
  if (e == cudaSuccess) e = cudaMalloc(&dW, 4 * (size_t)k * n);
  if (e != cudaSuccess) {
    cudaGetLastError();
    cudaFree(dW);
    dc_weight_free(w);
    return dc_fail(ctx, DC_E_NOMEM, "weight_register: device allocation failed");
  }
  int rc = DC_OK;
  e = cudaMemcpyAsync(dW, W, 4 * (size_t)k * n, cudaMemcpyHostToDevice, ctx->stream);
  if (e != cudaSuccess) rc = dc_cuda_fail(ctx, e, "weight upload");
  if (!rc) rc = dc_launch_quant_cols_t(ctx, dW, k, n, w->qt, w->ldw, w->cs, ctx->stream);
  if (!rc) rc = dc_sync(ctx);
  cudaFree(dW);
  if (rc) {
    dc_weight_free(w);
    return rc;
  }
  *out = w;
  return DC_OK;
}

extern "C" void dc_weight_free(dc_weight* w) {
  if (!w) return;
  if (w->owns) {
    cudaFree(w->qt);
    cudaFree(w->cs);
  }
  delete w;
}

extern "C" int dc_weight_info(const dc_weight* w, const int8_t** qt, int* ldw, const float** cs, int* k, int* n) {
  if (!w) return DC_E_INVAL;
  if (qt) *qt = w->qt;
  if (ldw) *ldw = w->ldw;
  if (cs) *cs = w->cs;
  if (k) *k = w->k;
  if (n) *n = w->n;
  return DC_OK;
}

extern "C" int dc_vgemm(dc_ctx* ctx, const float* X, int m, const dc_weight* w, unsigned flags, void* out) {
  if (!ctx || !w || m < 0 || (m && (!X || !out))) return dc_fail(ctx, DC_E_INVAL, "vgemm: bad arguments");
  if (m == 0) return DC_OK;
  const size_t bx = al256((size_t)m * w->ldw), brs = al256(4 * (size_t)m);
  void* base;
  int rc = dc_scratch(ctx, bx + brs, &base);
  if (rc) return rc;
  int8_t* xq = (int8_t*)base;
  float* rs = (float*)((char*)base + bx);
  if ((rc = dc_launch_quant_rows(ctx, X, m, w->k, xq, w->ldw, rs, ctx->stream))) return rc;
  return dc_gemm_dispatch(ctx, xq, w->ldw, w->qt, w->ldw, rs, w->cs, m, w->k, w->n, 1, flags, out, ctx->stream, 0);
}

// Prefetch a device range into L2 on the context's stream (asynchronous).
int dc_l2_prefetch_on(dc_ctx* ctx, const void* p, size_t bytes, cudaStream_t st) {
  if (!p || !bytes) return DC_OK;
  if (((uintptr_t)p & 15) || (bytes & 15)) return dc_fail(ctx, DC_E_INVAL, "l2_prefetch: range must be 16-byte aligned");
  const size_t npiece = (bytes + 65535) / 65536;
  const int blocks = (int)std::min<size_t>((npiece + 127) / 128, (size_t)ctx->sm_count);
  k_l2_prefetch<<<blocks, 128, 0, st>>>((const int8_t*)p, bytes);
  dc_count_launch();
  DC_CUDA(ctx, cudaGetLastError());
  return DC_OK;
}

extern "C" int dc_l2_prefetch(dc_ctx* ctx, const void* p, size_t bytes) {
  if (!ctx) return DC_E_INVAL;
  return dc_l2_prefetch_on(ctx, p, bytes, ctx->stream);
}
