// dc_quant.cu -- the two quantisers of the verified path, on the device.
//
// quantizeRows (public/verified_core.js:108-121): per-row absmax, the scale
// max(mx/127, 1e-8) in DOUBLE, q = clamp(Math.round(x / scale)) with that
// double scale; only the stored s[r] is rounded to f32.
// quantizeCols (verified_core.js:122-136): per-column absmax, s[c] rounded to
// f32 FIRST and q = clamp(Math.round(w / s[c])) with the rounded scale.
// Both refuse non-finite input (assertFinite, :16-27): here a kernel that sees
// one sets DC_ST_NONFINITE in the context status word, which the host reads at
// its next synchronisation point and turns into DC_E_NONFINITE.
//
// The absmax is a max of |x|: exact and order-independent, so a parallel
// reduction gives the reference's value.  The divide is IEEE double division
// (__ddiv_rn), correctly rounded like the JavaScript '/'.
#include "dc_internal.cuh"

namespace {

// One block per row.  HBM-bound: one read of the f32 row for the max, one
// (L1/L2-resident) re-read for the quotients, one int8 write.
__global__ void __launch_bounds__(256) k_quant_rows(const float* __restrict__ X, int rows, int cols,
                                                    int8_t* __restrict__ q, int ldq, float* __restrict__ s,
                                                    int* __restrict__ status) {
  const int r = blockIdx.x;
  if (r >= rows) return;
  const float* x = X + (int64_t)r * cols;
  float mx = 0.0f;
  bool bad = false;
  for (int c = threadIdx.x; c < cols; c += blockDim.x) {
    float v = x[c];
    if (!isfinite(v)) bad = true;
    mx = fmaxf(mx, fabsf(v));
  }
  // a warp vote, not a block vote: __syncthreads_or costs microseconds here
  if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) atomicOr(status, DC_ST_NONFINITE);
  __shared__ float red[32];
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  double sc = __ddiv_rn((double)red[0], 127.0);
  if (!(sc > 1e-8)) sc = 1e-8;
  if (threadIdx.x == 0) s[r] = __double2float_rn(sc);
  int8_t* qr = q + (int64_t)r * ldq;
  for (int c = threadIdx.x; c < ldq; c += blockDim.x) {
    int8_t v = 0;
    if (c < cols) v = dc_clamp8(dc_js_round(__ddiv_rn((double)x[c], sc)));
    qr[c] = v;
  }
}

// Column absmax of a k x n row-major matrix: one thread per column, rows
// walked in order, so a warp reads 128 contiguous bytes per row.
__global__ void __launch_bounds__(256) k_col_scales(const float* __restrict__ W, int rows, int cols,
                                                    float* __restrict__ s, int* __restrict__ status) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= cols) return;
  float mx = 0.0f;
  bool bad = false;
  for (int r = 0; r < rows; r++) {
    float v = W[(int64_t)r * cols + c];
    if (!isfinite(v)) bad = true;
    mx = fmaxf(mx, fabsf(v));
  }
  if (bad) atomicOr(status, DC_ST_NONFINITE);
  double sc = __ddiv_rn((double)mx, 127.0);
  if (!(sc > 1e-8)) sc = 1e-8;
  s[c] = __double2float_rn(sc);
}

// Quantise with the f32 column scales and write the transpose (cols x ldq),
// through a 32 x 32 shared tile so both the read and the write are coalesced.
__global__ void __launch_bounds__(256) k_quant_cols_t(const float* __restrict__ W, int rows, int cols,
                                                      const float* __restrict__ s, int8_t* __restrict__ qt,
                                                      int ldq) {
  __shared__ int8_t tile[32][33];
  const int r0 = blockIdx.y * 32, c0 = blockIdx.x * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8
  for (int i = ty; i < 32; i += 8) {
    int r = r0 + i, c = c0 + tx;
    int8_t v = 0;
    if (r < rows && c < cols) v = dc_clamp8(dc_js_round(__ddiv_rn((double)W[(int64_t)r * cols + c], (double)s[c])));
    tile[i][tx] = v;
  }
  __syncthreads();
  for (int i = ty; i < 32; i += 8) {
    int c = c0 + i, r = r0 + tx;
    if (c < cols && r < ldq) qt[(int64_t)c * ldq + r] = (r < rows) ? tile[tx][i] : (int8_t)0;
  }
}

// int8 transpose of batch x (k x n) into batch x (n x ldw), zero past k.
__global__ void __launch_bounds__(256) k_transpose_i8(const int8_t* __restrict__ W, int k, int n,
                                                      int8_t* __restrict__ Wt, int ldw) {
  __shared__ int8_t tile[32][33];
  const int bz = blockIdx.z;
  const int8_t* Wb = W + (int64_t)bz * k * n;
  int8_t* Wtb = Wt + (int64_t)bz * n * ldw;
  const int r0 = blockIdx.y * 32, c0 = blockIdx.x * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  for (int i = ty; i < 32; i += 8) {
    int r = r0 + i, c = c0 + tx;
    tile[i][tx] = (r < k && c < n) ? Wb[(int64_t)r * n + c] : (int8_t)0;
  }
  __syncthreads();
  for (int i = ty; i < 32; i += 8) {
    int c = c0 + i, r = r0 + tx;
    if (c < n && r < ldw) Wtb[(int64_t)c * ldw + r] = (r < k) ? tile[tx][i] : (int8_t)0;
  }
}

}  // namespace

int dc_launch_quant_rows(dc_ctx* ctx, const float* X, int rows, int cols, int8_t* q, int ldq, float* s,
                         cudaStream_t st) {
  if (rows <= 0) return DC_OK;
  k_quant_rows<<<rows, 256, 0, st>>>(X, rows, cols, q, ldq, s, ctx->d_status); dc_count_launch();
  DC_CUDA(ctx, cudaGetLastError());
  return DC_OK;
}

int dc_launch_quant_cols_t(dc_ctx* ctx, const float* W, int rows, int cols, int8_t* qt, int ldq, float* s,
                           cudaStream_t st) {
  if (cols <= 0) return DC_OK;
  k_col_scales<<<(cols + 255) / 256, 256, 0, st>>>(W, rows, cols, s, ctx->d_status); dc_count_launch();
  DC_CUDA(ctx, cudaGetLastError());
  dim3 grid((cols + 31) / 32, (ldq + 31) / 32);
  k_quant_cols_t<<<grid, 256, 0, st>>>(W, rows, cols, s, qt, ldq); dc_count_launch();
  DC_CUDA(ctx, cudaGetLastError());
  return DC_OK;
}

int dc_launch_transpose_i8(dc_ctx* ctx, const int8_t* W, int k, int n, int8_t* Wt, int ldw, int batch,
                           cudaStream_t st) {
  if (n <= 0 || batch <= 0) return DC_OK;
  dim3 grid((n + 31) / 32, (ldw + 31) / 32, batch);
  k_transpose_i8<<<grid, 256, 0, st>>>(W, k, n, Wt, ldw); dc_count_launch();
  DC_CUDA(ctx, cudaGetLastError());
  return DC_OK;
}

extern "C" int dc_quantize_rows(dc_ctx* ctx, const float* X, int rows, int cols, int8_t* q, int ldq, float* s) {
  if (!ctx || rows < 0 || cols < 0 || ldq < cols || (rows && (!X || !q || !s)))
    return dc_fail(ctx, DC_E_INVAL, "dc_quantize_rows: bad arguments");
  return dc_launch_quant_rows(ctx, X, rows, cols, q, ldq, s, ctx->stream);
}

extern "C" int dc_quantize_cols_t(dc_ctx* ctx, const float* W, int rows, int cols, int8_t* qt, int ldq, float* s) {
  if (!ctx || rows < 0 || cols < 0 || ldq < rows || (cols && (!W || !qt || !s)))
    return dc_fail(ctx, DC_E_INVAL, "dc_quantize_cols_t: bad arguments");
  return dc_launch_quant_cols_t(ctx, W, rows, cols, qt, ldq, s, ctx->stream);
}
