// dc_gemm_noalloc.cu -- the device-buffer GEMM for callers that must not allocate.
//
// dc_bgemm_dev grows a per-context split-K buffer with cudaMalloc the first time
// a tensor-core shape needs more than it holds, and cudaFree's the old one.
// Some callers cannot let that happen: a host that plans every byte of HBM up
// front (weights and KV cache sized to the GPU) and treats any later
// allocation as a failure, and an embedding runtime that owns all device
// allocation itself.  cudaFree also synchronises the whole device, which
// stalls every other stream of a process that keeps several pipeline stages or
// copies in flight.
//
// This entry point takes the same arguments and picks the same kernels as
// dc_bgemm_dev (the one-row GEMV up to 8 rows, the tcgen05 kernel above, the
// SIMT kernel when the tcgen05 kernel failed its init gate or cannot take the
// operands), but gives the tcgen05 kernel its split-K scratch from a fixed
// array compiled into the library (g_noalloc_scratch below), so no call ever
// reaches cudaMalloc, cudaFree or any allocating routine.  The array is
// DC_NOALLOC_MAX_OUT int32 partial sums plus DC_NOALLOC_MAX_TILES tile
// counters (about 4.2 MB); every GPU that loads the library holds it until the
// process exits.  Calls whose output (batch * m * n elements) is larger are
// refused with DC_E_INVAL.
//
// All calls on one device share the array.  A call that splits K clears the
// part it uses (cudaMemsetAsync on the call's stream) before its kernel runs,
// so it does not depend on what an earlier call left behind; calls that
// overlap on the GPU (two streams, or two contexts on the same device) race on
// it and must be serialised by the caller.
//
// The array's device address is looked up (cudaGetSymbolAddress, with the
// context's device current) by the first call made on each context and kept
// in the context; make that first call before any stream capture begins.
#include "dc_internal.cuh"

namespace {

constexpr size_t kPartialElems = DC_NOALLOC_MAX_OUT;
constexpr size_t kCounters = DC_NOALLOC_MAX_TILES;

// partial sums first, tile counters after them
static __device__ __align__(256) int32_t g_noalloc_scratch[kPartialElems + kCounters];

// Device address of the scratch array on ctx's device.
int scratch_on(dc_ctx* ctx, int32_t** out) {
  if (!ctx->noalloc_scratch) {
    int prev = -1;
    DC_CUDA(ctx, cudaGetDevice(&prev));
    if (prev != ctx->device) DC_CUDA(ctx, cudaSetDevice(ctx->device));
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (prev != ctx->device) cudaSetDevice(prev);
    if (e != cudaSuccess) return dc_cuda_fail(ctx, e, "cudaGetSymbolAddress(g_noalloc_scratch)");
    ctx->noalloc_scratch = (int32_t*)p;
  }
  *out = ctx->noalloc_scratch;
  return DC_OK;
}

}  // namespace

extern "C" int dc_bgemm_dev_noalloc(dc_ctx* ctx, const int8_t* Xq, int ldx, const int8_t* Wt, int ldw,
                                    const float* rs, const float* cs, int m, int k, int n, int batch, unsigned flags,
                                    void* out) {
  if (!ctx) return DC_E_INVAL;
  if (m < 0 || k < 0 || n < 0 || batch < 1 || ldx < k || ldw < k || (ldx & 15) || (ldw & 15))
    return dc_fail(ctx, DC_E_INVAL, "bgemm_dev_noalloc: bad shape or leading dimension");
  if (k > DC_MAX_INT32_K)
    return dc_fail(ctx, DC_E_ACCBOUND, "bgemm_dev_noalloc: contraction length %d exceeds %d", k, DC_MAX_INT32_K);
  if ((int64_t)m * n * batch == 0) return DC_OK;
  if (!out || !rs || !cs || (k > 0 && (!Xq || !Wt)))
    return dc_fail(ctx, DC_E_INVAL, "bgemm_dev_noalloc: null buffer");
  const size_t outs = (size_t)batch * m * n;
  const size_t tiles = (size_t)((n + 127) / 128) * ((m + 15) / 16) * batch;
  if (outs > kPartialElems || tiles > kCounters)
    return dc_fail(ctx, DC_E_INVAL,
                   "bgemm_dev_noalloc: output of %zu elements (%zu tiles) exceeds the fixed scratch of %zu elements "
                   "(%zu tiles); use dc_bgemm_dev",
                   outs, tiles, kPartialElems, kCounters);
  if (m > 8 && k > 0 && ctx->tc_enabled) {
    int32_t* scratch = nullptr;
    if (int rc = scratch_on(ctx, &scratch)) return rc;
    const int rc = dc_gemm_tc_with(ctx, Xq, ldx, Wt, ldw, rs, cs, m, k, n, batch, flags, out, ctx->stream, scratch,
                                   (int*)(scratch + kPartialElems), kPartialElems, kCounters, 1);
    if (rc != DC_E_INVAL) return rc;
    // operands the tensor-core kernel does not take (alignment): the SIMT kernel, as dc_bgemm_dev does
  }
  // the one-row GEMV (m <= 8), the SIMT kernel otherwise (k == 0 included): neither uses scratch
  return dc_gemm_untimed(ctx, Xq, ldx, Wt, ldw, rs, cs, m, k, n, batch, flags, out, ctx->stream, m <= 8 ? 1 : 2);
}
