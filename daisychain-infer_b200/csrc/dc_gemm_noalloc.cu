// dc_gemm_noalloc.cu -- the tensor-core GEMM for callers that must not allocate.
//
// dc_bgemm_dev grows a per-context split-K buffer with cudaMalloc the first time
// a shape needs more than it holds, and cudaFree's the old one.  Some callers
// cannot let that happen: a host that plans every byte of HBM up front (weights
// and KV cache sized to the GPU) and treats any later allocation as a failure,
// and an embedding runtime that owns all device allocation itself.  cudaFree
// also synchronises the whole device, which stalls every other stream of a
// process that keeps several pipeline stages or copies in flight.
//
// This entry point runs the same tcgen05 kernel with its split-K scratch in a
// fixed array compiled into the library (g_noalloc_scratch below), so it never
// calls cudaMalloc, cudaFree or any allocating routine.  The array is
// DC_NOALLOC_MAX_OUT int32 partial sums plus DC_NOALLOC_MAX_TILES tile counters
// (about 4.2 MB); every GPU that loads the library holds it until the process
// exits.  Calls whose output (batch * m * n elements) is larger are refused with
// DC_E_INVAL.
//
// All calls on one device share the array.  Each call clears the part it uses
// (cudaMemsetAsync, on the call's stream) before the kernel runs, so it does not
// depend on what an earlier call left behind; calls that overlap on the GPU
// (two streams, or two contexts on the same device) race on it and must be
// serialised by the caller.
//
// The device address of the array is looked up once per device, with that
// device current, by the first call made on it; make that first call before
// any stream capture begins on the device.
#include <mutex>

#include "dc_internal.cuh"

// The launcher in dc_gemm_tc.cu that takes caller-provided split-K scratch.
int dc_gemm_tc_with(dc_ctx* ctx, const int8_t* Xq, int ldx, const int8_t* Wt, int ldw, const float* rs,
                    const float* cs, int m, int k, int n, int batch, unsigned flags, void* out, cudaStream_t st,
                    int32_t* partial, int* counters, size_t partial_cap, size_t counter_cap);

namespace {

constexpr size_t kPartialElems = DC_NOALLOC_MAX_OUT;
constexpr size_t kCounters = DC_NOALLOC_MAX_TILES;

// partial sums first, tile counters after them
static __device__ __align__(256) int32_t g_noalloc_scratch[kPartialElems + kCounters];

constexpr int kMaxDevices = 64;
std::mutex g_lock;
int32_t* g_addr[kMaxDevices] = {nullptr};

// Device address of the scratch array on ctx's device (looked up once).
int scratch_on(dc_ctx* ctx, int32_t** out) {
  if (ctx->device < 0 || ctx->device >= kMaxDevices)
    return dc_fail(ctx, DC_E_INVAL, "bgemm_dev_noalloc: device %d out of range", ctx->device);
  std::lock_guard<std::mutex> guard(g_lock);
  if (!g_addr[ctx->device]) {
    int prev = -1;
    DC_CUDA(ctx, cudaGetDevice(&prev));
    if (prev != ctx->device) DC_CUDA(ctx, cudaSetDevice(ctx->device));
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (prev != ctx->device) cudaSetDevice(prev);
    if (e != cudaSuccess) return dc_cuda_fail(ctx, e, "cudaGetSymbolAddress(g_noalloc_scratch)");
    g_addr[ctx->device] = (int32_t*)p;
  }
  *out = g_addr[ctx->device];
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
  if (k == 0) return dc_fail(ctx, DC_E_INVAL, "bgemm_dev_noalloc: k must be at least 1");
  const size_t outs = (size_t)batch * m * n;
  const size_t tiles = (size_t)((n + 127) / 128) * ((m + 15) / 16) * batch;
  if (outs > kPartialElems || tiles > kCounters)
    return dc_fail(ctx, DC_E_INVAL,
                   "bgemm_dev_noalloc: output of %zu elements (%zu tiles) exceeds the fixed scratch of %zu elements "
                   "(%zu tiles); use dc_bgemm_dev",
                   outs, tiles, kPartialElems, kCounters);
  int32_t* scratch = nullptr;
  int rc = scratch_on(ctx, &scratch);
  if (rc) return rc;
  int32_t* partial = scratch;
  int* counters = (int*)(scratch + kPartialElems);
  DC_CUDA(ctx, cudaMemsetAsync(partial, 0, 4 * outs, ctx->stream));
  DC_CUDA(ctx, cudaMemsetAsync(counters, 0, 4 * tiles, ctx->stream));
  return dc_gemm_tc_with(ctx, Xq, ldx, Wt, ldw, rs, cs, m, k, n, batch, flags, out, ctx->stream, partial, counters,
                         kPartialElems, kCounters);
}
