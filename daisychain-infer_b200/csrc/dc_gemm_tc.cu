// dc_gemm_tc.cu -- tcgen05 tensor-core path (placeholder until the kernel lands).
#include "dc_internal.cuh"

int dc_gemm_tc(dc_ctx* ctx, const int8_t*, int, const int8_t*, int, const float*, const float*, int, int, int, int,
               unsigned, void*, cudaStream_t) {
  return dc_fail(ctx, DC_E_INVAL, "tcgen05 path not built");
}
