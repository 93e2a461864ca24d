// tcgen05 grouped expert GEMMs (placeholder until the kernels land).
#include "llq_common.cuh"

namespace llq {

bool tc_supported(int, int, int, int, int, bool) { return false; }

int gemm1_tc(const void*, const int32_t*, int64_t, int, int, int, const int8_t*, const float*, int,
             int, void*, cudaStream_t) {
  return fail(LLQ_EUNSUPPORTED, "tcgen05 GEMM1 not built");
}

int gemm2_tc(const void*, const int32_t*, const int32_t*, const float*, int64_t, int, int, int,
             const int8_t*, const float*, int, int, void*, cudaStream_t) {
  return fail(LLQ_EUNSUPPORTED, "tcgen05 GEMM2 not built");
}

}  // namespace llq
