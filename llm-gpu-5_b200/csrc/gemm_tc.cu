// tcgen05 tensor-core GEMM (placeholder until the sm_100a kernel lands).
#include "common.cuh"
namespace attn {
bool tc_gemm_supported(int, int, int, int64_t, int, int64_t, int, const void*, const void*) { return false; }
int gemm_tc(const void*, int64_t, int, const void*, int64_t, int, void*, int64_t, int, const float*,
            int, int, int, int, cudaStream_t) {
  set_error("tensor-core GEMM not built");
  return ATTN_ERR_UNSUPPORTED;
}
}  // namespace attn
