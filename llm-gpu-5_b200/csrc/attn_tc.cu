// tcgen05 tensor-core attention (placeholder until the sm_100a kernels land).
#include "common.cuh"
namespace attn {
bool tc_fwd_supported(int, int) { return false; }
int attn_fwd_tc(const void*, const void*, const void*, void*, float*, int, int, int, int,
                const int64_t*, float, cudaStream_t) {
  set_error("tensor-core attention not built");
  return ATTN_ERR_UNSUPPORTED;
}
bool tc_bwd_supported(int, int) { return false; }
size_t attn_bwd_tc_ws(int, int, int, int) { return 0; }
int attn_bwd_tc(const void*, const void*, const void*, const void*, const void*, const float*, void*,
                void*, void*, void*, int, int, int, int, const int64_t*, float, cudaStream_t) {
  set_error("tensor-core attention not built");
  return ATTN_ERR_UNSUPPORTED;
}
}  // namespace attn
