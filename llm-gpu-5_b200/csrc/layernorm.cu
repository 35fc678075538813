// LayerNorm feeding the attention path: y = (x - mean) * rsqrt(var + eps) * gamma + beta per row,
// var the biased variance (layernorm_kernel, core/kernels.py:75-110, computes mean and variance in
// two passes over the row and uses eps = 1e-5).  Written either as float32 or as the bf16 input of
// the QKV projection, optionally followed by a ones column (see attn_cast_rows_ones_bf16), so the
// pre-attention LayerNorm of a transformer block (model/gpt.py:778) writes the GEMM operand
// directly instead of a float32 tensor that a cast then reads again.
//
// One warp per row.  When C % 4 == 0 and C <= 4 * 32 * KMAX the row stays in registers (float4
// chunks c = lane + 32 k), so x is read once; otherwise a three-pass loop re-reads the row.
#include "common.cuh"

namespace attn {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ void store4(float* y, float a, float b, float c, float d) {
  *reinterpret_cast<float4*>(y) = make_float4(a, b, c, d);
}
__device__ __forceinline__ void store4(__nv_bfloat16* y, float a, float b, float c, float d) {
  __nv_bfloat162 p0 = __floats2bfloat162_rn(a, b), p1 = __floats2bfloat162_rn(c, d);
  uint2 u;
  u.x = *reinterpret_cast<uint32_t*>(&p0);
  u.y = *reinterpret_cast<uint32_t*>(&p1);
  *reinterpret_cast<uint2*>(y) = u;
}

// columns C .. ldy-1 of a row: 1 at column C when ones_col, else 0
template <typename TO>
__device__ __forceinline__ void pad_row(TO* yr, int C, int64_t ldy, int ones_col, int lane) {
  for (int64_t j = C + lane; j < ldy; j += 32) Elem<TO>::store(yr + j, (ones_col && j == C) ? 1.f : 0.f);
}

template <int KMAX, typename TO>
__global__ void layernorm_rows_kernel(const float* __restrict__ x, int64_t ldx, const float* __restrict__ gamma,
                                      const float* __restrict__ beta, int M, int C, float eps, TO* __restrict__ y,
                                      int64_t ldy, int ones_col) {
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + warp;
  if (row >= M) return;
  const float* xr = x + row * ldx;
  TO* yr = y + row * ldy;
  const int nch = C / 4;
  float4 v[KMAX];
  float s = 0.f;
#pragma unroll
  for (int k = 0; k < KMAX; ++k) {
    const int c = lane + 32 * k;
    v[k] = c < nch ? *reinterpret_cast<const float4*>(xr + 4 * c) : make_float4(0.f, 0.f, 0.f, 0.f);
    s += (v[k].x + v[k].y) + (v[k].z + v[k].w);
  }
  const float mean = warp_sum(s) / C;
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < KMAX; ++k) {
    if (lane + 32 * k < nch) {
      const float a = v[k].x - mean, b = v[k].y - mean, c = v[k].z - mean, d = v[k].w - mean;
      ss += (a * a + b * b) + (c * c + d * d);
    }
  }
  const float rstd = rsqrtf(warp_sum(ss) / C + eps);
#pragma unroll
  for (int k = 0; k < KMAX; ++k) {
    const int c = lane + 32 * k;
    if (c < nch) {
      const float4 g = *reinterpret_cast<const float4*>(gamma + 4 * c);
      const float4 b = *reinterpret_cast<const float4*>(beta + 4 * c);
      store4(yr + 4 * c, (v[k].x - mean) * rstd * g.x + b.x, (v[k].y - mean) * rstd * g.y + b.y,
             (v[k].z - mean) * rstd * g.z + b.z, (v[k].w - mean) * rstd * g.w + b.w);
    }
  }
  pad_row(yr, C, ldy, ones_col, lane);
}

template <typename TO>
__global__ void layernorm_rows_generic_kernel(const float* __restrict__ x, int64_t ldx,
                                              const float* __restrict__ gamma, const float* __restrict__ beta,
                                              int M, int C, float eps, TO* __restrict__ y, int64_t ldy,
                                              int ones_col) {
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + warp;
  if (row >= M) return;
  const float* xr = x + row * ldx;
  TO* yr = y + row * ldy;
  float s = 0.f;
  for (int c = lane; c < C; c += 32) s += xr[c];
  const float mean = warp_sum(s) / C;
  float ss = 0.f;
  for (int c = lane; c < C; c += 32) {
    const float d = xr[c] - mean;
    ss += d * d;
  }
  const float rstd = rsqrtf(warp_sum(ss) / C + eps);
  for (int c = lane; c < C; c += 32) Elem<TO>::store(yr + c, (xr[c] - mean) * rstd * gamma[c] + beta[c]);
  pad_row(yr, C, ldy, ones_col, lane);
}

template <typename TO>
static void launch_ln(const float* x, int64_t ldx, const float* gamma, const float* beta, int M, int C, float eps,
                      TO* y, int64_t ldy, int ones_col, cudaStream_t s) {
  const int warps = 8;  // rows per 256-thread block
  const unsigned blocks = (unsigned)(((int64_t)M + warps - 1) / warps);
  const bool vec = C % 4 == 0 && ldx % 4 == 0 && ldy % 4 == 0 && aligned(x, 16) && aligned(gamma, 16) &&
                   aligned(beta, 16) && aligned(y, 4 * sizeof(TO));
  if (vec && C <= 4 * 32 * 8)
    layernorm_rows_kernel<8, TO><<<blocks, 32 * warps, 0, s>>>(x, ldx, gamma, beta, M, C, eps, y, ldy, ones_col);
  else if (vec && C <= 4 * 32 * 32)
    layernorm_rows_kernel<32, TO><<<blocks, 32 * warps, 0, s>>>(x, ldx, gamma, beta, M, C, eps, y, ldy, ones_col);
  else
    layernorm_rows_generic_kernel<TO><<<blocks, 32 * warps, 0, s>>>(x, ldx, gamma, beta, M, C, eps, y, ldy,
                                                                    ones_col);
}

int layernorm_rows(const float* x, int64_t ldx, const float* gamma, const float* beta, int M, int C, float eps,
                   void* y, int64_t ldy, int y_dtype, int ones_col, cudaStream_t s) {
  if (y_dtype == ATTN_BF16)
    launch_ln(x, ldx, gamma, beta, M, C, eps, (__nv_bfloat16*)y, ldy, ones_col, s);
  else
    launch_ln(x, ldx, gamma, beta, M, C, eps, (float*)y, ldy, ones_col, s);
  count_launch();
  return check_launch("layernorm_rows_kernel");
}

}  // namespace attn
