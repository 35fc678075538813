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

// ---------------------------------------------------------------------------------------------
// LayerNorm backward (layernorm_backward_kernel, core/kernels.py:361-416): per row, with
// x_hat = (x - mean) * rstd and g = dy * gamma,
//   dx = rstd / C * (C * g - sum(g) - x_hat * sum(g * x_hat)),
//   dgamma += sum over rows of dy * x_hat,   dbeta += sum over rows of dy.
// dx is written, or added to dx's current contents (accumulate_dx: the residual branch of
// TransformerBlock.backward, dX0 = dX1 + dLN, model/gpt.py:826-838, done in place).  A persistent
// grid walks the rows one warp per row; every lane keeps the dgamma/dbeta partials of its own
// columns in registers across rows, the CTA's warps combine them in shared memory, and the CTA
// adds its sums to the outputs once (2 C global atomics per CTA).
template <int KMAX>
__global__ void layernorm_bwd_rows_kernel(const float* __restrict__ dy, const float* __restrict__ x,
                                          const float* __restrict__ gamma, int M, int C, float eps,
                                          float* __restrict__ dx, int accumulate_dx, float* __restrict__ dgamma,
                                          float* __restrict__ dbeta) {
  const int lane = threadIdx.x % 32;
  const int64_t wid = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int64_t nw = (int64_t)gridDim.x * (blockDim.x / 32);
  const int nch = C / 4;
  __shared__ float s_pg[4 * 32 * KMAX], s_pb[4 * 32 * KMAX];
  for (int i = threadIdx.x; i < C; i += blockDim.x) s_pg[i] = s_pb[i] = 0.f;
  __syncthreads();
  float4 pg[KMAX], pb[KMAX];
#pragma unroll
  for (int k = 0; k < KMAX; ++k) pg[k] = pb[k] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int64_t row = wid; row < M; row += nw) {
    const float* xr = x + row * C;
    const float* dyr = dy + row * C;
    float4 xv[KMAX], gv[KMAX];
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < KMAX; ++k) {
      const int c = lane + 32 * k;
      xv[k] = c < nch ? *reinterpret_cast<const float4*>(xr + 4 * c) : make_float4(0.f, 0.f, 0.f, 0.f);
      s += (xv[k].x + xv[k].y) + (xv[k].z + xv[k].w);
    }
    const float mean = warp_sum(s) / C;
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < KMAX; ++k) {
      if (lane + 32 * k < nch) {
        xv[k].x -= mean; xv[k].y -= mean; xv[k].z -= mean; xv[k].w -= mean;
        ss += (xv[k].x * xv[k].x + xv[k].y * xv[k].y) + (xv[k].z * xv[k].z + xv[k].w * xv[k].w);
      }
    }
    const float rstd = rsqrtf(warp_sum(ss) / C + eps);
    float sg = 0.f, sgx = 0.f;
#pragma unroll
    for (int k = 0; k < KMAX; ++k) {
      const int c = lane + 32 * k;
      if (c < nch) {
        const float4 d = *reinterpret_cast<const float4*>(dyr + 4 * c);
        const float4 g = *reinterpret_cast<const float4*>(gamma + 4 * c);
        xv[k].x *= rstd; xv[k].y *= rstd; xv[k].z *= rstd; xv[k].w *= rstd;  // x_hat
        pg[k].x += d.x * xv[k].x; pg[k].y += d.y * xv[k].y; pg[k].z += d.z * xv[k].z; pg[k].w += d.w * xv[k].w;
        pb[k].x += d.x; pb[k].y += d.y; pb[k].z += d.z; pb[k].w += d.w;
        gv[k] = make_float4(d.x * g.x, d.y * g.y, d.z * g.z, d.w * g.w);
        sg += (gv[k].x + gv[k].y) + (gv[k].z + gv[k].w);
        sgx += (gv[k].x * xv[k].x + gv[k].y * xv[k].y) + (gv[k].z * xv[k].z + gv[k].w * xv[k].w);
      }
    }
    sg = warp_sum(sg);
    sgx = warp_sum(sgx);
    const float f = rstd / C;
    float* dxr = dx + row * C;
#pragma unroll
    for (int k = 0; k < KMAX; ++k) {
      const int c = lane + 32 * k;
      if (c < nch) {
        float4 o;
        o.x = f * (C * gv[k].x - sg - xv[k].x * sgx);
        o.y = f * (C * gv[k].y - sg - xv[k].y * sgx);
        o.z = f * (C * gv[k].z - sg - xv[k].z * sgx);
        o.w = f * (C * gv[k].w - sg - xv[k].w * sgx);
        if (accumulate_dx) {
          const float4 a = *reinterpret_cast<const float4*>(dxr + 4 * c);
          o.x += a.x; o.y += a.y; o.z += a.z; o.w += a.w;
        }
        *reinterpret_cast<float4*>(dxr + 4 * c) = o;
      }
    }
  }
#pragma unroll
  for (int k = 0; k < KMAX; ++k) {
    const int c = lane + 32 * k;
    if (c < nch) {
      atomicAdd(s_pg + 4 * c, pg[k].x); atomicAdd(s_pg + 4 * c + 1, pg[k].y);
      atomicAdd(s_pg + 4 * c + 2, pg[k].z); atomicAdd(s_pg + 4 * c + 3, pg[k].w);
      atomicAdd(s_pb + 4 * c, pb[k].x); atomicAdd(s_pb + 4 * c + 1, pb[k].y);
      atomicAdd(s_pb + 4 * c + 2, pb[k].z); atomicAdd(s_pb + 4 * c + 3, pb[k].w);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < C; i += blockDim.x) {
    atomicAdd(dgamma + i, s_pg[i]);
    atomicAdd(dbeta + i, s_pb[i]);
  }
}

// Any C: one warp per row, scalar, parameter gradients by per-element atomics.
__global__ void layernorm_bwd_rows_generic_kernel(const float* __restrict__ dy, const float* __restrict__ x,
                                                  const float* __restrict__ gamma, int M, int C, float eps,
                                                  float* __restrict__ dx, int accumulate_dx,
                                                  float* __restrict__ dgamma, float* __restrict__ dbeta) {
  const int lane = threadIdx.x % 32;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  if (row >= M) return;
  const float* xr = x + row * C;
  const float* dyr = dy + row * C;
  float s = 0.f;
  for (int c = lane; c < C; c += 32) s += xr[c];
  const float mean = warp_sum(s) / C;
  float ss = 0.f;
  for (int c = lane; c < C; c += 32) ss += (xr[c] - mean) * (xr[c] - mean);
  const float rstd = rsqrtf(warp_sum(ss) / C + eps);
  float sg = 0.f, sgx = 0.f;
  for (int c = lane; c < C; c += 32) {
    const float xh = (xr[c] - mean) * rstd, g = dyr[c] * gamma[c];
    atomicAdd(dgamma + c, dyr[c] * xh);
    atomicAdd(dbeta + c, dyr[c]);
    sg += g;
    sgx += g * xh;
  }
  sg = warp_sum(sg);
  sgx = warp_sum(sgx);
  for (int c = lane; c < C; c += 32) {
    const float xh = (xr[c] - mean) * rstd;
    const float o = rstd / C * (C * dyr[c] * gamma[c] - sg - xh * sgx);
    dx[row * C + c] = accumulate_dx ? dx[row * C + c] + o : o;
  }
}

int layernorm_bwd_rows(const float* dy, const float* x, const float* gamma, int M, int C, float eps, float* dx,
                       int accumulate_dx, float* dgamma, float* dbeta, int accumulate_params, cudaStream_t s,
                       int sms) {
  if (!accumulate_params) {
    ATTN_CUDA_TRY(cudaMemsetAsync(dgamma, 0, (size_t)C * sizeof(float), s));
    ATTN_CUDA_TRY(cudaMemsetAsync(dbeta, 0, (size_t)C * sizeof(float), s));
  }
  const int warps = 8;
  const bool vec = C % 4 == 0 && aligned(dy, 16) && aligned(x, 16) && aligned(gamma, 16) && aligned(dx, 16);
  const int64_t row_blocks = ((int64_t)M + warps - 1) / warps;
  if (vec && C <= 4 * 32 * 8) {
    const int64_t cap = (int64_t)sms * 4;  // persistent: the lanes' parameter partials live across rows
    layernorm_bwd_rows_kernel<8><<<(unsigned)(row_blocks < cap ? row_blocks : cap), 32 * warps, 0, s>>>(
        dy, x, gamma, M, C, eps, dx, accumulate_dx, dgamma, dbeta);
  } else {
    layernorm_bwd_rows_generic_kernel<<<(unsigned)row_blocks, 32 * warps, 0, s>>>(dy, x, gamma, M, C, eps, dx,
                                                                                  accumulate_dx, dgamma, dbeta);
  }
  count_launch();
  return check_launch("layernorm_bwd_rows_kernel");
}

}  // namespace attn
