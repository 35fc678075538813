// CUDA-core GEMM for the float32 projection path: C[M,N] = op(A) op(B) (+bias) (+= C).
//
// Same contract as matmul_2d_kernel (core/kernels.py:119-140: fp32 accumulate, bias added after
// the dot) generalised to the transposed operands of the projection gradients
// (model/gpt.py:666-689).  64x64 output tile per CTA, 256 threads with a 4x4 register tile each,
// K staged through shared memory 16 at a time with coalesced global reads for either majorness.
#include "common.cuh"

namespace attn {

constexpr int SG_BM = 64, SG_BN = 64, SG_BK = 16;

template <typename TI, typename TO>
__global__ void __launch_bounds__(256)
gemm_simt_kernel(const TI* __restrict__ A, int64_t lda, int a_trans, const TI* __restrict__ Bm,
                 int64_t ldb, int b_trans, TO* __restrict__ C, int64_t ldc,
                 const float* __restrict__ bias, int M, int N, int K, int accumulate) {
  __shared__ __align__(16) float As[SG_BK][SG_BM];
  __shared__ __align__(16) float Bs[SG_BK][SG_BN];
  const int tid = threadIdx.x, tx = tid % 16, ty = tid / 16;
  const int m0 = blockIdx.y * SG_BM, n0 = blockIdx.x * SG_BN;
  float acc[4][4] = {};

  for (int k0 = 0; k0 < K; k0 += SG_BK) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int e = tid + 256 * i;
      int mm, kk;
      if (a_trans) { kk = e / SG_BM; mm = e % SG_BM; } else { mm = e / SG_BK; kk = e % SG_BK; }
      const int gm = m0 + mm, gk = k0 + kk;
      float val = 0.f;
      if (gm < M && gk < K)
        val = Elem<TI>::load(A + (a_trans ? (int64_t)gk * lda + gm : (int64_t)gm * lda + gk));
      As[kk][mm] = val;
      int nn;
      if (b_trans) { nn = e / SG_BK; kk = e % SG_BK; } else { kk = e / SG_BN; nn = e % SG_BN; }
      const int gn = n0 + nn, gk2 = k0 + kk;
      float bv = 0.f;
      if (gn < N && gk2 < K)
        bv = Elem<TI>::load(Bm + (b_trans ? (int64_t)gn * ldb + gk2 : (int64_t)gk2 * ldb + gn));
      Bs[kk][nn] = bv;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < SG_BK; ++kk) {
      const float4 a = *reinterpret_cast<const float4*>(&As[kk][ty * 4]);
      const float4 b = *reinterpret_cast<const float4*>(&Bs[kk][tx * 4]);
      const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int gm = m0 + ty * 4 + i;
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int gn = n0 + tx * 4 + j;
      if (gn >= N) continue;
      float val = acc[i][j];
      if (bias) val += bias[gn];
      TO* dst = C + (int64_t)gm * ldc + gn;
      if (accumulate) val += Elem<TO>::load(dst);
      Elem<TO>::store(dst, val);
    }
  }
}

int gemm_simt(const void* A, int64_t lda, int a_trans, const void* B, int64_t ldb, int b_trans,
              int ab_dtype, void* C, int64_t ldc, int c_dtype, const float* bias, int M, int N,
              int K, int accumulate, cudaStream_t s) {
  dim3 grid((N + SG_BN - 1) / SG_BN, (M + SG_BM - 1) / SG_BM);
  if (ab_dtype == ATTN_F32 && c_dtype == ATTN_F32)
    gemm_simt_kernel<float, float><<<grid, 256, 0, s>>>((const float*)A, lda, a_trans, (const float*)B,
        ldb, b_trans, (float*)C, ldc, bias, M, N, K, accumulate);
  else if (ab_dtype == ATTN_F32 && c_dtype == ATTN_BF16)
    gemm_simt_kernel<float, __nv_bfloat16><<<grid, 256, 0, s>>>((const float*)A, lda, a_trans,
        (const float*)B, ldb, b_trans, (__nv_bfloat16*)C, ldc, bias, M, N, K, accumulate);
  else if (ab_dtype == ATTN_BF16 && c_dtype == ATTN_F32)
    gemm_simt_kernel<__nv_bfloat16, float><<<grid, 256, 0, s>>>((const __nv_bfloat16*)A, lda, a_trans,
        (const __nv_bfloat16*)B, ldb, b_trans, (float*)C, ldc, bias, M, N, K, accumulate);
  else
    gemm_simt_kernel<__nv_bfloat16, __nv_bfloat16><<<grid, 256, 0, s>>>((const __nv_bfloat16*)A, lda,
        a_trans, (const __nv_bfloat16*)B, ldb, b_trans, (__nv_bfloat16*)C, ldc, bias, M, N, K,
        accumulate);
  count_launch();
  return check_launch("gemm_simt_kernel");
}

// ------------------------------------------------------------------------------------------
// layout adapters, casts, column sums
// ------------------------------------------------------------------------------------------

// split_heads_kernel semantics (core/mha_kernels.py:534-558), one thread per output element.
__global__ void split_heads_kernel(const float* __restrict__ qkv, float* __restrict__ q,
                                   float* __restrict__ k, float* __restrict__ v, int B, int T,
                                   int NH, int HD) {
  const int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int C = NH * HD;
  const int64_t total = (int64_t)B * T * NH * HD;
  if (idx >= total) return;
  const int hd = idx % HD;
  const int nh = (idx / HD) % NH;
  const int t = (idx / ((int64_t)HD * NH)) % T;
  const int64_t b = idx / ((int64_t)HD * NH * T);
  const int64_t row = b * T + t;
  const int col = nh * HD + hd;
  const int64_t out = (b * NH + nh) * T * HD + (int64_t)t * HD + hd;
  q[out] = qkv[row * 3 * C + col];
  k[out] = qkv[row * 3 * C + C + col];
  v[out] = qkv[row * 3 * C + 2 * C + col];
}

// merge_heads_kernel semantics (core/mha_kernels.py:567-584).
__global__ void merge_heads_kernel(const float* __restrict__ ch, float* __restrict__ ctx, int B,
                                   int T, int NH, int HD) {
  const int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t total = (int64_t)B * T * NH * HD;
  if (idx >= total) return;
  const int hd = idx % HD;
  const int nh = (idx / HD) % NH;
  const int t = (idx / ((int64_t)HD * NH)) % T;
  const int64_t b = idx / ((int64_t)HD * NH * T);
  const int64_t in = (b * NH + nh) * T * HD + (int64_t)t * HD + hd;
  const int64_t out = (b * T + t) * (int64_t)(NH * HD) + nh * HD + hd;
  ctx[out] = ch[in];
}

int split_heads(const float* qkv, float* q, float* k, float* v, int B, int T, int NH, int HD,
                cudaStream_t s) {
  const int64_t total = (int64_t)B * T * NH * HD;
  split_heads_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(qkv, q, k, v, B, T, NH, HD);
  count_launch();
  return check_launch("split_heads_kernel");
}

int merge_heads(const float* ch, float* ctx, int B, int T, int NH, int HD, cudaStream_t s) {
  const int64_t total = (int64_t)B * T * NH * HD;
  merge_heads_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(ch, ctx, B, T, NH, HD);
  count_launch();
  return check_launch("merge_heads_kernel");
}

// fp32 -> bf16, 8 elements per thread per step when 16-byte aligned (grid-stride).
__global__ void cast_f32_bf16_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ y,
                                     int64_t n, int vec) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (vec) {
    const int64_t n8 = n / 8;
    for (int64_t j = i; j < n8; j += stride) {
      const float4 a = reinterpret_cast<const float4*>(x)[2 * j];
      const float4 b = reinterpret_cast<const float4*>(x)[2 * j + 1];
      __nv_bfloat162 p0 = __floats2bfloat162_rn(a.x, a.y), p1 = __floats2bfloat162_rn(a.z, a.w);
      __nv_bfloat162 p2 = __floats2bfloat162_rn(b.x, b.y), p3 = __floats2bfloat162_rn(b.z, b.w);
      uint4 u;
      u.x = *reinterpret_cast<uint32_t*>(&p0);
      u.y = *reinterpret_cast<uint32_t*>(&p1);
      u.z = *reinterpret_cast<uint32_t*>(&p2);
      u.w = *reinterpret_cast<uint32_t*>(&p3);
      reinterpret_cast<uint4*>(y)[j] = u;
    }
    for (int64_t j = n8 * 8 + i; j < n; j += stride) y[j] = __float2bfloat16_rn(x[j]);
  } else {
    for (int64_t j = i; j < n; j += stride) y[j] = __float2bfloat16_rn(x[j]);
  }
}

int cast_f32_bf16(const float* x, void* y, int64_t n, cudaStream_t s, int sm_count) {
  const int vec = aligned(x, 16) && aligned(y, 16);
  int64_t want = (n / 8 + 255) / 256;
  int blocks = (int)(want < 1 ? 1 : (want > 8 * sm_count ? 8 * sm_count : want));
  cast_f32_bf16_kernel<<<blocks, 256, 0, s>>>(x, (__nv_bfloat16*)y, n, vec);
  count_launch();
  return check_launch("cast_f32_bf16_kernel");
}

// Column sums: pass 1 writes one partial row per split of M; pass 2 adds the partials in a fixed
// order (deterministic), optionally onto the existing output.
static int colsum_splits(int M, int N) {
  const int col_blocks = (N + 31) / 32;
  int s = (600 + col_blocks - 1) / col_blocks;
  const int max_s = (M + 63) / 64;
  if (s > max_s) s = max_s;
  if (s > 256) s = 256;
  return s < 1 ? 1 : s;
}

size_t colsum_ws(int M, int N) { return (size_t)colsum_splits(M, N) * N * sizeof(float); }

template <typename T>
__global__ void __launch_bounds__(256)
colsum_partial_kernel(const T* __restrict__ X, int64_t ldx, int M, int N, int rows_per_split,
                      float* __restrict__ part) {
  __shared__ float red[8][33];
  const int tx = threadIdx.x % 32, ty = threadIdx.x / 32;
  const int n = blockIdx.x * 32 + tx;
  const int r0 = blockIdx.y * rows_per_split;
  const int r1 = min(M, r0 + rows_per_split);
  float acc = 0.f;
  if (n < N)
    for (int r = r0 + ty; r < r1; r += 8) acc += Elem<T>::load(X + (int64_t)r * ldx + n);
  red[ty][tx] = acc;
  __syncthreads();
  if (ty == 0 && n < N) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) s += red[i][tx];
    part[(int64_t)blockIdx.y * N + n] = s;
  }
}

__global__ void colsum_combine_kernel(const float* __restrict__ part, int splits, int N,
                                      float* __restrict__ out, int accumulate) {
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= N) return;
  float s = 0.f;
  for (int i = 0; i < splits; ++i) s += part[(int64_t)i * N + n];
  out[n] = accumulate ? out[n] + s : s;
}

int colsum(const void* X, int x_dtype, int64_t ldx, int M, int N, float* out, int accumulate,
           void* ws, cudaStream_t s) {
  const int splits = colsum_splits(M, N);
  const int rps = (M + splits - 1) / splits;
  dim3 g1((N + 31) / 32, splits);
  float* part = (float*)ws;
  if (x_dtype == ATTN_F32)
    colsum_partial_kernel<float><<<g1, 256, 0, s>>>((const float*)X, ldx, M, N, rps, part);
  else
    colsum_partial_kernel<__nv_bfloat16><<<g1, 256, 0, s>>>((const __nv_bfloat16*)X, ldx, M, N, rps,
                                                            part);
  count_launch();
  int rc = check_launch("colsum_partial_kernel");
  if (rc) return rc;
  colsum_combine_kernel<<<(N + 255) / 256, 256, 0, s>>>(part, splits, N, out, accumulate);
  count_launch();
  return check_launch("colsum_combine_kernel");
}

}  // namespace attn
