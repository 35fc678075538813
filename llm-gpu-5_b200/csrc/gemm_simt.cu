// CUDA-core GEMM for the float32 projection path: C[M,N] = op(A) op(B) (+bias) (+= C).
//
// Same contract as matmul_2d_kernel (core/kernels.py:119-140: fp32 accumulate, bias added after
// the dot) generalised to the transposed operands of the projection gradients
// (model/gpt.py:666-689).  Two tile shapes: 128x128 per CTA with an 8x8 register tile per thread
// and double-buffered stages of 8 K (large outputs), and 64x64 with 4x4 per thread and stages of
// 16 K (small outputs, and K ranges over 8,192, where its chunk sums get Kahan compensation); both
// with coalesced global reads for either majorness.
// The epilogue applies the feed-forward activations of the tensor-core GEMM (ACT_GELU with an
// optional pre-activation output, ACT_GELU_BWD scaling by gelu'(aux)) with tanhf, in float32.
#include "common.cuh"

namespace attn {

constexpr int SG_BM = 64, SG_BN = 64, SG_BK = 16;

template <typename TI, typename TO>
__global__ void __launch_bounds__(256)
gemm_simt_kernel(const TI* __restrict__ A, int64_t lda, int a_trans, const TI* __restrict__ Bm,
                 int64_t ldb, int b_trans, TO* __restrict__ C, int64_t ldc,
                 const float* __restrict__ bias, int M, int N, int K, int accumulate, int k_chunk, int act,
                 void* __restrict__ aux, int64_t ldaux, int aux_bf16) {
  __shared__ __align__(16) float As[SG_BK][SG_BM];
  __shared__ __align__(16) float Bs[SG_BK][SG_BN];
  const int tid = threadIdx.x, tx = tid % 16, ty = tid / 16;
  const int m0 = blockIdx.y * SG_BM, n0 = blockIdx.x * SG_BN;
  const int k_begin = blockIdx.z * k_chunk, k_end = min(K, k_begin + k_chunk);
  const bool split = gridDim.z > 1;
  // Long reductions (the weight gradients sum over every token: K = 262,144 at batch 512, T = 512)
  // lose float32 accuracy in one running sum.  Each 256-deep chunk of K is summed on its own in
  // acc, and the chunk sums are added into tot with Kahan compensation (comp).  For K <= 256 the
  // result is the plain running sum.
  float acc[4][4] = {}, tot[4][4] = {}, comp[4][4] = {};
  auto fold = [&]() {
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float y = acc[i][j] - comp[i][j];
        const float t = tot[i][j] + y;
        comp[i][j] = (t - tot[i][j]) - y;
        tot[i][j] = t;
        acc[i][j] = 0.f;
      }
  };
  int tiles_in_chunk = 0;

  for (int k0 = k_begin; k0 < k_end; k0 += SG_BK) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int e = tid + 256 * i;
      int mm, kk;
      if (a_trans) { kk = e / SG_BM; mm = e % SG_BM; } else { mm = e / SG_BK; kk = e % SG_BK; }
      const int gm = m0 + mm, gk = k0 + kk;
      float val = 0.f;
      if (gm < M && gk < k_end)
        val = Elem<TI>::load(A + (a_trans ? (int64_t)gk * lda + gm : (int64_t)gm * lda + gk));
      As[kk][mm] = val;
      int nn;
      if (b_trans) { nn = e / SG_BK; kk = e % SG_BK; } else { kk = e / SG_BN; nn = e % SG_BN; }
      const int gn = n0 + nn, gk2 = k0 + kk;
      float bv = 0.f;
      if (gn < N && gk2 < k_end)
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
    if (++tiles_in_chunk == 256 / SG_BK) {
      fold();
      tiles_in_chunk = 0;
    }
  }
  fold();
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int gm = m0 + ty * 4 + i;
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int gn = n0 + tx * 4 + j;
      if (gn >= N) continue;
      float val = tot[i][j];
      if (bias && blockIdx.z == 0) val += bias[gn];
      if (act == ACT_GELU) {
        if (aux) {
          if (aux_bf16)
            reinterpret_cast<__nv_bfloat16*>(aux)[(int64_t)gm * ldaux + gn] = __float2bfloat16_rn(val);
          else
            reinterpret_cast<float*>(aux)[(int64_t)gm * ldaux + gn] = val;
        }
        val = gelu_fwd<false>(val);
      } else if (act == ACT_GELU_BWD) {
        const float x = aux_bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(aux)[(int64_t)gm * ldaux + gn])
                                 : reinterpret_cast<const float*>(aux)[(int64_t)gm * ldaux + gn];
        val *= gelu_grad<false>(x);
      }
      TO* dst = C + (int64_t)gm * ldc + gn;
      if (split) {  // float32 C only (host-checked)
        atomicAdd(reinterpret_cast<float*>(dst), val);
        continue;
      }
      if (accumulate) val += Elem<TO>::load(dst);
      Elem<TO>::store(dst, val);
    }
  }
}

// The same GEMM on 128x128 tiles: 256 threads with an 8x8 register tile each (two 4-row by two
// 4-column blocks, so every shared-memory read is a conflict-free float4), K staged 8 at a time
// in two shared-memory buffers, the next stage's global loads issued before the current stage's
// FMAs.  Four float4 reads feed 64 FMAs, twice the 4x4 kernel's ratio.  Each 256-deep chunk of K is
// summed on its own and the chunk sums are added into the result; the host sends a K range over
// 8,192 (at most 32 chunk sums) to the 4x4 kernel, whose chunk sums get Kahan compensation.
constexpr int SB_BM = 128, SB_BN = 128, SB_BK = 8, SB_PAD = 4;
constexpr int SB_MAX_K = 8192;

template <typename TI, typename TO>
__global__ void __launch_bounds__(256, 1)
gemm_simt_big_kernel(const TI* __restrict__ A, int64_t lda, int a_trans, const TI* __restrict__ Bm,
                     int64_t ldb, int b_trans, TO* __restrict__ C, int64_t ldc,
                     const float* __restrict__ bias, int M, int N, int K, int accumulate, int k_chunk, int act,
                     void* __restrict__ aux, int64_t ldaux, int aux_bf16) {
  __shared__ __align__(16) float As[2][SB_BK][SB_BM + SB_PAD];
  __shared__ __align__(16) float Bs[2][SB_BK][SB_BN + SB_PAD];
  const int tid = threadIdx.x, tx = tid % 16, ty = tid / 16;
  const int m0 = blockIdx.y * SB_BM, n0 = blockIdx.x * SB_BN;
  const int k_begin = blockIdx.z * k_chunk, k_end = min(K, k_begin + k_chunk);
  const bool split = gridDim.z > 1;
  float acc[8][8] = {}, tot[8][8] = {};
  float ra[4], rb[4];  // the next stage, in registers
  // element e = tid + 256 i of a stage: (row, k) of A and (k, column) of B, coalesced for either majorness
  auto load = [&](int k0) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int e = tid + 256 * i;
      int mm, kk;
      if (a_trans) { kk = e / SB_BM; mm = e % SB_BM; } else { mm = e / SB_BK; kk = e % SB_BK; }
      const int gm = m0 + mm, gk = k0 + kk;
      ra[i] = (gm < M && gk < k_end) ? Elem<TI>::load(A + (a_trans ? (int64_t)gk * lda + gm : (int64_t)gm * lda + gk))
                                     : 0.f;
      int nn;
      if (b_trans) { nn = e / SB_BK; kk = e % SB_BK; } else { kk = e / SB_BN; nn = e % SB_BN; }
      const int gn = n0 + nn, gk2 = k0 + kk;
      rb[i] = (gn < N && gk2 < k_end) ? Elem<TI>::load(Bm + (b_trans ? (int64_t)gn * ldb + gk2 : (int64_t)gk2 * ldb + gn))
                                      : 0.f;
    }
  };
  auto store = [&](int buf) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int e = tid + 256 * i;
      if (a_trans) As[buf][e / SB_BM][e % SB_BM] = ra[i]; else As[buf][e % SB_BK][e / SB_BK] = ra[i];
      if (b_trans) Bs[buf][e % SB_BK][e / SB_BK] = rb[i]; else Bs[buf][e / SB_BN][e % SB_BN] = rb[i];
    }
  };
  auto fold = [&]() {
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        tot[i][j] += acc[i][j];
        acc[i][j] = 0.f;
      }
  };
  int buf = 0, tiles_in_chunk = 0;
  if (k_begin < k_end) {
    load(k_begin);
    store(0);
  }
  __syncthreads();
  for (int k0 = k_begin; k0 < k_end; k0 += SB_BK) {
    const bool more = k0 + SB_BK < k_end;
    if (more) load(k0 + SB_BK);
#pragma unroll
    for (int kk = 0; kk < SB_BK; ++kk) {
      const float4 a0 = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 4]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[buf][kk][64 + ty * 4]);
      const float4 b0 = *reinterpret_cast<const float4*>(&Bs[buf][kk][tx * 4]);
      const float4 b1 = *reinterpret_cast<const float4*>(&Bs[buf][kk][64 + tx * 4]);
      const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    // the other buffer was last read before the barrier that ended the previous stage
    if (more) store(buf ^ 1);
    __syncthreads();
    buf ^= 1;
    if (++tiles_in_chunk == 256 / SB_BK) {
      fold();
      tiles_in_chunk = 0;
    }
  }
  fold();
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int gm = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + i - 4);
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int gn = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + j - 4);
      if (gn >= N) continue;
      float val = tot[i][j];
      if (bias && blockIdx.z == 0) val += bias[gn];
      if (act == ACT_GELU) {
        if (aux) {
          if (aux_bf16)
            reinterpret_cast<__nv_bfloat16*>(aux)[(int64_t)gm * ldaux + gn] = __float2bfloat16_rn(val);
          else
            reinterpret_cast<float*>(aux)[(int64_t)gm * ldaux + gn] = val;
        }
        val = gelu_fwd<false>(val);
      } else if (act == ACT_GELU_BWD) {
        const float x = aux_bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(aux)[(int64_t)gm * ldaux + gn])
                                 : reinterpret_cast<const float*>(aux)[(int64_t)gm * ldaux + gn];
        val *= gelu_grad<false>(x);
      }
      TO* dst = C + (int64_t)gm * ldc + gn;
      if (split) {  // float32 C only (host-checked)
        atomicAdd(reinterpret_cast<float*>(dst), val);
        continue;
      }
      if (accumulate) val += Elem<TO>::load(dst);
      Elem<TO>::store(dst, val);
    }
  }
}

// K splits for a grid of `tiles` output tiles: enough units for two waves of `slots` CTAs when the
// tiles alone fill less (float32 C without an activation only), each at least 256 deep in K.
static int simt_splits(int64_t tiles, int64_t slots, int K, int c_dtype, int act) {
  int splits = 1;
  const int64_t want = 2 * slots;
  if (c_dtype == ATTN_F32 && act == ACT_NONE && tiles < want && K >= 512) {
    splits = (int)((want + tiles - 1) / tiles);
    const int max_splits = K / 256;
    if (splits > max_splits) splits = max_splits;
    if (splits > 64) splits = 64;
  }
  return splits;
}

int gemm_simt(const void* A, int64_t lda, int a_trans, const void* B, int64_t ldb, int b_trans,
              int ab_dtype, void* C, int64_t ldc, int c_dtype, const float* bias, int M, int N,
              int K, int accumulate, cudaStream_t s, int act, void* aux, int64_t ldaux, int aux_dtype) {
  const int aux_bf16 = aux_dtype == ATTN_BF16;
  // 128x128 tiles where both output dimensions fill them, the units fill the SMs and each CTA's K
  // range stays within SB_MAX_K; otherwise 64x64 tiles (Kahan-compensated chunk sums for any K).
  // At B=256 T=128 C=256 (float32) the six projection GEMMs take 2.16 ms on 128x128 tiles against
  // 3.57 ms on 64x64.
  bool big = M >= SB_BM && N >= SB_BN;
  int splits = 1, k_chunk = K;
  dim3 grid;
  for (int attempt = 0; attempt < 2; ++attempt) {
    const int bm = big ? SB_BM : SG_BM, bn = big ? SB_BN : SG_BN, bk = big ? SB_BK : SG_BK;
    grid = dim3((N + bn - 1) / bn, (M + bm - 1) / bm);
    splits = simt_splits((int64_t)grid.x * grid.y, 148, K, c_dtype, act);
    k_chunk = K;
    if (splits > 1) {
      k_chunk = ((K + splits - 1) / splits + bk - 1) / bk * bk;
      splits = (K + k_chunk - 1) / k_chunk;
    }
    // the 8x8 kernel runs one CTA per SM: it needs a full wave of (tile, split) units
    if (!big || (k_chunk <= SB_MAX_K && (int64_t)grid.x * grid.y * splits >= 148)) break;
    big = false;
  }
  if (splits > 1 && !accumulate) {
    cudaError_t e = cudaMemset2DAsync(C, (size_t)ldc * 4, 0, (size_t)N * 4, (size_t)M, s);
    if (e != cudaSuccess) {
      set_error("gemm_simt: clearing C for the K splits failed: %s", cudaGetErrorString(e));
      return ATTN_ERR_CUDA;
    }
  }
  grid.z = splits;
#define SG_LAUNCH(TI, TO)                                                                                  \
  do {                                                                                                     \
    if (big)                                                                                               \
      gemm_simt_big_kernel<TI, TO><<<grid, 256, 0, s>>>((const TI*)A, lda, a_trans, (const TI*)B, ldb, b_trans, \
                                                        (TO*)C, ldc, bias, M, N, K, accumulate, k_chunk, act, aux, \
                                                        ldaux, aux_bf16);                                  \
    else                                                                                                   \
      gemm_simt_kernel<TI, TO><<<grid, 256, 0, s>>>((const TI*)A, lda, a_trans, (const TI*)B, ldb, b_trans,     \
                                                    (TO*)C, ldc, bias, M, N, K, accumulate, k_chunk, act, aux,  \
                                                    ldaux, aux_bf16);                                      \
  } while (0)
  if (ab_dtype == ATTN_F32 && c_dtype == ATTN_F32)
    SG_LAUNCH(float, float);
  else if (ab_dtype == ATTN_F32 && c_dtype == ATTN_BF16)
    SG_LAUNCH(float, __nv_bfloat16);
  else if (ab_dtype == ATTN_BF16 && c_dtype == ATTN_F32)
    SG_LAUNCH(__nv_bfloat16, float);
  else
    SG_LAUNCH(__nv_bfloat16, __nv_bfloat16);
#undef SG_LAUNCH
  count_launch();
  return check_launch(big ? "gemm_simt_big_kernel" : "gemm_simt_kernel");
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

// fp32 [M][ldx] -> bf16 [M][ldy] with a ones column appended: y[m, n] = bf16(x[m, n]) for n < N,
// y[m, N] = 1, y[m, n] = 0 for N < n < ldy.  One thread writes 8 columns (16 bytes) of a row
// (grid-stride over rows x ldy/8 chunks).  A GEMM with y^T as its left operand then produces the
// column sums of its right operand as one extra output row.
__global__ void cast_rows_ones_kernel(const float* __restrict__ x, int64_t ldx, int M, int N,
                                      __nv_bfloat16* __restrict__ y, int64_t ldy, int vec) {
  grid_dependency_wait();  // x is complete, and the earlier readers of y are done
  grid_dependents_launch();
  const int64_t chunks = ldy / 8, total = (int64_t)M * chunks;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += stride) {
    const int64_t m = i / chunks;
    const int n0 = (int)(i - m * chunks) * 8;
    const float* xr = x + m * ldx;
    float v[8];
    if (vec && n0 + 8 <= N) {
      const float4 a = *reinterpret_cast<const float4*>(xr + n0);
      const float4 b = *reinterpret_cast<const float4*>(xr + n0 + 4);
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = n0 + j < N ? xr[n0 + j] : (n0 + j == N ? 1.f : 0.f);
    }
    uint4 u;
    __nv_bfloat162 p0 = __floats2bfloat162_rn(v[0], v[1]), p1 = __floats2bfloat162_rn(v[2], v[3]);
    __nv_bfloat162 p2 = __floats2bfloat162_rn(v[4], v[5]), p3 = __floats2bfloat162_rn(v[6], v[7]);
    u.x = *reinterpret_cast<uint32_t*>(&p0);
    u.y = *reinterpret_cast<uint32_t*>(&p1);
    u.z = *reinterpret_cast<uint32_t*>(&p2);
    u.w = *reinterpret_cast<uint32_t*>(&p3);
    *reinterpret_cast<uint4*>(y + m * ldy + n0) = u;
  }
}

int cast_rows_ones(const float* x, int64_t ldx, int M, int N, void* y, int64_t ldy, cudaStream_t s,
                   int sms) {
  const int vec = (N % 4 == 0) && (ldx % 4 == 0) && aligned(x, 16);
  const int64_t total = (int64_t)M * (ldy / 8);
  int64_t blocks = (total + 255) / 256;
  const int64_t cap = (int64_t)sms * 8;
  if (blocks > cap) blocks = cap;
  const cudaError_t launched = launch_pdl(cast_rows_ones_kernel, dim3((unsigned)blocks), dim3(256), 0, s, x, ldx, M,
                                          N, (__nv_bfloat16*)y, ldy, vec);
  count_launch();
  return check_launch("cast_rows_ones_kernel", launched);
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
// order (deterministic), optionally onto the existing output.  Pass 1 reads 16-byte vectors: a
// CTA covers 256 columns with 256/V threads per row (V = 4 fp32 or 8 bf16 elements per thread) and
// 4 or 8 rows in flight.  The fp32 variant can also write the bf16 copy of X in the same pass
// (the dY cast and the output-projection bias gradient of model/gpt.py:667 read dY once).
constexpr int CS_COLS = 256;

__device__ __forceinline__ uint32_t bf16x2_bits(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

static int colsum_splits(int M, int N) {
  const int col_blocks = (N + CS_COLS - 1) / CS_COLS;
  int s = (4 * 148 + col_blocks - 1) / col_blocks;
  const int max_s = (M + 63) / 64;
  if (s > max_s) s = max_s;
  if (s > 1024) s = 1024;
  return s < 1 ? 1 : s;
}

size_t colsum_ws(int M, int N) { return (size_t)colsum_splits(M, N) * N * sizeof(float); }

template <typename T, bool CAST>
__global__ void __launch_bounds__(256)
colsum_partial_kernel(const T* __restrict__ X, int64_t ldx, int M, int N, int rows_per_split,
                      float* __restrict__ part, __nv_bfloat16* __restrict__ Y, int64_t ldy, int vec) {
  constexpr int V = 16 / sizeof(T);
  constexpr int TX = CS_COLS / V;  // threads along the columns
  constexpr int TY = 256 / TX;     // rows in flight
  __shared__ float red[TY][CS_COLS + 4];
  grid_dependency_wait();  // X is complete, and the earlier readers of part and Y are done
  grid_dependents_launch();
  const int tx = threadIdx.x % TX, ty = threadIdx.x / TX;
  const int c0 = blockIdx.x * CS_COLS + tx * V;
  const int r0 = blockIdx.y * rows_per_split;
  const int r1 = min(M, r0 + rows_per_split);
  float acc[V];
#pragma unroll
  for (int i = 0; i < V; ++i) acc[i] = 0.f;
  const bool full = vec && (c0 + V <= N);
  // U rows per thread per step, their loads issued before any use (memory-level parallelism):
  // 4 for float32 (0.263 -> 0.213 ms for the [262144, 768] dY cast + column sums); the bf16 form
  // measured slower unrolled (0.284 -> 0.521 ms at [262144, 2304]) and keeps one row per step
  constexpr int U = sizeof(T) == 4 ? 4 : 1;
  for (int rb = r0 + ty; rb < r1; rb += U * TY) {
    float v[U][V];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int r = rb + u * TY;
      const T* row = X + (int64_t)r * ldx + c0;
      if (r >= r1) {
#pragma unroll
        for (int i = 0; i < V; ++i) v[u][i] = 0.f;
      } else if (full) {
        if constexpr (sizeof(T) == 4) {
          const float4 a = __ldg(reinterpret_cast<const float4*>(row));
          v[u][0] = a.x; v[u][1] = a.y; v[u][2] = a.z; v[u][3] = a.w;
        } else {
          const uint4 q = __ldg(reinterpret_cast<const uint4*>(row));
          const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
            v[u][2 * i] = f.x;
            v[u][2 * i + 1] = f.y;
          }
        }
      } else {
#pragma unroll
        for (int i = 0; i < V; ++i) v[u][i] = (c0 + i < N) ? Elem<T>::load(row + i) : 0.f;
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
#pragma unroll
      for (int i = 0; i < V; ++i) acc[i] += v[u][i];
      const int r = rb + u * TY;
      if constexpr (CAST) {
        if (r < r1) {
          __nv_bfloat16* y = Y + (int64_t)r * ldy + c0;
          if (full) {
            *reinterpret_cast<uint2*>(y) = make_uint2(bf16x2_bits(v[u][0], v[u][1]), bf16x2_bits(v[u][2], v[u][3]));
          } else {
            for (int i = 0; i < V; ++i)
              if (c0 + i < N) y[i] = __float2bfloat16_rn(v[u][i]);
          }
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < V; ++i) red[ty][tx * V + i] = acc[i];
  __syncthreads();
  for (int c = threadIdx.x; c < CS_COLS; c += 256) {
    const int n = blockIdx.x * CS_COLS + c;
    if (n >= N) continue;
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < TY; ++i) s += red[i][c];
    part[(int64_t)blockIdx.y * N + n] = s;
  }
}

// Sum of the splits' partial rows: a block covers 32 columns, its eight warps take every eighth
// partial row (four loads in flight per thread) and meet in shared memory, so the few hundred
// partial rows are read by N/32 blocks in parallel instead of by one dependent chain per column.
// The order of the additions is fixed, so the result is deterministic.
__global__ void __launch_bounds__(256) colsum_combine_kernel(const float* __restrict__ part, int splits, int N,
                                                             float* __restrict__ out, int accumulate) {
  __shared__ float red[8][33];
  grid_dependency_wait();  // the partial rows are complete
  grid_dependents_launch();
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int n = blockIdx.x * 32 + lane;
  float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
  if (n < N) {
    int i = w;
    for (; i + 24 < splits; i += 32) {
      a0 += part[(int64_t)i * N + n];
      a1 += part[(int64_t)(i + 8) * N + n];
      a2 += part[(int64_t)(i + 16) * N + n];
      a3 += part[(int64_t)(i + 24) * N + n];
    }
    for (; i < splits; i += 8) a0 += part[(int64_t)i * N + n];
  }
  red[w][lane] = (a0 + a1) + (a2 + a3);
  __syncthreads();
  if (w == 0 && n < N) {
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) s += red[k][lane];
    out[n] = accumulate ? out[n] + s : s;
  }
}

static int colsum_launch(const void* X, int x_dtype, int64_t ldx, int M, int N, float* out,
                         int accumulate, void* ws, __nv_bfloat16* Y, int64_t ldy, cudaStream_t s) {
  const int splits = colsum_splits(M, N);
  const int rps = (M + splits - 1) / splits;
  dim3 g1((N + CS_COLS - 1) / CS_COLS, splits);
  float* part = (float*)ws;
  const size_t es = x_dtype == ATTN_F32 ? 4 : 2;
  int vec = aligned(X, 16) && ((ldx * es) % 16 == 0);
  if (Y) vec = vec && aligned(Y, 8) && ((ldy * 2) % 8 == 0);
  cudaError_t launched;
  if (x_dtype == ATTN_F32) {
    if (Y)
      launched = launch_pdl(colsum_partial_kernel<float, true>, g1, dim3(256), 0, s, (const float*)X, ldx, M, N, rps,
                            part, Y, ldy, vec);
    else
      launched = launch_pdl(colsum_partial_kernel<float, false>, g1, dim3(256), 0, s, (const float*)X, ldx, M, N, rps,
                            part, (__nv_bfloat16*)nullptr, (int64_t)0, vec);
  } else {
    launched = launch_pdl(colsum_partial_kernel<__nv_bfloat16, false>, g1, dim3(256), 0, s, (const __nv_bfloat16*)X,
                          ldx, M, N, rps, part, (__nv_bfloat16*)nullptr, (int64_t)0, vec);
  }
  count_launch();
  int rc = check_launch("colsum_partial_kernel", launched);
  if (rc) return rc;
  launched = launch_pdl(colsum_combine_kernel, dim3((N + 31) / 32), dim3(256), 0, s, (const float*)part, splits, N,
                        out, accumulate);
  count_launch();
  return check_launch("colsum_combine_kernel", launched);
}

int colsum(const void* X, int x_dtype, int64_t ldx, int M, int N, float* out, int accumulate,
           void* ws, cudaStream_t s) {
  return colsum_launch(X, x_dtype, ldx, M, N, out, accumulate, ws, nullptr, 0, s);
}

int cast_colsum(const float* X, int64_t ldx, int M, int N, void* Y, int64_t ldy, float* out,
                int accumulate, void* ws, cudaStream_t s) {
  return colsum_launch(X, ATTN_F32, ldx, M, N, out, accumulate, ws, (__nv_bfloat16*)Y, ldy, s);
}

}  // namespace attn
