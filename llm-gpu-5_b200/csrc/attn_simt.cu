// CUDA-core (FP32 FMA) causal attention forward/backward for any head_dim in {4,8,16,32,64,128}.
//
// This is the exact path used for float32 problems (the reference's own precision) and the
// generic path for bf16 head dims the tensor-core kernels do not cover.  Math follows the
// reference: scores = scale * q.k over keys j <= i (core/mha_kernels.py:429-445), a softmax with
// expf (core/mha_kernels.py:466-470; the reference compiles with --use_fast_math, so its expf is the
// hardware exponential) computed here as 2^x on log2-scaled scores with the ex2.approx instruction,
// O = P.V (core/mha_kernels.py:501-520); backward is
// the VJP of model/gpt.py:672-680 with the scale applied to dS (model/gpt.py:677).
//
// Instead of materialising P[T,T] the forward keeps an online softmax per row and writes the
// row log-sum-exp; the backward recomputes P = exp(scale*q.k - lse).
//
// Thread layout: each query (forward, dQ) or key (dK/dV) row is owned by TPR threads that each
// hold DPT = D/TPR of its elements in registers, interleaved in float4 groups
// (element d = (v*TPR + part)*4 + c) so that the TPR threads of a row read adjacent 16-byte
// words of a shared-memory row (no bank conflicts).  Dot products finish with a TPR-wide
// butterfly of warp shuffles, which leaves the identical sum in every lane of the row.
#include "common.cuh"
#include <math.h>

namespace attn {

template <int D> struct RowSplit {
  // threads per row: 32 elements per thread from D = 64 up, 16 at D = 32 (B=256 T=128 NH=8: forward
  // 0.168 -> 0.147 ms, backward 0.476 -> 0.454 ms; four threads per row measured slower), one below
  static constexpr int TPR = D > 32 ? D / 32 : (D == 32 ? 2 : 1);
  static constexpr int DPT = D / TPR;              // elements per thread
  static constexpr int NV = DPT / 4;               // float4 groups per thread
  static_assert(D % 4 == 0 && DPT % 4 == 0, "head_dim must be a multiple of 4");
};

constexpr float kLog2e = 1.4426950408889634f, kLn2 = 0.6931471805599453f;

// 2^x by the special-function unit (ex2.approx.ftz.f32); the softmax works in log2 units.
__device__ __forceinline__ float exp2_fast(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float dot4(float4 a, float4 b) {
  return a.x * b.x + a.y * b.y + a.z * b.z + a.w * b.w;
}
__device__ __forceinline__ void axpy4(float4& acc, float s, float4 x) {
  acc.x += s * x.x; acc.y += s * x.y; acc.z += s * x.z; acc.w += s * x.w;
}
__device__ __forceinline__ void scale4(float4& a, float s) { a.x *= s; a.y *= s; a.z *= s; a.w *= s; }

// x as the tf32 tensor cores read it (the 13 low mantissa bits ignored), when TF32S; else x.
// The backward after a tf32 forward recomputes its scores from these values, so that
// P = exp(scale*q.k - lse) matches the probabilities the forward's lse was computed from.
template <bool TF32S>
__device__ __forceinline__ float4 score_operand(float4 x) {
  if constexpr (TF32S) {
    const uint32_t m = 0xffffe000u;
    return make_float4(__uint_as_float(__float_as_uint(x.x) & m), __uint_as_float(__float_as_uint(x.y) & m),
                       __uint_as_float(__float_as_uint(x.z) & m), __uint_as_float(__float_as_uint(x.w) & m));
  } else {
    return x;
  }
}

template <int TPR> __device__ __forceinline__ float row_reduce(float v) {
#pragma unroll
  for (int off = TPR / 2; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

struct AttnStrides {
  int64_t in_sb, in_st, in_sh, out_sb, out_st, out_sh;
};

// ------------------------------------------------------------------------------------------
// forward: one CTA = 64 query rows of one (b, h); K/V tiles of 32 keys staged in shared memory
// ------------------------------------------------------------------------------------------
constexpr int FWD_BM = 64, FWD_BN = 32;

template <typename T, int D>
__global__ void __launch_bounds__(FWD_BM * RowSplit<D>::TPR)
attn_fwd_simt_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                     T* __restrict__ o, float* __restrict__ lse, int NH, int T_, AttnStrides st,
                     float scale) {
  using RS = RowSplit<D>;
  const float scale_log2 = scale * kLog2e;
  constexpr int TPR = RS::TPR, NV = RS::NV, D4 = D / 4;
  __shared__ float4 Ks[FWD_BN][D4];
  __shared__ float4 Vs[FWD_BN][D4];

  const int bh = blockIdx.y, b = bh / NH, h = bh % NH;
  const int qtile = gridDim.x - 1 - blockIdx.x;  // longest causal rows first
  const int tid = threadIdx.x, part = tid % TPR, r = tid / TPR;
  const int row = qtile * FWD_BM + r;
  const T* qb = q + b * st.in_sb + h * st.in_sh;
  const T* kb = k + b * st.in_sb + h * st.in_sh;
  const T* vb = v + b * st.in_sb + h * st.in_sh;

  float4 qr[NV], acc[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    qr[i] = row < T_ ? load4(qb + row * st.in_st + (i * TPR + part) * 4) : make_float4(0, 0, 0, 0);
    acc[i] = make_float4(0, 0, 0, 0);
  }
  float m = -INFINITY, l = 0.f;
  const int last_row = min(T_ - 1, qtile * FWD_BM + FWD_BM - 1);
  const int nkt = last_row / FWD_BN + 1;

  for (int kt = 0; kt < nkt; ++kt) {
    const int k0 = kt * FWD_BN;
    __syncthreads();
    for (int e = tid; e < FWD_BN * D4; e += blockDim.x) {
      const int j = e / D4, c4 = e % D4, key = k0 + j;
      float4 kv = make_float4(0, 0, 0, 0), vv = kv;
      if (key < T_) {
        kv = load4(kb + key * st.in_st + c4 * 4);
        vv = load4(vb + key * st.in_st + c4 * 4);
      }
      Ks[j][c4] = kv;
      Vs[j][c4] = vv;
    }
    __syncthreads();

    float s[FWD_BN];
    float tile_max = -INFINITY;
#pragma unroll
    for (int j = 0; j < FWD_BN; ++j) {
      float p = 0.f;
#pragma unroll
      for (int i = 0; i < NV; ++i) p += dot4(qr[i], Ks[j][i * TPR + part]);
      p = row_reduce<TPR>(p) * scale_log2;  // log2 units
      const int key = k0 + j;
      s[j] = (key <= row && key < T_) ? p : -INFINITY;
      tile_max = fmaxf(tile_max, s[j]);
    }
    // key 0 is in tile 0 and visible to every row, so m_new is finite from the first tile on
    const float m_new = fmaxf(m, tile_max);
    const float corr = exp2_fast(m - m_new);
    l *= corr;
#pragma unroll
    for (int i = 0; i < NV; ++i) scale4(acc[i], corr);
#pragma unroll
    for (int j = 0; j < FWD_BN; ++j) {
      const float p = exp2_fast(s[j] - m_new);
      l += p;
#pragma unroll
      for (int i = 0; i < NV; ++i) axpy4(acc[i], p, Vs[j][i * TPR + part]);
    }
    m = m_new;
  }

  if (row < T_) {
    const float inv = 1.f / l;
    T* ob = o + b * st.out_sb + h * st.out_sh + row * st.out_st;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      float4 a = acc[i];
      scale4(a, inv);
      store4(ob + (i * TPR + part) * 4, a);
    }
    if (part == 0) lse[(int64_t)bh * T_ + row] = (m + __log2f(l)) * kLn2;  // natural-log units
  }
}

// ------------------------------------------------------------------------------------------
// backward step 1: delta[b,h,t] = sum_d dO * O   (the row dot of the softmax VJP, gpt.py:675)
// ------------------------------------------------------------------------------------------
template <typename T, int D>
__global__ void __launch_bounds__(256)
attn_bwd_delta_kernel(const T* __restrict__ o, const T* __restrict__ dout, float* __restrict__ delta,
                      int NH, int T_, int64_t rows, AttnStrides st) {
  constexpr int LPR = D / 4;  // lanes per row (1..32)
  constexpr int RPW = 32 / LPR;
  const int lane = threadIdx.x & 31;
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t row = warp * RPW + lane / LPR;
  const int c4 = lane % LPR;
  float acc = 0.f;
  if (row < rows) {
    const int64_t bh = row / T_;
    const int t = (int)(row % T_);
    const int b = (int)(bh / NH), h = (int)(bh % NH);
    const int64_t off = b * st.out_sb + h * st.out_sh + t * st.out_st + c4 * 4;
    acc = dot4(load4(o + off), load4(dout + off));
  }
#pragma unroll
  for (int w = LPR / 2; w > 0; w >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, w);
  if (row < rows && c4 == 0) delta[row] = acc;
}

// ------------------------------------------------------------------------------------------
// backward step 2: dK, dV.  One CTA = 64 keys of one (b, h); query tiles of 64 rows (32 at head_dim
// 16 and below and at 128) staged in shared memory, from the first query that can see these keys to
// the end of the sequence.
// ------------------------------------------------------------------------------------------
constexpr int KV_BN = 64, KV_BQ = 32;

template <typename T, int D, bool TF32S = false>
__global__ void __launch_bounds__(KV_BN * RowSplit<D>::TPR)
attn_bwd_dkdv_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                     const T* __restrict__ dout, const float* __restrict__ lse,
                     const float* __restrict__ delta, T* __restrict__ dk, T* __restrict__ dv,
                     int NH, int T_, AttnStrides st, float scale) {
  using RS = RowSplit<D>;
  // 64 queries per stage for D = 32 .. 64 (fewer barriers; about 2 % faster at D = 32, bit-identical)
  constexpr int KQ = D >= 32 && D <= 64 ? 64 : KV_BQ;
  const float scale_log2 = scale * kLog2e;
  constexpr int TPR = RS::TPR, NV = RS::NV, D4 = D / 4;
  __shared__ float4 Qs[KQ][D4];
  // tf32-scored backward at D = 32: Q staged a second time as the scores read it, truncated once per
  // tile instead of by every thread per query (0.491 -> 0.471 ms at B=256 T=128 NH=8, the same
  // results; slower at D = 16 and 64, which truncate in the loop)
  constexpr bool QT = TF32S && D == 32;
  __shared__ float4 Qt[QT ? KQ : 1][D4];
  __shared__ float4 Gs[KQ][D4];
  __shared__ float Ls[KQ], Ds[KQ];

  const int bh = blockIdx.y, b = bh / NH, h = bh % NH;
  const int ktile = blockIdx.x;
  const int tid = threadIdx.x, part = tid % TPR, r = tid / TPR;
  const int key = ktile * KV_BN + r;
  const int64_t in_off = b * st.in_sb + h * st.in_sh;
  const int64_t out_off = b * st.out_sb + h * st.out_sh;

  float4 kr[NV], vr[NV], dkr[NV], dvr[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int64_t e = in_off + key * st.in_st + (i * TPR + part) * 4;
    kr[i] = key < T_ ? score_operand<TF32S>(load4(k + e)) : make_float4(0, 0, 0, 0);  // scores only
    vr[i] = key < T_ ? load4(v + e) : make_float4(0, 0, 0, 0);
    dkr[i] = make_float4(0, 0, 0, 0);
    dvr[i] = make_float4(0, 0, 0, 0);
  }

  const int qstart = (ktile * KV_BN) / KQ * KQ;
  for (int q0 = qstart; q0 < T_; q0 += KQ) {
    __syncthreads();
    for (int e = tid; e < KQ * D4; e += blockDim.x) {
      const int i = e / D4, c4 = e % D4, qi = q0 + i;
      float4 qv = make_float4(0, 0, 0, 0), gv = qv;
      if (qi < T_) {
        qv = load4(q + in_off + qi * st.in_st + c4 * 4);
        gv = load4(dout + out_off + qi * st.out_st + c4 * 4);
      }
      Qs[i][c4] = qv;
      if constexpr (QT) Qt[i][c4] = score_operand<true>(qv);
      Gs[i][c4] = gv;
    }
    for (int i = tid; i < KQ; i += blockDim.x) {
      const int qi = q0 + i;
      Ls[i] = qi < T_ ? lse[(int64_t)bh * T_ + qi] * kLog2e : 0.f;  // log2 units
      Ds[i] = qi < T_ ? delta[(int64_t)bh * T_ + qi] : 0.f;
    }
    __syncthreads();
#pragma unroll 4
    for (int i = 0; i < KQ; ++i) {
      const int qi = q0 + i;
      float s = 0.f, dp = 0.f;
#pragma unroll
      for (int c = 0; c < NV; ++c) {
        s += dot4(QT ? Qt[QT ? i : 0][c * TPR + part] : score_operand<TF32S>(Qs[i][c * TPR + part]), kr[c]);
        dp += dot4(Gs[i][c * TPR + part], vr[c]);
      }
      s = row_reduce<TPR>(s);
      dp = row_reduce<TPR>(dp);
      const bool valid = key <= qi && qi < T_ && key < T_;
      const float p = valid ? exp2_fast(s * scale_log2 - Ls[i]) : 0.f;
      const float ds = p * (dp - Ds[i]) * scale;
#pragma unroll
      for (int c = 0; c < NV; ++c) {
        axpy4(dvr[c], p, Gs[i][c * TPR + part]);
        axpy4(dkr[c], ds, Qs[i][c * TPR + part]);
      }
    }
  }
  if (key < T_) {
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int64_t e = in_off + key * st.in_st + (i * TPR + part) * 4;
      store4(dk + e, dkr[i]);
      store4(dv + e, dvr[i]);
    }
  }
}

// ------------------------------------------------------------------------------------------
// backward step 3: dQ.  One CTA = 64 query rows; K/V tiles of 64 keys (32 at head_dim 16 and below
// and at 128) up to the diagonal.
// ------------------------------------------------------------------------------------------
constexpr int DQ_BM = 64, DQ_BN = 32;

template <typename T, int D, bool TF32S = false>
__global__ void __launch_bounds__(DQ_BM * RowSplit<D>::TPR)
attn_bwd_dq_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                   const T* __restrict__ dout, const float* __restrict__ lse,
                   const float* __restrict__ delta, T* __restrict__ dq, int NH, int T_,
                   AttnStrides st, float scale) {
  using RS = RowSplit<D>;
  constexpr int KB = D >= 32 && D <= 64 ? 64 : DQ_BN;  // 64 keys per stage, as KQ above
  const float scale_log2 = scale * kLog2e;
  constexpr int TPR = RS::TPR, NV = RS::NV, D4 = D / 4;
  __shared__ float4 Ks[KB][D4];
  constexpr bool KT = TF32S && D == 32;  // K staged as the scores read it, as Q in the dK/dV kernel
  __shared__ float4 Kt[KT ? KB : 1][D4];
  __shared__ float4 Vs[KB][D4];

  const int bh = blockIdx.y, b = bh / NH, h = bh % NH;
  const int qtile = gridDim.x - 1 - blockIdx.x;
  const int tid = threadIdx.x, part = tid % TPR, r = tid / TPR;
  const int row = qtile * DQ_BM + r;
  const int64_t in_off = b * st.in_sb + h * st.in_sh;
  const int64_t out_off = b * st.out_sb + h * st.out_sh;

  float4 qr[NV], gr[NV], dqr[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    qr[i] = row < T_ ? score_operand<TF32S>(load4(q + in_off + row * st.in_st + (i * TPR + part) * 4))
                     : make_float4(0, 0, 0, 0);  // scores only
    gr[i] = row < T_ ? load4(dout + out_off + row * st.out_st + (i * TPR + part) * 4) : make_float4(0, 0, 0, 0);
    dqr[i] = make_float4(0, 0, 0, 0);
  }
  const float L = row < T_ ? lse[(int64_t)bh * T_ + row] * kLog2e : 0.f;  // log2 units
  const float Dl = row < T_ ? delta[(int64_t)bh * T_ + row] : 0.f;
  const int last_row = min(T_ - 1, qtile * DQ_BM + DQ_BM - 1);
  const int nkt = last_row / KB + 1;

  for (int kt = 0; kt < nkt; ++kt) {
    const int k0 = kt * KB;
    __syncthreads();
    for (int e = tid; e < KB * D4; e += blockDim.x) {
      const int j = e / D4, c4 = e % D4, key = k0 + j;
      float4 kv = make_float4(0, 0, 0, 0), vv = kv;
      if (key < T_) {
        kv = load4(k + in_off + key * st.in_st + c4 * 4);
        vv = load4(v + in_off + key * st.in_st + c4 * 4);
      }
      Ks[j][c4] = kv;
      if constexpr (KT) Kt[j][c4] = score_operand<true>(kv);
      Vs[j][c4] = vv;
    }
    __syncthreads();
#pragma unroll 4
    for (int j = 0; j < KB; ++j) {
      const int key = k0 + j;
      float s = 0.f, dp = 0.f;
#pragma unroll
      for (int c = 0; c < NV; ++c) {
        s += dot4(qr[c], KT ? Kt[KT ? j : 0][c * TPR + part] : score_operand<TF32S>(Ks[j][c * TPR + part]));
        dp += dot4(gr[c], Vs[j][c * TPR + part]);
      }
      s = row_reduce<TPR>(s);
      dp = row_reduce<TPR>(dp);
      const bool valid = key <= row && key < T_ && row < T_;
      const float p = valid ? exp2_fast(s * scale_log2 - L) : 0.f;
      const float ds = p * (dp - Dl) * scale;
#pragma unroll
      for (int c = 0; c < NV; ++c) axpy4(dqr[c], ds, Ks[j][c * TPR + part]);
    }
  }
  if (row < T_) {
#pragma unroll
    for (int i = 0; i < NV; ++i) store4(dq + in_off + row * st.in_st + (i * TPR + part) * 4, dqr[i]);
  }
}

// ------------------------------------------------------------------------------------------
// host launchers
// ------------------------------------------------------------------------------------------
template <typename T, int D>
static int fwd_simt_d(const void* q, const void* k, const void* v, void* o, float* lse, int B,
                      int NH, int T_, AttnStrides st, float scale, cudaStream_t s) {
  dim3 grid((T_ + FWD_BM - 1) / FWD_BM, B * NH);
  attn_fwd_simt_kernel<T, D><<<grid, FWD_BM * RowSplit<D>::TPR, 0, s>>>(
      (const T*)q, (const T*)k, (const T*)v, (T*)o, lse, NH, T_, st, scale);
  count_launch();
  return check_launch("attn_fwd_simt_kernel");
}

template <typename T, int D, bool TF32S = false>
static int bwd_simt_d(const void* q, const void* k, const void* v, const void* o, const void* dout,
                      const float* lse, void* dq, void* dk, void* dv, float* delta, int B, int NH,
                      int T_, AttnStrides st, float scale, cudaStream_t s) {
  const int64_t rows = (int64_t)B * NH * T_;
  constexpr int RPW = 32 / (D / 4);
  const int64_t warps = (rows + RPW - 1) / RPW;
  attn_bwd_delta_kernel<T, D><<<(unsigned)((warps * 32 + 255) / 256), 256, 0, s>>>(
      (const T*)o, (const T*)dout, delta, NH, T_, rows, st);
  count_launch();
  int rc = check_launch("attn_bwd_delta_kernel");
  if (rc) return rc;
  dim3 g1((T_ + KV_BN - 1) / KV_BN, B * NH);
  attn_bwd_dkdv_kernel<T, D, TF32S><<<g1, KV_BN * RowSplit<D>::TPR, 0, s>>>(
      (const T*)q, (const T*)k, (const T*)v, (const T*)dout, lse, delta, (T*)dk, (T*)dv, NH, T_,
      st, scale);
  count_launch();
  rc = check_launch("attn_bwd_dkdv_kernel");
  if (rc) return rc;
  dim3 g2((T_ + DQ_BM - 1) / DQ_BM, B * NH);
  attn_bwd_dq_kernel<T, D, TF32S><<<g2, DQ_BM * RowSplit<D>::TPR, 0, s>>>(
      (const T*)q, (const T*)k, (const T*)v, (const T*)dout, lse, delta, (T*)dq, NH, T_, st,
      scale);
  count_launch();
  return check_launch("attn_bwd_dq_kernel");
}

#define ATTN_DISPATCH_D(D_, FN, ...)                 \
  switch (D_) {                                      \
    case 4: return FN<4>(__VA_ARGS__);               \
    case 8: return FN<8>(__VA_ARGS__);               \
    case 16: return FN<16>(__VA_ARGS__);             \
    case 32: return FN<32>(__VA_ARGS__);             \
    case 64: return FN<64>(__VA_ARGS__);             \
    case 128: return FN<128>(__VA_ARGS__);           \
    default: set_error("head_dim %d not supported (4, 8, 16, 32, 64, 128)", D_); \
      return ATTN_ERR_UNSUPPORTED;                   \
  }

template <int D>
static int fwd_f32(const void* q, const void* k, const void* v, void* o, float* lse, int B, int NH,
                   int T_, AttnStrides st, float scale, cudaStream_t s) {
  return fwd_simt_d<float, D>(q, k, v, o, lse, B, NH, T_, st, scale, s);
}
template <int D>
static int fwd_bf16(const void* q, const void* k, const void* v, void* o, float* lse, int B, int NH,
                    int T_, AttnStrides st, float scale, cudaStream_t s) {
  return fwd_simt_d<__nv_bfloat16, D>(q, k, v, o, lse, B, NH, T_, st, scale, s);
}
template <int D>
static int bwd_f32(const void* q, const void* k, const void* v, const void* o, const void* dout,
                   const float* lse, void* dq, void* dk, void* dv, float* delta, int B, int NH,
                   int T_, AttnStrides st, float scale, cudaStream_t s) {
  return bwd_simt_d<float, D>(q, k, v, o, dout, lse, dq, dk, dv, delta, B, NH, T_, st, scale, s);
}
template <int D>
static int bwd_tf32(const void* q, const void* k, const void* v, const void* o, const void* dout,
                    const float* lse, void* dq, void* dk, void* dv, float* delta, int B, int NH,
                    int T_, AttnStrides st, float scale, cudaStream_t s) {
  return bwd_simt_d<float, D, true>(q, k, v, o, dout, lse, dq, dk, dv, delta, B, NH, T_, st, scale, s);
}
template <int D>
static int bwd_bf16(const void* q, const void* k, const void* v, const void* o, const void* dout,
                    const float* lse, void* dq, void* dk, void* dv, float* delta, int B, int NH,
                    int T_, AttnStrides st, float scale, cudaStream_t s) {
  return bwd_simt_d<__nv_bfloat16, D>(q, k, v, o, dout, lse, dq, dk, dv, delta, B, NH, T_, st,
                                      scale, s);
}

int attn_fwd_simt(const void* q, const void* k, const void* v, void* o, float* lse, int B, int NH,
                  int T_, int D, const int64_t* strides, float scale, int dtype, cudaStream_t s) {
  AttnStrides st{strides[0], strides[1], strides[2], strides[3], strides[4], strides[5]};
  if (dtype == ATTN_F32) {
    ATTN_DISPATCH_D(D, fwd_f32, q, k, v, o, lse, B, NH, T_, st, scale, s);
  }
  ATTN_DISPATCH_D(D, fwd_bf16, q, k, v, o, lse, B, NH, T_, st, scale, s);
}

int attn_bwd_simt(const void* q, const void* k, const void* v, const void* o, const void* dout,
                  const float* lse, void* dq, void* dk, void* dv, float* delta, int B, int NH,
                  int T_, int D, const int64_t* strides, float scale, int dtype, cudaStream_t s) {
  AttnStrides st{strides[0], strides[1], strides[2], strides[3], strides[4], strides[5]};
  if (dtype == ATTN_F32) {
    ATTN_DISPATCH_D(D, bwd_f32, q, k, v, o, dout, lse, dq, dk, dv, delta, B, NH, T_, st, scale, s);
  }
  if (dtype == ATTN_TF32) {  // float32 storage after a tf32 forward: scores from tf32 q and k
    ATTN_DISPATCH_D(D, bwd_tf32, q, k, v, o, dout, lse, dq, dk, dv, delta, B, NH, T_, st, scale, s);
  }
  ATTN_DISPATCH_D(D, bwd_bf16, q, k, v, o, dout, lse, dq, dk, dv, delta, B, NH, T_, st, scale, s);
}

// ------------------------------------------------------------------------------------------
// debug accessor: P[b,h,i,j] = exp(scale*q_i.k_j - lse_i) for j <= i (0 above the diagonal)
// ------------------------------------------------------------------------------------------
template <typename T>
__global__ void attn_probs_kernel(const T* __restrict__ q, const T* __restrict__ k,
                                  const float* __restrict__ lse, float* __restrict__ P, int NH,
                                  int T_, int D, int64_t sb, int64_t st, int64_t sh, float scale,
                                  int64_t total) {
  const int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const int j = idx % T_;
  const int i = (idx / T_) % T_;
  const int64_t bh = idx / ((int64_t)T_ * T_);
  const int b = (int)(bh / NH), h = (int)(bh % NH);
  float p = 0.f;
  if (j <= i) {
    const T* qi = q + b * sb + h * sh + i * st;
    const T* kj = k + b * sb + h * sh + j * st;
    float s = 0.f;
    for (int d = 0; d < D; ++d) s += Elem<T>::load(qi + d) * Elem<T>::load(kj + d);
    p = expf(s * scale - lse[bh * T_ + i]);
  }
  P[idx] = p;
}

int attn_probs_launch(const void* q, const void* k, const float* lse, float* P, int B, int NH,
                      int T_, int D, int64_t sb, int64_t st, int64_t sh, float scale, int dtype,
                      cudaStream_t s) {
  const int64_t total = (int64_t)B * NH * T_ * T_;
  const unsigned blocks = (unsigned)((total + 255) / 256);
  if (dtype == ATTN_F32)
    attn_probs_kernel<float><<<blocks, 256, 0, s>>>((const float*)q, (const float*)k, lse, P, NH, T_,
                                                    D, sb, st, sh, scale, total);
  else
    attn_probs_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>((const __nv_bfloat16*)q,
        (const __nv_bfloat16*)k, lse, P, NH, T_, D, sb, st, sh, scale, total);
  count_launch();
  return check_launch("attn_probs_kernel");
}

}  // namespace attn
