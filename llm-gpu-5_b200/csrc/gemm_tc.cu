// tcgen05 tensor-core GEMM for the attention projections (bf16 operands, fp32 accumulation).
//
// C[M,N] (=|+=) op(A)[M,K] . op(B)[K,N] (+ bias[N]), C float32 or bf16.  Serves the QKV and
// output projections of MultiHeadAttention.forward (model/gpt.py:558, :629; matmul_2d_kernel,
// core/kernels.py:119-140) and the projection gradients of its backward (model/gpt.py:666-689).
//
// Persistent, warp-specialised kernel, one CTA per SM:
//   warp 0      TMA producer: 128x64 A and 256x64 B tiles (128-byte swizzle) into a 4-stage ring
//   warp 1      TMEM allocation and the single MMA-issuing thread: 4 x tcgen05.mma (128x256x16)
//               per 64-deep K block, accumulating in TMEM
//   warps 2-5   epilogue: tcgen05.ld of the 128x256 fp32 accumulator (one row per thread), bias,
//               conversion, then 128-byte-wide column chunks staged in swizzled shared memory and
//               written by TMA stores (or TMA reduce-adds when accumulating into C)
// The accumulator is double-buffered in TMEM (2 x 256 columns) so the epilogue of one tile
// overlaps the main loop of the next.  Either operand may be K-major or MN-major (the transposed
// operands of the weight gradients); TMA writes both in the canonical 128B-swizzled layouts.
// Weight-gradient shapes (M, N = d_model, K = tokens) are split along K; the splits add their
// partial tiles into C with TMA reduce-adds (C is zeroed first unless accumulating).  Outputs
// without a 16-byte row pitch fall back to direct per-row stores (fp32 atomics for K splits).
//
// The epilogue can also apply the feed-forward block's activation (FeedForward, model/gpt.py:
// 327-456): ACT_GELU writes gelu(acc + bias) to C and, when an aux output is given, the
// pre-activation acc + bias to it through a second TMA map (matmul_2d_kernel + the in-place
// activation_kernel + the cache_pre_act copy, model/gpt.py:345-361); ACT_GELU_BWD multiplies the
// accumulator by gelu'(aux[m, n]) (dHidden = dOut W^T followed by gelu_backward_kernel,
// model/gpt.py:437-438).  Activations run without K splits and without accumulation.
#include "tc_common.cuh"

#include <string.h>

namespace attn {

constexpr int GT_BM = 128, GT_BN = 256, GT_BK = 64, GT_STAGES = 4;
constexpr int GT_THREADS = 192;
constexpr int GT_A_BYTES = GT_BM * GT_BK * 2;  // 16 KB
constexpr int GT_B_BYTES = GT_BN * GT_BK * 2;  // 32 KB
constexpr int GT_STAGE_BYTES = GT_A_BYTES + GT_B_BYTES;
constexpr int GT_EPI_BYTES = GT_BM * 128;      // one 128-row x 128-byte output chunk (16 KB)
constexpr int GT_SMEM = GT_STAGES * GT_STAGE_BYTES + 2 * GT_EPI_BYTES + GT_BN * 4 /*bias*/ + 1024 + 256;
constexpr uint32_t GT_TMEM_COLS = 512;

struct GemmParams {
  int M, N, K;
  int a_mn, b_mn;
  int tiles_m, tiles_n, kb_total, kb_per_split, units;
  void* C;
  int64_t ldc;
  int c_bf16, vec_ok, accumulate, atomic;
  int tma_epi;  // 1: stage output chunks in swizzled smem and write them with TMA
  int reduce;   // with tma_epi: add into C (accumulate or K splits) instead of storing
  const float* bias;
  int act;          // ACT_NONE, ACT_GELU, ACT_GELU_BWD (tma_epi only)
  const void* aux;  // ACT_GELU: pre-activation output (C's dtype) or null; ACT_GELU_BWD: input
  int64_t ldaux;
  int aux_bf16;
  int* err;
};

// The aux operand of ACT_GELU_BWD for one accumulator row: columns n0 .. n0+cols-1 as floats
// (columns past N read as 0).  A thread reads its own row (a whole 128-byte line or two).
__device__ __forceinline__ void load_aux_row(const GemmParams& p, int64_t m, int n0, int cols, float (&a)[64]) {
  const bool full = n0 + cols <= p.N;
  if (p.aux_bf16) {
    const __nv_bfloat16* src = reinterpret_cast<const __nv_bfloat16*>(p.aux) + m * p.ldaux + n0;
    if (full) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (8 * i < cols) {
          const uint4 u = reinterpret_cast<const uint4*>(src)[i];
          const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[j]));
            a[8 * i + 2 * j] = f.x;
            a[8 * i + 2 * j + 1] = f.y;
          }
        }
      }
    } else {
#pragma unroll
      for (int i = 0; i < 64; ++i) a[i] = i < cols && n0 + i < p.N ? __bfloat162float(src[i]) : 0.f;
    }
  } else {
    const float* src = reinterpret_cast<const float*>(p.aux) + m * p.ldaux + n0;
    if (full) {
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        if (4 * i < cols) {
          const float4 f = reinterpret_cast<const float4*>(src)[i];
          a[4 * i] = f.x; a[4 * i + 1] = f.y; a[4 * i + 2] = f.z; a[4 * i + 3] = f.w;
        }
      }
    } else {
#pragma unroll
      for (int i = 0; i < 64; ++i) a[i] = i < cols && n0 + i < p.N ? src[i] : 0.f;
    }
  }
}

__device__ __forceinline__ void unit_coords(const GemmParams& p, int unit, int& tm, int& tn, int& kb0,
                                            int& kb1) {
  tn = unit % p.tiles_n;
  tm = (unit / p.tiles_n) % p.tiles_m;
  const int split = unit / (p.tiles_n * p.tiles_m);
  kb0 = split * p.kb_per_split;
  kb1 = min(p.kb_total, kb0 + p.kb_per_split);
}

__device__ __forceinline__ void epilogue_store32(const GemmParams& p, int m, int n0, const uint32_t (&r)[32],
                                                 bool add_bias) {
  float v[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
  if (add_bias && p.bias) {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (n0 + i < p.N) v[i] += __ldg(p.bias + n0 + i);
  }
  const bool full = n0 + 32 <= p.N;
  if (p.c_bf16) {
    __nv_bfloat16* c = reinterpret_cast<__nv_bfloat16*>(p.C) + (int64_t)m * p.ldc + n0;
    if (full && p.vec_ok) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint4 u;
        u.x = pack_bf16x2(v[8 * i + 0], v[8 * i + 1]);
        u.y = pack_bf16x2(v[8 * i + 2], v[8 * i + 3]);
        u.z = pack_bf16x2(v[8 * i + 4], v[8 * i + 5]);
        u.w = pack_bf16x2(v[8 * i + 6], v[8 * i + 7]);
        reinterpret_cast<uint4*>(c)[i] = u;
      }
    } else {
      for (int i = 0; i < 32; ++i)
        if (n0 + i < p.N) c[i] = __float2bfloat16_rn(v[i]);
    }
    return;
  }
  float* c = reinterpret_cast<float*>(p.C) + (int64_t)m * p.ldc + n0;
  if (p.atomic) {
    for (int i = 0; i < 32; ++i)
      if (n0 + i < p.N) atomicAdd(c + i, v[i]);
    return;
  }
  if (full && p.vec_ok) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float4 o = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
      if (p.accumulate) {
        const float4 e = reinterpret_cast<const float4*>(c)[i];
        o.x += e.x; o.y += e.y; o.z += e.z; o.w += e.w;
      }
      reinterpret_cast<float4*>(c)[i] = o;
    }
  } else {
    for (int i = 0; i < 32; ++i)
      if (n0 + i < p.N) c[i] = p.accumulate ? c[i] + v[i] : v[i];
  }
}

__global__ void __launch_bounds__(GT_THREADS, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmAux,
               const GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* epi = smem + GT_STAGES * GT_STAGE_BYTES;  // [2] output staging chunks
  float* s_bias = reinterpret_cast<float*>(epi + 2 * GT_EPI_BYTES);  // the tile's bias columns
  uint64_t* full = reinterpret_cast<uint64_t*>(s_bias + GT_BN);
  uint64_t* empty = full + GT_STAGES;
  uint64_t* tfull = empty + GT_STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    for (int s = 0; s < GT_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 128);
    }
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, GT_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int unit = blockIdx.x; unit < p.units && ok; unit += gridDim.x) {
        int tm, tn, kb0, kb1;
        unit_coords(p, unit, tm, tn, kb0, kb1);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1, p.err, 101)) { ok = false; break; }
          uint8_t* sa = smem + s * GT_STAGE_BYTES;
          uint8_t* sb = sa + GT_A_BYTES;
          mbar_arrive_expect_tx(&full[s], GT_STAGE_BYTES);
          const int k0 = kb * GT_BK;
          if (!p.a_mn) {
            tma_load_2d(sa, &tmA, &full[s], k0, tm * GT_BM);
          } else {
            tma_load_2d(sa, &tmA, &full[s], tm * GT_BM, k0);
            tma_load_2d(sa + 8192, &tmA, &full[s], tm * GT_BM + 64, k0);
          }
          if (!p.b_mn) {
            tma_load_2d(sb, &tmB, &full[s], k0, tn * GT_BN);
          } else {
#pragma unroll
            for (int j = 0; j < GT_BN / 64; ++j) tma_load_2d(sb + j * 8192, &tmB, &full[s], tn * GT_BN + 64 * j, k0);
          }
          if (++s == GT_STAGES) { s = 0; ph ^= 1; }
        }
      }
      // tail: wait until the MMA thread has released every stage, so no asynchronous arrive is
      // still in flight to this CTA's shared memory when it exits
      for (int i = 0; i < GT_STAGES && ok; ++i) {
        ok = mbar_wait(&empty[s], ph ^ 1, p.err, 105);
        if (++s == GT_STAGES) { s = 0; ph ^= 1; }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(GT_BM, GT_BN, p.a_mn, p.b_mn);
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      int local = 0;
      for (int unit = blockIdx.x; unit < p.units && ok; unit += gridDim.x, ++local) {
        int tm, tn, kb0, kb1;
        unit_coords(p, unit, tm, tn, kb0, kb1);
        const int acc = local & 1;
        const uint32_t acc_ph = (local >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_ph ^ 1, p.err, 102)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * GT_BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[s], ph, p.err, 103)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * GT_STAGE_BYTES);
          const uint32_t sb = sa + GT_A_BYTES;
#pragma unroll
          for (int k = 0; k < GT_BK / 16; ++k) {
            const uint64_t ad = p.a_mn ? smem_desc_sw128(sa + k * 2048, 8192, 1024)
                                       : smem_desc_sw128(sa + k * 32, 16, 1024);
            const uint64_t bd = p.b_mn ? smem_desc_sw128(sb + k * 2048, 8192, 1024)
                                       : smem_desc_sw128(sb + k * 32, 16, 1024);
            umma_ss(d_tmem, ad, bd, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&empty[s]);  // frees the stage once these MMAs have read it
          if (++s == GT_STAGES) { s = 0; ph ^= 1; }
        }
        if (ok) umma_commit(&tfull[acc]);  // accumulator ready for the epilogue
      }
    }
  } else if (p.tma_epi) {
    // Epilogue through shared memory: each thread owns one accumulator row; a chunk of 128 bytes
    // per row (32 fp32 or 64 bf16 columns) goes to a 128B-swizzled staging buffer (conflict-free
    // 16-byte stores) and one thread writes the 128-row chunk with a TMA store, or a TMA
    // reduce-add when accumulating or splitting K.  Two staging buffers alternate.
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const bool leader = (warp == 2 && lane == 0);
    const int cols = p.c_bf16 ? 64 : 32;  // columns per 128-byte chunk
    int buf = 0;
    // stage 32 packed words per thread (one 128-byte chunk row) and write the 128-row chunk at
    // column n0 through `map`; two staging buffers alternate
    auto emit = [&](const CUtensorMap* map, const uint32_t (&w)[32], int n0, int m0, bool reduce) {
      if (leader) bulk_wait_read1();  // the store that last used this buffer has read it
      named_bar_sync(1, 128);
      uint8_t* rowp = epi + buf * GT_EPI_BYTES + row * 128;
#pragma unroll
      for (int ch = 0; ch < 8; ++ch)
        *reinterpret_cast<uint4*>(rowp + ((ch ^ (row & 7)) << 4)) =
            make_uint4(w[4 * ch], w[4 * ch + 1], w[4 * ch + 2], w[4 * ch + 3]);
      fence_proxy_async_smem();
      named_bar_sync(1, 128);
      if (leader) {
        if (reduce)
          tma_reduce_add_2d(map, epi + buf * GT_EPI_BYTES, n0, m0);
        else
          tma_store_2d(map, epi + buf * GT_EPI_BYTES, n0, m0);
        bulk_commit();
      }
      buf ^= 1;
    };
    auto pack = [&](const float (&v)[64], uint32_t (&w)[32]) {
      if (p.c_bf16) {
#pragma unroll
        for (int i = 0; i < 32; ++i) w[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) w[i] = __float_as_uint(v[i]);
      }
    };
    int local = 0;
    for (int unit = blockIdx.x; unit < p.units; unit += gridDim.x, ++local) {
      int tm, tn, kb0, kb1;
      unit_coords(p, unit, tm, tn, kb0, kb1);
      const int acc = local & 1;
      const uint32_t acc_ph = (local >> 1) & 1;
      const bool ok = __all_sync(0xffffffffu, mbar_wait(&tfull[acc], acc_ph, p.err, 104));
      if (!ok) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + acc * GT_BN;
      const bool add_bias = p.bias && kb0 == 0;
      if (add_bias) {  // the tile's 256 bias values, read once into shared memory
        // (every thread has passed the previous tile's last read of s_bias: it precedes that
        // chunk's first barrier)
#pragma unroll
        for (int i = 0; i < GT_BN / 128; ++i) {
          const int n = tn * GT_BN + row + 128 * i;
          s_bias[row + 128 * i] = n < p.N ? __ldg(p.bias + n) : 0.f;
        }
        named_bar_sync(1, 128);
      }
#pragma unroll 1
      for (int c0 = 0; c0 < GT_BN; c0 += cols) {
        const int n0 = tn * GT_BN + c0;
        const int64_t m = (int64_t)tm * GT_BM + row;
        float a[64];
        if (p.act == ACT_GELU_BWD && n0 < p.N && m < p.M) load_aux_row(p, m, n0, cols, a);  // in flight
        uint32_t r[64];
        tmem_ld32(taddr + c0, *reinterpret_cast<uint32_t(*)[32]>(r));
        if (p.c_bf16) tmem_ld32(taddr + c0 + 32, *reinterpret_cast<uint32_t(*)[32]>(r + 32));
        tmem_wait_ld();
        if (c0 + cols >= GT_BN) {  // accumulator fully read: hand it back to the MMA thread
          tc_fence_before();
          mbar_arrive(&tempty[acc]);
        }
        if (n0 >= p.N) continue;  // uniform across the CTA
        float v[64];
#pragma unroll
        for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
        if (add_bias) {  // broadcast reads; columns past N hold 0
          const float4* b4 = reinterpret_cast<const float4*>(s_bias + c0);
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            if (4 * i < cols) {
              const float4 bb = b4[i];
              v[4 * i] += bb.x;
              v[4 * i + 1] += bb.y;
              v[4 * i + 2] += bb.z;
              v[4 * i + 3] += bb.w;
            }
          }
        }
        uint32_t w[32];
        if (p.act == ACT_GELU) {
          if (p.aux) {  // the pre-activation, for the backward
            pack(v, w);
            emit(&tmAux, w, n0, tm * GT_BM, false);
          }
#pragma unroll
          for (int i = 0; i < 64; ++i)
            if (i < cols) v[i] = gelu_fwd<true>(v[i]);
        } else if (p.act == ACT_GELU_BWD) {
          if (m < p.M) {
#pragma unroll
            for (int i = 0; i < 64; ++i)
              if (i < cols) v[i] *= gelu_grad<true>(a[i]);
          }
        }
        pack(v, w);
        emit(&tmC, w, n0, tm * GT_BM, p.reduce != 0);
      }
    }
    if (leader) bulk_wait0();
  } else {
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int row = q * 32 + lane;
    int local = 0;
    for (int unit = blockIdx.x; unit < p.units; unit += gridDim.x, ++local) {
      int tm, tn, kb0, kb1;
      unit_coords(p, unit, tm, tn, kb0, kb1);
      const int acc = local & 1;
      const uint32_t acc_ph = (local >> 1) & 1;
      const bool ok = __all_sync(0xffffffffu, mbar_wait(&tfull[acc], acc_ph, p.err, 104));
      if (!ok) break;
      tc_fence_after();
      const int m = tm * GT_BM + row;
      const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + acc * GT_BN;
#pragma unroll 1
      for (int c0 = 0; c0 < GT_BN; c0 += 32) {
        uint32_t r[32];
        tmem_ld32(taddr + c0, r);
        tmem_wait_ld();
        const int n0 = tn * GT_BN + c0;
        if (m < p.M && n0 < p.N) epilogue_store32(p, m, n0, r, kb0 == 0);
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, GT_TMEM_COLS);
  }
}

// ------------------------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------------------------
static int g_sms = 0;

static int num_sms() {
  if (g_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_sms, cudaDevAttrMultiProcessorCount, dev);
    if (g_sms <= 0) g_sms = 148;
  }
  return g_sms;
}

bool tc_gemm_supported(int M, int N, int K, int64_t lda, int a_trans, int64_t ldb, int b_trans,
                       const void* A, const void* B) {
  (void)a_trans;
  (void)b_trans;
  return aligned(A, 16) && aligned(B, 16) && lda % 8 == 0 && ldb % 8 == 0 && K >= 16 &&
         (int64_t)M * N * K >= (int64_t)1 << 21;
}

// Pick the number of K splits so that the work units fill the SMs in near-whole waves.
static int choose_splits(int tiles, int kb_total, int sms) {
  if (tiles >= sms || kb_total < 16) return 1;
  int best = 1;
  double best_eff = (double)tiles / (double)(((tiles + sms - 1) / sms) * sms);
  for (int s = 2; s <= 64 && kb_total / s >= 4; ++s) {
    const int units = tiles * s;
    const double eff = (double)units / (double)(((units + sms - 1) / sms) * sms);
    if (eff > best_eff + 0.02) {
      best = s;
      best_eff = eff;
    }
    if (best_eff > 0.95) break;
  }
  return best;
}

// Whether the epilogue can apply `act` here: it needs the TMA epilogue (16-byte aligned C and row
// pitch), an aux output of C's dtype for ACT_GELU, and 16-byte aligned aux rows for vector reads.
bool tc_gemm_act_ok(const void* C, int64_t ldc, int c_dtype, int act, const void* aux, int64_t ldaux,
                    int aux_dtype) {
  const int64_t cq = c_dtype == ATTN_BF16 ? 8 : 4, aq = aux_dtype == ATTN_BF16 ? 8 : 4;
  if (act == ACT_NONE) return true;
  if (!aligned(C, 16) || ldc % cq != 0) return false;
  if (!aux) return act == ACT_GELU;
  if (act == ACT_GELU && aux_dtype != c_dtype) return false;
  return aligned(aux, 16) && ldaux % aq == 0;
}

int gemm_tc(const void* A, int64_t lda, int a_trans, const void* B, int64_t ldb, int b_trans, void* C,
            int64_t ldc, int c_dtype, const float* bias, int M, int N, int K, int accumulate,
            cudaStream_t s, int act, const void* aux, int64_t ldaux, int aux_dtype) {
  if (act != ACT_NONE && (accumulate || !tc_gemm_act_ok(C, ldc, c_dtype, act, aux, ldaux, aux_dtype))) {
    set_error("gemm_tc: activation epilogue unsupported for this output layout");
    return ATTN_ERR_UNSUPPORTED;
  }
  CUtensorMap tmA, tmB;
  {
    uint64_t dims[2], strides[1];
    uint32_t box[2];
    if (!a_trans) {  // A stored [M][lda], K contiguous
      dims[0] = K; dims[1] = M; box[0] = 64; box[1] = GT_BM;
    } else {         // A stored [K][lda], M contiguous
      dims[0] = M; dims[1] = K; box[0] = 64; box[1] = 64;
    }
    strides[0] = (uint64_t)lda * 2;
    if (!make_tmap_bf16(&tmA, A, 2, dims, strides, box)) return ATTN_ERR_CUDA;
  }
  {
    uint64_t dims[2], strides[1];
    uint32_t box[2];
    if (b_trans) {   // B stored [N][ldb], K contiguous
      dims[0] = K; dims[1] = N; box[0] = 64; box[1] = GT_BN;
    } else {         // B stored [K][ldb], N contiguous
      dims[0] = N; dims[1] = K; box[0] = 64; box[1] = 64;
    }
    strides[0] = (uint64_t)ldb * 2;
    if (!make_tmap_bf16(&tmB, B, 2, dims, strides, box)) return ATTN_ERR_CUDA;
  }
  GemmParams p{};
  p.M = M; p.N = N; p.K = K;
  p.a_mn = a_trans ? 1 : 0;
  p.b_mn = b_trans ? 0 : 1;
  p.tiles_m = (M + GT_BM - 1) / GT_BM;
  p.tiles_n = (N + GT_BN - 1) / GT_BN;
  p.kb_total = (K + GT_BK - 1) / GT_BK;
  const int sms = num_sms();
  const int tiles = p.tiles_m * p.tiles_n;
  int splits = c_dtype == ATTN_F32 && act == ACT_NONE ? choose_splits(tiles, p.kb_total, sms) : 1;
  p.kb_per_split = (p.kb_total + splits - 1) / splits;
  splits = (p.kb_total + p.kb_per_split - 1) / p.kb_per_split;  // no empty split
  p.units = tiles * splits;
  p.C = C;
  p.ldc = ldc;
  p.c_bf16 = c_dtype == ATTN_BF16;
  p.accumulate = accumulate;
  p.atomic = splits > 1;
  p.bias = bias;
  p.act = act;
  p.aux = aux;
  p.ldaux = ldaux;
  p.aux_bf16 = aux_dtype == ATTN_BF16;
  p.vec_ok = aligned(C, 16) && (ldc % (p.c_bf16 ? 8 : 4) == 0);
  p.err = dev_error_ptr();
  if (!p.err) return ATTN_ERR_CUDA;
  // TMA epilogue whenever C is 16-byte aligned with 16-byte row pitch
  CUtensorMap tmC, tmAux;
  memset(&tmC, 0, sizeof(tmC));
  memset(&tmAux, 0, sizeof(tmAux));
  p.tma_epi = p.vec_ok ? 1 : 0;
  p.reduce = (accumulate || p.atomic) ? 1 : 0;
  if (p.tma_epi) {
    const uint64_t dims[2] = {(uint64_t)N, (uint64_t)M};
    const uint64_t strides[1] = {(uint64_t)ldc * (p.c_bf16 ? 2 : 4)};
    const uint32_t box[2] = {(uint32_t)(p.c_bf16 ? 64 : 32), (uint32_t)GT_BM};
    const bool ok = p.c_bf16 ? make_tmap_bf16(&tmC, C, 2, dims, strides, box)
                             : make_tmap_f32(&tmC, C, 2, dims, strides, box);
    if (!ok) return ATTN_ERR_CUDA;
    if (act == ACT_GELU && aux) {  // the pre-activation output, same geometry as C
      const uint64_t astr[1] = {(uint64_t)ldaux * (p.c_bf16 ? 2 : 4)};
      const bool ok2 = p.c_bf16 ? make_tmap_bf16(&tmAux, aux, 2, dims, astr, box)
                                : make_tmap_f32(&tmAux, aux, 2, dims, astr, box);
      if (!ok2) return ATTN_ERR_CUDA;
    }
  }
  if (p.atomic && !accumulate)
    ATTN_CUDA_TRY(cudaMemset2DAsync(C, (size_t)ldc * 4, 0, (size_t)N * 4, (size_t)M, s));
  static bool attr_set = false;
  if (!attr_set) {
    ATTN_CUDA_TRY(cudaFuncSetAttribute(gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, GT_SMEM));
    attr_set = true;
  }
  const int grid = p.units < sms ? p.units : sms;
  gemm_tc_kernel<<<grid, GT_THREADS, GT_SMEM, s>>>(tmA, tmB, tmC, tmAux, p);
  count_launch();
  return check_launch("gemm_tc_kernel");
}

}  // namespace attn
