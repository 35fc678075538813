// tcgen05 tensor-core GEMM for the attention projections: bf16 operands (kind::f16) or float32
// operands read as tf32 (kind::tf32), fp32 accumulation.
//
// C[M,N] (=|+=) op(A)[M,K] . op(B)[K,N] (+ bias[N]), C float32 or bf16.  Serves the QKV and
// output projections of MultiHeadAttention.forward (model/gpt.py:558, :629; matmul_2d_kernel,
// core/kernels.py:119-140) and the projection gradients of its backward (model/gpt.py:666-689).
//
// Persistent, warp-specialised kernel, one CTA per SM:
//   warp 0      TMA producer: 128-row A and 256-row B tiles, 128 bytes of K per row (64 bf16 or
//               32 tf32 elements; 128-byte swizzle), into a 4-stage ring
//   warp 1      TMEM allocation and the single MMA-issuing thread: 4 x tcgen05.mma (128x256x16
//               bf16 or 128x256x8 tf32) per K block, accumulating in TMEM
//   warps 2..   epilogue, groups of four warps (one warp per TMEM lane quarter in each), each group
//               owning a column span of the tile: tcgen05.ld of the fp32 accumulator (one row per
//               thread), bias, activation, conversion, then column chunks staged in swizzled shared
//               memory (two buffers per group) and written by TMA stores (or TMA reduce-adds when
//               accumulating into C).  Two shapes, a template parameter: four epilogue warps with
//               128-byte chunk rows (the default), or eight warps in two groups of 128 columns with
//               64-byte chunk rows, which doubles the epilogue's issue slots and memory parallelism
//               for ACT_GELU_BWD (its epilogue reads a second operand).
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
#include "attn_tc_common.cuh"

#include <stdlib.h>
#include <string.h>

namespace attn {

constexpr int GT_BM = 128, GT_BN = 256, GT_STAGES = 4;
constexpr int GT_A_BYTES = GT_BM * 128;  // 16 KB: 128 rows x 128 bytes of K (64 bf16 / 32 tf32)
constexpr int GT_B_BYTES = GT_BN * 128;  // 32 KB
constexpr int GT_STAGE_BYTES = GT_A_BYTES + GT_B_BYTES;

// Operand ring of one CTA.  Alone, a CTA loads a 128-row A tile and a 256-row B tile per K block
// into four 48 KB stages.  In a CTA pair (PAIR: one 256x256 tile per pair, tcgen05.mma.cta_group::2
// issued by the pair's first CTA), each CTA loads its 128 rows of A and its 128 of the tile's 256
// B columns, 32 KB per K block, into six stages of the same 192 KB: a third fewer operand bytes
// per SM per K block for the same tensor work.
template <bool PAIR>
struct Ring {
  static constexpr int b_rows = PAIR ? GT_BN / 2 : GT_BN;  // B rows (tile columns) this CTA loads
  static constexpr int stage_bytes = GT_A_BYTES + b_rows * 128;
  static constexpr int stages = PAIR ? 6 : 4;
  static constexpr int m_tile = PAIR ? 2 * GT_BM : GT_BM;  // rows of one work unit
};
static_assert(Ring<true>::stages * Ring<true>::stage_bytes == GT_STAGES * GT_STAGE_BYTES &&
                  Ring<false>::stages * Ring<false>::stage_bytes == GT_STAGES * GT_STAGE_BYTES,
              "both rings fill the same shared memory");
constexpr int GT_EPI_STAGING = 32 * 1024;      // output staging: two buffers per epilogue group
// No alignment pad: the kernel checks that its dynamic shared memory starts 1024-byte aligned (the
// 128-byte swizzle needs it; error site 106 otherwise), which leaves room on the SM for a small
// CTA beside it (the gradient all-reduce that overlaps the dX GEMM).
constexpr int GT_SMEM = GT_STAGES * GT_STAGE_BYTES + GT_EPI_STAGING + GT_BN * 4 /*bias*/ + 256;
constexpr int GT_SITE_SMEM_ALIGN = 106;

// Epilogue shape for EW epilogue warps (4 or 8).
template <int EW>
struct Epi {
  static constexpr int threads = 32 * EW;             // epilogue threads
  static constexpr int kthreads = 64 + threads;       // whole CTA
  static constexpr int groups = EW / 4;
  static constexpr int span = GT_BN / groups;         // tile columns per group
  static constexpr int row_bytes = EW == 8 ? 64 : 128;  // one chunk row: 16/32 fp32 or 32/64 bf16 columns
  static constexpr int vecs = row_bytes / 16;         // 16-byte pieces per chunk row
  static constexpr int words = row_bytes / 4;         // 32-bit words per chunk row
  static constexpr int buf_bytes = GT_BM * row_bytes;
  static_assert(groups * 2 * buf_bytes == GT_EPI_STAGING, "staging layout");
};
constexpr uint32_t GT_TMEM_COLS = 512;
static_assert(GT_SMEM <= 227 * 1024, "GEMM shared memory exceeds the per-CTA limit");

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

// The aux operand of ACT_GELU_BWD (C's dtype) for one accumulator row and one 64-byte output chunk
// starting at column n0, as raw words (columns past N read as 0; rows past M are not read).  The
// thread reads its own row: one 64-byte piece of a line, issued a chunk ahead of its use.
template <int V>
__device__ __forceinline__ void fetch_aux_chunk(const GemmParams& p, int64_t m, int n0, uint4 (&dst)[V]) {
  constexpr int W = 4 * V;  // words per chunk row
  const int cols = p.c_bf16 ? 2 * W : W;
  if (m >= p.M || n0 >= p.N) return;
  const int esz = p.c_bf16 ? 2 : 4;
  const uint8_t* src = reinterpret_cast<const uint8_t*>(p.aux) + (m * p.ldaux + n0) * esz;
  if (n0 + cols <= p.N) {
#pragma unroll
    for (int j = 0; j < V; ++j) dst[j] = __ldg(reinterpret_cast<const uint4*>(src) + j);
    return;
  }
  uint32_t t[W];
  if (p.c_bf16) {
    const unsigned short* s16 = reinterpret_cast<const unsigned short*>(src);
#pragma unroll
    for (int i = 0; i < W; ++i) {
      const uint32_t lo = n0 + 2 * i < p.N ? s16[2 * i] : 0u;
      const uint32_t hi = n0 + 2 * i + 1 < p.N ? s16[2 * i + 1] : 0u;
      t[i] = lo | (hi << 16);
    }
  } else {
    const uint32_t* s32 = reinterpret_cast<const uint32_t*>(src);
#pragma unroll
    for (int i = 0; i < W; ++i) t[i] = n0 + i < p.N ? s32[i] : 0u;
  }
#pragma unroll
  for (int j = 0; j < V; ++j) dst[j] = make_uint4(t[4 * j], t[4 * j + 1], t[4 * j + 2], t[4 * j + 3]);
}

// Word w of a raw aux chunk (w a compile-time index after unrolling).
template <int V>
__device__ __forceinline__ uint32_t aux_word(const uint4 (&raw)[V], int w) {
  const uint4 q = raw[w >> 2];
  return (w & 3) == 0 ? q.x : (w & 3) == 1 ? q.y : (w & 3) == 2 ? q.z : q.w;
}

__device__ __forceinline__ void unit_coords(const GemmParams& p, int unit, int& tm, int& tn, int& kb0,
                                            int& kb1) {
  tn = unit % p.tiles_n;
  tm = (unit / p.tiles_n) % p.tiles_m;
  const int split = unit / (p.tiles_n * p.tiles_m);
  kb0 = split * p.kb_per_split;
  kb1 = min(p.kb_total, kb0 + p.kb_per_split);
}

// Direct per-row stores of one chunk (C without a 16-byte row pitch): cols values of row m from
// column n0, bias already added; fp32 atomics for K splits, read-add-write when accumulating.
template <int NV>
__device__ __forceinline__ void store_chunk_direct(const GemmParams& p, int64_t m, int n0, const float (&v)[NV],
                                                   int cols) {
  if (p.c_bf16) {
    __nv_bfloat16* c = reinterpret_cast<__nv_bfloat16*>(p.C) + m * p.ldc + n0;
#pragma unroll
    for (int i = 0; i < NV; ++i)
      if (i < cols && n0 + i < p.N) c[i] = __float2bfloat16_rn(v[i]);
    return;
  }
  float* c = reinterpret_cast<float*>(p.C) + m * p.ldc + n0;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    if (i < cols && n0 + i < p.N) {
      if (p.atomic)
        atomicAdd(c + i, v[i]);
      else
        c[i] = p.accumulate ? c[i] + v[i] : v[i];
    }
  }
}

template <int EW, bool TF32, bool PAIR>
__global__ void __launch_bounds__(Epi<EW>::kthreads, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmAux,
               const GemmParams p) {
  static_assert(!(PAIR && TF32), "CTA pairs run bf16 operands");
  using R = Ring<PAIR>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const WaitErr werr = wait_err(p.err);
  // uniform over the CTA and over both CTAs of a pair (the same kernel and layout), so every thread
  // of a pair leaves before any set-up or pair barrier
  if (smem_u32(smem_raw) & 1023u) {
    if (threadIdx.x == 0) record_wait_error(werr, GT_SITE_SMEM_ALIGN);
    return;
  }
  // work units: one per CTA, or one per pair (cluster of two CTAs, rank crank)
  const uint32_t crank = PAIR ? cluster_ctarank() : 0u;
  const int ufirst = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int ustep = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  const int row0 = PAIR ? (int)crank * GT_BM : 0;  // this CTA's first row of a unit's tile
  uint8_t* smem = smem_raw;
  using E = Epi<EW>;
  // A K block is 128 bytes of K per row: 64 bf16 or 32 tf32 elements.  MN-major operands arrive as
  // boxes MNW elements (128 bytes) wide and one K block deep; one MMA-K step spans 16 bf16 / 8 tf32
  // K rows of such a box.
  constexpr int BKE = TF32 ? 32 : 64;
  constexpr int MNW = TF32 ? 32 : 64;
  constexpr uint32_t MN_BOX = 128u * BKE;        // bytes of one MN-major box
  constexpr uint32_t MN_KSTEP = 128u * (BKE / 4); // bytes per MMA-K step in an MN-major box
  // MN-major operands: bf16 in the 128-byte swizzle (8-row atoms), tf32 in the 128-byte swizzle with
  // 32-byte atomicity (4-row atoms), the only MN-major layout the tf32 MMA reads
  auto mn_desc = [&](uint32_t addr) {
    return TF32 ? smem_desc_sw128_atom32(addr, MN_BOX, 512) : smem_desc_sw128(addr, MN_BOX, 1024);
  };
  uint8_t* epi = smem + GT_STAGES * GT_STAGE_BYTES;  // output staging buffers, two per epilogue group
  float* s_bias = reinterpret_cast<float*>(epi + GT_EPI_STAGING);  // the tile's bias columns
  uint64_t* full = reinterpret_cast<uint64_t*>(s_bias + GT_BN);
  uint64_t* empty = full + R::stages;
  uint64_t* tfull = empty + R::stages;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    for (int s = 0; s < R::stages; ++s) {
      mbar_init(&full[s], 1);   // pair: used in the first CTA, which counts both CTAs' bytes
      mbar_init(&empty[s], 1);  // pair: one commit arrival in each CTA
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      // pair: one arrival per epilogue warp of both CTAs, in the first CTA
      mbar_init(&tempty[a], PAIR ? 2 * EW : E::threads);
    }
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_slot, GT_TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, GT_TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) pair_sync();  // both CTAs' barriers exist before either CTA signals the other's
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  grid_dependency_wait();    // the operands (and an accumulated C) are complete
  grid_dependents_launch();  // the next kernel's CTAs may take SMs as this grid's CTAs leave

  if (warp == 0) {
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      // a tile load into this CTA's stage s, counted on full[s] (pair: the first CTA's full[s])
      auto load = [&](void* dst, const CUtensorMap* map, int s_, int c0, int c1) {
        if constexpr (PAIR)
          tma_load_2d_pair(dst, map, cluster_addr(&full[s_], 0), c0, c1);
        else
          tma_load_2d(dst, map, &full[s_], c0, c1);
      };
      for (int unit = ufirst; unit < p.units && ok; unit += ustep) {
        int tm, tn, kb0, kb1;
        unit_coords(p, unit, tm, tn, kb0, kb1);
        const int ar = tm * R::m_tile + row0;               // this CTA's A rows
        const int bn = tn * GT_BN + (int)crank * R::b_rows;  // this CTA's B rows (tile columns)
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1, werr, 101)) { ok = false; break; }
          uint8_t* sa = smem + s * R::stage_bytes;
          uint8_t* sb = sa + GT_A_BYTES;
          if (!PAIR || crank == 0) mbar_arrive_expect_tx(&full[s], (PAIR ? 2 : 1) * R::stage_bytes);
          const int k0 = kb * BKE;
          if (!p.a_mn) {
            load(sa, &tmA, s, k0, ar);
          } else {
#pragma unroll
            for (int j = 0; j < GT_BM / MNW; ++j) load(sa + j * MN_BOX, &tmA, s, ar + MNW * j, k0);
          }
          if (!p.b_mn) {
            load(sb, &tmB, s, k0, bn);
          } else {
#pragma unroll
            for (int j = 0; j < R::b_rows / MNW; ++j) load(sb + j * MN_BOX, &tmB, s, bn + MNW * j, k0);
          }
          if (++s == R::stages) { s = 0; ph ^= 1; }
        }
      }
      // tail: wait until the MMA thread has released every stage, so no asynchronous arrive is
      // still in flight to this CTA's shared memory when it exits
      for (int i = 0; i < R::stages && ok; ++i) {
        ok = mbar_wait(&empty[s], ph ^ 1, werr, 105);
        if (++s == R::stages) { s = 0; ph ^= 1; }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && crank == 0) {  // pair: the first CTA issues the pair's MMAs
      const uint32_t idesc = TF32 ? idesc_tf32_f32(GT_BM, GT_BN, p.a_mn, p.b_mn)
                                  : idesc_bf16_f32(R::m_tile, GT_BN, p.a_mn, p.b_mn);
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      int local = 0;
      for (int unit = ufirst; unit < p.units && ok; unit += ustep, ++local) {
        int tm, tn, kb0, kb1;
        unit_coords(p, unit, tm, tn, kb0, kb1);
        const int acc = local & 1;
        const uint32_t acc_ph = (local >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_ph ^ 1, werr, 102)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * GT_BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[s], ph, werr, 103)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * R::stage_bytes);
          const uint32_t sb = sa + GT_A_BYTES;
#pragma unroll
          for (int k = 0; k < 4; ++k) {  // four MMA-K steps of 32 bytes per 128-byte K block
            const uint64_t ad = p.a_mn ? mn_desc(sa + k * MN_KSTEP) : smem_desc_sw128(sa + k * 32, 16, 1024);
            const uint64_t bd = p.b_mn ? mn_desc(sb + k * MN_KSTEP) : smem_desc_sw128(sb + k * 32, 16, 1024);
            if constexpr (TF32)
              umma_ss_tf32(d_tmem, ad, bd, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
            else if constexpr (PAIR)
              umma_ss_pair(d_tmem, ad, bd, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
            else
              umma_ss(d_tmem, ad, bd, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          // frees the stage (in both CTAs of a pair) once these MMAs have read it
          if constexpr (PAIR) umma_commit_pair(&empty[s]); else umma_commit(&empty[s]);
          if (++s == R::stages) { s = 0; ph ^= 1; }
        }
        if (ok) {  // accumulator ready for the epilogue (of both CTAs of a pair)
          if constexpr (PAIR) umma_commit_pair(&tfull[acc]); else umma_commit(&tfull[acc]);
        }
      }
    }
  } else {
    // Epilogue: each thread owns one accumulator row of its group's column span.  A chunk of
    // E::row_bytes per row goes to a swizzled staging buffer (conflict-free 16-byte stores; the
    // 128B or 64B swizzle of C's tensor map) and the group's leader writes the 128-row chunk with
    // a TMA store, or a TMA reduce-add when accumulating or splitting K.  Each group alternates two
    // staging buffers and synchronises on its own named barrier.  Without a 16-byte row pitch (no
    // TMA map for C) the threads store their rows directly instead.
    constexpr int V = E::vecs, W = E::words;
    const int ew = warp - 2;
    const int h = ew >> 2;                 // the group: tile columns h * E::span ..
    const int q = warp & 3;                // TMEM lane quarter this warp may access
    const int row = q * 32 + lane;
    const int bar = 1 + h;
    const bool leader = (ew & 3) == 0 && lane == 0;
    const int cols = p.c_bf16 ? 2 * W : W;  // columns per chunk
    const int nchunks = E::span / cols;
    const bool bwd = p.act == ACT_GELU_BWD;
    const int sw = E::row_bytes == 128 ? (row & 7) : ((row >> 1) & 3);  // swizzle of this row's pieces
    uint8_t* gepi = epi + 2 * h * E::buf_bytes;
    float* gbias = s_bias + h * E::span;
    int buf = 0;
    auto emit = [&](const CUtensorMap* map, const uint32_t (&w)[W], int n0, int m0, bool reduce) {
      if (leader) bulk_wait_read1();  // the store that last used this buffer has read it
      named_bar_sync(bar, 128);
      uint8_t* rowp = gepi + buf * E::buf_bytes + row * E::row_bytes;
#pragma unroll
      for (int j = 0; j < V; ++j)
        *reinterpret_cast<uint4*>(rowp + ((j ^ sw) << 4)) = make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
      fence_proxy_async_smem();
      named_bar_sync(bar, 128);
      if (leader) {
        if (reduce)
          tma_reduce_add_2d(map, gepi + buf * E::buf_bytes, n0, m0);
        else
          tma_store_2d(map, gepi + buf * E::buf_bytes, n0, m0);
        bulk_commit();
      }
      buf ^= 1;
    };
    auto pack = [&](const float (&v)[2 * W], uint32_t (&w)[W]) {
      if (p.c_bf16) {
#pragma unroll
        for (int i = 0; i < W; ++i) w[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
      } else {
#pragma unroll
        for (int i = 0; i < W; ++i) w[i] = __float_as_uint(v[i]);
      }
    };
    uint4 pf[V] = {};  // ACT_GELU_BWD: the aux chunk of the next (tile, chunk), fetched a chunk ahead
    if (bwd && ufirst < p.units) {
      int tm, tn, kb0, kb1;
      unit_coords(p, ufirst, tm, tn, kb0, kb1);
      fetch_aux_chunk<V>(p, (int64_t)tm * R::m_tile + row0 + row, tn * GT_BN + h * E::span, pf);
    }
    int local = 0;
    for (int unit = ufirst; unit < p.units; unit += ustep, ++local) {
      int tm, tn, kb0, kb1;
      unit_coords(p, unit, tm, tn, kb0, kb1);
      const int acc = local & 1;
      const uint32_t acc_ph = (local >> 1) & 1;
      const bool ok = __all_sync(0xffffffffu, mbar_wait(&tfull[acc], acc_ph, werr, 104));
      if (!ok) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + acc * GT_BN + h * E::span;
      const int m0 = tm * R::m_tile + row0;  // this CTA's first output row of the tile
      const int64_t m = (int64_t)m0 + row;
      const bool add_bias = p.bias && kb0 == 0;
      if (add_bias) {  // the group's bias values, read once into shared memory (every thread of the
        // group has passed the barriers that follow its last read of the previous tile's)
#pragma unroll
        for (int i = 0; i < E::span / 128; ++i) {
          const int n = tn * GT_BN + h * E::span + row + 128 * i;
          gbias[row + 128 * i] = n < p.N ? __ldg(p.bias + n) : 0.f;
        }
        named_bar_sync(bar, 128);
      }
#pragma unroll 1
      for (int c = 0; c < nchunks; ++c) {
        const int n0 = tn * GT_BN + h * E::span + c * cols;
        uint4 cur[V];
        if (bwd) {
#pragma unroll
          for (int j = 0; j < V; ++j) cur[j] = pf[j];
          if (c + 1 < nchunks) {
            fetch_aux_chunk<V>(p, m, n0 + cols, pf);
          } else if (unit + ustep < p.units) {
            int tm2, tn2, k0, k1;
            unit_coords(p, unit + ustep, tm2, tn2, k0, k1);
            fetch_aux_chunk<V>(p, (int64_t)tm2 * R::m_tile + row0 + row, tn2 * GT_BN + h * E::span, pf);
          }
        }
        uint32_t r[2 * W];
        if (n0 < p.N) {  // uniform across the group
          const uint32_t ta = taddr + c * cols;
          if constexpr (W == 32) {
            tmem_ld32(ta, *reinterpret_cast<uint32_t(*)[32]>(r));
            if (p.c_bf16) tmem_ld32(ta + 32, *reinterpret_cast<uint32_t(*)[32]>(r + 32));
          } else {
            if (p.c_bf16)
              tmem_ld32(ta, *reinterpret_cast<uint32_t(*)[32]>(r));
            else
              tmem_ld16(ta, *reinterpret_cast<uint32_t(*)[16]>(r));
          }
          tmem_wait_ld();
        }
        if (c + 1 == nchunks) {  // accumulator fully read: hand it back to the MMA thread
          tc_fence_before();
          if constexpr (PAIR) {  // one arrival per warp, on the first CTA's barrier
            __syncwarp();
            if (lane == 0) mbar_arrive_remote(cluster_addr(&tempty[acc], 0));
          } else {
            mbar_arrive(&tempty[acc]);
          }
        }
        // columns past N; a pair's second CTA past the last row (M < its rows): nothing to write
        if (n0 >= p.N || m0 >= p.M) continue;
        float v[2 * W];
#pragma unroll
        for (int i = 0; i < 2 * W; ++i) v[i] = __uint_as_float(r[i]);
        if (add_bias) {  // broadcast reads; columns past N hold 0
          const float4* b4 = reinterpret_cast<const float4*>(gbias + c * cols);
#pragma unroll
          for (int i = 0; i < 2 * W / 4; ++i) {
            if (4 * i < cols) {
              const float4 bb = b4[i];
              v[4 * i] += bb.x;
              v[4 * i + 1] += bb.y;
              v[4 * i + 2] += bb.z;
              v[4 * i + 3] += bb.w;
            }
          }
        }
        if (!p.tma_epi) {  // activations always take the TMA path (host-checked)
          if (m < p.M) store_chunk_direct(p, m, n0, v, cols);
          continue;
        }
        uint32_t w[W];
        if (p.act == ACT_GELU) {
          if (p.aux) {  // the pre-activation, for the backward
            pack(v, w);
            emit(&tmAux, w, n0, m0, false);
          }
#pragma unroll
          for (int i = 0; i < 2 * W; ++i)
            if (i < cols) v[i] = gelu_fwd<true>(v[i]);
        } else if (bwd) {
          if (p.c_bf16) {
#pragma unroll
            for (int i = 0; i < 2 * W; ++i) {
              const uint32_t u = aux_word(cur, i >> 1);
              v[i] *= gelu_grad<true>(__uint_as_float((i & 1) ? (u & 0xffff0000u) : (u << 16)));
            }
          } else {
#pragma unroll
            for (int i = 0; i < W; ++i) v[i] *= gelu_grad<true>(__uint_as_float(aux_word(cur, i)));
          }
        }
        pack(v, w);
        emit(&tmC, w, n0, m0, p.reduce != 0);
      }
    }
    if (leader) bulk_wait0();
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) pair_sync();  // the other CTA is done with this CTA's barriers and operands
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR) tmem_dealloc_pair(tmem_base, GT_TMEM_COLS); else tmem_dealloc(tmem_base, GT_TMEM_COLS);
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

// CTA pairs are used when the environment variable ATTN_GEMM_PAIRS is "1" at the library's first
// GEMM launch.  They are off by default.  Measured at cfg 5 on one B200, they cut the operand bytes
// each SM reads per K block by a third but did not make the step faster: 6.12-6.17 ms against
// 6.01-6.08. The QKV projection gained inside the step (0.77 vs 0.83 ms), the output projection and
// dWqkv lost, and the runs held lower SM clocks. These GEMMs run near the power-capped sustained
// tensor rate, not at an L2 limit.
static bool gemm_pairs_enabled() {
  static const bool on = [] {
    const char* v = getenv("ATTN_GEMM_PAIRS");
    return v && strcmp(v, "1") == 0;
  }();
  return on;
}

// Pairs that can be resident at once (clusters of two CTAs of 229 KB shared memory), at most
// sms / 2; 0 when the runtime cannot say, and the one-CTA kernel is used.
static int g_pairs = -1;
static int pair_capacity(int sms) {
  if (g_pairs < 0) {
    g_pairs = 0;
    auto k = gemm_tc_kernel<4, false, true>;
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, GT_SMEM) == cudaSuccess) {
      cudaLaunchAttribute a[1];
      a[0].id = cudaLaunchAttributeClusterDimension;
      a[0].val.clusterDim.x = 2;
      a[0].val.clusterDim.y = 1;
      a[0].val.clusterDim.z = 1;
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(2 * (num_sms() / 2));
      cfg.blockDim = dim3(Epi<4>::kthreads);
      cfg.dynamicSmemBytes = GT_SMEM;
      cfg.attrs = a;
      cfg.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, k, &cfg) == cudaSuccess) g_pairs = n;
    }
    cudaGetLastError();  // a refused query leaves no error behind for the next launch check
  }
  const int half = sms / 2;
  return g_pairs < half ? g_pairs : half;
}

bool tc_gemm_supported(int M, int N, int K, int64_t lda, int a_trans, int64_t ldb, int b_trans,
                       const void* A, const void* B, int tf32) {
  (void)a_trans;
  (void)b_trans;
  const int64_t q = tf32 ? 4 : 8;  // elements per 16 bytes
  return aligned(A, 16) && aligned(B, 16) && lda % q == 0 && ldb % q == 0 && K >= 16 &&
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
// pitch) and an aux operand of C's dtype with 16-byte aligned rows.
bool tc_gemm_act_ok(const void* C, int64_t ldc, int c_dtype, int act, const void* aux, int64_t ldaux,
                    int aux_dtype) {
  const int64_t cq = c_dtype == ATTN_BF16 ? 8 : 4, aq = aux_dtype == ATTN_BF16 ? 8 : 4;
  if (act == ACT_NONE) return true;
  if (!aligned(C, 16) || ldc % cq != 0) return false;
  if (!aux) return act == ACT_GELU;
  return aux_dtype == c_dtype && aligned(aux, 16) && ldaux % aq == 0;
}

int gemm_tc(const void* A, int64_t lda, int a_trans, const void* B, int64_t ldb, int b_trans, void* C,
            int64_t ldc, int c_dtype, const float* bias, int M, int N, int K, int accumulate,
            cudaStream_t s, int act, const void* aux, int64_t ldaux, int aux_dtype, int tf32, int max_ctas) {
  if (act != ACT_NONE && (accumulate || !tc_gemm_act_ok(C, ldc, c_dtype, act, aux, ldaux, aux_dtype))) {
    set_error("gemm_tc: activation epilogue unsupported for this output layout");
    return ATTN_ERR_UNSUPPORTED;
  }
  // persistent CTAs: one per SM, or max_ctas when the caller leaves SMs to a kernel on another stream
  const int sms = max_ctas > 0 && max_ctas < num_sms() ? max_ctas : num_sms();
  // CTA pairs (256x256 tiles, tcgen05.mma.cta_group::2) for bf16 operands with at least two 128-row
  // tiles; as many pairs as fit on the SMs at once
  const int pair_slots = tf32 || M < 2 * GT_BM || !gemm_pairs_enabled() ? 0 : pair_capacity(sms);
  const bool pair = pair_slots > 0;
  // operand boxes are 128 bytes wide: 64 bf16 or 32 tf32 elements (one K block, or one MN-major
  // block of a K block's rows)
  const uint32_t w = tf32 ? 32 : 64;
  const uint64_t esz = tf32 ? 4 : 2;
  auto make_op_map = [&](CUtensorMap* m, const void* base, const uint64_t* dims, const uint64_t* strides,
                         const uint32_t* box, bool mn_major) {
    return tf32 ? make_tmap_f32(m, base, 2, dims, strides, box, mn_major ? SWIZZLE_128B_ATOM32 : 128)
                : make_tmap_bf16(m, base, 2, dims, strides, box);
  };
  CUtensorMap tmA, tmB;
  {
    uint64_t dims[2], strides[1];
    uint32_t box[2];
    if (!a_trans) {  // A stored [M][lda], K contiguous
      dims[0] = K; dims[1] = M; box[0] = w; box[1] = GT_BM;
    } else {         // A stored [K][lda], M contiguous
      dims[0] = M; dims[1] = K; box[0] = w; box[1] = w;
    }
    strides[0] = (uint64_t)lda * esz;
    if (!make_op_map(&tmA, A, dims, strides, box, a_trans != 0)) return ATTN_ERR_CUDA;
  }
  {
    uint64_t dims[2], strides[1];
    uint32_t box[2];
    if (b_trans) {   // B stored [N][ldb], K contiguous; a pair's CTA loads half the tile's rows
      dims[0] = K; dims[1] = N; box[0] = w; box[1] = pair ? Ring<true>::b_rows : GT_BN;
    } else {         // B stored [K][ldb], N contiguous
      dims[0] = N; dims[1] = K; box[0] = w; box[1] = w;
    }
    strides[0] = (uint64_t)ldb * esz;
    if (!make_op_map(&tmB, B, dims, strides, box, b_trans == 0)) return ATTN_ERR_CUDA;
  }
  GemmParams p{};
  p.M = M; p.N = N; p.K = K;
  p.a_mn = a_trans ? 1 : 0;
  p.b_mn = b_trans ? 0 : 1;
  const int m_tile = pair ? Ring<true>::m_tile : GT_BM;
  p.tiles_m = (M + m_tile - 1) / m_tile;
  p.tiles_n = (N + GT_BN - 1) / GT_BN;
  p.kb_total = (K + (int)w - 1) / (int)w;
  const int slots = pair ? pair_slots : sms;  // concurrent work units
  const int tiles = p.tiles_m * p.tiles_n;
  int splits = c_dtype == ATTN_F32 && act == ACT_NONE ? choose_splits(tiles, p.kb_total, slots) : 1;
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
  // Eight epilogue warps with 64-byte chunk rows: for ACT_GELU_BWD (its aux reads), and for fp32
  // outputs with a short K, where the 128 KB fp32 tile's epilogue is long next to the main loop
  // (the output projection, M=262144 N=768 K=768: 0.354 -> 0.343 ms).
  const bool wide = act == ACT_GELU_BWD || (!p.c_bf16 && K <= 1024);
  const int row_bytes = wide ? Epi<8>::row_bytes : Epi<4>::row_bytes;
  if (p.tma_epi) {
    const uint64_t dims[2] = {(uint64_t)N, (uint64_t)M};
    const uint64_t strides[1] = {(uint64_t)ldc * (p.c_bf16 ? 2 : 4)};
    const uint32_t box[2] = {(uint32_t)(row_bytes / (p.c_bf16 ? 2 : 4)), (uint32_t)GT_BM};  // one chunk
    const bool ok = p.c_bf16 ? make_tmap_bf16(&tmC, C, 2, dims, strides, box, row_bytes)
                             : make_tmap_f32(&tmC, C, 2, dims, strides, box, row_bytes);
    if (!ok) return ATTN_ERR_CUDA;
    if (act == ACT_GELU && aux) {  // the pre-activation output, same geometry as C
      const uint64_t astr[1] = {(uint64_t)ldaux * (p.c_bf16 ? 2 : 4)};
      const bool ok2 = p.c_bf16 ? make_tmap_bf16(&tmAux, aux, 2, dims, astr, box, row_bytes)
                                : make_tmap_f32(&tmAux, aux, 2, dims, astr, box, row_bytes);
      if (!ok2) return ATTN_ERR_CUDA;
    }
  }
  if (p.atomic && !accumulate)
    ATTN_CUDA_TRY(cudaMemset2DAsync(C, (size_t)ldc * 4, 0, (size_t)N * 4, (size_t)M, s));
  static CtxOnce attr[6];
  const int units_run = p.units < slots ? p.units : slots;
  const int grid = pair ? 2 * units_run : units_run;
  cudaError_t launched = cudaSuccess;
#define GT_LAUNCH(EW, TF, PR, slot)                                                                    \
  do {                                                                                                 \
    if (!set_smem_limit_once(gemm_tc_kernel<EW, TF, PR>, GT_SMEM, attr[slot])) return ATTN_ERR_CUDA;   \
    if (PR)                                                                                            \
      launched = launch_pdl_pairs(gemm_tc_kernel<EW, TF, PR>, dim3(grid), dim3(Epi<EW>::kthreads), GT_SMEM, s, \
                                  tmA, tmB, tmC, tmAux, p);                                            \
    else                                                                                               \
      launched = launch_pdl(gemm_tc_kernel<EW, TF, PR>, dim3(grid), dim3(Epi<EW>::kthreads), GT_SMEM, s, tmA, \
                            tmB, tmC, tmAux, p);                                                       \
  } while (0)
  if (pair && wide)
    GT_LAUNCH(8, false, true, 5);
  else if (pair)
    GT_LAUNCH(4, false, true, 4);
  else if (wide && tf32)
    GT_LAUNCH(8, true, false, 3);
  else if (wide)
    GT_LAUNCH(8, false, false, 2);
  else if (tf32)
    GT_LAUNCH(4, true, false, 1);
  else
    GT_LAUNCH(4, false, false, 0);
#undef GT_LAUNCH
  count_launch();
  return check_launch("gemm_tc_kernel", launched);
}

}  // namespace attn
