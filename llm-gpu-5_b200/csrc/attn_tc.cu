// tcgen05 tensor-core causal attention for head_dim 64, bf16 operands, fp32 accumulation.
//
// Forward (replaces fused_attention_forward_kernel, core/mha_kernels.py:404-521): one CTA per
// (b, h, 128-row query tile), two CTAs per SM.  Per 128-key K/V block:
//   S = Q K^T           tcgen05.mma, A = Q and B = K from shared memory (TMA, 128B swizzle),
//                       fp32 accumulator in TMEM columns [0,128)
//   softmax             4 warps, one query row per thread (tcgen05.ld of its TMEM lane): causal
//                       mask on the diagonal block, row max, 2^(s*scale*log2e - m), row sum; P is
//                       packed to bf16 and written back over S in TMEM columns [0,64)
//   O += P V            tcgen05.mma with A = P read from TMEM, B = V (MN-major) from shared
//                       memory, fp32 accumulator in TMEM columns [128,192)
// The running max is only moved (and O rescaled in TMEM) when it grows by more than 2^8, so
// rescaling is rare.  The row's log-sum-exp is written instead of the T x T probabilities.
//
// Backward (replaces model/gpt.py:669-680 and core/mha_kernels.py:195-236, 592-680): a prep
// kernel computes delta = rowsum(dO * O) (model/gpt.py:675) and copies lse into a padded
// log2-domain array; then one CTA per (b, h, 128-key block) keeps K, V and the dK/dV accumulators
// resident and streams the query tiles that can see its keys:
//   S^T = K Q^T, dP^T = V dO^T            SS MMAs into TMEM
//   P^T = 2^(S^T*scale*log2e - lse2),  dS^T = P^T (dP^T - delta) * scale   (one key row per thread)
//   dV += P^T dO, dK += dS^T Q            MMAs with A = P^T / dS^T from TMEM
//   dQ_tile = dS K                        SS MMA with A = dS^T in shared memory (read MN-major)
// dQ tiles are added into an fp32 accumulator in the workspace with bulk reduce-adds
// (cp.reduce.async.bulk ... add.f32), then converted to bf16 by a last small kernel.
//
// Every mbarrier wait is bounded (tc_common.cuh): a wait that gives up sets the library's device
// error word and the kernel skips its remaining work instead of hanging.
#include "tc_common.cuh"

#include <math.h>

namespace attn {

constexpr int AT_TILE = 128;                     // query / key rows per tile
constexpr int AT_D = 64;                         // head_dim handled here
constexpr int AT_TILE_BYTES = AT_TILE * AT_D * 2;  // 16 KB bf16 tile, 128 B per row
constexpr float LOG2E = 1.4426950408889634f;
constexpr float LN2 = 0.6931471805599453f;

struct TileMap {
  CUtensorMap map;
  int h_first;  // 1: dims {D, NH, T, B}; 0: dims {D, T, NH, B}
};

__device__ __forceinline__ void load_tile(void* dst, const TileMap& tm, uint64_t* bar, int b, int h,
                                          int t0) {
  if (tm.h_first)
    tma_load_4d(dst, &tm.map, bar, 0, h, t0, b);
  else
    tma_load_4d(dst, &tm.map, bar, 0, t0, h, b);
}

// ==========================================================================================
// forward
// ==========================================================================================
constexpr int FA_THREADS = 192;  // warp 0 TMA, warp 1 MMA + TMEM, warps 2-5 softmax/epilogue
constexpr int FA_STAGES = 2;
constexpr uint32_t FA_TMEM_COLS = 256;  // S/P [0,128), O [128,192)
constexpr int FA_SMEM = AT_TILE_BYTES * (1 + 2 * FA_STAGES) + 1024 + 256;

struct FwdMaps {
  TileMap q, k, v;
};

struct FwdParams {
  int NH, T, nq;
  float scale_log2;
  __nv_bfloat16* o;
  int64_t o_sb, o_st, o_sh;
  float* lse;
  int* err;
};

__global__ void __launch_bounds__(FA_THREADS, 2)
attn_fwd_tc_kernel(const __grid_constant__ FwdMaps maps, const FwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = smem + AT_TILE_BYTES;                      // [FA_STAGES]
  uint8_t* sV = sK + FA_STAGES * AT_TILE_BYTES;            // [FA_STAGES]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + FA_STAGES * AT_TILE_BYTES);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* v_full = k_full + FA_STAGES;
  uint64_t* kv_empty = v_full + FA_STAGES;
  uint64_t* s_full = kv_empty + FA_STAGES;
  uint64_t* p_ready = s_full + 1;
  uint64_t* pv_done = p_ready + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(pv_done + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int bh = blockIdx.x / p.nq;
  const int qt = p.nq - 1 - (int)(blockIdx.x % p.nq);  // longest causal rows first within a head
  const int b = bh / p.NH, h = bh % p.NH;
  const int n_kv = qt + 1;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < FA_STAGES; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(p_ready, 128);
    mbar_init(pv_done, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, FA_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tP = tmem, tO = tmem + 128;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&maps.q.map);
      tma_prefetch_desc(&maps.k.map);
      tma_prefetch_desc(&maps.v.map);
      mbar_arrive_expect_tx(q_full, AT_TILE_BYTES);
      load_tile(sQ, maps.q, q_full, b, h, qt * AT_TILE);
      bool ok = true;
      for (int j = 0; j < n_kv && ok; ++j) {
        const int st = j % FA_STAGES;
        const uint32_t ph = (j / FA_STAGES) & 1;
        if (!mbar_wait(&kv_empty[st], ph ^ 1, p.err, 201)) { ok = false; break; }
        mbar_arrive_expect_tx(&k_full[st], AT_TILE_BYTES);
        load_tile(sK + st * AT_TILE_BYTES, maps.k, &k_full[st], b, h, j * AT_TILE);
        mbar_arrive_expect_tx(&v_full[st], AT_TILE_BYTES);
        load_tile(sV + st * AT_TILE_BYTES, maps.v, &v_full[st], b, h, j * AT_TILE);
      }
      // tail: every stage released by the MMA thread before the CTA may exit
      for (int j = n_kv; j < n_kv + FA_STAGES && ok; ++j)
        ok = mbar_wait(&kv_empty[j % FA_STAGES], ((j / FA_STAGES) & 1) ^ 1, p.err, 202);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc_s = idesc_bf16_f32(128, 128, 0, 0);  // Q K-major, K K-major
      const uint32_t idesc_o = idesc_bf16_f32(128, 64, 0, 1);   // P from TMEM, V MN-major
      bool ok = mbar_wait(q_full, 0, p.err, 203);
      const uint32_t q_addr = smem_u32(sQ);
      for (int j = 0; j < n_kv && ok; ++j) {
        const int st = j % FA_STAGES;
        const uint32_t ph = (j / FA_STAGES) & 1;
        if (!mbar_wait(&k_full[st], ph, p.err, 204)) break;
        if (j > 0 && !mbar_wait(pv_done, (j - 1) & 1, p.err, 205)) break;  // P_{j-1} consumed
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sK + st * AT_TILE_BYTES);
#pragma unroll
        for (int k = 0; k < AT_D / 16; ++k)
          umma_ss(tS, smem_desc_sw128(q_addr + k * 32, 16, 1024), smem_desc_sw128(k_addr + k * 32, 16, 1024),
                  idesc_s, k > 0 ? 1u : 0u);
        umma_commit(s_full);
        if (!mbar_wait(p_ready, j & 1, p.err, 206)) break;
        if (!mbar_wait(&v_full[st], ph, p.err, 207)) break;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(sV + st * AT_TILE_BYTES);
#pragma unroll
        for (int k = 0; k < AT_TILE / 16; ++k)
          umma_ts(tO, tP + k * 8, smem_desc_sw128(v_addr + k * 2048, 8192, 1024), idesc_o,
                  (j > 0 || k > 0) ? 1u : 0u);
        umma_commit(pv_done);
        umma_commit(&kv_empty[st]);
      }
    }
  } else {
    // ---------------- softmax warpgroup: one query row per thread ----------------
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int grow = qt * AT_TILE + row;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const float sl2 = p.scale_log2;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      ok = __all_sync(0xffffffffu, mbar_wait(s_full, j & 1, p.err, 208));
      if (!ok) break;
      tc_fence_after();
      const bool diag = (j == qt);
      // pass 1: row max of the scaled scores (log2 domain)
      float mx = -INFINITY;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        tmem_ld32(tS + lane_off + c * 32, r);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float s = __uint_as_float(r[i]);
          const bool masked = diag && (c * 32 + i > row);
          mx = masked ? mx : fmaxf(mx, s);
        }
      }
      const float m_cand = mx * sl2;
      // move the max (and rescale O) only when it grows by more than 8 in log2 units
      const bool grow_m = (j == 0) || (m_cand > m + 8.0f);
      if (j > 0 && __any_sync(0xffffffffu, grow_m)) {
        const float alpha = grow_m ? ex2_approx(m - m_cand) : 1.f;
        // O holds exactly PV_0..PV_{j-1}: S_j was issued only after PV_{j-1} completed
        uint32_t o0[32], o1[32];
        tmem_ld32(tO + lane_off, o0);
        tmem_ld32(tO + lane_off + 32, o1);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          o0[i] = __float_as_uint(__uint_as_float(o0[i]) * alpha);
          o1[i] = __float_as_uint(__uint_as_float(o1[i]) * alpha);
        }
        uint32_t w[16];
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          const uint32_t* src = q4 < 2 ? o0 + 16 * q4 : o1 + 16 * (q4 - 2);
#pragma unroll
          for (int i = 0; i < 16; ++i) w[i] = src[i];
          tmem_st16(tO + lane_off + 16 * q4, w);
        }
        l *= alpha;
      }
      if (grow_m) m = m_cand;
      // pass 2: probabilities, row sum, P (bf16) over the first 64 columns of S
      float sum = 0.f;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        tmem_ld32(tS + lane_off + c * 32, r);
        tmem_wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const bool m0 = diag && (c * 32 + i > row);
          const bool m1 = diag && (c * 32 + i + 1 > row);
          const float p0 = m0 ? 0.f : ex2_approx(fmaf(__uint_as_float(r[i]), sl2, -m));
          const float p1 = m1 ? 0.f : ex2_approx(fmaf(__uint_as_float(r[i + 1]), sl2, -m));
          sum += p0 + p1;
          pk[i / 2] = pack_bf16x2(p0, p1);
        }
        tmem_st16(tP + lane_off + c * 16, pk);
      }
      tmem_wait_st();
      l += sum;
      tc_fence_before();
      mbar_arrive(p_ready);
    }
    // epilogue: O / l -> bf16 rows, lse = (m + log2 l) * ln 2
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(pv_done, (n_kv - 1) & 1, p.err, 209));
    if (ok) {
      tc_fence_after();
      uint32_t o0[32], o1[32];
      tmem_ld32(tO + lane_off, o0);
      tmem_ld32(tO + lane_off + 32, o1);
      tmem_wait_ld();
      if (grow < p.T) {
        const float inv = 1.f / l;
        __nv_bfloat16* dst = p.o + (int64_t)b * p.o_sb + (int64_t)grow * p.o_st + (int64_t)h * p.o_sh;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint32_t* src = c < 4 ? o0 + 8 * c : o1 + 8 * (c - 4);
          uint4 u;
          u.x = pack_bf16x2(__uint_as_float(src[0]) * inv, __uint_as_float(src[1]) * inv);
          u.y = pack_bf16x2(__uint_as_float(src[2]) * inv, __uint_as_float(src[3]) * inv);
          u.z = pack_bf16x2(__uint_as_float(src[4]) * inv, __uint_as_float(src[5]) * inv);
          u.w = pack_bf16x2(__uint_as_float(src[6]) * inv, __uint_as_float(src[7]) * inv);
          reinterpret_cast<uint4*>(dst)[c] = u;
        }
        p.lse[(int64_t)bh * p.T + grow] = (m + __log2f(l)) * LN2;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, FA_TMEM_COLS);
  }
}

// ==========================================================================================
// backward
// ==========================================================================================
constexpr int BA_THREADS = 320;  // warp 0 TMA, warp 1 MMA, warps 2-5 dS, warps 6-9 dQ drain
constexpr uint32_t BA_TMEM_COLS = 512;
// TMEM columns: S^T [0,128) (P^T bf16 over [0,64)), dP^T [128,256) (dS^T bf16 over [128,192)),
// dV [256,320), dK [320,384), dQ [384,448)
constexpr int BA_QSTAGE = 2 * AT_TILE_BYTES + 2 * AT_TILE * 4;  // Q, dO, lse2, delta
constexpr int BA_SMEM = 2 * AT_TILE_BYTES /*K,V*/ + 2 * BA_QSTAGE + 2 * AT_TILE_BYTES /*dS^T*/ +
                        AT_TILE * AT_D * 4 /*dQ staging*/ + 1024 + 256;

struct BwdMaps {
  TileMap q, k, v, dout;
  CUtensorMap dq_acc;  // fp32 [BH*Tp rows][64], box 32 x 128, 128B swizzle
};

struct BwdParams {
  int NH, T, nq, Tp;
  float scale, scale_log2;
  const float* lse2;    // [BH][Tp] lse * log2 e (+inf on padding rows)
  const float* delta;   // [BH][Tp]
  float* dq_acc;        // [BH][Tp][64] fp32
  __nv_bfloat16 *dk, *dv;
  int64_t sb, st, sh;   // strides of dk/dv (same as q/k/v)
  int* err;
};

__global__ void attn_bwd_prep_kernel(const __nv_bfloat16* __restrict__ o,
                                     const __nv_bfloat16* __restrict__ dout,
                                     const float* __restrict__ lse, float* __restrict__ lse2,
                                     float* __restrict__ delta, int NH, int T, int Tp,
                                     int64_t o_sb, int64_t o_st, int64_t o_sh, int64_t rows) {
  const int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (idx >= rows) return;
  const int64_t bh = idx / Tp;
  const int t = (int)(idx % Tp);
  if (t >= T) {
    lse2[idx] = INFINITY;  // padding rows: P = 2^(s - inf) = 0
    delta[idx] = 0.f;
    return;
  }
  const int b = (int)(bh / NH), h = (int)(bh % NH);
  const int64_t off = b * o_sb + (int64_t)t * o_st + (int64_t)h * o_sh;
  const uint4* po = reinterpret_cast<const uint4*>(o + off);
  const uint4* pd = reinterpret_cast<const uint4*>(dout + off);
  float acc = 0.f;
#pragma unroll
  for (int c = 0; c < AT_D / 8; ++c) {
    const uint4 a = po[c], g = pd[c];
    const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, gw[4] = {g.x, g.y, g.z, g.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 fa = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&aw[i]));
      const float2 fg = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&gw[i]));
      acc = fmaf(fa.x, fg.x, acc);
      acc = fmaf(fa.y, fg.y, acc);
    }
  }
  delta[idx] = acc;
  lse2[idx] = lse[bh * T + t] * LOG2E;
}

__global__ void __launch_bounds__(BA_THREADS, 1)
attn_bwd_tc_kernel(const __grid_constant__ BwdMaps maps, const BwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem;
  uint8_t* sV = sK + AT_TILE_BYTES;
  uint8_t* sStage = sV + AT_TILE_BYTES;  // [2] x {Q, dO, lse2[128], delta[128]}
  uint8_t* sDS = sStage + 2 * BA_QSTAGE;  // dS^T, two 64-query atom blocks of [128 keys][64] bf16
  // dQ staging: two 32-column halves of [128 q][32] fp32 in the 128B-swizzled layout the
  // reduce's tensor map expects (16 KB each)
  float* sDQ = reinterpret_cast<float*>(sDS + 2 * AT_TILE_BYTES);
  uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(sDQ) + AT_TILE * AT_D * 4);
  uint64_t* kv_full = bars;
  uint64_t* q_full = bars + 1;      // [2]
  uint64_t* q_empty = q_full + 2;   // [2]
  uint64_t* sdp_full = q_empty + 2;
  uint64_t* ds_ready = sdp_full + 1;
  uint64_t* pd_free = ds_ready + 1;
  uint64_t* dq_full = pd_free + 1;
  uint64_t* dq_free = dq_full + 1;
  uint64_t* kv_done = dq_free + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(kv_done + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int nkv = p.nq;
  const int bh = blockIdx.x / nkv;
  const int jt = (int)(blockIdx.x % nkv);  // key tile; tile 0 sees the most query tiles
  const int b = bh / p.NH, h = bh % p.NH;
  const int n_it = p.nq - jt;              // query tiles jt .. nq-1

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&q_full[s], 1);
      mbar_init(&q_empty[s], 1);
    }
    mbar_init(sdp_full, 1);
    mbar_init(ds_ready, 128);
    mbar_init(pd_free, 1);
    mbar_init(dq_full, 1);
    mbar_init(dq_free, 128);
    mbar_init(kv_done, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, BA_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tP = tmem, tdP = tmem + 128, tdS = tmem + 128;
  const uint32_t tdV = tmem + 256, tdK = tmem + 320, tdQ = tmem + 384;

  auto stage_q = [&](int s) { return sStage + s * BA_QSTAGE; };
  auto stage_do = [&](int s) { return sStage + s * BA_QSTAGE + AT_TILE_BYTES; };
  auto stage_lse = [&](int s) { return reinterpret_cast<float*>(sStage + s * BA_QSTAGE + 2 * AT_TILE_BYTES); };
  auto stage_delta = [&](int s) { return stage_lse(s) + AT_TILE; };

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&maps.q.map);
      tma_prefetch_desc(&maps.k.map);
      tma_prefetch_desc(&maps.v.map);
      tma_prefetch_desc(&maps.dout.map);
      mbar_arrive_expect_tx(kv_full, 2 * AT_TILE_BYTES);
      load_tile(sK, maps.k, kv_full, b, h, jt * AT_TILE);
      load_tile(sV, maps.v, kv_full, b, h, jt * AT_TILE);
      bool ok = true;
      for (int it = 0; it < n_it && ok; ++it) {
        const int s = it & 1;
        const uint32_t ph = (it >> 1) & 1;
        if (!mbar_wait(&q_empty[s], ph ^ 1, p.err, 301)) { ok = false; break; }
        const int q0 = (jt + it) * AT_TILE;
        mbar_arrive_expect_tx(&q_full[s], 2 * AT_TILE_BYTES + 2 * AT_TILE * 4);
        load_tile(stage_q(s), maps.q, &q_full[s], b, h, q0);
        load_tile(stage_do(s), maps.dout, &q_full[s], b, h, q0);
        bulk_load(stage_lse(s), p.lse2 + (int64_t)bh * p.Tp + q0, AT_TILE * 4, &q_full[s]);
        bulk_load(stage_delta(s), p.delta + (int64_t)bh * p.Tp + q0, AT_TILE * 4, &q_full[s]);
      }
      for (int it = n_it; it < n_it + 2 && ok; ++it)
        ok = mbar_wait(&q_empty[it & 1], ((it >> 1) & 1) ^ 1, p.err, 302);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc_sdp = idesc_bf16_f32(128, 128, 0, 0);  // K/V and Q/dO all K-major
      const uint32_t idesc_kv = idesc_bf16_f32(128, 64, 0, 1);    // A from TMEM, B MN-major
      const uint32_t idesc_q = idesc_bf16_f32(128, 64, 1, 1);     // A = dS (MN-major), B = K MN-major
      const uint32_t k_addr = smem_u32(sK), v_addr = smem_u32(sV), ds_addr = smem_u32(sDS);
      bool ok = mbar_wait(kv_full, 0, p.err, 303);
      for (int it = 0; it < n_it && ok; ++it) {
        const int s = it & 1;
        const uint32_t ph = (it >> 1) & 1;
        if (!mbar_wait(&q_full[s], ph, p.err, 304)) { ok = false; break; }
        if (it > 0 && !mbar_wait(pd_free, (it - 1) & 1, p.err, 305)) { ok = false; break; }
        tc_fence_after();
        const uint32_t q_addr = smem_u32(stage_q(s)), do_addr = smem_u32(stage_do(s));
#pragma unroll
        for (int k = 0; k < AT_D / 16; ++k)
          umma_ss(tS, smem_desc_sw128(k_addr + k * 32, 16, 1024), smem_desc_sw128(q_addr + k * 32, 16, 1024),
                  idesc_sdp, k > 0 ? 1u : 0u);
#pragma unroll
        for (int k = 0; k < AT_D / 16; ++k)
          umma_ss(tdP, smem_desc_sw128(v_addr + k * 32, 16, 1024), smem_desc_sw128(do_addr + k * 32, 16, 1024),
                  idesc_sdp, k > 0 ? 1u : 0u);
        umma_commit(sdp_full);
        if (!mbar_wait(ds_ready, it & 1, p.err, 306)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < AT_TILE / 16; ++k)  // dV += P^T dO
          umma_ts(tdV, tP + k * 8, smem_desc_sw128(do_addr + k * 2048, 8192, 1024), idesc_kv,
                  (it > 0 || k > 0) ? 1u : 0u);
#pragma unroll
        for (int k = 0; k < AT_TILE / 16; ++k)  // dK += dS^T Q
          umma_ts(tdK, tdS + k * 8, smem_desc_sw128(q_addr + k * 2048, 8192, 1024), idesc_kv,
                  (it > 0 || k > 0) ? 1u : 0u);
        umma_commit(pd_free);
        if (it > 0 && !mbar_wait(dq_free, (it - 1) & 1, p.err, 307)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < AT_TILE / 16; ++k)  // dQ = dS K  (k over keys)
          umma_ss(tdQ, smem_desc_sw128(ds_addr + k * 2048, 16384, 1024),
                  smem_desc_sw128(k_addr + k * 2048, 8192, 1024), idesc_q, k > 0 ? 1u : 0u);
        umma_commit(dq_full);
        umma_commit(&q_empty[s]);
      }
      if (ok) umma_commit(kv_done);
    }
  } else if (warp < 6) {
    // ---------------- dS warpgroup: one key row per thread ----------------
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // key row within the tile
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    bool ok = true;
    for (int it = 0; it < n_it; ++it) {
      const int s = it & 1;
      const uint32_t ph = (it >> 1) & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(sdp_full, it & 1, p.err, 308) &&
                                       mbar_wait(&q_full[s], ph, p.err, 309));
      if (!ok) break;
      tc_fence_after();
      const bool diag = (it == 0);  // query tile jt: key r visible to query q iff r <= q
      const float* lse2 = stage_lse(s);
      const float* dl = stage_delta(s);
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t sr[32], dr[32];
        tmem_ld32(tS + lane_off + c * 32, sr);
        tmem_ld32(tdP + lane_off + c * 32, dr);
        tmem_wait_ld();
        uint32_t pk[16], dk[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const int q = c * 32 + i;
          float p0 = ex2_approx(fmaf(__uint_as_float(sr[i]), p.scale_log2, -lse2[q]));
          float p1 = ex2_approx(fmaf(__uint_as_float(sr[i + 1]), p.scale_log2, -lse2[q + 1]));
          if (diag && q < r) p0 = 0.f;
          if (diag && q + 1 < r) p1 = 0.f;
          const float d0 = p0 * (__uint_as_float(dr[i]) - dl[q]) * p.scale;
          const float d1 = p1 * (__uint_as_float(dr[i + 1]) - dl[q + 1]) * p.scale;
          pk[i / 2] = pack_bf16x2(p0, p1);
          dk[i / 2] = pack_bf16x2(d0, d1);
        }
        tmem_st16(tP + lane_off + c * 16, pk);
        tmem_st16(tdS + lane_off + c * 16, dk);
        // dS^T row r, queries 32c..32c+31 -> 128B-swizzled [64-query block][key row][64] layout
        uint8_t* blk = sDS + (c >> 1) * AT_TILE_BYTES + r * 128;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int chunk = (c & 1) * 4 + u;
          uint4 v4 = make_uint4(dk[4 * u], dk[4 * u + 1], dk[4 * u + 2], dk[4 * u + 3]);
          *reinterpret_cast<uint4*>(blk + ((chunk ^ (r & 7)) << 4)) = v4;
        }
      }
      tmem_wait_st();
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(ds_ready);
    }
    // dK, dV epilogue
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(kv_done, 0, p.err, 310));
    if (ok) {
      tc_fence_after();
      const int key = jt * AT_TILE + r;
#pragma unroll 1
      for (int which = 0; which < 2; ++which) {
        const uint32_t src_col = which == 0 ? tdV : tdK;
        uint32_t a0[32], a1[32];
        tmem_ld32(src_col + lane_off, a0);
        tmem_ld32(src_col + lane_off + 32, a1);
        tmem_wait_ld();
        if (key < p.T) {
          __nv_bfloat16* dst = (which == 0 ? p.dv : p.dk) + (int64_t)b * p.sb + (int64_t)key * p.st +
                               (int64_t)h * p.sh;
#pragma unroll
          for (int cc = 0; cc < 8; ++cc) {
            const uint32_t* src = cc < 4 ? a0 + 8 * cc : a1 + 8 * (cc - 4);
            uint4 u;
            u.x = pack_bf16x2(__uint_as_float(src[0]), __uint_as_float(src[1]));
            u.y = pack_bf16x2(__uint_as_float(src[2]), __uint_as_float(src[3]));
            u.z = pack_bf16x2(__uint_as_float(src[4]), __uint_as_float(src[5]));
            u.w = pack_bf16x2(__uint_as_float(src[6]), __uint_as_float(src[7]));
            reinterpret_cast<uint4*>(dst)[cc] = u;
          }
        }
      }
    }
  } else {
    // ---------------- dQ drain warpgroup: one query row per thread ----------------
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const bool leader = (warp == 6 && lane == 0);
    for (int it = 0; it < n_it; ++it) {
      const bool ok = __all_sync(0xffffffffu, mbar_wait(dq_full, it & 1, p.err, 311));
      if (!ok) break;
      tc_fence_after();
      uint32_t a0[32], a1[32];
      tmem_ld32(tdQ + lane_off, a0);
      tmem_ld32(tdQ + lane_off + 32, a1);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(dq_free);
      // the previous bulk reduce must have finished reading the staging buffer
      if (leader) bulk_wait_read0();
      named_bar_sync(1, 128);
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        uint8_t* rowp = reinterpret_cast<uint8_t*>(sDQ) + hf * (AT_TILE * 128) + row * 128;
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) {
          const uint32_t* src = (hf == 0 ? a0 : a1) + 4 * ch;
          *reinterpret_cast<uint4*>(rowp + ((ch ^ (row & 7)) << 4)) = make_uint4(src[0], src[1], src[2], src[3]);
        }
      }
      fence_proxy_async_smem();
      named_bar_sync(1, 128);
      if (leader) {
        const int grow = bh * p.Tp + (jt + it) * AT_TILE;
        tma_reduce_add_2d(&maps.dq_acc, sDQ, 0, grow);
        tma_reduce_add_2d(&maps.dq_acc, reinterpret_cast<uint8_t*>(sDQ) + AT_TILE * 128, 32, grow);
        bulk_commit();
      }
    }
    if (leader) bulk_wait0();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, BA_TMEM_COLS);
  }
}

__global__ void attn_dq_convert_kernel(const float* __restrict__ dq_acc, __nv_bfloat16* __restrict__ dq,
                                       int NH, int T, int Tp, int64_t sb, int64_t st, int64_t sh,
                                       int64_t n8) {
  const int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;  // one thread per 8 elements
  if (idx >= n8) return;
  const int c8 = (int)(idx % (AT_D / 8));
  const int64_t rowi = idx / (AT_D / 8);
  const int t = (int)(rowi % T);
  const int64_t bh = rowi / T;
  const int b = (int)(bh / NH), h = (int)(bh % NH);
  const float4* src = reinterpret_cast<const float4*>(dq_acc + ((bh * Tp + t) * AT_D + c8 * 8));
  const float4 a = src[0], c = src[1];
  uint4 u;
  u.x = pack_bf16x2(a.x, a.y);
  u.y = pack_bf16x2(a.z, a.w);
  u.z = pack_bf16x2(c.x, c.y);
  u.w = pack_bf16x2(c.z, c.w);
  *reinterpret_cast<uint4*>(dq + b * sb + (int64_t)t * st + (int64_t)h * sh + c8 * 8) = u;
}

// ==========================================================================================
// host side
// ==========================================================================================
static bool strides_ok(int64_t sb, int64_t st, int64_t sh) {
  if (sb % 8 || st % 8 || sh % 8) return false;  // 16-byte TMA strides
  if (st < AT_D) return false;
  return true;
}

bool tc_fwd_supported(int D, int dtype) { return D == AT_D && dtype == ATTN_BF16; }
bool tc_bwd_supported(int D, int dtype) { return D == AT_D && dtype == ATTN_BF16; }

static size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

size_t attn_bwd_tc_ws(int B, int NH, int T, int D) {
  const size_t Tp = (size_t)((T + AT_TILE - 1) / AT_TILE) * AT_TILE;
  const size_t BH = (size_t)B * NH;
  return 2 * align256(BH * Tp * 4) + align256(BH * Tp * D * 4);
}

// 4D map over a [B][T][NH][64] (or [B][NH][T][64]) bf16 tensor given element strides.
static bool make_head_map(TileMap* tm, const void* base, int B, int NH, int T, int64_t sb, int64_t st,
                          int64_t sh) {
  uint64_t dims[4], strides[3];
  uint32_t box[4];
  tm->h_first = sh <= st ? 1 : 0;
  dims[0] = AT_D;
  box[0] = AT_D;
  if (tm->h_first) {
    dims[1] = NH; dims[2] = T; dims[3] = B;
    strides[0] = sh * 2; strides[1] = st * 2; strides[2] = sb * 2;
    box[1] = 1; box[2] = AT_TILE; box[3] = 1;
  } else {
    dims[1] = T; dims[2] = NH; dims[3] = B;
    strides[0] = st * 2; strides[1] = sh * 2; strides[2] = sb * 2;
    box[1] = AT_TILE; box[2] = 1; box[3] = 1;
  }
  return make_tmap_bf16(&tm->map, base, 4, dims, strides, box);
}

int attn_fwd_tc(const void* q, const void* k, const void* v, void* o, float* lse, int B, int NH, int T,
                int D, const int64_t* s, float scale, cudaStream_t stream) {
  (void)D;
  if (!strides_ok(s[0], s[1], s[2]) || !strides_ok(s[3], s[4], s[5]) || !aligned(q, 16) || !aligned(k, 16) ||
      !aligned(v, 16) || !aligned(o, 16)) {
    set_error("attn_fwd: the tensor-core path needs 16-byte aligned bf16 tensors with strides that are "
              "multiples of 8 elements");
    return ATTN_ERR_ARG;
  }
  FwdMaps maps;
  if (!make_head_map(&maps.q, q, B, NH, T, s[0], s[1], s[2]) ||
      !make_head_map(&maps.k, k, B, NH, T, s[0], s[1], s[2]) ||
      !make_head_map(&maps.v, v, B, NH, T, s[0], s[1], s[2]))
    return ATTN_ERR_CUDA;
  FwdParams p;
  p.NH = NH;
  p.T = T;
  p.nq = (T + AT_TILE - 1) / AT_TILE;
  p.scale_log2 = scale * LOG2E;
  p.o = reinterpret_cast<__nv_bfloat16*>(o);
  p.o_sb = s[3];
  p.o_st = s[4];
  p.o_sh = s[5];
  p.lse = lse;
  p.err = dev_error_ptr();
  if (!p.err) return ATTN_ERR_CUDA;
  static bool attr = false;
  if (!attr) {
    ATTN_CUDA_TRY(cudaFuncSetAttribute(attn_fwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, FA_SMEM));
    attr = true;
  }
  const int64_t grid = (int64_t)B * NH * p.nq;
  attn_fwd_tc_kernel<<<(unsigned)grid, FA_THREADS, FA_SMEM, stream>>>(maps, p);
  count_launch();
  return check_launch("attn_fwd_tc_kernel");
}

int attn_bwd_tc(const void* q, const void* k, const void* v, const void* o, const void* dout,
                const float* lse, void* dq, void* dk, void* dv, void* ws, int B, int NH, int T, int D,
                const int64_t* s, float scale, cudaStream_t stream) {
  (void)D;
  if (!strides_ok(s[0], s[1], s[2]) || !strides_ok(s[3], s[4], s[5]) || !aligned(q, 16) || !aligned(k, 16) ||
      !aligned(v, 16) || !aligned(o, 16) || !aligned(dout, 16) || !aligned(dq, 16) || !aligned(dk, 16) ||
      !aligned(dv, 16)) {
    set_error("attn_bwd: the tensor-core path needs 16-byte aligned bf16 tensors with strides that are "
              "multiples of 8 elements");
    return ATTN_ERR_ARG;
  }
  const int nq = (T + AT_TILE - 1) / AT_TILE;
  const int Tp = nq * AT_TILE;
  const size_t BH = (size_t)B * NH;
  uint8_t* w = reinterpret_cast<uint8_t*>(ws);
  float* lse2 = reinterpret_cast<float*>(w);
  float* delta = reinterpret_cast<float*>(w + align256(BH * Tp * 4));
  float* dq_acc = reinterpret_cast<float*>(w + 2 * align256(BH * Tp * 4));
  ATTN_CUDA_TRY(cudaMemsetAsync(dq_acc, 0, BH * Tp * AT_D * 4, stream));
  const int64_t rows = (int64_t)BH * Tp;
  attn_bwd_prep_kernel<<<(unsigned)((rows + 255) / 256), 256, 0, stream>>>(
      (const __nv_bfloat16*)o, (const __nv_bfloat16*)dout, lse, lse2, delta, NH, T, Tp, s[3], s[4], s[5], rows);
  count_launch();
  if (int rc = check_launch("attn_bwd_prep_kernel")) return rc;

  BwdMaps maps;
  if (!make_head_map(&maps.q, q, B, NH, T, s[0], s[1], s[2]) ||
      !make_head_map(&maps.k, k, B, NH, T, s[0], s[1], s[2]) ||
      !make_head_map(&maps.v, v, B, NH, T, s[0], s[1], s[2]) ||
      !make_head_map(&maps.dout, dout, B, NH, T, s[3], s[4], s[5]))
    return ATTN_ERR_CUDA;
  {
    const uint64_t dims[2] = {(uint64_t)AT_D, (uint64_t)BH * Tp};
    const uint64_t strides[1] = {AT_D * 4};
    const uint32_t box[2] = {32, AT_TILE};
    if (!make_tmap_f32(&maps.dq_acc, dq_acc, 2, dims, strides, box)) return ATTN_ERR_CUDA;
  }
  BwdParams p;
  p.NH = NH;
  p.T = T;
  p.nq = nq;
  p.Tp = Tp;
  p.scale = scale;
  p.scale_log2 = scale * LOG2E;
  p.lse2 = lse2;
  p.delta = delta;
  p.dq_acc = dq_acc;
  p.dk = reinterpret_cast<__nv_bfloat16*>(dk);
  p.dv = reinterpret_cast<__nv_bfloat16*>(dv);
  p.sb = s[0];
  p.st = s[1];
  p.sh = s[2];
  p.err = dev_error_ptr();
  if (!p.err) return ATTN_ERR_CUDA;
  static bool attr = false;
  if (!attr) {
    ATTN_CUDA_TRY(cudaFuncSetAttribute(attn_bwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, BA_SMEM));
    attr = true;
  }
  attn_bwd_tc_kernel<<<(unsigned)(BH * nq), BA_THREADS, BA_SMEM, stream>>>(maps, p);
  count_launch();
  if (int rc = check_launch("attn_bwd_tc_kernel")) return rc;
  const int64_t n8 = (int64_t)BH * T * (AT_D / 8);
  attn_dq_convert_kernel<<<(unsigned)((n8 + 255) / 256), 256, 0, stream>>>(dq_acc, (__nv_bfloat16*)dq, NH, T,
                                                                          Tp, s[0], s[1], s[2], n8);
  count_launch();
  return check_launch("attn_dq_convert_kernel");
}

}  // namespace attn
