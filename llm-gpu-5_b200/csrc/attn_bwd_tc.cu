// tcgen05 causal attention backward for head_dim 64 (bf16 operands, fp32 accumulation).
//
// Replaces the NumPy backward of model/gpt.py:669-680 (and the unwired GPU kernels
// softmax_fused_backward / matmul_grad_{q,k,v}, core/mha_kernels.py:195-236, 592-680):
//   dV = P^T dO,  dP = dO V^T,  dS = P (dP - rowsum(dP P)) * scale,  dQ = dS K,  dK = dS^T Q
// with rowsum(dP P) = rowsum(dO O) = delta (model/gpt.py:675-677), and P recomputed from the
// forward's log-sum-exp instead of being stored.
//
// 1. attn_bwd_prep_kernel: delta = rowsum(dO * O) and lse in log2 units, both padded to whole
//    128-row tiles (padding rows get lse = +inf so their probabilities are exactly 0).
// 2. attn_bwd_tc_kernel: one CTA per (b, h, 128-key tile).  K, V and the dK/dV accumulators stay
//    resident; the query tiles that can see these keys stream through a 2-stage TMA ring.  Each
//    query tile is processed as two halves of 64 queries, double-buffered in TMEM so that the
//    tensor core works on one half while the dS warpgroup works on the other:
//      MMA thread     S^T = K Q_h^T and dP^T = V dO_h^T (128x64 each) into TMEM buffer h,
//                     then dV += P^T dO_h and dK += dS^T Q_h with P^T, dS^T read from TMEM,
//                     and per query tile dQ = dS K (128x64) with dS read from shared memory
//      dS warps       one key row per thread: P^T = 2^(S^T*scale*log2e - lse2), dS^T =
//                     P^T (dP^T - delta) scale; bf16 P^T and dS^T back to TMEM (over the S^T /
//                     dP^T columns already read) and dS^T to shared memory for the dQ MMA
//      dQ warps       drain each dQ tile from TMEM to swizzled shared memory and add it into an
//                     fp32 accumulator in the workspace with TMA reduce-adds (done in L2)
//    TMEM: half-buffers [0,128) and [128,256) (S^T | dP^T, 64 columns each), dV [256,320),
//    dK [320,384), dQ [384,448).
// 3. attn_dq_convert_kernel: fp32 dQ accumulator -> bf16 dQ in the caller's layout.
//
// Every mbarrier wait is bounded (tc_common.cuh): a wait that gives up sets the library's device
// error word and the kernel skips its remaining work instead of hanging.
#include "attn_tc_common.cuh"

#include <math.h>

namespace attn {

constexpr int BA_THREADS = 320;  // warp 0 TMA, warp 1 MMA, warps 2-5 dS, warps 6-9 dQ drain
constexpr uint32_t BA_TMEM_COLS = 512;
constexpr int BA_QSTAGE = 2 * AT_TILE_BYTES + 2 * AT_TILE * 4;  // Q, dO, lse2, delta
constexpr int BA_DS_BYTES = 2 * AT_TILE_BYTES;                   // dS^T of one query tile
constexpr int BA_SMEM = 2 * AT_TILE_BYTES /*K,V*/ + 2 * BA_QSTAGE + 2 * BA_DS_BYTES +
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
  uint8_t* sStage = sV + AT_TILE_BYTES;         // [2] x {Q, dO, lse2[128], delta[128]}
  uint8_t* sDS = sStage + 2 * BA_QSTAGE;         // [2] x dS^T: two 64-query blocks of [128 keys][64]
  uint8_t* sDQ = sDS + 2 * BA_DS_BYTES;          // dQ staging: two [128 q][32 fp32] swizzled halves
  uint64_t* bars = reinterpret_cast<uint64_t*>(sDQ + AT_TILE * AT_D * 4);
  uint64_t* kv_full = bars;
  uint64_t* q_full = bars + 1;       // [2] per query-tile stage
  uint64_t* q_empty = q_full + 2;    // [2]
  uint64_t* sdp_full = q_empty + 2;  // [2] per TMEM half-buffer
  uint64_t* ds_ready = sdp_full + 2; // [2]
  uint64_t* buf_free = ds_ready + 2; // [2]
  uint64_t* ds_free = buf_free + 2;  // [2] per dS^T shared-memory buffer
  uint64_t* dq_full = ds_free + 2;
  uint64_t* dq_free = dq_full + 1;
  uint64_t* kv_done = dq_free + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(kv_done + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int nkv = p.nq;
  const int bh = blockIdx.x / nkv;
  const int jt = (int)(blockIdx.x % nkv);  // key tile; tile 0 sees the most query tiles
  const int b = bh / p.NH, h = bh % p.NH;
  const int n_it = p.nq - jt;              // query tiles jt .. nq-1
  const int n_half = 2 * n_it;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&q_full[s], 1);
      mbar_init(&q_empty[s], 1);
      mbar_init(&sdp_full[s], 1);
      mbar_init(&ds_ready[s], 128);
      mbar_init(&buf_free[s], 1);
      mbar_init(&ds_free[s], 1);
    }
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
  const uint32_t tdV = tmem + 256, tdK = tmem + 320, tdQ = tmem + 384;

  auto stage_q = [&](int s) { return sStage + s * BA_QSTAGE; };
  auto stage_do = [&](int s) { return sStage + s * BA_QSTAGE + AT_TILE_BYTES; };
  auto stage_lse = [&](int s) { return reinterpret_cast<float*>(sStage + s * BA_QSTAGE + 2 * AT_TILE_BYTES); };
  auto stage_delta = [&](int s) { return stage_lse(s) + AT_TILE; };

  if (warp == 0) {
    // ---------------- TMA producer ----------------
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
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc_sdp = idesc_bf16_f32(128, 64, 0, 0);  // K/V and Q/dO all K-major
      const uint32_t idesc_kv = idesc_bf16_f32(128, 64, 0, 1);   // A from TMEM, B MN-major
      const uint32_t idesc_q = idesc_bf16_f32(128, 64, 1, 1);    // A = dS (MN-major), B = K MN-major
      const uint32_t k_addr = smem_u32(sK), v_addr = smem_u32(sV);
      bool ok = mbar_wait(kv_full, 0, p.err, 303);

      // S^T and dP^T of half n (query tile n/2, queries 64*(n%2) .. +63) into TMEM buffer n%2
      auto issue_sdp = [&](int n) -> bool {
        const int it = n >> 1, hf = n & 1, s = it & 1;
        if (hf == 0 && !mbar_wait(&q_full[s], (it >> 1) & 1, p.err, 304)) return false;
        tc_fence_after();
        const uint32_t tS = tmem + (n & 1) * 128, tdP = tS + 64;
        const uint32_t q_addr = smem_u32(stage_q(s)) + hf * 8192, do_addr = smem_u32(stage_do(s)) + hf * 8192;
#pragma unroll
        for (int k = 0; k < AT_D / 16; ++k)
          umma_ss(tS, smem_desc_sw128(k_addr + k * 32, 16, 1024), smem_desc_sw128(q_addr + k * 32, 16, 1024),
                  idesc_sdp, k > 0 ? 1u : 0u);
#pragma unroll
        for (int k = 0; k < AT_D / 16; ++k)
          umma_ss(tdP, smem_desc_sw128(v_addr + k * 32, 16, 1024), smem_desc_sw128(do_addr + k * 32, 16, 1024),
                  idesc_sdp, k > 0 ? 1u : 0u);
        umma_commit(&sdp_full[n & 1]);
        return true;
      };

      for (int n = 0; n < 2 && n < n_half && ok; ++n) ok = issue_sdp(n);
      for (int n = 0; n < n_half && ok; ++n) {
        const int it = n >> 1, hf = n & 1, s = it & 1, bb = n & 1;
        if (!mbar_wait(&ds_ready[bb], (n >> 1) & 1, p.err, 305)) { ok = false; break; }
        tc_fence_after();
        const uint32_t tP = tmem + bb * 128, tdS = tP + 64;
        const uint32_t q_addr = smem_u32(stage_q(s)) + hf * 8192, do_addr = smem_u32(stage_do(s)) + hf * 8192;
#pragma unroll
        for (int k = 0; k < 4; ++k)  // dV += P^T dO_h   (k over the 64 queries of the half)
          umma_ts(tdV, tP + k * 8, smem_desc_sw128(do_addr + k * 2048, 8192, 1024), idesc_kv,
                  (n > 0 || k > 0) ? 1u : 0u);
#pragma unroll
        for (int k = 0; k < 4; ++k)  // dK += dS^T Q_h
          umma_ts(tdK, tdS + k * 8, smem_desc_sw128(q_addr + k * 2048, 8192, 1024), idesc_kv,
                  (n > 0 || k > 0) ? 1u : 0u);
        umma_commit(&buf_free[bb]);
        if (hf == 1) {  // both halves of query tile `it` done: dQ = dS K
          if (it > 0 && !mbar_wait(dq_free, (it - 1) & 1, p.err, 306)) { ok = false; break; }
          tc_fence_after();
          const uint32_t ds_addr = smem_u32(sDS + (it & 1) * BA_DS_BYTES);
#pragma unroll
          for (int k = 0; k < AT_TILE / 16; ++k)
            umma_ss(tdQ, smem_desc_sw128(ds_addr + k * 2048, 16384, 1024),
                    smem_desc_sw128(k_addr + k * 2048, 8192, 1024), idesc_q, k > 0 ? 1u : 0u);
          umma_commit(dq_full);
          umma_commit(&ds_free[it & 1]);
          umma_commit(&q_empty[s]);
        }
        if (n + 2 < n_half) {
          // the half-buffer is rewritten only once dV/dK above have read P^T and dS^T from it
          if (!mbar_wait(&buf_free[bb], (n >> 1) & 1, p.err, 307)) { ok = false; break; }
          ok = issue_sdp(n + 2);
        }
      }
      if (ok) umma_commit(kv_done);
    }
  } else if (warp < 6) {
    // ---------------- dS warpgroup: one key row per thread ----------------
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // key row within the tile
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    bool ok = true;
    for (int n = 0; n < n_half; ++n) {
      const int it = n >> 1, hf = n & 1, s = it & 1, bb = n & 1;
      bool w = mbar_wait(&sdp_full[bb], (n >> 1) & 1, p.err, 308) &&
               mbar_wait(&q_full[s], (it >> 1) & 1, p.err, 309);
      if (w && hf == 0 && it >= 2) w = mbar_wait(&ds_free[it & 1], ((it >> 1) & 1) ^ 1, p.err, 310);
      ok = __all_sync(0xffffffffu, w);
      if (!ok) break;
      tc_fence_after();
      const bool diag = (it == 0);  // query tile jt: key r is visible to query q iff r <= q
      const float* lse2 = stage_lse(s) + hf * 64;
      const float* dl = stage_delta(s) + hf * 64;
      const uint32_t tS = tmem + bb * 128 + lane_off, tdP = tS + 64;
      uint8_t* dsrow = sDS + (it & 1) * BA_DS_BYTES + hf * AT_TILE_BYTES + r * 128;
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        uint32_t sr[32], dr[32];
        tmem_ld32(tS + c * 32, sr);
        tmem_ld32(tdP + c * 32, dr);
        tmem_wait_ld();
        uint32_t pk[16], dk[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const int ql = c * 32 + i;          // query within the half
          const int qt = hf * 64 + ql;        // query within the tile
          float p0 = ex2_approx(fmaf(__uint_as_float(sr[i]), p.scale_log2, -lse2[ql]));
          float p1 = ex2_approx(fmaf(__uint_as_float(sr[i + 1]), p.scale_log2, -lse2[ql + 1]));
          if (diag && qt < r) p0 = 0.f;
          if (diag && qt + 1 < r) p1 = 0.f;
          const float d0 = p0 * (__uint_as_float(dr[i]) - dl[ql]) * p.scale;
          const float d1 = p1 * (__uint_as_float(dr[i + 1]) - dl[ql + 1]) * p.scale;
          pk[i / 2] = pack_bf16x2(p0, p1);
          dk[i / 2] = pack_bf16x2(d0, d1);
        }
        tmem_st16(tS + c * 16, pk);   // P^T over S^T columns already read
        tmem_st16(tdP + c * 16, dk);  // dS^T over dP^T columns already read
#pragma unroll
        for (int u = 0; u < 4; ++u) {  // dS^T -> 128B-swizzled [key row][64 queries] block
          const int chunk = c * 4 + u;
          *reinterpret_cast<uint4*>(dsrow + ((chunk ^ (r & 7)) << 4)) =
              make_uint4(dk[4 * u], dk[4 * u + 1], dk[4 * u + 2], dk[4 * u + 3]);
        }
      }
      tmem_wait_st();
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&ds_ready[bb]);
    }
    // dK, dV epilogue
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(kv_done, 0, p.err, 311));
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
      const bool ok = __all_sync(0xffffffffu, mbar_wait(dq_full, it & 1, p.err, 312));
      if (!ok) break;
      tc_fence_after();
      uint32_t a0[32], a1[32];
      tmem_ld32(tdQ + lane_off, a0);
      tmem_ld32(tdQ + lane_off + 32, a1);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(dq_free);
      if (leader) bulk_wait_read0();  // the previous reduce has finished reading the staging buffer
      named_bar_sync(1, 128);
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        uint8_t* rowp = sDQ + hf * (AT_TILE * 128) + row * 128;
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
        tma_reduce_add_2d(&maps.dq_acc, sDQ + AT_TILE * 128, 32, grow);
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
bool tc_bwd_supported(int D, int dtype) { return D == AT_D && dtype == ATTN_BF16; }

size_t attn_bwd_tc_ws(int B, int NH, int T, int D) {
  const size_t Tp = (size_t)((T + AT_TILE - 1) / AT_TILE) * AT_TILE;
  const size_t BH = (size_t)B * NH;
  return 2 * align256(BH * Tp * 4) + align256(BH * Tp * D * 4);
}

int attn_bwd_tc(const void* q, const void* k, const void* v, const void* o, const void* dout,
                const float* lse, void* dq, void* dk, void* dv, void* ws, int B, int NH, int T, int D,
                const int64_t* s, float scale, cudaStream_t stream) {
  (void)D;
  if (!head_strides_ok(s[0], s[1], s[2]) || !head_strides_ok(s[3], s[4], s[5]) || !aligned(q, 16) ||
      !aligned(k, 16) || !aligned(v, 16) || !aligned(o, 16) || !aligned(dout, 16) || !aligned(dq, 16) ||
      !aligned(dk, 16) || !aligned(dv, 16)) {
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
