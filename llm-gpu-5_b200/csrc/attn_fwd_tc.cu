// tcgen05 tensor-core causal attention forward for head_dim 64, bf16 operands, fp32 accumulation.
//
// Replaces fused_attention_forward_kernel (core/mha_kernels.py:404-521).  A persistent kernel:
// one CTA per SM walks a static list of items.  An item is two consecutive 128-row query tiles
// (A = 2m, B = 2m+1) of one (batch, head); they share one stream of 128-key K/V blocks.  Items
// are walked in pairs (m, nI-1-m) so that every pair costs the same number of blocks.
//
//   MMA thread     per block j: S_X = Q_X K_j^T (X = A, B; tcgen05.mma, A and B operands from
//                  shared memory, fp32 accumulator in TMEM), then O_X += P_X V_{j-1} for the
//                  previous block (A = P_X read from TMEM, B = V MN-major from shared memory)
//   softmax A, B   two warpgroups, one per query tile, one query row per thread: the row of S
//                  is read from TMEM once (128 columns), causal mask on the diagonal block only,
//                  row max, 2^(s*scale*log2e - m), row sum; P packed to bf16 into the tile's own
//                  TMEM P columns, so the next S can be computed while P V runs
// While one warpgroup computes its softmax the tensor core works for the other, and the two
// warpgroups give each SM sub-partition two softmax warps.  The running max is only moved (and O
// rescaled in TMEM) when it grows by more than 2^8, so rescaling is rare.  The row's log-sum-exp
// is written instead of the T x T probabilities.
//
// TMEM columns: S_A [0,128), S_B [128,256), P_A [256,320), P_B [320,384), O_A [384,448),
// O_B [448,512).
//
// Every mbarrier wait is bounded (tc_common.cuh): a wait that gives up sets the library's device
// error word and the kernel skips its remaining work instead of hanging.
#include "attn_tc_common.cuh"

#include <math.h>

namespace attn {

constexpr int FA_THREADS = 320;  // warp 0 TMA, warp 1 MMA + TMEM, warps 2-5 softmax A, 6-9 softmax B
constexpr int FA_KV = 3;         // K/V ring stages
constexpr uint32_t FA_TMEM_COLS = 512;
constexpr uint32_t FA_TM_S = 0, FA_TM_P = 256, FA_TM_O = 384;
constexpr int FA_SMEM = 1024 + AT_TILE_BYTES * (4 + 2 * FA_KV + 2) + 256;

struct FwdMaps {
  TileMap q, k, v, o;
};

struct FwdParams {
  int NH, T, nq, n_items, n_units, BH;  // n_items = ceil(nq/2) per head, n_units = ceil(n_items/2)
  float scale_log2;
  __nv_bfloat16* o;
  int64_t o_sb, o_st, o_sh;
  float* lse;
  int* err;
};

// The item list every role of a CTA walks in the same order: units w = blockIdx.x, +gridDim.x,
// ...; unit w is head bh = w / n_units with items m = u and n_items-1-u (u = w % n_units; one
// item when they coincide).  Item m covers query tiles 2m and 2m+1 (tB = -1 past the end).
// fn(bh, tA, tB) returns false to stop the walk.
template <typename Fn>
__device__ __forceinline__ void for_each_item(const FwdParams& p, Fn&& fn) {
  for (int w = blockIdx.x; w < p.BH * p.n_units; w += gridDim.x) {
    const int bh = w / p.n_units, u = w % p.n_units;
    const int m0 = p.n_items - 1 - u, m1 = u;  // the longer item first
    int tB = 2 * m0 + 1 < p.nq ? 2 * m0 + 1 : -1;
    if (!fn(bh, 2 * m0, tB)) return;
    if (m1 != m0) {
      tB = 2 * m1 + 1 < p.nq ? 2 * m1 + 1 : -1;
      if (!fn(bh, 2 * m1, tB)) return;
    }
  }
}

// The same walk as an explicit cursor, for the producer, which loads the next item's Q while
// streaming the current item's K/V blocks.
struct ItemCursor {
  int w, second;  // unit index and which item of the unit
  int bh, tA, tB;
  __device__ __forceinline__ void set(const FwdParams& p) {
    const int u = w % p.n_units;
    const int m = second ? u : p.n_items - 1 - u;
    bh = w / p.n_units;
    tA = 2 * m;
    tB = 2 * m + 1 < p.nq ? 2 * m + 1 : -1;
  }
  __device__ __forceinline__ bool valid(const FwdParams& p) const { return w < p.BH * p.n_units; }
  __device__ __forceinline__ void start(const FwdParams& p) {
    w = blockIdx.x;
    second = 0;
    if (valid(p)) set(p);
  }
  __device__ __forceinline__ void next(const FwdParams& p) {
    const int u = w % p.n_units;
    if (!second && u != p.n_items - 1 - u) {
      second = 1;
    } else {
      second = 0;
      w += gridDim.x;
    }
    if (valid(p)) set(p);
  }
};

__global__ void __launch_bounds__(FA_THREADS, 1)
attn_fwd_tc_kernel(const __grid_constant__ FwdMaps maps, const FwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                               // [2 slots][A, B]
  uint8_t* sK = sQ + 4 * AT_TILE_BYTES;             // [FA_KV]
  uint8_t* sV = sK + FA_KV * AT_TILE_BYTES;         // [FA_KV]
  uint8_t* sO = sV + FA_KV * AT_TILE_BYTES;         // [2] epilogue staging per softmax warpgroup
  uint64_t* bars = reinterpret_cast<uint64_t*>(sO + 2 * AT_TILE_BYTES);
  uint64_t* q_full = bars;              // [2] per Q slot (both tiles of an item)
  uint64_t* q_empty = q_full + 2;       // [2]
  uint64_t* k_full = q_empty + 2;       // [FA_KV]
  uint64_t* v_full = k_full + FA_KV;    // [FA_KV]
  uint64_t* kv_empty = v_full + FA_KV;  // [FA_KV]
  uint64_t* s_full = kv_empty + FA_KV;  // [2] per query tile X: S_X is in TMEM
  uint64_t* p_ready = s_full + 2;       // [2] S_X read and P_X written (128 arrivals)
  uint64_t* pv_done = p_ready + 2;      // [2] the P_X V MMA has completed
  uint64_t* wg_bar = pv_done + 2;       // [2] sync of softmax warpgroup X (128 arrivals)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(wg_bar + 2);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&q_full[s], 1);
      mbar_init(&q_empty[s], 1);
      mbar_init(&s_full[s], 1);
      mbar_init(&p_ready[s], 128);
      mbar_init(&pv_done[s], 1);
      mbar_init(&wg_bar[s], 128);
    }
    for (int s = 0; s < FA_KV; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
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

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      tma_prefetch_desc(&maps.q.map);
      tma_prefetch_desc(&maps.k.map);
      tma_prefetch_desc(&maps.v.map);
      auto load_q = [&](const ItemCursor& c, int it) -> bool {
        const int qs = it & 1;
        if (!mbar_wait(&q_empty[qs], ((it >> 1) & 1) ^ 1, p.err, 201)) return false;
        const int b = c.bh / p.NH, h = c.bh % p.NH;
        mbar_arrive_expect_tx(&q_full[qs], (c.tB >= 0 ? 2 : 1) * AT_TILE_BYTES);
        load_tile(sQ + (2 * qs) * AT_TILE_BYTES, maps.q, &q_full[qs], b, h, c.tA * AT_TILE);
        if (c.tB >= 0) load_tile(sQ + (2 * qs + 1) * AT_TILE_BYTES, maps.q, &q_full[qs], b, h, c.tB * AT_TILE);
        return true;
      };
      ItemCursor cur;
      cur.start(p);
      bool ok = !cur.valid(p) || load_q(cur, 0);
      int it = 0, g = 0;
      while (ok && cur.valid(p)) {
        ItemCursor nxt = cur;
        nxt.next(p);
        const int b = cur.bh / p.NH, h = cur.bh % p.NH;
        const int jmax = cur.tB >= 0 ? cur.tB : cur.tA;
        for (int j = 0; j <= jmax && ok; ++j, ++g) {
          const int st = g % FA_KV;
          if (!mbar_wait(&kv_empty[st], ((g / FA_KV) & 1) ^ 1, p.err, 202)) { ok = false; break; }
          mbar_arrive_expect_tx(&k_full[st], AT_TILE_BYTES);
          load_tile(sK + st * AT_TILE_BYTES, maps.k, &k_full[st], b, h, j * AT_TILE);
          mbar_arrive_expect_tx(&v_full[st], AT_TILE_BYTES);
          load_tile(sV + st * AT_TILE_BYTES, maps.v, &v_full[st], b, h, j * AT_TILE);
          // the next item's Q, as soon as this item's first block is on its way
          if (j == 0 && nxt.valid(p) && !load_q(nxt, it + 1)) ok = false;
        }
        cur = nxt;
        ++it;
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc_s = idesc_bf16_f32(128, 128, 0, 0);  // Q K-major, K K-major
      const uint32_t idesc_o = idesc_bf16_f32(128, 64, 0, 1);   // P from TMEM, V MN-major
      int cnt[2] = {0, 0};  // S MMAs issued per query tile X (= softmax steps of X)
      int it = 0, g = 0;
      bool ok = true;
      for_each_item(p, [&](int bh, int tA, int tB) -> bool {
        (void)bh;
        const int qs = it & 1;
        const int tX[2] = {tA, tB};
        if (!mbar_wait(&q_full[qs], (it >> 1) & 1, p.err, 203)) return ok = false;
        const int jmax = tB >= 0 ? tB : tA;
        // block j: S_X(j) for the tiles that see it, then P_X V_{j-1}; a last pass (j = jmax+1)
        // issues only the final P V products
        for (int j = 0; j <= jmax + 1; ++j) {
          const int st = (g + j) % FA_KV, pst = (g + j - 1) % FA_KV;
          if (j <= jmax && !mbar_wait(&k_full[st], ((g + j) / FA_KV) & 1, p.err, 204)) return ok = false;
          if (j > 0 && !mbar_wait(&v_full[pst], ((g + j - 1) / FA_KV) & 1, p.err, 205)) return ok = false;
          for (int x = 0; x < 2; ++x) {
            const bool now = j <= tX[x], prev = j >= 1 && j - 1 <= tX[x];
            if (!now && !prev) continue;
            // S_X is rewritten (and P_X read by the MMA) once softmax X has finished its step
            if (cnt[x] > 0 && !mbar_wait(&p_ready[x], (cnt[x] - 1) & 1, p.err, 206)) return ok = false;
            tc_fence_after();
            if (now) {
              const uint64_t q_desc = smem_desc_sw128(smem_u32(sQ + (2 * qs + x) * AT_TILE_BYTES), 16, 1024);
              const uint64_t k_desc = smem_desc_sw128(smem_u32(sK + st * AT_TILE_BYTES), 16, 1024);
              const uint32_t tS = tmem + FA_TM_S + x * 128;
#pragma unroll
              for (int k = 0; k < AT_D / 16; ++k)
                umma_ss(tS, desc_step(q_desc, k * 32), desc_step(k_desc, k * 32),
                        idesc_s, k > 0 ? 1u : 0u);
              umma_commit(&s_full[x]);
              ++cnt[x];
            }
            if (prev) {
              const uint64_t v_desc = smem_desc_sw128(smem_u32(sV + pst * AT_TILE_BYTES), 8192, 1024);
              const uint32_t tP = tmem + FA_TM_P + x * 64, tO = tmem + FA_TM_O + x * 64;
#pragma unroll
              for (int k = 0; k < AT_TILE / 16; ++k)
                umma_ts(tO, tP + k * 8, desc_step(v_desc, k * 2048), idesc_o,
                        (j == 1 && k == 0) ? 0u : 1u);
              umma_commit(&pv_done[x]);
            }
          }
          if (j == jmax) umma_commit(&q_empty[qs]);  // the item's last S MMAs read Q
          if (j > 0) umma_commit(&kv_empty[pst]);
        }
        g += jmax + 1;
        ++it;
        return true;
      });
    }
  } else {
    // ---------------- softmax warpgroups: X = 0 (tile A) warps 2-5, X = 1 (tile B) warps 6-9 ----------------
    const int x = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t tS = tmem + FA_TM_S + x * 128 + lane_off;
    const uint32_t tP = tmem + FA_TM_P + x * 64 + lane_off;
    const uint32_t tO = tmem + FA_TM_O + x * 64 + lane_off;
    const float sl2 = p.scale_log2;
    int c = 0;  // softmax steps done by this warpgroup
    const bool leader = (warp & 3) == 2 && lane == 0;  // first warp of the warpgroup
    bool first_store = true;
    uint32_t wg_phase = 0;
    auto wg_sync = [&]() -> bool {  // bounded barrier over the 128 threads of warpgroup X
      mbar_arrive(&wg_bar[x]);
      const bool w = mbar_wait(&wg_bar[x], wg_phase & 1, p.err, 210);
      ++wg_phase;
      return __all_sync(0xffffffffu, w);
    };
    for_each_item(p, [&](int bh, int tA, int tB) -> bool {
      const int t = x == 0 ? tA : tB;
      if (t < 0) return true;
      float m = -INFINITY, l = 0.f;
      for (int j = 0; j <= t; ++j, ++c) {
        if (!__all_sync(0xffffffffu, mbar_wait(&s_full[x], c & 1, p.err, 207))) return false;
        tc_fence_after();
        uint32_t sr[128];
        tmem_ld32(tS, *reinterpret_cast<uint32_t(*)[32]>(sr));
        tmem_ld32(tS + 32, *reinterpret_cast<uint32_t(*)[32]>(sr + 32));
        tmem_ld32(tS + 64, *reinterpret_cast<uint32_t(*)[32]>(sr + 64));
        tmem_ld32(tS + 96, *reinterpret_cast<uint32_t(*)[32]>(sr + 96));
        tmem_wait_ld();
        const bool diag = (j == t);
        if (diag) {  // key column k is visible to query row r iff k <= r
#pragma unroll
          for (int i = 0; i < 128; ++i)
            if (i > row) sr[i] = __float_as_uint(-INFINITY);
        }
        float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
#pragma unroll
        for (int i = 0; i < 128; i += 8) {
          mx0 = fmax3(mx0, __uint_as_float(sr[i]), __uint_as_float(sr[i + 1]));
          mx1 = fmax3(mx1, __uint_as_float(sr[i + 2]), __uint_as_float(sr[i + 3]));
          mx2 = fmax3(mx2, __uint_as_float(sr[i + 4]), __uint_as_float(sr[i + 5]));
          mx3 = fmax3(mx3, __uint_as_float(sr[i + 6]), __uint_as_float(sr[i + 7]));
        }
        const float m_cand = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3)) * sl2;
        // move the max (and rescale O) only when it grows by more than 8 in log2 units
        const bool grow_m = (j == 0) || (m_cand > m + 8.0f);
        const bool rescale = j > 0 && __any_sync(0xffffffffu, grow_m);
        const float alpha = (j > 0 && grow_m) ? ex2_approx(m - m_cand) : 1.f;
        if (grow_m) m = m_cand;
        // P_X and O_X are touched once the previous step's P V has completed
        if (j > 0 && !__all_sync(0xffffffffu, mbar_wait(&pv_done[x], (c - 1) & 1, p.err, 208))) return false;
        tc_fence_after();
        float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 32; i += 4) {
            const float a0 = ex2_approx(fmaf(__uint_as_float(sr[cc * 32 + i]), sl2, -m));
            const float a1 = ex2_approx(fmaf(__uint_as_float(sr[cc * 32 + i + 1]), sl2, -m));
            const float a2 = ex2_approx(fmaf(__uint_as_float(sr[cc * 32 + i + 2]), sl2, -m));
            const float a3 = ex2_approx(fmaf(__uint_as_float(sr[cc * 32 + i + 3]), sl2, -m));
            s0 += a0;
            s1 += a1;
            s2 += a2;
            s3 += a3;
            pk[i / 2] = pack_bf16x2(a0, a1);
            pk[i / 2 + 1] = pack_bf16x2(a2, a3);
          }
          tmem_st16(tP + cc * 16, pk);
        }
        if (rescale) {  // O *= 2^(m_old - m_new) on the rows whose max moved (before this P V)
          uint32_t o[64];
          tmem_ld32(tO, *reinterpret_cast<uint32_t(*)[32]>(o));
          tmem_ld32(tO + 32, *reinterpret_cast<uint32_t(*)[32]>(o + 32));
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 64; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) tmem_st16(tO + 16 * q4, *reinterpret_cast<const uint32_t(*)[16]>(o + 16 * q4));
        }
        l *= alpha;
        l += (s0 + s1) + (s2 + s3);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&p_ready[x]);
      }
      // epilogue: O / l -> bf16 rows, lse = (m + log2 l) * ln 2
      if (!__all_sync(0xffffffffu, mbar_wait(&pv_done[x], (c - 1) & 1, p.err, 209))) return false;
      tc_fence_after();
      uint32_t o[64];
      tmem_ld32(tO, *reinterpret_cast<uint32_t(*)[32]>(o));
      tmem_ld32(tO + 32, *reinterpret_cast<uint32_t(*)[32]>(o + 32));
      tmem_wait_ld();
      tc_fence_before();
      // O rows -> swizzled staging tile -> one TMA store (rows past T are clipped)
      const float inv = 1.f / l;
      uint8_t* stg = sO + x * AT_TILE_BYTES;
      if (leader && !first_store) bulk_wait_read0();  // the previous store has read the staging tile
      if (!wg_sync()) return false;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const uint32_t* src = o + 8 * k;
        uint4 u;
        u.x = pack_bf16x2(__uint_as_float(src[0]) * inv, __uint_as_float(src[1]) * inv);
        u.y = pack_bf16x2(__uint_as_float(src[2]) * inv, __uint_as_float(src[3]) * inv);
        u.z = pack_bf16x2(__uint_as_float(src[4]) * inv, __uint_as_float(src[5]) * inv);
        u.w = pack_bf16x2(__uint_as_float(src[6]) * inv, __uint_as_float(src[7]) * inv);
        *reinterpret_cast<uint4*>(stg + row * 128 + ((k ^ (row & 7)) << 4)) = u;
      }
      fence_proxy_async_smem();
      if (!wg_sync()) return false;
      const int b = bh / p.NH, h = bh % p.NH;
      if (leader) {
        store_tile(maps.o, stg, b, h, t * AT_TILE);
        bulk_commit();
      }
      first_store = false;
      const int grow = t * AT_TILE + row;
      if (grow < p.T) p.lse[(int64_t)bh * p.T + grow] = (m + __log2f(l)) * LN2;
      return true;
    });
  }
  if (warp >= 2 && (warp & 3) == 2 && lane == 0) bulk_wait0();  // epilogue stores done with smem
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, FA_TMEM_COLS);
  }
}

// ==========================================================================================
// host side
// ==========================================================================================
bool tc_fwd_supported(int D, int dtype) { return D == AT_D && dtype == ATTN_BF16; }

int attn_fwd_tc(const void* q, const void* k, const void* v, void* o, float* lse, int B, int NH, int T,
                int D, const int64_t* s, float scale, cudaStream_t stream) {
  (void)D;
  if (!head_strides_ok(s[0], s[1], s[2]) || !head_strides_ok(s[3], s[4], s[5]) || !aligned(q, 16) || !aligned(k, 16) ||
      !aligned(v, 16) || !aligned(o, 16)) {
    set_error("attn_fwd: the tensor-core path needs 16-byte aligned bf16 tensors with strides that are "
              "multiples of 8 elements");
    return ATTN_ERR_ARG;
  }
  FwdMaps maps;
  if (!make_head_map(&maps.q, q, B, NH, T, s[0], s[1], s[2]) ||
      !make_head_map(&maps.k, k, B, NH, T, s[0], s[1], s[2]) ||
      !make_head_map(&maps.v, v, B, NH, T, s[0], s[1], s[2]) ||
      !make_head_map(&maps.o, o, B, NH, T, s[3], s[4], s[5]))
    return ATTN_ERR_CUDA;
  FwdParams p;
  p.NH = NH;
  p.T = T;
  p.nq = (T + AT_TILE - 1) / AT_TILE;
  p.n_items = (p.nq + 1) / 2;
  p.n_units = (p.n_items + 1) / 2;
  p.BH = B * NH;
  p.scale_log2 = scale * LOG2E;
  p.o = reinterpret_cast<__nv_bfloat16*>(o);
  p.o_sb = s[3];
  p.o_st = s[4];
  p.o_sh = s[5];
  p.lse = lse;
  p.err = dev_error_ptr();
  if (!p.err) return ATTN_ERR_CUDA;
  static uint64_t attr_done = 0;
  if (!set_smem_limit_once(attn_fwd_tc_kernel, FA_SMEM, attr_done)) return ATTN_ERR_CUDA;
  const int64_t units = (int64_t)p.BH * p.n_units;
  const int sms = current_device_sms();
  const int grid = (int)(units < sms ? units : sms);
  attn_fwd_tc_kernel<<<grid, FA_THREADS, FA_SMEM, stream>>>(maps, p);
  count_launch();
  return check_launch("attn_fwd_tc_kernel");
}

}  // namespace attn
