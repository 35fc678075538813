// tcgen05 tensor-core causal attention forward for head_dim a multiple of 8 up to 64 (64-wide
// tiles; TMA zero-fills the columns of narrower heads), bf16 operands, fp32 accumulation.
//
// Replaces fused_attention_forward_kernel (core/mha_kernels.py:404-521).  A persistent kernel:
// one CTA per SM walks a static list of work units (below).  Inside a CTA two
// independent streams X = 0, 1 each process a list of 128-row query tiles; every stream has its
// own TMA thread, MMA thread, softmax warpgroup, Q slots, K and V rings and TMEM columns, so one
// stream's epilogue or short diagonal tile never stalls the other, and the two softmax
// warpgroups keep the special-function units of every SM sub-partition busy between them.
//
// Work is handed out in units of two query tiles (nq-1-k, k) of one head, which cost nq+1 key
// blocks together (the middle tile of an odd count is a unit of its own); a CTA's units alternate
// between its two streams.  When that leaves fewer than eight units per stream (few heads, long
// sequences), whole units would leave the last round part-empty, so the units are then single
// query tiles taken longest first (all heads' last tile, then the one before, ...).
//
//   TMA thread     Q of the tile (the next tile's Q is fetched while this tile streams), then
//                  K_j and V_j for the key blocks j = 0 .. t into two-stage rings (K and V are
//                  released separately: K after S, V after P V)
//   MMA thread     S(j) = Q K_j^T (A and B from shared memory, fp32 in TMEM) as soon as softmax
//                  has loaded S(j-1), then O += P(j-1) V_{j-1} (A = P from TMEM, B = V MN-major)
//   softmax        one query row per thread: the row of S is read from TMEM once (128 columns)
//                  and S released at once, so S(j+1) runs on the tensor core while this step
//                  exponentiates; causal mask on the diagonal block only, row max,
//                  2^(s*scale*log2e - m) packed to bf16 in registers, row sum; P then goes to
//                  TMEM as soon as the previous P V has read it.  The running max is only moved
//                  (and O rescaled in TMEM) when it grows by more than 2^8, so rescaling is rare.
//                  Epilogue: O / l through a swizzled staging tile and one TMA store; the row's
//                  log-sum-exp is written instead of the T x T probabilities.
//
// TMEM columns of stream X: S [256X, 256X+128), P [256X+128, +64), O [256X+192, +64).
//
// Every mbarrier wait is bounded (tc_common.cuh): a wait that gives up sets the library's device
// error word and the kernel skips its remaining work instead of hanging.
#include "attn_tc_common.cuh"

#include <math.h>

namespace attn {

// Three warpgroups: 0 = TMA 0, MMA 0, TMA 1, MMA 1 (one warp each); 1 = softmax of stream 0;
// 2 = softmax of stream 1.  Launched at 168 registers per thread (the most a 384-thread CTA can
// have); warpgroup 0 gives registers back to the softmax warpgroups: per SM sub-partition (one
// warp of each warpgroup) FA_REG_LOW + 2 * FA_REG_SOFT <= 3 x 168.
constexpr int FA_THREADS = 384;
constexpr int FA_LAUNCH_REGS = 168;  // registers per thread at launch (384 threads); checked on the host
constexpr int FA_REG_LOW = 56, FA_REG_SOFT = 224;
static_assert(FA_REG_LOW + 2 * FA_REG_SOFT <= 3 * FA_LAUNCH_REGS, "register split exceeds the launch allocation");
constexpr uint32_t FA_TMEM_COLS = 512;
constexpr uint32_t FA_TM_S = 0, FA_TM_P = 128, FA_TM_O = 192, FA_TM_STREAM = 256;
constexpr int FA_STREAM_BYTES = 7 * AT_TILE_BYTES;  // Q[2], K[2], V[2], O staging
constexpr int FA_BAR_BYTES = 512;
constexpr int FA_SMEM = 1024 + 2 * FA_STREAM_BYTES + FA_BAR_BYTES;

struct FwdMaps {
  TileMap q, k, v, o;
};

struct FwdParams {
  int NH, T, nq, npairs, BH;  // npairs = ceil(nq / 2) units per head
  float scale_log2;
  float* lse;
  int* err;
};

// The tiles of one stream, in the order all of the stream's roles visit them.  Work is cut into
// units w = (head bh, pair k): query tiles nq-1-k and k of that head (the middle tile alone when
// nq is odd), nq+1 key blocks per full pair; or, with SINGLES (a template parameter, so the pair
// walk compiles as it would alone), units w = single tiles ordered by cost, tile nq-1-(w / BH) of
// head w % BH.  The CTA takes units w = blockIdx.x + n*gridDim.x;
// stream X takes its n = X, X+2, X+4, ...
template <bool SINGLES>
struct TileWalk {
  int n, second;  // unit index within the CTA, and which tile of the unit
  int bh, t;
  __device__ __forceinline__ bool valid(const FwdParams& p) const { return bh < p.BH; }
  __device__ __forceinline__ void set(const FwdParams& p) {
    const int w = blockIdx.x + n * gridDim.x;
    if constexpr (SINGLES) {
      const int level = w / p.BH;
      t = p.nq - 1 - level;
      bh = level < p.nq ? w - level * p.BH : p.BH;  // past the last tile: not valid
      return;
    }
    bh = w / p.npairs;
    const int k = w - bh * p.npairs;
    t = second ? k : p.nq - 1 - k;
  }
  __device__ __forceinline__ void start(const FwdParams& p, int X) {
    n = X;
    second = 0;
    set(p);
  }
  __device__ __forceinline__ void next(const FwdParams& p, int) {
    if (!SINGLES && !second && t != p.nq - 1 - t) {
      second = 1;  // the pair's short tile
    } else {
      second = 0;
      n += 2;
    }
    set(p);
  }
};

struct StreamBars {
  uint64_t q_full[2], q_empty[2], k_full[2], k_empty[2], v_full[2], v_empty[2];
  uint64_t s_full, s_free, p_ready, pv_done, wg_bar;
};
static_assert(2 * sizeof(StreamBars) + 16 <= FA_BAR_BYTES, "barrier area too small");

template <bool SINGLES, bool TF32>
__global__ void __launch_bounds__(FA_THREADS, 1)
attn_fwd_tc_kernel(const __grid_constant__ FwdMaps maps, const FwdParams p) {
  using TileWalk = attn::TileWalk<SINGLES>;
  extern __shared__ uint8_t smem_raw[];
  const WaitErr werr = wait_err(p.err);
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  StreamBars* sbars = reinterpret_cast<StreamBars*>(smem + 2 * FA_STREAM_BYTES);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sbars + 2);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int x = 0; x < 2; ++x) {
      StreamBars& b = sbars[x];
      for (int s = 0; s < 2; ++s) {
        mbar_init(&b.q_full[s], 1);
        mbar_init(&b.q_empty[s], 1);
        mbar_init(&b.k_full[s], 1);
        mbar_init(&b.k_empty[s], 1);
        mbar_init(&b.v_full[s], 1);
        mbar_init(&b.v_empty[s], 1);
      }
      mbar_init(&b.s_full, 1);
      mbar_init(&b.s_free, 128);
      mbar_init(&b.p_ready, 128);
      mbar_init(&b.pv_done, 1);
      mbar_init(&b.wg_bar, 128);
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
  grid_dependency_wait();    // Q, K, V (and dO, lse, delta) are complete
  grid_dependents_launch();  // the next kernel's CTAs may take SMs as this grid's CTAs leave

  if (warp < 4) {
    reg_dealloc<FA_REG_LOW>();
    const int X = warp >> 1;  // warps 0, 1: stream 0; warps 2, 3: stream 1
    StreamBars& sb = sbars[X];
    uint8_t* sQ = smem + X * FA_STREAM_BYTES;  // [2]
    uint8_t* sK = sQ + 2 * AT_TILE_BYTES;      // [2]
    uint8_t* sV = sK + 2 * AT_TILE_BYTES;      // [2]
    if ((warp & 1) == 0) {
      // ---------------- TMA producer of stream X ----------------
      if (lane == 0) {
        if (X == 0) {
          tma_prefetch_desc(&maps.q.map);
          tma_prefetch_desc(&maps.k.map);
          tma_prefetch_desc(&maps.v.map);
        }
        auto load_q = [&](const TileWalk& c, int it) -> bool {
          const int qs = it & 1;
          if (!mbar_wait(&sb.q_empty[qs], ((it >> 1) & 1) ^ 1, werr, 201)) return false;
          mbar_arrive_expect_tx(&sb.q_full[qs], AT_TILE_BYTES);
          load_tile(sQ + qs * AT_TILE_BYTES, maps.q, &sb.q_full[qs], c.bh / p.NH, c.bh % p.NH, c.t * AT_TILE);
          return true;
        };
        TileWalk cur;
        cur.start(p, X);
        bool ok = !cur.valid(p) || load_q(cur, 0);
        int it = 0, kg = 0, vg = 0;
        while (ok && cur.valid(p)) {
          TileWalk nxt = cur;
          nxt.next(p, X);
          const int b = cur.bh / p.NH, h = cur.bh % p.NH;
          for (int j = 0; j <= cur.t && ok; ++j, ++kg, ++vg) {
            const int ks = kg & 1, vs = vg & 1;
            if (!mbar_wait(&sb.k_empty[ks], ((kg >> 1) & 1) ^ 1, werr, 202)) { ok = false; break; }
            mbar_arrive_expect_tx(&sb.k_full[ks], AT_TILE_BYTES);
            load_tile(sK + ks * AT_TILE_BYTES, maps.k, &sb.k_full[ks], b, h, j * AT_TILE);
            if (!mbar_wait(&sb.v_empty[vs], ((vg >> 1) & 1) ^ 1, werr, 212)) { ok = false; break; }
            mbar_arrive_expect_tx(&sb.v_full[vs], AT_TILE_BYTES);
            load_tile(sV + vs * AT_TILE_BYTES, maps.v, &sb.v_full[vs], b, h, j * AT_TILE);
            // the next tile's Q, as soon as this tile's first block is on its way
            if (j == 0 && nxt.valid(p) && !load_q(nxt, it + 1)) ok = false;
          }
          cur = nxt;
          ++it;
        }
      }
    } else {
      // ---------------- MMA issuer of stream X ----------------
      if (lane == 0 && TF32) {
        // tf32: P(j) is written over S(j)'s TMEM columns (as float32 it needs all 128), so S(j+1)
        // waits until P(j) V(j) has read them; per stream the tensor core alternates P V and S
        // while the other stream's softmax runs.  Q and K K-major (128-byte swizzle), V MN-major
        // in the 128-byte swizzle with 32-byte atomicity (the tf32 MMA's only MN-major layout).
        const uint32_t idesc_s = idesc_tf32_f32(128, 128, 0, 0);
        const uint32_t idesc_o = idesc_tf32_f32(128, AT_D / 2, 0, 1);
        const uint32_t tS = tmem + X * FA_TM_STREAM + FA_TM_S;
        const uint32_t tO = tmem + X * FA_TM_STREAM + FA_TM_O;
        int pcnt = 0;  // P V MMAs issued
        int it = 0, kg = 0, vg = 0;
        bool ok = true;
        TileWalk cur;
        for (cur.start(p, X); ok && cur.valid(p); cur.next(p, X), ++it) {
          const int qs = it & 1;
          if (!mbar_wait(&sb.q_full[qs], (it >> 1) & 1, werr, 203)) { ok = false; break; }
          const uint64_t q_desc = smem_desc_sw128(smem_u32(sQ + qs * AT_TILE_BYTES), 16, 1024);
          for (int j = 0; j <= cur.t + 1 && ok; ++j) {
            if (j > 0) {
              // O += P(j-1) V_{j-1} once softmax has written P(j-1) (and rescaled O)
              const int vs = vg & 1;
              if (!mbar_wait(&sb.v_full[vs], (vg >> 1) & 1, werr, 205)) { ok = false; break; }
              if (!mbar_wait(&sb.p_ready, pcnt & 1, werr, 211)) { ok = false; break; }
              tc_fence_after();
              const uint32_t v_addr = smem_u32(sV + vs * AT_TILE_BYTES);
#pragma unroll
              for (int k = 0; k < AT_TILE / 8; ++k)
                umma_ts_tf32(tO, tS + k * 8, smem_desc_sw128_atom32(v_addr + k * 1024, AT_TILE_BYTES, 512),
                             idesc_o, (j == 1 && k == 0) ? 0u : 1u);
              umma_commit(&sb.pv_done);
              umma_commit(&sb.v_empty[vs]);
              ++pcnt;
              ++vg;
            }
            if (j <= cur.t) {
              // S(j) = Q K_j^T over the columns of P(j-1) (or of the previous tile's last P) once
              // that P V has completed
              const int ks = kg & 1;
              if (!mbar_wait(&sb.k_full[ks], (kg >> 1) & 1, werr, 204)) { ok = false; break; }
              if (pcnt > 0 && !mbar_wait(&sb.pv_done, (pcnt - 1) & 1, werr, 213)) { ok = false; break; }
              tc_fence_after();
              const uint64_t k_desc = smem_desc_sw128(smem_u32(sK + ks * AT_TILE_BYTES), 16, 1024);
#pragma unroll
              for (int k = 0; k < AT_D / 16; ++k)
                umma_ss_tf32(tS, desc_step(q_desc, k * 32), desc_step(k_desc, k * 32), idesc_s, k > 0 ? 1u : 0u);
              umma_commit(&sb.s_full);
              umma_commit(&sb.k_empty[ks]);
              if (j == cur.t) umma_commit(&sb.q_empty[qs]);  // the tile's last S read Q
              ++kg;
            }
          }
        }
      } else if (lane == 0) {
        const uint32_t idesc_s = idesc_bf16_f32(128, 128, 0, 0);  // Q K-major, K K-major
        const uint32_t idesc_o = idesc_bf16_f32(128, 64, 0, 1);   // P from TMEM, V MN-major
        const uint32_t tS = tmem + X * FA_TM_STREAM + FA_TM_S;
        const uint32_t tP = tmem + X * FA_TM_STREAM + FA_TM_P;
        const uint32_t tO = tmem + X * FA_TM_STREAM + FA_TM_O;
        int scnt = 0, pcnt = 0;  // S and P V MMAs issued (= softmax steps started / finished)
        int it = 0, kg = 0, vg = 0;
        bool ok = true;
        TileWalk cur;
        for (cur.start(p, X); ok && cur.valid(p); cur.next(p, X), ++it) {
          const int qs = it & 1;
          if (!mbar_wait(&sb.q_full[qs], (it >> 1) & 1, werr, 203)) { ok = false; break; }
          const uint64_t q_desc = smem_desc_sw128(smem_u32(sQ + qs * AT_TILE_BYTES), 16, 1024);
          for (int j = 0; j <= cur.t + 1 && ok; ++j) {
            if (j <= cur.t) {
              // S(j) = Q K_j^T once softmax has loaded S(j-1)
              const int ks = kg & 1;
              if (!mbar_wait(&sb.k_full[ks], (kg >> 1) & 1, werr, 204)) { ok = false; break; }
              if (scnt > 0 && !mbar_wait(&sb.s_free, (scnt - 1) & 1, werr, 206)) { ok = false; break; }
              tc_fence_after();
              const uint64_t k_desc = smem_desc_sw128(smem_u32(sK + ks * AT_TILE_BYTES), 16, 1024);
#pragma unroll
              for (int k = 0; k < AT_D / 16; ++k)
                umma_ss(tS, desc_step(q_desc, k * 32), desc_step(k_desc, k * 32), idesc_s, k > 0 ? 1u : 0u);
              umma_commit(&sb.s_full);
              umma_commit(&sb.k_empty[ks]);
              if (j == cur.t) umma_commit(&sb.q_empty[qs]);  // the tile's last S read Q
              ++scnt;
              ++kg;
            }
            if (j > 0) {
              // O += P(j-1) V_{j-1} once softmax has written P(j-1) (and rescaled O)
              const int vs = vg & 1;
              if (!mbar_wait(&sb.v_full[vs], (vg >> 1) & 1, werr, 205)) { ok = false; break; }
              if (!mbar_wait(&sb.p_ready, pcnt & 1, werr, 211)) { ok = false; break; }
              tc_fence_after();
              const uint64_t v_desc = smem_desc_sw128(smem_u32(sV + vs * AT_TILE_BYTES), 8192, 1024);
#pragma unroll
              for (int k = 0; k < AT_TILE / 16; ++k)
                umma_ts(tO, tP + k * 8, desc_step(v_desc, k * 2048), idesc_o, (j == 1 && k == 0) ? 0u : 1u);
              umma_commit(&sb.pv_done);
              umma_commit(&sb.v_empty[vs]);
              ++pcnt;
              ++vg;
            }
          }
        }
      }
    }
  } else {
    reg_alloc<FA_REG_SOFT>();
    // ---------------- softmax warpgroup of stream X (warps 4-7: X = 0, 8-11: X = 1) ----------------
    const int X = (warp - 4) >> 2;
    StreamBars& sb = sbars[X];
    uint8_t* stg = smem + X * FA_STREAM_BYTES + 6 * AT_TILE_BYTES;  // O staging tile
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t tS = tmem + X * FA_TM_STREAM + FA_TM_S + lane_off;
    const uint32_t tP = tmem + X * FA_TM_STREAM + FA_TM_P + lane_off;
    const uint32_t tO = tmem + X * FA_TM_STREAM + FA_TM_O + lane_off;
    const float sl2 = p.scale_log2;
    int c = 0;  // softmax steps done by this warpgroup
    const bool leader = (warp & 3) == 0 && lane == 0;  // first thread of the warpgroup
    bool first_store = true;
    uint32_t wg_phase = 0;
    auto wg_sync = [&]() -> bool {  // bounded barrier over the 128 threads of the warpgroup
      mbar_arrive(&sb.wg_bar);
      const bool w = mbar_wait(&sb.wg_bar, wg_phase & 1, werr, 210);
      ++wg_phase;
      return __all_sync(0xffffffffu, w);
    };
    TileWalk cur;
    for (cur.start(p, X); cur.valid(p); cur.next(p, X)) {
      const int t = cur.t;
      float m = -INFINITY, l = 0.f;
      bool ok = true;
      for (int j = 0; j <= t; ++j, ++c) {
        if (!__all_sync(0xffffffffu, mbar_wait(&sb.s_full, c & 1, werr, 207))) { ok = false; break; }
        tc_fence_after();
        uint32_t sr[128];
        tmem_ld32(tS, *reinterpret_cast<uint32_t(*)[32]>(sr));
        tmem_ld32(tS + 32, *reinterpret_cast<uint32_t(*)[32]>(sr + 32));
        tmem_ld32(tS + 64, *reinterpret_cast<uint32_t(*)[32]>(sr + 64));
        tmem_ld32(tS + 96, *reinterpret_cast<uint32_t(*)[32]>(sr + 96));
        tmem_wait_ld();
        tc_fence_before();
        if constexpr (!TF32) mbar_arrive(&sb.s_free);  // S is in registers: the next S may be computed
        if (j == t) {  // diagonal block: key column k is visible to query row r iff k <= r
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
        // P = 2^(s*scale*log2e - m), the row sum in fp32; bf16: packed in registers for the P V MMA;
        // tf32: float32 in place of S (the MMA reads its upper 19 bits)
        float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
        uint32_t pk[TF32 ? 1 : 64];
#pragma unroll
        for (int i = 0; i < 128; i += 4) {
          const float a0 = ex2_approx(fmaf(__uint_as_float(sr[i]), sl2, -m));
          const float a1 = ex2_approx(fmaf(__uint_as_float(sr[i + 1]), sl2, -m));
          const float a2 = ex2_approx(fmaf(__uint_as_float(sr[i + 2]), sl2, -m));
          const float a3 = ex2_approx(fmaf(__uint_as_float(sr[i + 3]), sl2, -m));
          s0 += a0;
          s1 += a1;
          s2 += a2;
          s3 += a3;
          if constexpr (TF32) {
            sr[i] = __float_as_uint(a0);
            sr[i + 1] = __float_as_uint(a1);
            sr[i + 2] = __float_as_uint(a2);
            sr[i + 3] = __float_as_uint(a3);
          } else {
            pk[i / 2] = pack_bf16x2(a0, a1);
            pk[i / 2 + 1] = pack_bf16x2(a2, a3);
          }
        }
        // P and O are rewritten once the previous step's P V has completed (tf32: already implied,
        // this step's S was computed after it)
        if (j > 0 && !__all_sync(0xffffffffu, mbar_wait(&sb.pv_done, (c - 1) & 1, werr, 208))) { ok = false; break; }
        tc_fence_after();
        constexpr int OC = TF32 ? AT_D / 2 : AT_D;  // O columns
        if constexpr (TF32) {
#pragma unroll
          for (int cc = 0; cc < 8; ++cc) tmem_st16(tS + cc * 16, *reinterpret_cast<const uint32_t(*)[16]>(sr + 16 * cc));
        } else {
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) tmem_st16(tP + cc * 16, *reinterpret_cast<const uint32_t(*)[16]>(pk + 16 * cc));
        }
        if (rescale) {  // O *= 2^(m_old - m_new) on the rows whose max moved (before this P V)
          uint32_t o[OC];
#pragma unroll
          for (int q = 0; q < OC / 32; ++q) tmem_ld32(tO + 32 * q, *reinterpret_cast<uint32_t(*)[32]>(o + 32 * q));
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < OC; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
#pragma unroll
          for (int q4 = 0; q4 < OC / 16; ++q4) tmem_st16(tO + 16 * q4, *reinterpret_cast<const uint32_t(*)[16]>(o + 16 * q4));
        }
        l *= alpha;
        l += (s0 + s1) + (s2 + s3);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&sb.p_ready);
      }
      if (!ok) break;
      // epilogue: O / l -> bf16 rows, lse = (m + log2 l) * ln 2
      if (!__all_sync(0xffffffffu, mbar_wait(&sb.pv_done, (c - 1) & 1, werr, 209))) break;
      tc_fence_after();
      constexpr int OC = TF32 ? AT_D / 2 : AT_D;  // O columns: 128 bytes of output per row either way
      uint32_t o[OC];
#pragma unroll
      for (int q = 0; q < OC / 32; ++q) tmem_ld32(tO + 32 * q, *reinterpret_cast<uint32_t(*)[32]>(o + 32 * q));
      tmem_wait_ld();
      tc_fence_before();
      // O rows -> swizzled staging tile -> one TMA store (rows past T are clipped)
      const float inv = 1.f / l;
      if (leader && !first_store) bulk_wait_read0();  // the previous store has read the staging tile
      if (!wg_sync()) break;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        uint4 u;
        if constexpr (TF32) {
          const uint32_t* src = o + 4 * k;
          u = make_uint4(__float_as_uint(__uint_as_float(src[0]) * inv), __float_as_uint(__uint_as_float(src[1]) * inv),
                         __float_as_uint(__uint_as_float(src[2]) * inv), __float_as_uint(__uint_as_float(src[3]) * inv));
        } else {
          const uint32_t* src = o + 8 * k;
          u.x = pack_bf16x2(__uint_as_float(src[0]) * inv, __uint_as_float(src[1]) * inv);
          u.y = pack_bf16x2(__uint_as_float(src[2]) * inv, __uint_as_float(src[3]) * inv);
          u.z = pack_bf16x2(__uint_as_float(src[4]) * inv, __uint_as_float(src[5]) * inv);
          u.w = pack_bf16x2(__uint_as_float(src[6]) * inv, __uint_as_float(src[7]) * inv);
        }
        *reinterpret_cast<uint4*>(stg + row * 128 + ((k ^ (row & 7)) << 4)) = u;
      }
      fence_proxy_async_smem();
      if (!wg_sync()) break;
      const int b = cur.bh / p.NH, h = cur.bh % p.NH;
      if (leader) {
        store_tile(maps.o, stg, b, h, t * AT_TILE);
        bulk_commit();
      }
      first_store = false;
      const int grow = t * AT_TILE + row;
      if (grow < p.T) p.lse[(int64_t)cur.bh * p.T + grow] = (m + __log2f(l)) * LN2;
    }
    if (leader) bulk_wait0();  // epilogue stores done with shared memory
  }
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
bool tc_fwd_supported(int D, int dtype) {
  return dtype == ATTN_BF16 ? tc_head_dim_ok(D) : dtype == ATTN_TF32 ? tc_head_dim_ok_tf32(D) : false;
}

// Whether n tensors with the element strides s[0..5] (input b/t/h, output b/t/h) can go through
// the TMA maps of the tensor-core kernels: 16-byte aligned bases, strides in 16-byte steps.
bool tc_attn_layout_ok(const void* const* ptrs, int n, const int64_t* s, int D, int esz) {
  auto ok = [&](int64_t sb, int64_t st, int64_t sh) {
    return esz == 4 ? head_strides_ok_f32(sb, st, sh, D) : head_strides_ok(sb, st, sh, D);
  };
  if (!ok(s[0], s[1], s[2]) || !ok(s[3], s[4], s[5])) return false;
  for (int i = 0; i < n; ++i)
    if (!aligned(ptrs[i], 16)) return false;
  return true;
}

// tf32 != 0: float32 q/k/v/o (head_dim <= 32) multiplied as tf32; otherwise bf16 (head_dim <= 64).
int attn_fwd_tc(const void* q, const void* k, const void* v, void* o, float* lse, int B, int NH, int T,
                int D, const int64_t* s, float scale, cudaStream_t stream, int tf32) {
  const void* tens[4] = {q, k, v, o};
  if (!tc_attn_layout_ok(tens, 4, s, D, tf32 ? 4 : 2)) {
    set_error("attn_fwd: the tensor-core path needs 16-byte aligned tensors with strides in 16-byte steps");
    return ATTN_ERR_ARG;
  }
  FwdMaps maps;
  if (tf32) {
    if (!make_head_map_f32(&maps.q, q, B, NH, T, D, s[0], s[1], s[2], 128) ||
        !make_head_map_f32(&maps.k, k, B, NH, T, D, s[0], s[1], s[2], 128) ||
        !make_head_map_f32(&maps.v, v, B, NH, T, D, s[0], s[1], s[2], SWIZZLE_128B_ATOM32) ||
        !make_head_map_f32(&maps.o, o, B, NH, T, D, s[3], s[4], s[5], 128))
      return ATTN_ERR_CUDA;
  } else if (!make_head_map(&maps.q, q, B, NH, T, D, s[0], s[1], s[2]) ||
             !make_head_map(&maps.k, k, B, NH, T, D, s[0], s[1], s[2]) ||
             !make_head_map(&maps.v, v, B, NH, T, D, s[0], s[1], s[2]) ||
             !make_head_map(&maps.o, o, B, NH, T, D, s[3], s[4], s[5])) {
    return ATTN_ERR_CUDA;
  }
  FwdParams p;
  p.NH = NH;
  p.T = T;
  p.nq = (T + AT_TILE - 1) / AT_TILE;
  p.npairs = (p.nq + 1) / 2;
  p.BH = B * NH;
  p.scale_log2 = scale * LOG2E;
  p.lse = lse;
  p.err = dev_error_ptr();
  if (!p.err) return ATTN_ERR_CUDA;
  const int sms = current_device_sms();
  const bool singles = (int64_t)p.BH * p.npairs < (int64_t)8 * 2 * sms;
  const int64_t units = (int64_t)p.BH * (singles ? p.nq : p.npairs);
  const int grid = (int)((units + 1) / 2 < sms ? (units + 1) / 2 : sms);  // at least a unit per stream
  static CtxOnce attr[4];
  static int regs[4] = {0, 0, 0, 0};
  cudaError_t launched = cudaSuccess;
#define FA_LAUNCH(SG, TF, slot)                                                                          \
  do {                                                                                                   \
    if (!set_smem_limit_once(attn_fwd_tc_kernel<SG, TF>, FA_SMEM, attr[slot]) ||                         \
        !launch_regs_match(attn_fwd_tc_kernel<SG, TF>, FA_LAUNCH_REGS, regs[slot], "attn_fwd_tc_kernel")) \
      return ATTN_ERR_CUDA;                                                                              \
    launched = launch_pdl(attn_fwd_tc_kernel<SG, TF>, dim3(grid), dim3(FA_THREADS), FA_SMEM, stream, maps, p); \
  } while (0)
  if (singles && tf32)
    FA_LAUNCH(true, true, 3);
  else if (singles)
    FA_LAUNCH(true, false, 1);
  else if (tf32)
    FA_LAUNCH(false, true, 2);
  else
    FA_LAUNCH(false, false, 0);
#undef FA_LAUNCH
  count_launch();
  return check_launch("attn_fwd_tc_kernel", launched);
}

}  // namespace attn
