// tcgen05 causal attention backward for head_dim a multiple of 8 up to 64 (64-wide tiles; TMA
// zero-fills the columns of narrower heads), bf16 operands, fp32 accumulation.
//
// Replaces the NumPy backward of model/gpt.py:669-680 (and the unwired GPU kernels
// softmax_fused_backward / matmul_grad_{q,k,v}, core/mha_kernels.py:195-236, 592-680):
//   dV = P^T dO,  dP = dO V^T,  dS = P (dP - rowsum(dP P)) * scale,  dQ = dS K,  dK = dS^T Q
// with rowsum(dP P) = rowsum(dO O) = delta (model/gpt.py:675-677), and P recomputed from the
// forward's log-sum-exp instead of being stored.  The softmax scale is applied when dQ and dK are
// written out (both are linear in dS).
//
// 1. attn_bwd_prep_kernel: delta = rowsum(dO * O) and lse in log2 units, both padded to whole
//    128-row tiles (padding rows get lse = +inf so their probabilities are exactly 0).
// 2. attn_bwd_tc_kernel, persistent: one CTA per SM walks the heads (b, h) assigned to it; for
//    each head it visits the 128-key tiles jt = nq-1 .. 0, keeps K_jt, V_jt and the dK/dV
//    accumulators resident and streams the query tiles i = jt .. nq-1 that can see those keys:
//      TMA warps      K/V per key tile (two stages), Q and lse2 per query tile (three stages),
//                     dO and delta per query tile (two stages)
//      MMA thread     S^T = K Q_i^T and dP^T = V dO_i^T (128 x 128 each) into TMEM;
//                     dV += P^T dO_i and dK += dS^T Q_i with P^T, dS^T read from TMEM;
//                     dQ_i(partial) = dS K with dS read from shared memory
//      8 P/dS warps   one key row per thread and 64 of the 128 queries per warpgroup:
//                     P^T = 2^(S^T*scale*log2e - lse2) into its own TMEM columns (so S^T of the
//                     next tile can be computed while dS is formed), dS^T = P^T (dP^T - delta)
//                     to TMEM over the dP^T columns already read and to shared memory for dQ
//                     (two dS buffers, so tile n's dS never waits for tile n-1's dQ MMA)
//      4 drain warps  per tile: the dQ partial from TMEM to a per-CTA fp32 accumulator (a TMA
//                     store from the diagonal key tile, which reaches a query tile first, TMA
//                     reduce-adds after it, all into L2-resident memory); for key tile 0 (each
//                     query tile's last contribution) the accumulator row is read back, the
//                     partial added, and scale * dQ written as bf16.  Per key tile: dK (times
//                     scale) and dV out.
//    Because one CTA owns a head, the dQ accumulator needs no zeroing and no atomics between
//    CTAs, and no separate conversion pass.
//    TMEM: S^T [0,128), dP^T / dS^T [128,256), P^T [256,320), dV [320,384), dK [384,448),
//    dQ [448,512).
//
// Every mbarrier wait is bounded (tc_common.cuh): a wait that gives up sets the library's device
// error word and the kernel skips its remaining work instead of hanging.
#include "attn_tc_common.cuh"

#include <math.h>

namespace attn {

// Four warpgroups: 0 = TMA for K/V (warp 0), MMA (warp 1), TMA for Q and lse2 (warp 2), TMA for dO
// and delta (warp 3); 1-2 = P/dS; 3 = drain.
// Launched at 128 registers per thread (512 threads); warpgroup 0 gives registers back so the
// P/dS warpgroups can hold more: per SM sub-partition (one warp of each warpgroup)
// BA_REG_LOW + 2 * BA_REG_PDS + 128 <= 4 x 128.
constexpr int BA_THREADS = 512;
constexpr int BA_LAUNCH_REGS = 128;  // registers per thread at launch (512 threads); checked on the host
constexpr int BA_REG_LOW = 96, BA_REG_PDS = 144;
static_assert(BA_REG_LOW + 2 * BA_REG_PDS + BA_LAUNCH_REGS <= 4 * BA_LAUNCH_REGS,
              "register split exceeds the launch allocation");
constexpr uint32_t BA_TMEM_COLS = 512;
constexpr uint32_t BA_TM_S = 0, BA_TM_DP = 128, BA_TM_P = 256, BA_TM_DV = 320, BA_TM_DK = 384, BA_TM_DQ = 448;
constexpr int BA_MAX_CTAS = 160;  // the dQ accumulator workspace is sized for this many CTAs
// Q (+ lse2) has three stages: S^T(n+1) reads Q(n+1) while dK(n-1) may still read Q(n-1).  dO
// (+ delta) has two: dP^T(n+1) comes late in tile n+1, after dV(n) and dK(n), the last readers of
// the stage it reuses.  With two dS^T buffers that fills shared memory with no room for an
// alignment pad; the kernel checks that the dynamic shared memory starts 1024-byte aligned.
constexpr int BA_QS = 3, BA_OS = 2;
constexpr int BA_SMEM = 4 * AT_TILE_BYTES /*K,V x2*/ + (BA_QS + BA_OS) * AT_TILE_BYTES /*Q, dO*/ +
                        4 * AT_TILE_BYTES /*dS^T, two buffers*/ + AT_TILE * 128 /*dQ staging, half a tile*/ +
                        (BA_QS + BA_OS) * AT_TILE * 4 /*lse2, delta*/ + 256;
static_assert(BA_SMEM <= 232448, "over the per-block shared memory limit");
constexpr int BA_SITE_SMEM_ALIGN = 300;  // error site: dynamic shared memory not 1024-byte aligned

struct BwdMaps {
  TileMap q, k, v, dout;
  CUtensorMap dq_acc;  // fp32 [grid * Tp rows][64], box 32 x 128, 128B swizzle
};

struct BwdParams {
  int NH, T, nq, Tp, BH, D;  // D = head_dim (<= 64; the tiles are 64 wide)
  float scale, scale_log2;
  const float* lse2;    // [BH][Tp] lse * log2 e (+inf on padding rows)
  const float* delta;   // [BH][Tp]
  float* dq_acc;        // [gridDim.x][Tp][64]
  __nv_bfloat16 *dq, *dk, *dv;
  int64_t sb, st, sh;   // strides of dq/dk/dv (same as q/k/v)
  int* err;
};

// Eight lanes per row: lane c of a row reads the row's 16-byte pieces c (O and dO), so a row's 128
// bytes of each are read by one coalesced request; the partial dot products meet by shuffles.
// Grid (BH, Tp / 32), 256 threads: a block covers 32 rows of one head, so no thread divides a
// flat row index.
__global__ void attn_bwd_prep_kernel(const __nv_bfloat16* __restrict__ o,
                                     const __nv_bfloat16* __restrict__ dout,
                                     const float* __restrict__ lse, float* __restrict__ lse2,
                                     float* __restrict__ delta, int NH, int T, int Tp, int D,
                                     int64_t o_sb, int64_t o_st, int64_t o_sh) {
  grid_dependency_wait();  // O and dO are complete
  grid_dependents_launch();
  const int bh = blockIdx.x;
  const int t = blockIdx.y * 32 + (threadIdx.x >> 3);  // < Tp
  const int c = threadIdx.x & 7;
  float acc = 0.f;
  if (t < T && c < D / 8) {
    const int b = bh / NH, h = bh - b * NH;
    const int64_t off = b * o_sb + (int64_t)t * o_st + (int64_t)h * o_sh;
    const uint4 a = __ldg(reinterpret_cast<const uint4*>(o + off) + c);
    const uint4 g = __ldg(reinterpret_cast<const uint4*>(dout + off) + c);
    const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, gw[4] = {g.x, g.y, g.z, g.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 fa = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&aw[i]));
      const float2 fg = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&gw[i]));
      acc = fmaf(fa.x, fg.x, acc);
      acc = fmaf(fa.y, fg.y, acc);
    }
  }
  acc += __shfl_xor_sync(0xffffffffu, acc, 1);
  acc += __shfl_xor_sync(0xffffffffu, acc, 2);
  acc += __shfl_xor_sync(0xffffffffu, acc, 4);
  if (c != 0) return;
  const int64_t idx = (int64_t)bh * Tp + t;
  if (t >= T) {
    lse2[idx] = INFINITY;  // padding rows: P = 2^(s - inf) = 0
    delta[idx] = 0.f;
    return;
  }
  delta[idx] = acc;
  lse2[idx] = lse[(int64_t)bh * T + t] * LOG2E;
}

__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Wait until at most n of this thread's most recent bulk groups are pending (n clamped to 7).
__device__ __forceinline__ void bulk_wait_upto(int n) {
  switch (n) {
    case 0: asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); break;
    case 1: asm volatile("cp.async.bulk.wait_group 1;" ::: "memory"); break;
    case 2: asm volatile("cp.async.bulk.wait_group 2;" ::: "memory"); break;
    case 3: asm volatile("cp.async.bulk.wait_group 3;" ::: "memory"); break;
    case 4: asm volatile("cp.async.bulk.wait_group 4;" ::: "memory"); break;
    case 5: asm volatile("cp.async.bulk.wait_group 5;" ::: "memory"); break;
    case 6: asm volatile("cp.async.bulk.wait_group 6;" ::: "memory"); break;
    default: asm volatile("cp.async.bulk.wait_group 7;" ::: "memory"); break;
  }
}

// 64 fp32 values (two TMEM loads of 32 columns) times `mul` -> 32 packed bf16 pairs.
__device__ __forceinline__ void pack_row_bf16(uint32_t (&out)[32], const uint32_t (&a0)[32],
                                              const uint32_t (&a1)[32], float mul) {
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    out[j] = pack_bf16x2(__uint_as_float(a0[2 * j]) * mul, __uint_as_float(a0[2 * j + 1]) * mul);
    out[16 + j] = pack_bf16x2(__uint_as_float(a1[2 * j]) * mul, __uint_as_float(a1[2 * j + 1]) * mul);
  }
}

// The first D of 64 packed bf16 values (32 pairs) -> D/8 x 16 B at dst (one head row).
__device__ __forceinline__ void store_packed_row(__nv_bfloat16* dst, const uint32_t (&w)[32], int D) {
#pragma unroll
  for (int c = 0; c < 8; ++c)
    if (c < D / 8)
      reinterpret_cast<uint4*>(dst)[c] = make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
}

__global__ void __launch_bounds__(BA_THREADS, 1)
attn_bwd_tc_kernel(const __grid_constant__ BwdMaps maps, const BwdParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const WaitErr werr = wait_err(p.err);
  if (smem_u32(smem_raw) & 1023u) {  // the swizzled tiles need it; uniform, so every thread leaves
    if (threadIdx.x == 0) record_wait_error(werr, BA_SITE_SMEM_ALIGN);
    return;
  }
  uint8_t* smem = smem_raw;
  uint8_t* sK = smem;                          // [2]
  uint8_t* sV = sK + 2 * AT_TILE_BYTES;        // [2]
  uint8_t* sQ = sV + 2 * AT_TILE_BYTES;        // [BA_QS]
  uint8_t* sDO = sQ + BA_QS * AT_TILE_BYTES;   // [BA_OS]
  uint8_t* sDS = sDO + BA_OS * AT_TILE_BYTES;  // dS^T [2 buffers]: two 64-query blocks of [128 keys][64]
  uint8_t* sDQ = sDS + 4 * AT_TILE_BYTES;      // dQ staging: one [128 q][32 fp32] swizzled half
  float* sLse = reinterpret_cast<float*>(sDQ + AT_TILE * 128);  // [BA_QS][128]
  float* sDelta = sLse + BA_QS * AT_TILE;                           // [BA_OS][128]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sDelta + BA_OS * AT_TILE);
  uint64_t* kv_full = bars;           // [2] per key tile (unit)
  uint64_t* kv_empty = kv_full + 2;   // [2]
  uint64_t* q_full = kv_empty + 2;    // [BA_QS] per query tile
  uint64_t* q_empty = q_full + BA_QS; // [BA_QS]
  uint64_t* o_full = q_empty + BA_QS; // [BA_OS] per query tile: dO and delta
  uint64_t* o_empty = o_full + BA_OS; // [BA_OS]
  uint64_t* s_full = o_empty + BA_OS; // S^T in TMEM
  uint64_t* dp_full = s_full + 1;     // dP^T in TMEM
  uint64_t* p_ready = dp_full + 1;    // S^T read, P^T written (256 arrivals)
  uint64_t* dv_done = p_ready + 1;    // the dV MMA reading P^T has completed
  uint64_t* ds_ready = dv_done + 1;   // dP^T read, dS^T written to TMEM and smem (256 arrivals)
  uint64_t* dk_done = ds_ready + 1;   // the dK MMA reading dS^T from TMEM has completed
  uint64_t* ds_free = dk_done + 1;    // [2] the dQ MMA reading that dS^T buffer has completed
  uint64_t* dq_full = ds_free + 2;
  uint64_t* dq_free = dq_full + 1;    // 128 arrivals
  uint64_t* dkdv_full = dq_free + 1;
  uint64_t* dkdv_free = dkdv_full + 1;  // 128 arrivals
  uint64_t* drain_bar = dkdv_free + 1;  // 128 arrivals: sync of the drain warpgroup
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int nq = p.nq;

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int s = 0; s < BA_QS; ++s) {
      mbar_init(&q_full[s], 1);
      mbar_init(&q_empty[s], 1);
    }
    for (int s = 0; s < BA_OS; ++s) {
      mbar_init(&o_full[s], 1);
      mbar_init(&o_empty[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(dp_full, 1);
    mbar_init(p_ready, 256);
    mbar_init(dv_done, 1);
    mbar_init(ds_ready, 256);
    mbar_init(dk_done, 1);
    mbar_init(&ds_free[0], 1);
    mbar_init(&ds_free[1], 1);
    mbar_init(dq_full, 1);
    mbar_init(dq_free, 128);
    mbar_init(dkdv_full, 1);
    mbar_init(dkdv_free, 128);
    mbar_init(drain_bar, 128);
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
  grid_dependency_wait();    // Q, K, V (and dO, lse, delta) are complete
  grid_dependents_launch();  // the next kernel's CTAs may take SMs as this grid's CTAs leave

  if (warp < 4) {  // TMA producers, MMA issuer
    reg_dealloc<BA_REG_LOW>();
    if (warp == 0) {
      // ---------------- TMA producer: K/V per key tile ----------------
      if (lane == 0) {
        tma_prefetch_desc(&maps.k.map);
        tma_prefetch_desc(&maps.v.map);
        int u = 0;
        bool ok = true;
        for (int bh = blockIdx.x; bh < p.BH && ok; bh += gridDim.x) {
          const int b = bh / p.NH, h = bh % p.NH;
          for (int jt = nq - 1; jt >= 0; --jt, ++u) {
            const int ks = u & 1;
            if (!mbar_wait(&kv_empty[ks], ((u >> 1) & 1) ^ 1, werr, 301)) { ok = false; break; }
            mbar_arrive_expect_tx(&kv_full[ks], 2 * AT_TILE_BYTES);
            load_tile(sK + ks * AT_TILE_BYTES, maps.k, &kv_full[ks], b, h, jt * AT_TILE);
            load_tile(sV + ks * AT_TILE_BYTES, maps.v, &kv_full[ks], b, h, jt * AT_TILE);
          }
        }
      }
    } else if (warp == 2 || warp == 3) {
      // ---------------- TMA producers per query tile (run ahead of K/V): warp 2 Q and lse2 into the
      // Q stages, warp 3 dO and delta into the dO stages ----------------
      if (lane == 0) {
        const bool isq = (warp == 2);
        const TileMap& map = isq ? maps.q : maps.dout;
        const float* vec = isq ? p.lse2 : p.delta;
        uint8_t* tiles = isq ? sQ : sDO;
        float* vecs = isq ? sLse : sDelta;
        uint64_t* full = isq ? q_full : o_full;
        uint64_t* empty = isq ? q_empty : o_empty;
        const int nst = isq ? BA_QS : BA_OS;
        tma_prefetch_desc(&map.map);
        int n = 0;
        bool ok = true;
        for (int bh = blockIdx.x; bh < p.BH && ok; bh += gridDim.x) {
          const int b = bh / p.NH, h = bh % p.NH;
          for (int jt = nq - 1; jt >= 0 && ok; --jt) {
            for (int i = jt; i < nq; ++i, ++n) {
              const int s = n % nst;
              if (!mbar_wait(&empty[s], ((n / nst) & 1) ^ 1, werr, isq ? 302 : 318)) { ok = false; break; }
              const int q0 = i * AT_TILE;
              mbar_arrive_expect_tx(&full[s], AT_TILE_BYTES + AT_TILE * 4);
              load_tile(tiles + s * AT_TILE_BYTES, map, &full[s], b, h, q0);
              bulk_load(vecs + s * AT_TILE, vec + (int64_t)bh * p.Tp + q0, AT_TILE * 4, &full[s]);
            }
          }
        }
      }
    } else if (warp == 1) {
      // ---------------- MMA issuer ----------------
      if (lane == 0) {
        const uint32_t idesc_sdp = idesc_bf16_f32(128, 128, 0, 0);  // K/V and Q/dO all K-major
        const uint32_t idesc_kv = idesc_bf16_f32(128, 64, 0, 1);    // A from TMEM, B MN-major
        const uint32_t idesc_q = idesc_bf16_f32(128, 64, 1, 1);     // A = dS (MN-major), B = K MN-major
        const uint32_t tS = tmem + BA_TM_S, tdP = tmem + BA_TM_DP, tP = tmem + BA_TM_P;
        const uint32_t tdV = tmem + BA_TM_DV, tdK = tmem + BA_TM_DK, tdQ = tmem + BA_TM_DQ;
        // shared-memory descriptors: K-major (row = 64 elements of the contraction) and MN-major
        // (row = 64 output columns), built per use from the stage's base address
        auto kmaj = [](const uint8_t* t) { return smem_desc_sw128(smem_u32(t), 16, 1024); };
        auto mnmaj = [](const uint8_t* t) { return smem_desc_sw128(smem_u32(t), 8192, 1024); };
        // The previous tile's dV and dK are issued after this tile's S^T, which goes to the tensor
        // core as soon as the P/dS warps have read the previous S^T; then this tile's dP^T (it only
        // waits for the dK MMA, which reads the dS^T columns dP^T overwrites), and the previous
        // tile's dQ last: it reads its own dS buffer in shared memory, so the P/dS warps get dP^T
        // early and can write the next dS into the other buffer meanwhile.
        int pn = -1, ps = 0, pso = 0, pks = 0, pu = 0;
        bool pfirst = false, plast = false;
        auto finish_dvdk = [&]() -> bool {
          // dV += P^T dO   (the first tile of a key tile starts dV/dK afresh once they are drained)
          if (pfirst && !mbar_wait(dkdv_free, (pu & 1) ^ 1, werr, 308)) return false;
          tc_fence_after();
          const uint64_t do_mn = mnmaj(sDO + pso * AT_TILE_BYTES);
  #pragma unroll
          for (int k = 0; k < AT_TILE / 16; ++k)
            umma_ts(tdV, tP + k * 8, desc_step(do_mn, k * 2048), idesc_kv, (pfirst && k == 0) ? 0u : 1u);
          umma_commit(dv_done);
          if (!mbar_wait(ds_ready, pn & 1, werr, 303)) return false;
          tc_fence_after();
          const uint64_t q_mn = mnmaj(sQ + ps * AT_TILE_BYTES);
  #pragma unroll
          for (int k = 0; k < AT_TILE / 16; ++k)  // dK += dS^T Q   (k over the 128 queries)
            umma_ts(tdK, tdP + (k >> 2) * 64 + (k & 3) * 8, desc_step(q_mn, k * 2048),
                    idesc_kv, (pfirst && k == 0) ? 0u : 1u);
          umma_commit(dk_done);
          umma_commit(&q_empty[ps]);   // dK was the last MMA to read Q
          umma_commit(&o_empty[pso]);  // dV the last for dO, and delta has been read before ds_ready
          return true;
        };
        auto finish_dq = [&]() -> bool {
          if (!mbar_wait(dq_free, (pn & 1) ^ 1, werr, 304)) return false;
          tc_fence_after();
          const uint64_t k_mn = mnmaj(sK + pks * AT_TILE_BYTES);
          const uint64_t ds_mn = smem_desc_sw128(smem_u32(sDS + (pn & 1) * 2 * AT_TILE_BYTES), 16384, 1024);
  #pragma unroll
          for (int k = 0; k < AT_TILE / 16; ++k)  // dQ = dS K   (k over the 128 keys)
            umma_ss(tdQ, desc_step(ds_mn, k * 2048), desc_step(k_mn, k * 2048), idesc_q, k > 0 ? 1u : 0u);
          umma_commit(dq_full);
          umma_commit(&ds_free[pn & 1]);
          if (plast) {
            umma_commit(dkdv_full);
            umma_commit(&kv_empty[pks]);
          }
          return true;
        };
        int u = 0, n = 0;
        bool ok = true;
        for (int bh = blockIdx.x; bh < p.BH && ok; bh += gridDim.x) {
          for (int jt = nq - 1; jt >= 0 && ok; --jt, ++u) {
            const int ks = u & 1;
            if (!mbar_wait(&kv_full[ks], (u >> 1) & 1, werr, 305)) { ok = false; break; }
            const uint64_t k_k = kmaj(sK + ks * AT_TILE_BYTES), v_k = kmaj(sV + ks * AT_TILE_BYTES);
            for (int i = jt; i < nq; ++i, ++n) {
              const int s = n % BA_QS, so = n % BA_OS;
              if (!mbar_wait(&q_full[s], (n / BA_QS) & 1, werr, 306)) { ok = false; break; }
              // S^T = K Q^T once the P/dS warps have read the previous S^T (and written its P^T)
              if (pn >= 0 && !mbar_wait(p_ready, pn & 1, werr, 309)) { ok = false; break; }
              tc_fence_after();
              const uint64_t q_k = kmaj(sQ + s * AT_TILE_BYTES), do_k = kmaj(sDO + so * AT_TILE_BYTES);
  #pragma unroll
              for (int k = 0; k < AT_D / 16; ++k)
                umma_ss(tS, desc_step(k_k, k * 32), desc_step(q_k, k * 32), idesc_sdp, k > 0 ? 1u : 0u);
              umma_commit(s_full);
              if (pn >= 0 && !finish_dvdk()) { ok = false; break; }
              // dP^T = V dO^T over the previous dS^T: wait for the dK MMA that reads it
              if (!mbar_wait(dk_done, (n & 1) ^ 1, werr, 307)) { ok = false; break; }
              if (!mbar_wait(&o_full[so], (n / BA_OS) & 1, werr, 319)) { ok = false; break; }
              tc_fence_after();
  #pragma unroll
              for (int k = 0; k < AT_D / 16; ++k)
                umma_ss(tdP, desc_step(v_k, k * 32), desc_step(do_k, k * 32), idesc_sdp, k > 0 ? 1u : 0u);
              umma_commit(dp_full);
              if (pn >= 0 && !finish_dq()) { ok = false; break; }
              pn = n;
              ps = s;
              pso = so;
              pks = ks;
              pu = u;
              pfirst = (i == jt);
              plast = (i == nq - 1);
            }
          }
        }
        if (ok && pn >= 0 && mbar_wait(p_ready, pn & 1, werr, 309) && finish_dvdk()) finish_dq();
      }
    }
  } else if (warp < 12) {
    reg_alloc<BA_REG_PDS>();
    // ---------------- P/dS warps: one key row per thread, 64 queries per warpgroup ----------------
    const int g = (warp - 4) >> 2;      // query half of the tile
    const int quarter = warp & 3;       // TMEM lane quarter
    const int r = quarter * 32 + lane;  // key row within the tile
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t tS = tmem + BA_TM_S + lane_off + g * 64;
    const uint32_t tdP = tmem + BA_TM_DP + lane_off + g * 64;
    const uint32_t tP = tmem + BA_TM_P + lane_off + g * 32;
    const float sl2 = p.scale_log2;
    int n = 0;
    bool ok = true;
    for (int bh = blockIdx.x; bh < p.BH && ok; bh += gridDim.x) {
      for (int jt = nq - 1; jt >= 0 && ok; --jt) {
        for (int i = jt; i < nq; ++i, ++n) {
          const int s = n % BA_QS;
          ok = __all_sync(0xffffffffu, mbar_wait(s_full, n & 1, werr, 310) &&
                                           mbar_wait(&q_full[s], (n / BA_QS) & 1, werr, 311));
          if (!ok) break;
          tc_fence_after();
          const bool diag = (i == jt);  // key r is visible to query q iff r <= q
          // ---- P^T = 2^(S^T * scale * log2 e - lse2)
          uint32_t pw[32];  // P^T as packed bf16 pairs: what the dV MMA reads, reused for dS
          {
            uint32_t a0[32], a1[32];  // both TMEM loads in flight before one wait
            tmem_ld32(tS, a0);
            tmem_ld32(tS + 32, a1);
            tmem_wait_ld();
            const float4* l4 = reinterpret_cast<const float4*>(sLse + s * AT_TILE + g * 64);
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const float4 lv = l4[j];
              const uint32_t* src = (j < 8 ? a0 : a1) + 4 * (j & 7);
              float p0 = ex2_approx(fmaf(__uint_as_float(src[0]), sl2, -lv.x));
              float p1 = ex2_approx(fmaf(__uint_as_float(src[1]), sl2, -lv.y));
              float p2 = ex2_approx(fmaf(__uint_as_float(src[2]), sl2, -lv.z));
              float p3 = ex2_approx(fmaf(__uint_as_float(src[3]), sl2, -lv.w));
              if (diag) {
                const int q = g * 64 + 4 * j;
                if (q < r) p0 = 0.f;
                if (q + 1 < r) p1 = 0.f;
                if (q + 2 < r) p2 = 0.f;
                if (q + 3 < r) p3 = 0.f;
              }
              pw[2 * j] = pack_bf16x2(p0, p1);
              pw[2 * j + 1] = pack_bf16x2(p2, p3);
            }
          }
          // the P^T columns are rewritten once the previous tile's dV MMA has read them
          ok = __all_sync(0xffffffffu, mbar_wait(dv_done, (n & 1) ^ 1, werr, 312));
          if (!ok) break;
          tc_fence_after();
          tmem_st16(tP, *reinterpret_cast<const uint32_t(*)[16]>(pw));
          tmem_st16(tP + 16, *reinterpret_cast<const uint32_t(*)[16]>(pw + 16));
          tmem_wait_st();
          tc_fence_before();
          mbar_arrive(p_ready);
          // ---- dS^T = P^T (dP^T - delta)
          const int so = n % BA_OS;
          ok = __all_sync(0xffffffffu, mbar_wait(dp_full, n & 1, werr, 313) &&
                                           mbar_wait(&o_full[so], (n / BA_OS) & 1, werr, 320) &&
                                           mbar_wait(&ds_free[n & 1], ((n >> 1) & 1) ^ 1, werr, 314));
          uint8_t* dsrow = sDS + (n & 1) * 2 * AT_TILE_BYTES + g * AT_TILE_BYTES + r * 128;
          if (!ok) break;
          tc_fence_after();
          {
            uint32_t a0[32], a1[32];
            tmem_ld32(tdP, a0);
            tmem_ld32(tdP + 32, a1);
            tmem_wait_ld();
            const float4* d4 = reinterpret_cast<const float4*>(sDelta + so * AT_TILE + g * 64);
#pragma unroll
            for (int c = 0; c < 2; ++c) {
              uint32_t dk[16];
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                const float4 dv = d4[c * 8 + j];
                const uint32_t* src = (c == 0 ? a0 : a1) + 4 * j;
                const uint32_t w0 = pw[c * 16 + 2 * j], w1 = pw[c * 16 + 2 * j + 1];
                // dS^T = P^T (dP^T - delta) as packed bf16x2 products: the differences in fp32,
                // rounded to bf16 pairs, times the packed P^T pairs (4 instructions per pair of
                // elements instead of 7 with unpacking and fp32 products)
                const uint32_t g0 = pack_bf16x2(__uint_as_float(src[0]) - dv.x, __uint_as_float(src[1]) - dv.y);
                const uint32_t g1 = pack_bf16x2(__uint_as_float(src[2]) - dv.z, __uint_as_float(src[3]) - dv.w);
                dk[2 * j] = mul_bf16x2(w0, g0);
                dk[2 * j + 1] = mul_bf16x2(w1, g1);
              }
              tmem_st16(tdP + c * 16, dk);  // dS^T over dP^T columns already read
#pragma unroll
              for (int u4 = 0; u4 < 4; ++u4) {  // dS^T -> 128B-swizzled [key row][64 queries] block
                const int ch = c * 4 + u4;
                *reinterpret_cast<uint4*>(dsrow + ((ch ^ (r & 7)) << 4)) =
                    make_uint4(dk[4 * u4], dk[4 * u4 + 1], dk[4 * u4 + 2], dk[4 * u4 + 3]);
              }
            }
          }
          tmem_wait_st();
          fence_proxy_async_smem();
          tc_fence_before();
          mbar_arrive(ds_ready);
        }
      }
    }
  } else {
    // ---------------- drain warps: dQ per tile, dK/dV per key tile ----------------
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;  // TMEM lane: query row of dQ, key row of dK/dV
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const bool leader = (warp == 12 && lane == 0);
    float* acc = p.dq_acc + (size_t)blockIdx.x * p.Tp * AT_D;
    uint32_t sync_phase = 0;
    auto drain_sync = [&]() -> bool {
      mbar_arrive(drain_bar);
      const bool w = mbar_wait(drain_bar, sync_phase & 1, werr, 315);
      ++sync_phase;
      return __all_sync(0xffffffffu, w);
    };
    int u = 0, n = 0;
    bool ok = true;
    for (int bh = blockIdx.x; bh < p.BH && ok; bh += gridDim.x) {
      const int b = bh / p.NH, h = bh % p.NH;
      for (int jt = nq - 1; jt >= 0 && ok; --jt, ++u) {
        for (int i = jt; i < nq; ++i, ++n) {
          if (i == nq - 1) {
            // key tile jt done: dV and scale * dK out first (committed together with this
            // tile's dQ), so the next key tile can start accumulating while dQ is drained
            ok = __all_sync(0xffffffffu, mbar_wait(dkdv_full, u & 1, werr, 317));
            if (!ok) break;
            tc_fence_after();
            // dV packed to bf16 first, then dK, so at most 64 fp32 values are live
            uint32_t pv[32];
            {
              uint32_t a0[32], a1[32];
              tmem_ld32(tmem + BA_TM_DV + lane_off, a0);
              tmem_ld32(tmem + BA_TM_DV + lane_off + 32, a1);
              tmem_wait_ld();
              pack_row_bf16(pv, a0, a1, 1.f);
            }
            uint32_t pkk[32];
            {
              uint32_t a0[32], a1[32];
              tmem_ld32(tmem + BA_TM_DK + lane_off, a0);
              tmem_ld32(tmem + BA_TM_DK + lane_off + 32, a1);
              tmem_wait_ld();
              tc_fence_before();
              mbar_arrive(dkdv_free);
              pack_row_bf16(pkk, a0, a1, p.scale);
            }
            const int key = jt * AT_TILE + row;
            if (key < p.T) {
              const int64_t off = (int64_t)b * p.sb + (int64_t)key * p.st + (int64_t)h * p.sh;
              store_packed_row(p.dv + off, pv, p.D);
              store_packed_row(p.dk + off, pkk, p.D);
            }
          }
          ok = __all_sync(0xffffffffu, mbar_wait(dq_full, n & 1, werr, 316));
          if (!ok) break;
          tc_fence_after();
          uint32_t a0[32], a1[32];
          tmem_ld32(tmem + BA_TM_DQ + lane_off, a0);
          tmem_ld32(tmem + BA_TM_DQ + lane_off + 32, a1);
          tmem_wait_ld();
          tc_fence_before();
          mbar_arrive(dq_free);
          const int qrow = i * AT_TILE + row;
          if (jt == 0) {
            // key tile 0 is this query tile's last contribution: finish dQ
            if (i > 0) {
              // the accumulator's last reduce-add for tile i came from key tile 1, whose later
              // tiles i+1 .. nq-1 may still be in flight
              if (leader) {
                bulk_wait_upto(2 * (nq - 1 - i));  // two bulk groups (halves) per tile
                fence_proxy_async_global();
              }
              if (!(ok = drain_sync())) break;
              const float4* src = reinterpret_cast<const float4*>(acc + (size_t)qrow * AT_D);
#pragma unroll
              for (int c = 0; c < 16; ++c) {
                const float4 v = src[c];
                uint32_t* d = c < 8 ? a0 + 4 * c : a1 + 4 * (c - 8);
                d[0] = __float_as_uint(__uint_as_float(d[0]) + v.x);
                d[1] = __float_as_uint(__uint_as_float(d[1]) + v.y);
                d[2] = __float_as_uint(__uint_as_float(d[2]) + v.z);
                d[3] = __float_as_uint(__uint_as_float(d[3]) + v.w);
              }
            }
            if (qrow < p.T) {
              uint32_t w[32];
              pack_row_bf16(w, a0, a1, p.scale);
              store_packed_row(p.dq + (int64_t)b * p.sb + (int64_t)qrow * p.st + (int64_t)h * p.sh, w, p.D);
            }
          } else {
            // an earlier contribution: into the accumulator in L2 (a TMA store from the diagonal
            // key tile, which reaches query tile i first, reduce-adds after it)
            // two halves (d 0..31, 32..63) through the one staging buffer
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
              if (leader) bulk_wait_read0();  // the previous bulk op has finished reading sDQ
              if (!(ok = drain_sync())) break;
              uint8_t* rowp = sDQ + row * 128;
#pragma unroll
              for (int ch = 0; ch < 8; ++ch) {
                const uint32_t* src = (hf == 0 ? a0 : a1) + 4 * ch;
                *reinterpret_cast<uint4*>(rowp + ((ch ^ (row & 7)) << 4)) = make_uint4(src[0], src[1], src[2], src[3]);
              }
              fence_proxy_async_smem();
              if (!(ok = drain_sync())) break;
              if (leader) {
                if (hf == 0) fence_proxy_async_global();  // earlier generic reads of these rows come first
                const int grow = blockIdx.x * p.Tp + i * AT_TILE;
                if (i == jt)
                  tma_store_2d(&maps.dq_acc, sDQ, 32 * hf, grow);
                else
                  tma_reduce_add_2d(&maps.dq_acc, sDQ, 32 * hf, grow);
                bulk_commit();
              }
            }
            if (!ok) break;
          }
        }
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

// ==========================================================================================
// host side
// ==========================================================================================
// The prep kernel's grid has T/32 rows in y (at most 65535), so the tensor-core backward takes T up
// to 16383 tiles of 128 rows; attn_bwd sends longer rows to the CUDA-core backward.
constexpr int kBwdTcMaxT = (65535 * 32 / AT_TILE) * AT_TILE;  // 2,097,024

bool tc_bwd_supported(int D, int T, int dtype) {
  return tc_head_dim_ok(D) && dtype == ATTN_BF16 && T <= kBwdTcMaxT;
}

static int bwd_grid(int BH) { return BH < BA_MAX_CTAS ? BH : BA_MAX_CTAS; }

size_t attn_bwd_tc_ws(int B, int NH, int T, int D) {
  const size_t Tp = (size_t)((T + AT_TILE - 1) / AT_TILE) * AT_TILE;
  const size_t BH = (size_t)B * NH;
  (void)D;  // the dQ accumulator rows are one 64-wide head tile whatever the head_dim
  return 2 * align256(BH * Tp * 4) + align256((size_t)bwd_grid((int)BH) * Tp * AT_D * 4);
}

int attn_bwd_tc(const void* q, const void* k, const void* v, const void* o, const void* dout,
                const float* lse, void* dq, void* dk, void* dv, void* ws, int B, int NH, int T, int D,
                const int64_t* s, float scale, cudaStream_t stream) {
  if (!head_strides_ok(s[0], s[1], s[2], D) || !head_strides_ok(s[3], s[4], s[5], D) || !aligned(q, 16) ||
      !aligned(k, 16) || !aligned(v, 16) || !aligned(o, 16) || !aligned(dout, 16) || !aligned(dq, 16) ||
      !aligned(dk, 16) || !aligned(dv, 16)) {
    set_error("attn_bwd: the tensor-core path needs 16-byte aligned bf16 tensors with strides that are "
              "multiples of 8 elements");
    return ATTN_ERR_ARG;
  }
  const int nq = (T + AT_TILE - 1) / AT_TILE;
  const int Tp = nq * AT_TILE;
  const int BH = B * NH;
  const int sms = current_device_sms();
  int grid = bwd_grid(BH);
  if (grid > sms) grid = sms;
  uint8_t* w = reinterpret_cast<uint8_t*>(ws);
  float* lse2 = reinterpret_cast<float*>(w);
  float* delta = reinterpret_cast<float*>(w + align256((size_t)BH * Tp * 4));
  float* dq_acc = reinterpret_cast<float*>(w + 2 * align256((size_t)BH * Tp * 4));
  if (T > kBwdTcMaxT) {  // the prep kernel's grid.y; attn_bwd routes such rows elsewhere first
    set_error("attn_bwd: T = %d exceeds the tensor-core backward's limit of %d", T, kBwdTcMaxT);
    return ATTN_ERR_UNSUPPORTED;
  }
  const cudaError_t prep = launch_pdl(attn_bwd_prep_kernel, dim3((unsigned)BH, (unsigned)(Tp / 32)), dim3(256), 0,
                                      stream, (const __nv_bfloat16*)o, (const __nv_bfloat16*)dout, lse, lse2,
                                      delta, NH, T, Tp, D, s[3], s[4], s[5]);
  count_launch();
  if (int rc = check_launch("attn_bwd_prep_kernel", prep)) return rc;

  BwdMaps maps;
  if (!make_head_map(&maps.q, q, B, NH, T, D, s[0], s[1], s[2]) ||
      !make_head_map(&maps.k, k, B, NH, T, D, s[0], s[1], s[2]) ||
      !make_head_map(&maps.v, v, B, NH, T, D, s[0], s[1], s[2]) ||
      !make_head_map(&maps.dout, dout, B, NH, T, D, s[3], s[4], s[5]))
    return ATTN_ERR_CUDA;
  {
    const uint64_t dims[2] = {(uint64_t)AT_D, (uint64_t)grid * Tp};
    const uint64_t strides[1] = {AT_D * 4};
    const uint32_t box[2] = {32, AT_TILE};
    if (!make_tmap_f32(&maps.dq_acc, dq_acc, 2, dims, strides, box)) return ATTN_ERR_CUDA;
  }
  BwdParams p;
  p.NH = NH;
  p.T = T;
  p.nq = nq;
  p.Tp = Tp;
  p.BH = BH;
  p.D = D;
  p.scale = scale;
  p.scale_log2 = scale * LOG2E;
  p.lse2 = lse2;
  p.delta = delta;
  p.dq_acc = dq_acc;
  p.dq = reinterpret_cast<__nv_bfloat16*>(dq);
  p.dk = reinterpret_cast<__nv_bfloat16*>(dk);
  p.dv = reinterpret_cast<__nv_bfloat16*>(dv);
  p.sb = s[0];
  p.st = s[1];
  p.sh = s[2];
  p.err = dev_error_ptr();
  if (!p.err) return ATTN_ERR_CUDA;
  static CtxOnce attr_done;
  if (!set_smem_limit_once(attn_bwd_tc_kernel, BA_SMEM, attr_done)) return ATTN_ERR_CUDA;
  static int launch_regs = 0;
  if (!launch_regs_match(attn_bwd_tc_kernel, BA_LAUNCH_REGS, launch_regs, "attn_bwd_tc_kernel")) return ATTN_ERR_CUDA;
  const cudaError_t launched = launch_pdl(attn_bwd_tc_kernel, dim3(grid), dim3(BA_THREADS), BA_SMEM, stream, maps, p);
  count_launch();
  return check_launch("attn_bwd_tc_kernel", launched);
}

}  // namespace attn
